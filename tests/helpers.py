"""Shared helpers for the GPU parity tests."""
import ctypes

import numpy as np

import dfssm_oracle as O
from dfssm_b200 import dfssm_format as fmt
from dfssm_b200 import synthetic


def weights(shape="tiny", n_layer=2, seed=0, vocab=None):
    return synthetic.make_weights(synthetic.make_dims(shape, n_layer, vocab), seed=seed)


def model(w, batch, **kw):
    from dfssm_b200.model import DFSSMModel
    return DFSSMModel(w, device="cuda", batch_size=batch, **kw)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def f16_ulp(x):
    """Spacing of fp16 numbers at |x|."""
    a = np.abs(np.asarray(x, np.float32)).astype(np.float16)
    return (np.nextafter(a, np.float16(np.inf)).astype(np.float32) - a.astype(np.float32))


def oracle_layer_parts(w, l, x16, conv_state, h_state):
    """The oracle's in_proj / conv / SSM / gate / out_proj for one layer, returning intermediates."""
    d, L = w.dims, w.layers[l]
    m = O.OracleModel.__new__(O.OracleModel)
    m.w, m.d, m.div_mode, m._signs, m.cache_signs = w, d, "cuda", {}, False
    m._lora = {l: (O.lora_dequant(L.in_proj), O.lora_dequant(L.out_proj))}
    proj = m.proj(O.rms_norm_f16(x16, L.ln_w), l, "in_proj")
    z = proj[:, :d.d_inner]
    xbc = O.conv_step(conv_state, proj[:, d.d_inner:d.d_inner + d.d_xbc].copy(), L.conv_w, L.conv_b)
    dt = proj[:, d.d_inner + d.d_xbc:]
    y = O.ssm_step(h_state, xbc[:, :d.d_inner], xbc[:, d.d_inner:d.d_inner + d.d_state],
                   xbc[:, d.d_inner + d.d_state:], dt, L.dt_bias, L.A_log, L.D)
    gated = O.gate(y, z)
    out = m.proj(O.rms_norm_f16(gated, L.norm_w), l, "out_proj")
    xo = (x16.astype(np.float32) + out.astype(np.float32)).astype(np.float16)
    return dict(z=z, xbc=xbc, dt=dt, y=y, gated=gated, x=xo)
