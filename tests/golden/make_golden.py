"""Generate golden vectors by running the reference's own decode driver.

Runs cs-cmyk/df-ssm's inference/gpu/df_ssm_inference.py (class DFSSMModel) on the
CPU of the build container, imported from the reference checkout given by
--ref (it is not available where the tests run, so its outputs are committed as
.npz fixtures next to this script).  Patches applied, all at run time:

  * module constants (df_ssm_inference.py:15-19) set from the synthetic dims,
    HEADDIM = 64 (the shipped 32 leaves half of the SSM channels unwritten);
  * the model is populated from the synthetic weights instead of `_load`, whose
    norm dtypes disagree with the exporter (df_ssm_inference.py:105-110), with the
    same tensor dtypes `_load` produces (LoRA dequantised to fp16, int8 +-1 weights
    transposed, fp16 norms);
  * `_graph` is replaced by a direct call of `_run_layers` (no CUDA graph on a CPU);
  * `df_ssm_kernels` (a CUDA extension) is replaced by the torch restatement of
    conv_step_kernel / ssm_step_kernel (df_ssm_kernels.cu:27-47, 53-103) in
    oracle/ref_torch.py.  That restatement is pinned separately against the real
    CUDA kernels on a GPU (tests/test_parity_ref_gpu.py);
  * variant "f32state" allocates h/conv state in fp32 instead of fp16
    (df_ssm_inference.py:114-121), the contract the B200 engine implements.

Usage:  python tests/golden/make_golden.py --ref <path to df-ssm checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from dfssm_b200 import synthetic  # noqa: E402

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
from ref_torch import conv_step_torch, make_ssm_step_torch  # noqa: E402


def load_reference(ref_root: str, d):
    stub = types.ModuleType("df_ssm_kernels")
    stub.conv_step = conv_step_torch
    stub.ssm_step = make_ssm_step_torch(d.d_inner, d.d_state, d.nheads, d.headdim)
    sys.modules["df_ssm_kernels"] = stub
    path = os.path.join(ref_root, "inference", "gpu", "df_ssm_inference.py")
    spec = importlib.util.spec_from_file_location("df_ssm_inference_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.D_MODEL, mod.D_INNER, mod.D_XBC = d.d_model, d.d_inner, d.d_xbc
    mod.D_STATE, mod.NHEADS, mod.HEADDIM = d.d_state, d.nheads, d.headdim
    mod.N_LAYERS, mod.VOCAB_SIZE, mod.IN_PROJ_OUT = d.n_layer, d.vocab, d.n_in
    mod.SSM_DIM = d.nheads * d.headdim
    return mod


def build_model(mod, w, batch, state_f32: bool):
    d = w.dims
    m = object.__new__(mod.DFSSMModel)
    m.device, m.batch_size, m.layers = "cpu", batch, []
    m.embedding = torch.from_numpy(w.embedding_f16().copy())
    from dfssm_b200.dfssm_format import unpack_signs
    for L in w.layers:
        lw = mod.LayerWeights()
        for name, p, k in (("in", L.in_proj, d.d_model), ("out", L.out_proj, d.d_inner)):
            signs = torch.from_numpy(unpack_signs(p.packed, k))
            setattr(lw, f"{name}_w_T", signs.T.contiguous())
            setattr(lw, f"{name}_scale", torch.from_numpy(p.scale.copy()))
            A = (torch.from_numpy(p.lora_A).float() * torch.from_numpy(p.lora_A_s).float()[:, None]).half()
            Bm = (torch.from_numpy(p.lora_B).float() * torch.from_numpy(p.lora_B_s).float()[:, None]).half()
            setattr(lw, f"{name}_lora_A", A)
            setattr(lw, f"{name}_lora_B", Bm)
        lw.conv_weight = torch.from_numpy(L.conv_w.copy())
        lw.conv_bias = torch.from_numpy(L.conv_b.copy())
        lw.A_log = torch.from_numpy(L.A_log.copy())
        lw.D = torch.from_numpy(L.D.copy())
        lw.dt_bias = torch.from_numpy(L.dt_bias.copy())
        lw.norm_weight = torch.from_numpy(L.norm_w).half()
        lw.layer_norm_weight = torch.from_numpy(L.ln_w).half()
        m.layers.append(lw)
    m.norm_f_weight = torch.from_numpy(w.norm_f).half()
    m._alloc_state()
    if state_f32:
        m.h_states = [h.float() for h in m.h_states]
        m.conv_states = [c.float() for c in m.conv_states]
    m._graph = types.SimpleNamespace(replay=m._run_layers)
    return m


def run(mod, w, batch, prompts, n_steps, state_f32):
    m = build_model(mod, w, batch, state_f32)
    m.reset_state()
    captured = []
    real_int_mm = torch._int_mm

    def spy(a, b):
        out = real_int_mm(a, b)
        if len(captured) < 2:
            captured.append((a.clone(), out.clone()))
        return out

    torch._int_mm = spy
    try:
        tok = None
        with torch.no_grad():
            for t in range(prompts.shape[1]):
                logits = m.forward(torch.from_numpy(prompts[:, t]))
                tok = logits.argmax(-1)
            toks, logs = [], []
            for _ in range(n_steps):
                toks.append(tok.numpy().copy())
                logits = m.forward(tok)
                logs.append(logits.numpy().copy())
                tok = logits.argmax(-1)
    finally:
        torch._int_mm = real_int_mm
    return dict(tokens=np.stack(toks), logits=np.stack(logs),
                h=[h.numpy().copy() for h in m.h_states], conv=[c.numpy().copy() for c in m.conv_states],
                mm0_in=captured[0][0].numpy(), mm0_out=captured[0][1].numpy())


CASES = {
    # name: (shape, n_layer, vocab, batch, prompt_len, n_steps, seed)
    "tiny": ("tiny", 2, None, 2, 4, 12, 0),
    "cfg0": ("1.3b", 2, None, 1, 16, 8, 0),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--cases", default=",".join(CASES))
    a = ap.parse_args()
    torch.set_num_threads(4)
    for name in a.cases.split(","):
        shape, nl, vocab, batch, plen, steps, seed = CASES[name]
        d = synthetic.make_dims(shape, nl, vocab)
        w = synthetic.make_weights(d, seed=seed)
        prompts = synthetic.make_prompts(d.vocab, batch, plen, seed=seed)
        mod = load_reference(a.ref, d)
        out = {}
        for variant, f32 in (("f16state", False), ("f32state", True)):
            r = run(mod, w, batch, prompts, steps, f32)
            B = batch
            nh_keep = min(2, d.nheads)
            out[f"{variant}_tokens"] = r["tokens"]
            if d.vocab <= 4096:
                out[f"{variant}_logits"] = r["logits"]
            else:
                lg = r["logits"].astype(np.float32)
                top = np.argsort(-lg, axis=-1, kind="stable")[..., :16]
                out[f"{variant}_top_idx"] = top.astype(np.int32)
                out[f"{variant}_top_val"] = np.take_along_axis(r["logits"], top, -1)
                out[f"{variant}_logits_head"] = r["logits"][..., :256]
            for l in range(nl):
                out[f"{variant}_h{l}"] = r["h"][l][:, :nh_keep].astype(np.float32)
                out[f"{variant}_hsum{l}"] = r["h"][l].astype(np.float64).sum(axis=(2, 3))
                out[f"{variant}_conv{l}"] = r["conv"][l].astype(np.float32)
            out[f"{variant}_mm0_in"] = r["mm0_in"][:B]
            out[f"{variant}_mm0_out"] = r["mm0_out"][:B]
        out["prompts"] = prompts
        np.savez_compressed(os.path.join(HERE, f"golden_{name}.npz"), **out)
        print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
