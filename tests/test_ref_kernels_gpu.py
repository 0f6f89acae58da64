"""Pins the oracle's restatement of the reference CUDA kernels (conv_step_kernel, ssm_step_kernel,
inference/gpu/df_ssm_kernels.cu:27-103) to the reference kernels themselves.  oracle/build_ref.py
--gpu-kernels compiles them from the reference checkout (HEADDIM patched to 64) into oracle/_ref/;
this test is skipped where that build is absent."""
import importlib.machinery
import importlib.util
import os

import numpy as np
import pytest

import dfssm_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
SO = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "ref_kernels", "df_ssm_kernels_h64.so")
B, H, P, N, D_INNER, D_XBC = 2, 64, 64, 128, 4096, 4352  # compile-time dims of the reference build


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(SO):
        pytest.skip("reference kernels not built (python oracle/build_ref.py --gpu-kernels)")
    loader = importlib.machinery.ExtensionFileLoader("df_ssm_kernels_h64", SO)
    spec = importlib.util.spec_from_loader("df_ssm_kernels_h64", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def test_conv_step_restatement_matches_reference_kernel(ref):
    rng = np.random.default_rng(0)
    state = rng.standard_normal((B, D_XBC, 3)).astype(np.float16)
    xbc = rng.standard_normal((B, D_XBC)).astype(np.float16)
    w = rng.normal(0, 0.5, (D_XBC, 4)).astype(np.float16)
    bias = rng.normal(0, 0.1, D_XBC).astype(np.float16)
    dev = torch.device("cuda")
    ts, tx = torch.from_numpy(state.copy()).to(dev), torch.from_numpy(xbc.copy()).to(dev)
    ref.conv_step(ts, tx, torch.from_numpy(w).to(dev), torch.from_numpy(bias).to(dev), D_XBC)
    torch.cuda.synchronize()
    st = state.copy()
    out = O.conv_step(st, xbc, w, bias)
    np.testing.assert_array_equal(ts.cpu().numpy(), st)
    np.testing.assert_allclose(tx.cpu().numpy().astype(np.float32), out.astype(np.float32), rtol=2**-10, atol=1e-5)


def test_ssm_step_restatement_matches_reference_kernel(ref):
    rng = np.random.default_rng(1)
    xbc = rng.standard_normal((B, D_XBC)).astype(np.float16)
    dt = rng.standard_normal((B, H)).astype(np.float16)
    dt_bias = rng.uniform(-4, 0, H).astype(np.float32)
    A_log = np.log(rng.uniform(1, 16, H)).astype(np.float32)
    Dp = rng.uniform(0.5, 1.5, H).astype(np.float32)
    h = (rng.standard_normal((B, H, P, N)) * 0.5).astype(np.float16)
    dev = torch.device("cuda")
    th = torch.from_numpy(h.copy()).to(dev)
    ty = torch.zeros(B, D_INNER, dtype=torch.float16, device=dev)
    ref.ssm_step(th, torch.from_numpy(xbc).to(dev), torch.from_numpy(dt).to(dev), torch.from_numpy(dt_bias).to(dev),
                 torch.from_numpy(A_log).to(dev), torch.from_numpy(Dp).to(dev), ty)
    torch.cuda.synchronize()
    hr = h.copy()  # fp16 storage, as the reference kernel keeps it
    y = O.ssm_step(hr, xbc[:, :D_INNER], xbc[:, D_INNER:D_INNER + N], xbc[:, D_INNER + N:], dt, dt_bias, A_log, Dp)
    got_h = th.cpu().numpy().astype(np.float32)
    want_h = hr.astype(np.float32)
    np.testing.assert_allclose(got_h, want_h, rtol=2**-10, atol=1e-6)  # one fp16 ulp (FMA contraction)
    np.testing.assert_allclose(ty.cpu().numpy().astype(np.float32), y.astype(np.float32), rtol=2e-3, atol=2e-3)
