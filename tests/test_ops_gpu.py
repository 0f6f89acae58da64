"""GPU parity of the stand-alone ops against the CPU oracle (and torch._int_mm)."""
import ctypes

import numpy as np
import pytest

import dfssm_oracle as O
from dfssm_b200 import _lib
from dfssm_b200 import dfssm_format as fmt
from helpers import ptr, stream

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


@pytest.mark.parametrize("N,K", [(8512, 2048), (2048, 4096), (10576, 2560), (2560, 5120)])
@pytest.mark.parametrize("M", [1, 8, 32, 64, 100, 128, 512])
def test_scaffold_gemm_bit_exact(lib, M, N, K):
    """Config 3: 1-bit packed x int8 -> int32, bit-exact vs the oracle and torch._int_mm
    (M < 8: dp4a GEMV; 8..95: mma.sync; >= 96: tcgen05 with the accumulator in TMEM, batch tiles of
    32, 64 or 128 rows by the tile count)."""
    rng = np.random.default_rng(M * 7 + N)
    packed = rng.integers(0, 2**32, size=(N, K // 32), dtype=np.uint32)
    x = rng.standard_normal((M, K)).astype(np.float16)
    _, q = O.quantize_int8(x)
    dev = torch.device("cuda")
    tp = torch.from_numpy(packed.view(np.int32)).to(dev)
    tq = torch.from_numpy(q).to(dev)
    acc = torch.empty(M, N, dtype=torch.int32, device=dev)
    ws = torch.empty(lib.dfssm_scaffold_gemm_workspace(M, K), dtype=torch.uint8, device=dev)
    _lib.check(lib.dfssm_scaffold_gemm(ptr(tp), ptr(tq), M, N, K, ptr(acc), ptr(ws), stream()))
    torch.cuda.synchronize()
    got = acc.cpu().numpy()
    signs = fmt.unpack_signs(packed.view(np.int32), K)
    np.testing.assert_array_equal(got, O.scaffold_int32(q, signs.astype(np.float32)))
    # the reference's own library call: torch._int_mm on the unpacked +-1 weights, padded rows
    mp = max(32, (M + 7) // 8 * 8)
    qp = torch.zeros(mp, K, dtype=torch.int8, device=dev)
    qp[:M] = tq
    ref = torch._int_mm(qp, torch.from_numpy(signs).to(dev).t().contiguous())[:M]
    np.testing.assert_array_equal(got, ref.cpu().numpy())


def test_scaffold_gemm_rejects_bad_k(lib):
    dev = torch.device("cuda")
    z = torch.zeros(1024, dtype=torch.int32, device=dev)
    rc = lib.dfssm_scaffold_gemm(ptr(z), ptr(z), 1, 4, 100, ptr(z), ptr(z), stream())
    assert rc == 1


@pytest.mark.parametrize("B", [1, 3])
def test_conv_step(lib, B):
    rng = np.random.default_rng(B)
    D = 4352
    state = rng.standard_normal((B, D, 3)).astype(np.float16).astype(np.float32)
    xbc = rng.standard_normal((B, D)).astype(np.float16)
    w = rng.normal(0, 0.5, (D, 4)).astype(np.float16)
    b = rng.normal(0, 0.1, D).astype(np.float16)
    dev = torch.device("cuda")
    ts = torch.from_numpy(np.ascontiguousarray(state.transpose(0, 2, 1))).to(dev)  # tap-major
    tx = torch.from_numpy(xbc).to(dev)
    tw, tb = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)  # keep alive across the launch
    _lib.check(lib.dfssm_conv_step(ptr(ts), ptr(tx), D, ptr(tw), ptr(tb), B, D, stream()))
    torch.cuda.synchronize()
    st = state.copy()
    ref = O.conv_step(st, xbc, w, b)
    np.testing.assert_array_equal(ts.cpu().numpy().transpose(0, 2, 1), st)
    got = tx.cpu().numpy().astype(np.float32)
    # one fp16 ulp of the output, plus fp32 cancellation in the 4-tap sum (FMA contraction differs)
    np.testing.assert_allclose(got, ref.astype(np.float32), rtol=2**-10, atol=1e-5)


@pytest.mark.parametrize("B,H", [(1, 64), (4, 8)])
def test_ssm_step(lib, B, H):
    rng = np.random.default_rng(H + B)
    P, N = 64, 128
    di = H * P
    xbc = rng.standard_normal((B, di + 2 * N)).astype(np.float16)
    dt = rng.standard_normal((B, H)).astype(np.float16)
    dt_bias = rng.uniform(-4, 0, H).astype(np.float32)
    A_log = np.log(rng.uniform(1, 16, H)).astype(np.float32)
    D = rng.uniform(0.5, 1.5, H).astype(np.float32)
    h = rng.standard_normal((B, H, P, N)).astype(np.float32)
    dev = torch.device("cuda")
    th = torch.from_numpy(h).to(dev)
    ty = torch.zeros(B, di, dtype=torch.float16, device=dev)
    args = [torch.from_numpy(a).to(dev) for a in (xbc, dt, dt_bias, A_log, D)]
    _lib.check(lib.dfssm_ssm_step(ptr(args[0]), di + 2 * N, ptr(args[1]), H, ptr(args[2]), ptr(args[3]),
                                  ptr(args[4]), ptr(th), ptr(ty), di, B, H, P, N, stream()))
    torch.cuda.synchronize()
    hr = h.copy()
    y = O.ssm_step(hr, xbc[:, :di], xbc[:, di:di + N], xbc[:, di + N:], dt, dt_bias, A_log, D)
    np.testing.assert_allclose(th.cpu().numpy(), hr, rtol=1e-5, atol=1e-5)
    yg = ty.cpu().numpy().astype(np.float32)
    yr = y.astype(np.float32)
    assert np.abs(yg - yr).max() <= 2 * float(np.abs(yr).max()) * 2**-11 + 1e-3


@pytest.mark.parametrize("B,V,d", [(1, 50280, 2048), (5, 3001, 256), (9, 1000, 2560)])
def test_lm_head_argmax(lib, B, V, d):
    rng = np.random.default_rng(V)
    Eq = rng.integers(-127, 128, (V, d), dtype=np.int8)
    Es = np.full(V, np.float16(0.01), np.float32)
    x = rng.standard_normal((B, d)).astype(np.float16)
    dev = torch.device("cuda")
    tE, tS, tx = (torch.from_numpy(a).to(dev) for a in (Eq, Es, x))
    lg = torch.empty(B, V, dtype=torch.float32, device=dev)
    nxt = torch.empty(B, dtype=torch.int32, device=dev)
    ws = torch.empty(lib.dfssm_lm_head_workspace(B), dtype=torch.uint8, device=dev)
    _lib.check(lib.dfssm_lm_head_argmax(ptr(tE), ptr(tS), V, d, ptr(tx), B, ptr(lg), ptr(nxt), ptr(ws), stream()))
    torch.cuda.synchronize()
    ref = (x.astype(np.float64) @ Eq.T.astype(np.float64)) * Es[None, :]
    got = lg.cpu().numpy()
    # fp32 accumulation (tensor-core accumulation for batch >= 8): 1e-5 of the logit scale
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    g16 = got.astype(np.float16)
    n = nxt.cpu().numpy()
    # argmax over the kernel's own fp16-rounded logits, first index on ties
    np.testing.assert_array_equal(n, np.argmax(g16, axis=-1))
    # and the oracle's choice is within one fp16 ulp of it
    r16 = ref.astype(np.float32).astype(np.float16)
    top = r16.max(-1)
    assert np.all(np.abs(r16[np.arange(B), n].astype(np.float32) - top.astype(np.float32)) <= 0.125)


def test_quantiser_division_matches_ieee(lib):
    """The activation quantiser divides by its scale with two FMAs and a reciprocal
    (common.cuh div_rn_rcp); over every finite fp16 dividend and positive fp16 divisor its
    quotient must equal IEEE fp32 division bit for bit."""
    out = (ctypes.c_ulonglong * 2)()
    assert lib.dfssm_selftest_division(0, out) == 0, lib.dfssm_last_error()
    assert (out[0], out[1]) == (0, 0)


# ---------------------------------------------------------------- sampling epilogue

def _sample(lib, logits, seen_mask, T, top_p, rep, seed=0, counters=None):
    import torch
    B, V = logits.shape
    W = (V + 31) // 32
    bits = np.zeros((B, W), np.uint32)
    for b, v in zip(*np.nonzero(seen_mask)):
        bits[b, v >> 5] |= np.uint32(1 << (v & 31))
    dev = "cuda"
    tl = torch.from_numpy(logits.astype(np.float32)).to(dev)
    tb = torch.from_numpy(bits.view(np.int32)).to(dev)
    ctr = counters if counters is not None else torch.zeros(B, dtype=torch.int64, device=dev)
    nxt = torch.empty(B, dtype=torch.int32, device=dev)
    mass = torch.empty(B, dtype=torch.float32, device=dev)
    cnt = torch.empty(B, dtype=torch.int32, device=dev)
    _lib.check(lib.dfssm_sample(ptr(tl), B, V, ptr(tb), T, top_p, rep, seed, ptr(ctr), ptr(nxt), ptr(mass),
                                ptr(cnt), stream()))
    torch.cuda.synchronize()
    return nxt.cpu().numpy(), mass.cpu().numpy(), cnt.cpu().numpy()


@pytest.mark.parametrize("top_p", [0.0, 0.3, 0.9, 1.0])
def test_sampling_nucleus_matches_reference_rule(lib, top_p):
    """Kept set (count, mass) and the drawn token against the sort-based rule of
    eval/gen_test.py:69-87 restated in the oracle; random logits have distinct probabilities."""
    rng = np.random.default_rng(1)
    B, V = 4, 3001
    logits = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    seen = rng.random((B, V)) < 0.1
    for seed in range(3):
        nxt, mass, cnt = _sample(lib, logits, seen, 0.7, top_p, 1.2, seed=seed)
        for b in range(B):
            kept, p, kmass = O.sample_nucleus(logits[b], seen[b], 0.7, top_p, 1.2)
            # the boundary token may flip only if its preceding mass is within fp32 summation error
            assert abs(int(cnt[b]) - len(kept)) <= 1, (b, cnt[b], len(kept))
            assert abs(float(mass[b]) - kmass) < 2e-4 + (p[kept[-1]] if abs(int(cnt[b]) - len(kept)) else 0)
            extended = set(kept.tolist()) | set(np.argsort(-p, kind="stable")[:len(kept) + 1].tolist())
            assert int(nxt[b]) in extended


def test_sampling_top_p_zero_is_penalised_argmax(lib):
    """top_p = 0 keeps only the most likely token; the repetition penalty divides the logit of a
    seen token whatever its sign (eval/gen_test.py:71-72), so a seen token with a negative logit
    becomes the most likely one when the others are more negative."""
    logits = np.full((2, 500), -8.0, np.float32)
    logits[0, 17] = -1.0          # unseen, best
    logits[1, 17] = -1.0
    logits[1, 42] = -2.0          # seen in row 1: -2 / 4 = -0.5 beats -1
    seen = np.zeros((2, 500), bool)
    seen[1, 42] = True
    nxt, mass, cnt = _sample(lib, logits, seen, 1.0, 0.0, 4.0)
    assert nxt.tolist() == [17, 42] and cnt.tolist() == [1, 1]


def test_sampling_distribution_matches_softmax(lib):
    """2000 draws (the per-row counter advances each call) follow the softmax within 5 sigma."""
    import torch
    logits = np.array([[1.0, 0.5, 0.0, -0.5, -1.0, 2.0]], np.float32)
    seen = np.zeros_like(logits, bool)
    ctr = torch.zeros(1, dtype=torch.int64, device="cuda")
    n = 2000
    counts = np.zeros(6)
    for _ in range(n):
        nxt, _, _ = _sample(lib, logits, seen, 1.0, 1.0, 1.0, seed=7, counters=ctr)
        counts[nxt[0]] += 1
    assert int(ctr.item()) == n
    p = np.exp(logits[0] - logits[0].max())
    p /= p.sum()
    sigma = np.sqrt(n * p * (1 - p))
    assert np.all(np.abs(counts - n * p) < 5 * sigma), (counts, n * p)
