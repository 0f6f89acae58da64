"""Allocation-free scaffold GEMM (dfssm_scaffold_gemm_noalloc).

Callers that cannot allocate device memory where they run the GEMM (allocator callbacks, plug-in
hosts that own the memory pool, loops that must not block on an allocation) use this entry point.
It keeps its scratch in a fixed array inside the library instead of a caller workspace.  This file
is collected last on purpose: it checks the variant against the workspace-based entry point,
through the C ABI, on two calls in a row, and must pass alone in a fresh process or after every
other test."""
import numpy as np
import pytest

import dfssm_oracle as O
from dfssm_b200 import _lib
from helpers import ptr, stream

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _inputs(rng, M, N, K, dev):
    packed = rng.integers(0, 2**32, size=(N, K // 32), dtype=np.uint32)
    _, q = O.quantize_int8(rng.standard_normal((M, K)).astype(np.float16))
    return torch.from_numpy(packed.view(np.int32)).to(dev), torch.from_numpy(q).to(dev)


def _int_mm_ref(tp, tq, N, K):
    """torch._int_mm on the unpacked +-1 weights (df_ssm_inference.py:23-29,157); needs M > 16."""
    import ref_torch as R
    return torch._int_mm(tq, R.unpack_to_int8(tp, N, K).T.contiguous())


# consecutive calls with different shapes and data, through every kernel the entry point can pick
# (1-bit GEMV below 8 rows, mma.sync, tcgen05), up to the documented limits M = 2048 and
# M * K = 2 MiB: the shared scratch keeps each call's contents, so every later result shows that
# nothing stale leaks into it
CASES = ((32, 8512, 2048), (7, 2048, 4096), (2048, 2048, 1024), (128, 8512, 2048))


def test_noalloc_matches_workspace_entry_point_twice():
    lib = _lib.load()
    dev = torch.device("cuda")
    rng = np.random.default_rng(11)
    for M, N, K in CASES:
        tp, tq = _inputs(rng, M, N, K, dev)
        want = torch.empty(M, N, dtype=torch.int32, device=dev)
        ws = torch.empty(lib.dfssm_scaffold_gemm_workspace(M, K), dtype=torch.uint8, device=dev)
        _lib.check(lib.dfssm_scaffold_gemm(ptr(tp), ptr(tq), M, N, K, ptr(want), ptr(ws), stream()))
        got = torch.full((M, N), -1, dtype=torch.int32, device=dev)
        _lib.check(lib.dfssm_scaffold_gemm_noalloc(ptr(tp), ptr(tq), M, N, K, ptr(got), stream()))
        torch.cuda.synchronize()
        # integer accumulators: the tolerance of the scaffold tests is exact equality
        np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())
        if M > 16:
            np.testing.assert_array_equal(got.cpu().numpy(), _int_mm_ref(tp, tq, N, K).cpu().numpy())


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    dev = torch.device("cuda")
    z = torch.zeros(16, dtype=torch.int32, device=dev)
    rc = lib.dfssm_scaffold_gemm_noalloc(ptr(z), ptr(z), 1024, 8, 4096, ptr(z), stream())  # M*K = 4 MiB
    assert rc == 1
    assert b"exceeds the fixed scratch" in lib.dfssm_last_error()
    rc = lib.dfssm_scaffold_gemm_noalloc(ptr(z), ptr(z), 2049, 8, 128, ptr(z), stream())  # M > 2048
    assert rc == 1
    assert b"exceeds the fixed scratch" in lib.dfssm_last_error()
