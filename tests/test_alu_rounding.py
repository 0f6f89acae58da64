"""CPU check of the exact ALU rounding used by the kernels in place of F2H/H2F conversions
(common.cuh: round_h, rint_alu, i8_to_f), emulated with the same IEEE fp32 operations."""
import numpy as np

F32 = np.float32


def round_h_alu(v):
    v = np.asarray(v, F32)
    e = (v.view(np.uint32) >> 23) & 0xFF
    e = np.clip(e, 113, 160)
    M = (((e + 13) << 23) | 0x400000).astype(np.uint32).view(F32)
    with np.errstate(over="ignore", invalid="ignore"):
        r = np.copysign((v + M) - M, v)  # numpy float32 add/sub: IEEE round-to-nearest-even
        return np.where(np.abs(r) > 65504, np.copysign(np.inf, v), r).astype(F32)


def test_round_h_matches_fp16_conversion():
    rng = np.random.default_rng(0)
    vals = [rng.standard_normal(200000).astype(F32) * F32(s) for s in (1e-7, 1e-5, 1e-3, 1, 30, 3e3, 6e4)]
    # exact ties halfway between fp16 neighbours, subnormals, overflow boundary, zeros
    h = rng.integers(0, 0x7BFF, 50000).astype(np.uint16).view(np.float16)
    nxt = np.nextafter(h, np.float16(np.inf))
    ties = ((h.astype(np.float64) + nxt.astype(np.float64)) / 2).astype(F32)
    edge = np.array([0.0, -0.0, 65504, 65519.99, 65520, -65520, 70000, 5.96e-8, 2.98e-8, 2.99e-8, 6.1e-5], F32)
    v = np.concatenate(vals + [ties, -ties, edge])
    ref = v.astype(np.float16).astype(F32)
    got = round_h_alu(v)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_rint_alu_matches_rne():
    v = np.concatenate([np.arange(-300, 300, 0.5, dtype=F32), np.random.default_rng(1).uniform(-1e6, 1e6, 10000).astype(F32)])
    got = (v + F32(12582912.0)) - F32(12582912.0)
    np.testing.assert_array_equal(got, np.rint(v))


def test_int8_magic_conversion():
    q = np.arange(-128, 128, dtype=np.int32)
    biased = (q + 128).astype(np.uint32)  # (byte ^ 0x80)
    f = (biased | np.uint32(0x4B000000)).view(F32) - F32(8388736.0)
    np.testing.assert_array_equal(f, q.astype(F32))
