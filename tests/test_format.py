"""CPU tests: .dfssm byte map, sign packing, synthetic generator, loader validation."""
import ctypes
import os
import struct

import numpy as np
import pytest

from dfssm_b200 import dfssm_format as fmt
from dfssm_b200 import synthetic


def tiny(n_layer=2, seed=0):
    d = synthetic.make_dims("tiny", n_layer)
    return synthetic.make_weights(d, seed=seed)


def test_header_matches_exporter_struct():
    # export_dfssm.py:106-119 packs '8s9I20s' = 64 bytes
    d = synthetic.make_dims("1.3b", 48)
    h = fmt.pack_header(d)
    assert len(h) == 64 == struct.calcsize("8s9I20s")
    vals = struct.unpack("8s9I20s", h)
    assert vals[0] == b"DFSSM001"
    assert vals[1:10] == (48, 2048, 4096, 128, 64, 64, 1, 50280, 4)


@pytest.mark.parametrize("emb_kind", [fmt.EMB_FP16, fmt.EMB_INT8])
def test_roundtrip(emb_kind):
    w = tiny()
    buf = fmt.to_bytes(w, emb_kind)
    assert len(buf) == fmt.file_size(w.dims, emb_kind)
    w2 = fmt.from_bytes(buf)
    assert w2.dims == w.dims
    np.testing.assert_array_equal(w2.embedding_f16(), w.embedding_f16())
    for a, b in zip(w.layers, w2.layers):
        np.testing.assert_array_equal(a.in_proj.packed, b.in_proj.packed)
        np.testing.assert_array_equal(a.out_proj.lora_B, b.out_proj.lora_B)
        np.testing.assert_array_equal(a.norm_w, b.norm_w)
    np.testing.assert_array_equal(w.norm_f, w2.norm_f)


def test_1p3b_layer_bytes():
    # per-layer weight bytes used in the roofline: packed 3,227,648 B
    d = synthetic.make_dims("1.3b", 1)
    assert d.n_in == 8512 and d.d_xbc == 4352
    packed = d.n_in * d.d_model // 8 + d.d_model * d.d_inner // 8
    assert packed == 3_227_648


def test_unpack_matches_reference_rule():
    # df_ssm_inference.py:23-29: bit b of word j -> column 32j+b, 1 -> +1, 0 -> -1
    rng = np.random.default_rng(1)
    packed = rng.integers(0, 2**32, size=(5, 4), dtype=np.uint32).view(np.int32)
    s = fmt.unpack_signs(packed, 128)
    for r in range(5):
        for c in range(128):
            bit = (int(packed[r, c // 32].view(np.uint32)) >> (c % 32)) & 1
            assert s[r, c] == (1 if bit else -1)
    np.testing.assert_array_equal(fmt.pack_signs((s > 0).astype(np.uint8)), packed)


def test_synthetic_distributions():
    w = synthetic.make_weights(synthetic.make_dims("tiny", 4), seed=3)
    L = w.layers[0]
    A = -np.exp(np.concatenate([l.A_log for l in w.layers]))
    assert np.all(A <= -1.0) and np.all(A >= -16.0)
    dt = np.log1p(np.exp(np.concatenate([l.dt_bias for l in w.layers]).astype(np.float64)))
    assert dt.min() >= 0.999e-3 and dt.max() <= 0.1001
    assert abs(float(np.std(L.conv_w.astype(np.float32))) - 0.5) < 0.05
    assert np.all(L.in_proj.scale > 0)
    bits = np.unpackbits(L.in_proj.packed.view(np.uint8))
    assert abs(bits.mean() - 0.5) < 0.01
    assert w.emb_q.min() >= -127 and w.emb_q.max() <= 127
    # deterministic
    w2 = synthetic.make_weights(synthetic.make_dims("tiny", 4), seed=3)
    np.testing.assert_array_equal(w2.layers[3].out_proj.packed, w.layers[3].out_proj.packed)


def test_reader_rejects_bad_images():
    w = tiny(1)
    buf = bytearray(fmt.to_bytes(w))
    with pytest.raises(ValueError):
        fmt.from_bytes(bytes(buf[:-1]))
    bad = bytearray(buf)
    bad[:8] = b"XXXXXXXX"
    with pytest.raises(ValueError):
        fmt.from_bytes(bytes(bad))
    bad = bytearray(buf)
    struct.pack_into("<I", bad, 8 + 4 * 5, 32)  # headdim 32 -> nheads*headdim != d_inner
    with pytest.raises(ValueError):
        fmt.from_bytes(bytes(bad))


def test_convert_cli_to_int8_embedding(tmp_path):
    w = tiny(1)
    src, dst = tmp_path / "a.dfssm", tmp_path / "b.dfssm"
    fmt.write(str(src), w, fmt.EMB_FP16)
    fmt.main(["convert", str(src), str(dst), "--int8-embedding"])
    w2 = fmt.read(str(dst))
    assert w2.emb_q is not None and w2.emb_f16 is None
    # per-row absmax/127 quantisation reconstructs every value within half a step (+ fp16 scale rounding)
    E = w.embedding_f16().astype(np.float32)
    deq = w2.emb_q.astype(np.float32) * w2.emb_s.astype(np.float32)[:, None]
    step = w2.emb_s.astype(np.float32)[:, None]
    assert np.all(np.abs(deq - E) <= 0.5 * step + 1e-3 * np.abs(E) + 1e-6)
    assert dst.stat().st_size < src.stat().st_size
