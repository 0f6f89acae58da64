"""`.dfssm` weight file: header, byte map, reader and writer.

The byte map is the one written by the reference exporter
(training/export_dfssm.py:104-193) and read by the reference CPU driver
(inference/cpu/cpu_inference_driver.py:89-141):

  header  64 B  struct '8s9I20s'  magic b'DFSSM001', n_layer, d_model, d_inner,
                d_state, nheads, headdim, ngroups, vocab, Kw, 20 reserved bytes
                (export_dfssm.py:106-119)
  embedding     fp16 [vocab, d_model]                    (export_dfssm.py:124-127)
  per layer, for in_proj (N = 2*d_inner + 2*ngroups*d_state + nheads, K = d_model)
  then out_proj (N = d_model, K = d_inner)               (export_dfssm.py:133-167):
                packed sign bits int32 [N, K/32]  (bit b of word j <-> column 32j+b,
                                                   bit 1 -> +1, bit 0 -> -1)
                scale fp16 [N]  (per-row abs-mean)
                lora_A int8 [N, 16], lora_A_scale fp16 [N]
                lora_B int8 [16, K], lora_B_scale fp16 [16]
                conv_w fp16 [D_XBC, d_conv], conv_b fp16 [D_XBC]   (:170-174)
                A_log f32 [nheads], D f32 [nheads], dt_bias f32 [nheads] (:177-179)
                mixer norm f32 [d_inner], layer norm f32 [d_model] (:182-185)
  final norm    f32 [d_model]                            (:193)

The norms are fp32 as the exporter writes them; the reference GPU loader reads
them as fp16 (inference/gpu/df_ssm_inference.py:105-110), which desynchronises it
on exporter-written files, so this reader follows the exporter.

Extension (no counterpart in the reference): reserved byte 0 == 1 marks an int8
tied embedding, stored as int8 [vocab, d_model] followed by a per-row fp16 scale
[vocab]; the dequantised row is int8 * scale.  Every dimension comes from the
header (the reference hard-codes them, df_ssm_inference.py:15-19).
"""
from __future__ import annotations

import dataclasses
import struct
from typing import List, Optional

import numpy as np

MAGIC = b"DFSSM001"
HEADER_FMT = "<8s9I20s"
HEADER_SIZE = 64
LORA_RANK = 16
D_CONV = 4
EMB_FP16 = 0
EMB_INT8 = 1


@dataclasses.dataclass(frozen=True)
class Dims:
    n_layer: int
    d_model: int
    d_inner: int
    d_state: int
    nheads: int
    headdim: int
    ngroups: int
    vocab: int
    Kw: int = 4

    @property
    def d_xbc(self) -> int:
        return self.d_inner + 2 * self.ngroups * self.d_state

    @property
    def n_in(self) -> int:
        return 2 * self.d_inner + 2 * self.ngroups * self.d_state + self.nheads

    def validate(self) -> None:
        if self.nheads * self.headdim != self.d_inner:
            raise ValueError(f"nheads*headdim={self.nheads * self.headdim} != d_inner={self.d_inner}")
        if self.ngroups != 1:
            raise ValueError("only ngroups == 1 is supported (as in the reference kernels)")
        if self.d_model % 128 or self.d_inner % 128:
            raise ValueError("d_model and d_inner must be multiples of 128")
        for f in ("n_layer", "d_model", "d_inner", "d_state", "nheads", "headdim", "vocab"):
            if getattr(self, f) <= 0:
                raise ValueError(f"{f} must be positive")


@dataclasses.dataclass
class Proj:
    """One scaffold projection: 1-bit signs + per-row scale + int8 rank-16 LoRA."""
    packed: np.ndarray    # int32 [N, K/32]
    scale: np.ndarray     # fp16 [N]
    lora_A: np.ndarray    # int8 [N, 16]
    lora_A_s: np.ndarray  # fp16 [N]
    lora_B: np.ndarray    # int8 [16, K]
    lora_B_s: np.ndarray  # fp16 [16]


@dataclasses.dataclass
class Layer:
    in_proj: Proj
    out_proj: Proj
    conv_w: np.ndarray     # fp16 [D_XBC, 4]
    conv_b: np.ndarray     # fp16 [D_XBC]
    A_log: np.ndarray      # f32 [nheads]
    D: np.ndarray          # f32 [nheads]
    dt_bias: np.ndarray    # f32 [nheads]
    norm_w: np.ndarray     # f32 [d_inner]  (mixer gate-norm)
    ln_w: np.ndarray       # f32 [d_model]  (pre-layer RMSNorm)


@dataclasses.dataclass
class Weights:
    dims: Dims
    layers: List[Layer]
    norm_f: np.ndarray                   # f32 [d_model]
    emb_q: Optional[np.ndarray] = None   # int8 [V, d_model]
    emb_s: Optional[np.ndarray] = None   # fp16 [V]
    emb_f16: Optional[np.ndarray] = None  # fp16 [V, d_model]

    def embedding_f16(self) -> np.ndarray:
        """The fp16 embedding the reference path uses (int8 * scale rounded to fp16)."""
        if self.emb_f16 is not None:
            return self.emb_f16
        return (self.emb_q.astype(np.float32) * self.emb_s.astype(np.float32)[:, None]).astype(np.float16)


def pack_header(d: Dims, emb_kind: int = EMB_FP16) -> bytes:
    reserved = bytes([emb_kind]) + b"\x00" * 19
    return struct.pack(HEADER_FMT, MAGIC, d.n_layer, d.d_model, d.d_inner, d.d_state,
                       d.nheads, d.headdim, d.ngroups, d.vocab, d.Kw, reserved)


def parse_header(buf: bytes):
    if len(buf) < HEADER_SIZE:
        raise ValueError(f"truncated .dfssm header ({len(buf)} bytes)")
    magic, nl, dm, di, ds, nh, hd, ng, v, kw, res = struct.unpack(HEADER_FMT, buf[:HEADER_SIZE])
    if magic != MAGIC:
        raise ValueError(f"bad .dfssm magic {magic!r}")
    d = Dims(nl, dm, di, ds, nh, hd, ng, v, kw)
    d.validate()
    return d, res[0]


def file_size(d: Dims, emb_kind: int) -> int:
    """Exact byte length of a .dfssm file with these dims."""
    def proj(n, k):
        return n * (k // 32) * 4 + n * 2 + n * LORA_RANK + n * 2 + LORA_RANK * k + LORA_RANK * 2
    per_layer = (proj(d.n_in, d.d_model) + proj(d.d_model, d.d_inner)
                 + d.d_xbc * D_CONV * 2 + d.d_xbc * 2 + 3 * d.nheads * 4
                 + d.d_inner * 4 + d.d_model * 4)
    emb = d.vocab * d.d_model * (2 if emb_kind == EMB_FP16 else 1) + (d.vocab * 2 if emb_kind == EMB_INT8 else 0)
    return HEADER_SIZE + emb + d.n_layer * per_layer + d.d_model * 4


def to_bytes(w: Weights, emb_kind: int = EMB_FP16) -> bytes:
    """Serialise in the exporter's byte order (export_dfssm.py:104-193)."""
    d = w.dims
    parts = [pack_header(d, emb_kind)]
    if emb_kind == EMB_FP16:
        parts.append(np.ascontiguousarray(w.embedding_f16(), np.float16).tobytes())
    else:
        parts.append(np.ascontiguousarray(w.emb_q, np.int8).tobytes())
        parts.append(np.ascontiguousarray(w.emb_s, np.float16).tobytes())
    for L in w.layers:
        for p in (L.in_proj, L.out_proj):
            parts += [np.ascontiguousarray(p.packed, np.int32).tobytes(),
                      np.ascontiguousarray(p.scale, np.float16).tobytes(),
                      np.ascontiguousarray(p.lora_A, np.int8).tobytes(),
                      np.ascontiguousarray(p.lora_A_s, np.float16).tobytes(),
                      np.ascontiguousarray(p.lora_B, np.int8).tobytes(),
                      np.ascontiguousarray(p.lora_B_s, np.float16).tobytes()]
        parts += [np.ascontiguousarray(L.conv_w, np.float16).tobytes(),
                  np.ascontiguousarray(L.conv_b, np.float16).tobytes(),
                  np.ascontiguousarray(L.A_log, np.float32).tobytes(),
                  np.ascontiguousarray(L.D, np.float32).tobytes(),
                  np.ascontiguousarray(L.dt_bias, np.float32).tobytes(),
                  np.ascontiguousarray(L.norm_w, np.float32).tobytes(),
                  np.ascontiguousarray(L.ln_w, np.float32).tobytes()]
    parts.append(np.ascontiguousarray(w.norm_f, np.float32).tobytes())
    out = b"".join(parts)
    assert len(out) == file_size(d, emb_kind)
    return out


def write(path: str, w: Weights, emb_kind: int = EMB_FP16) -> None:
    with open(path, "wb") as f:
        f.write(to_bytes(w, emb_kind))


def from_bytes(buf) -> Weights:
    """Parse a .dfssm image; every dimension comes from the header."""
    mv = memoryview(buf)
    d, emb_kind = parse_header(bytes(mv[:HEADER_SIZE]))
    if emb_kind not in (EMB_FP16, EMB_INT8):
        raise ValueError(f"unknown embedding kind {emb_kind}")
    need = file_size(d, emb_kind)
    if len(mv) != need:
        raise ValueError(f".dfssm size {len(mv)} != {need} expected from header")
    off = HEADER_SIZE

    def rd(shape, dt):
        nonlocal off
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        a = np.frombuffer(mv[off:off + n], dtype=dt).reshape(shape).copy()
        off += n
        return a

    w = Weights(dims=d, layers=[], norm_f=None)
    if emb_kind == EMB_FP16:
        w.emb_f16 = rd((d.vocab, d.d_model), np.float16)
    else:
        w.emb_q = rd((d.vocab, d.d_model), np.int8)
        w.emb_s = rd((d.vocab,), np.float16)
    for _ in range(d.n_layer):
        projs = []
        for n, k in ((d.n_in, d.d_model), (d.d_model, d.d_inner)):
            projs.append(Proj(rd((n, k // 32), np.int32), rd((n,), np.float16),
                              rd((n, LORA_RANK), np.int8), rd((n,), np.float16),
                              rd((LORA_RANK, k), np.int8), rd((LORA_RANK,), np.float16)))
        w.layers.append(Layer(projs[0], projs[1],
                              rd((d.d_xbc, D_CONV), np.float16), rd((d.d_xbc,), np.float16),
                              rd((d.nheads,), np.float32), rd((d.nheads,), np.float32),
                              rd((d.nheads,), np.float32),
                              rd((d.d_inner,), np.float32), rd((d.d_model,), np.float32)))
    w.norm_f = rd((d.d_model,), np.float32)
    assert off == len(mv)
    return w


def read(path: str) -> Weights:
    with open(path, "rb") as f:
        return from_bytes(f.read())


def unpack_signs(packed: np.ndarray, k: int) -> np.ndarray:
    """±1 int8 [N, K] from packed int32 [N, K/32] (df_ssm_inference.py:23-29)."""
    u = np.ascontiguousarray(packed).view(np.uint32)
    bits = np.unpackbits(u.view(np.uint8).reshape(u.shape[0], -1), axis=1, bitorder="little")
    return (bits[:, :k].astype(np.int8) * 2 - 1).astype(np.int8)


def pack_signs(signs01: np.ndarray) -> np.ndarray:
    """Inverse of unpack_signs for a 0/1 array [N, K] (export_dfssm.py:34-42)."""
    n, k = signs01.shape
    assert k % 32 == 0
    b = np.packbits(signs01.astype(np.uint8), axis=1, bitorder="little")
    return b.view(np.uint32).reshape(n, k // 32).view(np.int32)


def main(argv=None):
    """`python -m dfssm_b200.dfssm_format convert IN OUT [--int8-embedding]`: rewrite a .dfssm file,
    optionally storing the tied embedding as int8 + per-row fp16 scale (header reserved byte 0 = 1),
    which halves the embedding bytes (206 -> 103 MB at vocab 50280, d_model 2048)."""
    import argparse
    ap = argparse.ArgumentParser(prog="python -m dfssm_b200.dfssm_format")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("convert")
    c.add_argument("src")
    c.add_argument("dst")
    c.add_argument("--int8-embedding", action="store_true")
    i = sub.add_parser("info")
    i.add_argument("src")
    a = ap.parse_args(argv)
    if a.cmd == "info":
        with open(a.src, "rb") as fh:
            d, kind = parse_header(fh.read(HEADER_SIZE))
        print(d, "embedding", "int8" if kind == EMB_INT8 else "fp16")
        return
    w = read(a.src)
    if a.int8_embedding and w.emb_q is None:
        w.emb_q, w.emb_s = quantize_embedding_int8(w.emb_f16)
    write(a.dst, w, EMB_INT8 if a.int8_embedding else EMB_FP16)


def quantize_embedding_int8(E16: np.ndarray):
    """Per-row symmetric int8 (absmax / 127, fp16 scale) of an fp16 embedding."""
    Ef = E16.astype(np.float32)
    s32 = np.abs(Ef).max(axis=1) / np.float32(127.0)            # codes from the fp32 scale
    s32 = np.where(s32 > 0, s32, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(Ef / s32[:, None]), -127, 127).astype(np.int8)
    return q, s32.astype(np.float16)


if __name__ == "__main__":
    main()
