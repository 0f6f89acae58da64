"""Seeded synthetic DF-SSM weights and prompts (no checkpoints exist offline).

Distributions follow the workload definition of this engine's benchmark:
  * scaffold sign bits Bernoulli(0.5), packed 8 per byte (exporter layout,
    training/export_dfssm.py:34-42,144-145); per-row fp16 scale |N(0,0.02)|+1e-3;
  * LoRA: rank-16 A ~ N(0,1)/rank (the exporter stores lora_A*scaling,
    export_dfssm.py:154-155, scaling = 1/rank at alpha 1) and B ~ 0.1*N(0,1),
    each quantised per row to int8 with an fp16 scale exactly as
    export_dfssm.py:45-50 does.  Literal N(0,1) for both drives dt_raw past the
    softplus overflow in both reference paths (inference/cpu/cpu_inference.c:282,
    inference/gpu/df_ssm_kernels.cu:78) and yields NaN, hence the deviation;
  * tied embedding int8 U[-127,127] with per-row scale fp16(0.01);
  * A_log = log U[1,16]; dt ~ logU[1e-3,1e-1], dt_bias = softplus^-1(dt); D = 1;
    conv weights N(0,0.5) fp16; conv bias 0; all norms 1.
"""
from __future__ import annotations

import numpy as np

from .dfssm_format import D_CONV, LORA_RANK, Dims, Layer, Proj, Weights

# Named shapes (per-layer dims of Mamba-2 1.3B / 2.7B, headdim 64).
SHAPES = {
    "1.3b": dict(d_model=2048, d_inner=4096, d_state=128, nheads=64, headdim=64, ngroups=1, vocab=50280),
    "2.7b": dict(d_model=2560, d_inner=5120, d_state=128, nheads=80, headdim=64, ngroups=1, vocab=50280),
    # small shapes for fast tests (same head geometry as the real ones)
    "tiny": dict(d_model=256, d_inner=512, d_state=128, nheads=8, headdim=64, ngroups=1, vocab=512),
    "small": dict(d_model=512, d_inner=1024, d_state=128, nheads=16, headdim=64, ngroups=1, vocab=1000),
}


def make_dims(shape: str, n_layer: int, vocab: int | None = None) -> Dims:
    kw = dict(SHAPES[shape])
    if vocab is not None:
        kw["vocab"] = vocab
    d = Dims(n_layer=n_layer, **kw)
    d.validate()
    return d


def _quantize_rows_int8(w: np.ndarray):
    """Per-row symmetric int8 quantisation (export_dfssm.py:45-50), in fp32."""
    w = w.astype(np.float32)
    scale = (np.abs(w).max(axis=-1) / np.float32(127.0)).astype(np.float32)
    scale = np.maximum(scale, np.float32(1e-8))
    q = np.clip(np.rint(w / scale[:, None]), -128, 127).astype(np.int8)
    return q, scale.astype(np.float16)


def _proj(rng, n: int, k: int, lora_b_mag: float) -> Proj:
    packed = rng.integers(0, 2**32, size=(n, k // 32), dtype=np.uint32).view(np.int32)
    scale = (np.abs(rng.normal(0.0, 0.02, size=n)) + 1e-3).astype(np.float16)
    A = rng.standard_normal((n, LORA_RANK), dtype=np.float32) * np.float32(1.0 / LORA_RANK)
    B = rng.standard_normal((LORA_RANK, k), dtype=np.float32) * np.float32(lora_b_mag)
    Aq, As = _quantize_rows_int8(A)
    Bq, Bs = _quantize_rows_int8(B)
    return Proj(packed, scale, Aq, As, Bq, Bs)


def make_weights(dims: Dims, seed: int = 0, lora_b_mag: float = 0.1, emb_scale: float = 0.01) -> Weights:
    rng = np.random.default_rng(seed)
    d = dims
    emb_q = rng.integers(-127, 128, size=(d.vocab, d.d_model), dtype=np.int8)
    emb_s = np.full(d.vocab, emb_scale, dtype=np.float16)
    layers = []
    for _ in range(d.n_layer):
        inp = _proj(rng, d.n_in, d.d_model, lora_b_mag)
        outp = _proj(rng, d.d_model, d.d_inner, lora_b_mag)
        conv_w = rng.normal(0.0, 0.5, size=(d.d_xbc, D_CONV)).astype(np.float16)
        conv_b = np.zeros(d.d_xbc, dtype=np.float16)
        A_log = np.log(rng.uniform(1.0, 16.0, size=d.nheads)).astype(np.float32)
        dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), size=d.nheads))
        dt_bias = (dt + np.log(-np.expm1(-dt))).astype(np.float32)
        layers.append(Layer(inp, outp, conv_w, conv_b, A_log,
                            np.ones(d.nheads, np.float32), dt_bias,
                            np.ones(d.d_inner, np.float32), np.ones(d.d_model, np.float32)))
    return Weights(dims=d, layers=layers, norm_f=np.ones(d.d_model, np.float32),
                   emb_q=emb_q, emb_s=emb_s)


def make_prompts(vocab: int, batch: int, length: int = 16, seed: int = 0) -> np.ndarray:
    """Independent uniform-random prompts, int64 [batch, length]."""
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.integers(0, vocab, size=(batch, length), dtype=np.int64)
