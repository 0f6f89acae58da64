"""CPU oracle for the DF-SSM per-token decode path — TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of the reference GPU decode path
(inference/gpu/df_ssm_inference.py + inference/gpu/df_ssm_kernels.cu of
cs-cmyk/df-ssm) with HEADDIM = 64.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import it; the product (the dfssm_b200 package
and libdfssm.so) never does.

It reproduces the reference's fp16 rounding points one by one, so that a kernel
following the same points can be compared tightly:

  rms_norm      df_ssm_inference.py:141-145   fp32 mean of squares, x*rsqrt(.)*w
                                               in fp32, result stored fp16
  quantize      df_ssm_inference.py:147-152   scale = fp16(max(amax, fp16(1e-4))/127)
                                               (CUDA divides a tensor by a host scalar as
                                               a multiply by the fp32 reciprocal),
                                               q = rne(fp16(x/scale)) clamped to int8
  scaffold      df_ssm_inference.py:154-158   int32 = q . W(+-1)^T; fp16(fp16(fp16(acc)*xs)*ws)
  LoRA          df_ssm_inference.py:78-83,92-97,173,204
                                               A,B dequantised to fp16; t = fp16(x_norm.B^T);
                                               proj = fp16(proj + fp16(t.A^T)) on CUDA (the fp16
                                               addmm_ rounds the product first), fp16(proj + t.A^T)
                                               on the CPU
  split         df_ssm_inference.py:176-178
  conv_step     df_ssm_kernels.cu:27-47        shift register, 4-tap conv + bias, SiLU -> fp16
  ssm_step      df_ssm_kernels.cu:53-103       dt=softplus(dt_raw+dt_bias), Abar=exp(-dt*exp(A_log)),
                                               h = Abar*h + x*dt*B, y = sum_n C*h + D*x -> fp16
  gate + norm   df_ssm_inference.py:194-196   fp16(y*fp16(z*fp16(sigmoid(z)))) then rms_norm
  residual      df_ssm_inference.py:207       x = fp16(x + out)
  head          df_ssm_inference.py:210,224,236  final rms_norm, logits = fp16(norm_out.E^T),
                                               greedy argmax (first index on ties)
  sampling      eval/gen_test.py:54-95         temperature, repetition penalty, top-p nucleus

Options select the documented deviations of the B200 engine from the literal
reference: ``state_dtype`` ("f16" is the reference, "f32" the engine contract) and
``emb`` ("f16": logits from the fp16 embedding as the reference computes them;
"int8": logits = fp16(scale_v * sum_k q_vk*x_k), as the engine's int8 LM head).
``div_mode`` selects where the reference ran: "cuda" (its GPU path: the quantisation scale is a
multiply by the fp32 reciprocal of 127 and the LoRA product is rounded to fp16 before the add) or
"cpu" (true division, one rounding of the LoRA add; used only when checking against goldens made
on the CPU).
"""
from __future__ import annotations

import numpy as np

import dfssm_b200.dfssm_format as fmt

F16, F32 = np.float16, np.float32
RMS_EPS = F32(1e-5)


def rms_norm_f16(x16: np.ndarray, w: np.ndarray) -> np.ndarray:
    """df_ssm_inference.py:141-145 (x fp16 [B,K], w fp32 or fp16 [K]) -> fp16."""
    xf = x16.astype(F32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=F32).astype(F32)
    r = (F32(1.0) / np.sqrt(var + RMS_EPS, dtype=F32)).astype(F32)
    return ((xf * r).astype(F32) * w.astype(F32)).astype(F16)


def quantize_int8(x16: np.ndarray, div_mode: str = "cuda"):
    """df_ssm_inference.py:147-152 -> (scale fp16 [B,1], q int8 [B,K])."""
    amax = np.abs(x16).max(axis=-1, keepdims=True)
    amax = np.maximum(amax, F16(1e-4))
    if div_mode == "cuda":
        scale = (amax.astype(F32) * (F32(1.0) / F32(127.0))).astype(F16)
    else:
        scale = (amax.astype(F32) / F32(127.0)).astype(F16)
    t = (x16.astype(F32) / scale.astype(F32)).astype(F16).astype(F32)
    q = np.clip(np.rint(t), -128, 127).astype(np.int8)
    return scale, q


def scaffold_int32(q: np.ndarray, signs_f32: np.ndarray) -> np.ndarray:
    """Exact int32 q . W^T with W = +-1 (as float32: every partial sum is an integer < 2^24)."""
    return (q.astype(F32) @ signs_f32.T).astype(np.int64).astype(np.int32)


def dequant(acc: np.ndarray, xs16: np.ndarray, ws16: np.ndarray) -> np.ndarray:
    """df_ssm_inference.py:158: fp16(fp16(fp16(acc)*x_scale)*w_scale)."""
    a = acc.astype(F32).astype(F16).astype(F32)
    t = (a * xs16.astype(F32)).astype(F16).astype(F32)
    return (t * ws16.astype(F32)[None, :]).astype(F16)


def lora_dequant(p: fmt.Proj):
    A16 = (p.lora_A.astype(F32) * p.lora_A_s.astype(F32)[:, None]).astype(F16)
    B16 = (p.lora_B.astype(F32) * p.lora_B_s.astype(F32)[:, None]).astype(F16)
    return A16, B16


def lora_add(base16: np.ndarray, x16: np.ndarray, A16: np.ndarray, B16: np.ndarray, div_mode: str = "cuda") -> np.ndarray:
    """df_ssm_inference.py:173,204: base.addmm_(x @ B^T, A^T), fp32-or-better accumulate.
    t = fp16(x . B^T).  On CUDA (torch 2.11 / cuBLAS, measured on the B200) the fp16 addmm_ rounds
    the rank-16 product t . A^T to fp16 before adding it to base: fp16(base + fp16(t . A^T)); on
    the CPU it rounds once: fp16(base + t . A^T)."""
    t = (x16.astype(np.float64) @ B16.astype(np.float64).T).astype(F16)
    prod = t.astype(np.float64) @ A16.astype(np.float64).T
    if div_mode == "cuda":
        prod = prod.astype(F16).astype(np.float64)
    return (base16.astype(np.float64) + prod).astype(F16)


def silu_f32(v: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (v * (F32(1.0) / (F32(1.0) + np.exp(-v, dtype=F32)))).astype(F32)


def conv_step(conv_state: np.ndarray, xbc16: np.ndarray, w16: np.ndarray, b16: np.ndarray) -> np.ndarray:
    """df_ssm_kernels.cu:27-47.  conv_state [B, D_XBC, 3] (updated in place), returns fp16 SiLU(conv)."""
    s = conv_state.astype(F32)
    xv = xbc16.astype(F32)
    w = w16.astype(F32)
    out = (s[..., 0] * w[:, 0] + s[..., 1] * w[:, 1] + s[..., 2] * w[:, 2] + xv * w[:, 3]
           + b16.astype(F32)).astype(F32)
    conv_state[..., 0] = s[..., 1]
    conv_state[..., 1] = s[..., 2]
    conv_state[..., 2] = xv
    return silu_f32(out).astype(F16)


def softplus_f32(v: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return np.log1p(np.exp(v, dtype=F32), dtype=F32)


def ssm_step(h: np.ndarray, x16, B16, C16, dt16, dt_bias, A_log, Dp):
    """df_ssm_kernels.cu:53-103 for all heads.  h [B,H,P,N] updated in place (its dtype is the
    storage type); y uses the unrounded fp32 state as the kernel does.  Returns y fp16 [B,H*P]."""
    Bsz, H, P, N = h.shape
    dt = softplus_f32((dt16.astype(F32) + dt_bias.astype(F32)).astype(F32))       # [B,H]
    Abar = np.exp((dt * (-np.exp(A_log.astype(F32), dtype=F32))).astype(F32), dtype=F32)
    x = x16.astype(F32).reshape(Bsz, H, P)
    X = (x * dt[:, :, None]).astype(F32)                                          # [B,H,P]
    hn = (Abar[:, :, None, None] * h.astype(F32) + X[..., None] * B16.astype(F32)[:, None, None, :]).astype(F32)
    y = np.sum(hn * C16.astype(F32)[:, None, None, :], axis=-1, dtype=F32)
    y = (y + x * Dp.astype(F32)[None, :, None]).astype(F32)
    h[...] = hn.astype(h.dtype)
    return y.reshape(Bsz, H * P).astype(F16)


def gate(y16: np.ndarray, z16: np.ndarray) -> np.ndarray:
    """df_ssm_inference.py:194-195: fp16(y * fp16(z * fp16(sigmoid(z))))."""
    zf = z16.astype(F32)
    with np.errstate(over="ignore"):
        sig = (F32(1.0) / (F32(1.0) + np.exp(-zf, dtype=F32))).astype(F16)
    silu_z = (zf * sig.astype(F32)).astype(F16)
    return (y16.astype(F32) * silu_z.astype(F32)).astype(F16)


def sample_nucleus(logits: np.ndarray, seen: np.ndarray, temperature: float, top_p: float, rep_penalty: float):
    """The token-choice rule of the reference's generate() (eval/gen_test.py:69-87) for one row:
    logits / T (:69), seen tokens' logits / rep_penalty (:71-72), softmax (:74), descending sort,
    cumsum, drop tokens whose preceding mass exceeds top_p (:75-78), renormalise (:79-82).
    Returns (kept token ids in descending-probability order, softmax probabilities, kept mass).
    The draw itself (torch.multinomial, :84) is random; tests check its distribution."""
    l = logits.astype(np.float32) / np.float32(temperature)
    l = l.copy()
    l[seen] = l[seen] / np.float32(rep_penalty)
    e = np.exp((l - l.max()).astype(np.float64))
    p = e / e.sum()
    order = np.argsort(-p, kind="stable")
    sp = p[order]
    cs = np.cumsum(sp)
    keep = (cs - sp) <= top_p
    return order[keep], p, float(sp[keep].sum())


def argmax_first(v: np.ndarray) -> np.ndarray:
    return np.argmax(v, axis=-1)  # numpy returns the first maximal index, like torch


class OracleModel:
    """Per-token decode of a whole model, batch B, on the CPU."""

    def __init__(self, w: fmt.Weights, batch: int, state_dtype: str = "f32", emb: str = "int8",
                 div_mode: str = "cuda", cache_signs: bool = True):
        self.w, self.d, self.B = w, w.dims, batch
        self.state_dtype = {"f32": F32, "f16": F16}[state_dtype]
        self.emb_mode, self.div_mode = emb, div_mode
        self.E16 = w.embedding_f16()
        if emb == "int8":
            if w.emb_q is None:
                raise ValueError("int8 LM head needs an int8 embedding")
            self.Eq = w.emb_q.astype(F32)
            self.Es = w.emb_s.astype(F32)
        self._signs = {}
        self.cache_signs = cache_signs
        self._lora = [(lora_dequant(L.in_proj), lora_dequant(L.out_proj)) for L in w.layers]
        self.reset()

    def signs(self, l: int, which: str) -> np.ndarray:
        key = (l, which)
        if key in self._signs:
            return self._signs[key]
        p = getattr(self.w.layers[l], which)
        k = p.packed.shape[1] * 32
        s = fmt.unpack_signs(p.packed, k).astype(F32)
        if self.cache_signs:
            self._signs[key] = s
        return s

    def reset(self):
        d, B = self.d, self.B
        self.h = [np.zeros((B, d.nheads, d.headdim, d.d_state), self.state_dtype) for _ in range(d.n_layer)]
        self.conv = [np.zeros((B, d.d_xbc, 3), self.state_dtype) for _ in range(d.n_layer)]

    def proj(self, x16, l, which):
        p = getattr(self.w.layers[l], which)
        xs, q = quantize_int8(x16, self.div_mode)
        acc = scaffold_int32(q, self.signs(l, which))
        base = dequant(acc, xs, p.scale)
        A16, B16 = self._lora[l][0 if which == "in_proj" else 1]
        return lora_add(base, x16, A16, B16, self.div_mode)

    def layer(self, x16: np.ndarray, l: int) -> np.ndarray:
        d, L = self.d, self.w.layers[l]
        xn = rms_norm_f16(x16, L.ln_w)
        proj = self.proj(xn, l, "in_proj")
        z = proj[:, :d.d_inner]
        xbc = proj[:, d.d_inner:d.d_inner + d.d_xbc].copy()
        dt = proj[:, d.d_inner + d.d_xbc:]
        xbc = conv_step(self.conv[l], xbc, L.conv_w, L.conv_b)
        y = ssm_step(self.h[l], xbc[:, :d.d_inner], xbc[:, d.d_inner:d.d_inner + d.d_state],
                     xbc[:, d.d_inner + d.d_state:d.d_inner + 2 * d.d_state], dt,
                     L.dt_bias, L.A_log, L.D)
        yn = rms_norm_f16(gate(y, z), L.norm_w)
        out = self.proj(yn, l, "out_proj")
        return (x16.astype(F32) + out.astype(F32)).astype(F16)

    def logits(self, x16: np.ndarray):
        """Returns (fp16 logits the greedy argmax sees, fp32 pre-rounding logits)."""
        no = rms_norm_f16(x16, self.w.norm_f)
        if self.emb_mode == "int8":
            l32 = ((no.astype(np.float64) @ self.Eq.T.astype(np.float64)) * self.Es[None, :]).astype(F32)
        else:
            l32 = (no.astype(np.float64) @ self.E16.T.astype(np.float64)).astype(F32)
        return l32.astype(F16), l32

    def step(self, tokens: np.ndarray):
        """One decode step for token ids [B]; returns (logits fp16 [B,V], logits fp32, argmax)."""
        x = self.E16[np.asarray(tokens, np.int64)]
        for l in range(self.d.n_layer):
            x = self.layer(x, l)
        self.x_last = x
        l16, l32 = self.logits(x)
        return l16, l32, argmax_first(l16)

    def generate(self, prompts: np.ndarray, n_steps: int, teacher=None):
        """Feed prompts [B,T] one token at a time, then n_steps greedy steps.  Returns
        (tokens [n_steps,B], per-step fp16 logits list).  With `teacher` [n_steps,B] the
        decode inputs are forced (teacher forcing) instead of the own argmax."""
        prompts = np.asarray(prompts)
        tok = None
        for t in range(prompts.shape[1]):
            l16, _, tok = self.step(prompts[:, t])
        toks, logs = [], []
        for s in range(n_steps):
            toks.append(tok.copy())
            inp = tok if teacher is None else teacher[s]
            l16, _, tok = self.step(inp)
            logs.append(l16)
        return np.stack(toks), logs
