"""ctypes driver for the reference's CPU engine (TEST / BASELINE INFRASTRUCTURE ONLY).

Restates the per-token loop of inference/cpu/cpu_inference_driver.py:77-204 (class
CPUModel: fp32 copies of fp16 tensors, precompute_row_sums per projection,
embedding_lookup -> n_layer x layer_forward -> final_rms_norm -> fp32 numpy LM head
`norm_out @ embedding.T` -> argmax) over oracle/_ref/libcpu_inference_<shape>.so, the
reference's cpu_inference.c built by oracle/build_ref.py.  Dims come from the Weights
object instead of the driver's module constants (:19-30).  Used as bench.py's reference
arm and CPU baseline, and as a semantic cross-check of the oracle (the CPU engine
quantises activations asymmetrically to uint8, cpu_inference.c:65-97, so it is not a
bit-level oracle of the GPU path).
"""
from __future__ import annotations

import ctypes
import os
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F_P = ctypes.POINTER(ctypes.c_float)
I_P = ctypes.POINTER(ctypes.c_int)
I8_P = ctypes.POINTER(ctypes.c_int8)
U32_P = ctypes.POINTER(ctypes.c_uint32)


def lib_path(shape_key: str) -> str:
    return os.path.join(HERE, "_ref", f"libcpu_inference_{shape_key}.so")


def shape_key(d) -> str:
    return {2048: "1p3b", 2560: "2p7b", 256: "tiny"}[d.d_model]


def cpu_supports_reference() -> bool:
    """The reference engine needs AVX-512 F/BW/VL/DQ + VNNI."""
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return False
    return all(f in flags for f in ("avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512_vnni"))


def _p(a, t):
    return a.ctypes.data_as(t)


class RefCPUModel:
    def __init__(self, w, lib: str | None = None):
        self.d = d = w.dims
        path = lib or lib_path(shape_key(d))
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (python oracle/build_ref.py)")
        self.lib = L = ctypes.CDLL(path)
        L.layer_forward.restype = None
        L.layer_forward.argtypes = ([F_P, U32_P, F_P, I_P, U32_P, F_P, I_P] + [I8_P, F_P, I8_P, F_P] * 2
                                    + [F_P] * 7 + [F_P, F_P] + [F_P] * 4)
        L.precompute_row_sums.restype = None
        L.precompute_row_sums.argtypes = [U32_P, I_P, ctypes.c_int, ctypes.c_int]
        L.final_rms_norm.restype = None
        L.final_rms_norm.argtypes = [F_P, F_P, F_P, ctypes.c_int]
        L.embedding_lookup.restype = None
        L.embedding_lookup.argtypes = [F_P, ctypes.c_int, F_P, ctypes.c_int]
        f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)
        self.embedding = f32(w.embedding_f16())
        self.layers = []
        for Lw in w.layers:
            lw = {}
            for nm, p, n, k in (("in", Lw.in_proj, d.n_in, d.d_model), ("out", Lw.out_proj, d.d_model, d.d_inner)):
                packed = np.ascontiguousarray(p.packed.view(np.uint32))
                rs = np.empty(n, np.int32)
                L.precompute_row_sums(_p(packed, U32_P), _p(rs, I_P), n, k // 32)
                lw[nm] = (packed, f32(p.scale), rs, np.ascontiguousarray(p.lora_A), f32(p.lora_A_s),
                          np.ascontiguousarray(p.lora_B), f32(p.lora_B_s))
            lw["rest"] = tuple(f32(a) for a in (Lw.conv_w, Lw.conv_b, Lw.A_log, Lw.D, Lw.dt_bias, Lw.norm_w, Lw.ln_w))
            self.layers.append(lw)
        self.norm_f = f32(w.norm_f)
        self.x = np.empty(d.d_model, np.float32)
        self.x_norm = np.empty(d.d_model, np.float32)
        self.proj = np.empty(d.n_in, np.float32)
        self.y = np.empty(d.d_inner, np.float32)
        self.out = np.empty(d.d_model, np.float32)
        self.norm_out = np.empty(d.d_model, np.float32)
        self.reset()

    def reset(self):
        d = self.d
        self.h = [np.zeros((d.nheads, d.headdim, d.d_state), np.float32) for _ in range(d.n_layer)]
        self.conv = [np.zeros((d.d_xbc, 3), np.float32) for _ in range(d.n_layer)]

    def forward(self, token: int) -> np.ndarray:
        """cpu_inference_driver.py:159-184."""
        d, L = self.d, self.lib
        L.embedding_lookup(_p(self.embedding, F_P), int(token), _p(self.x, F_P), d.d_model)
        for l, lw in enumerate(self.layers):
            ip, op = lw["in"], lw["out"]
            cw, cb, al, dd, dtb, nw, lnw = lw["rest"]
            L.layer_forward(_p(self.x, F_P),
                            _p(ip[0], U32_P), _p(ip[1], F_P), _p(ip[2], I_P),
                            _p(op[0], U32_P), _p(op[1], F_P), _p(op[2], I_P),
                            _p(ip[3], I8_P), _p(ip[4], F_P), _p(ip[5], I8_P), _p(ip[6], F_P),
                            _p(op[3], I8_P), _p(op[4], F_P), _p(op[5], I8_P), _p(op[6], F_P),
                            _p(cw, F_P), _p(cb, F_P), _p(al, F_P), _p(dd, F_P), _p(dtb, F_P),
                            _p(nw, F_P), _p(lnw, F_P), _p(self.h[l], F_P), _p(self.conv[l], F_P),
                            _p(self.x_norm, F_P), _p(self.proj, F_P), _p(self.y, F_P), _p(self.out, F_P))
        L.final_rms_norm(_p(self.x, F_P), _p(self.norm_f, F_P), _p(self.norm_out, F_P), d.d_model)
        return self.norm_out @ self.embedding.T

    def decode(self, prompt, n_steps: int):
        """Feed prompt tokens, then n_steps greedy steps.  Returns (tokens, seconds of the decode loop)."""
        self.reset()
        tok = 0
        for t in prompt:
            tok = int(np.argmax(self.forward(int(t))))
        out = []
        t0 = time.perf_counter()
        for _ in range(n_steps):
            out.append(tok)
            tok = int(np.argmax(self.forward(tok)))
        return np.array(out), time.perf_counter() - t0


def _main():
    """Time the reference CPU engine on a synthetic config; prints one JSON line.
    Run in its own process so OMP_NUM_THREADS / OPENBLAS_NUM_THREADS take effect."""
    import argparse
    import json
    import sys
    sys.path.insert(0, os.path.dirname(HERE))
    from dfssm_b200 import synthetic
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="1.3b")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    w = synthetic.make_weights(synthetic.make_dims(a.shape, a.layers), seed=a.seed)
    prompts = synthetic.make_prompts(w.dims.vocab, a.batch, a.prompt, seed=a.seed)
    # one engine, one state set per sequence (the reference CPU path decodes one sequence)
    m = RefCPUModel(w)
    states = []
    for b in range(a.batch):
        m.reset()
        tok = 0
        for t in prompts[b]:
            tok = int(np.argmax(m.forward(int(t))))
        for _ in range(a.warmup):
            tok = int(np.argmax(m.forward(tok)))
        states.append((m.h, m.conv, tok))
    t0 = time.perf_counter()
    for _ in range(a.steps):
        for b in range(a.batch):
            h, c, tok = states[b]
            m.h, m.conv = h, c
            tok = int(np.argmax(m.forward(tok)))
            states[b] = (h, c, tok)
    el = time.perf_counter() - t0
    print(json.dumps({"tok_per_s": a.steps * a.batch / el, "seconds": el, "steps": a.steps,
                      "batch": a.batch, "threads": int(os.environ.get("OMP_NUM_THREADS", "0") or 0),
                      "tokens_last": [s[2] for s in states][:4]}))


if __name__ == "__main__":
    _main()
