"""DFSSMModel — drop-in for the reference GPU decode driver.

Mirrors class DFSSMModel of inference/gpu/df_ssm_inference.py:47-243 (constructor
`DFSSMModel(path, device="cuda", batch_size=1)`, `forward(token_ids) -> logits`,
`generate(n_tokens=128)`, `reset_state()`, attributes `h_states`, `conv_states`, `layers`,
`embedding`) and
its CLI (`model --batch_size B --n_tokens N`, :246-252).  All compute runs in
libdfssm.so (sm_100a kernels behind a C ABI); PyTorch only supplies device memory,
the current stream and tensor views.

Documented differences from the reference driver:
  * dims come from the .dfssm header; norms are read as fp32 (the exporter's dtype);
  * SSM/conv state is fp32 (the reference keeps fp16); `conv_states[l]` is the
    reference's [B, D_XBC, 3] layout as a strided view of the tap-major buffer;
  * `forward` returns fp32 logits (scale * int8-dot of the int8 tied embedding) and the
    greedy argmax is taken on their fp16 rounding, as the reference's fp16 logits;
  * `generate(n_tokens, prompt=None)` resets the state once and feeds the prompt token by
    token (token 0 when no prompt is given) instead of advancing the state twice on a
    warm-up token (df_ssm_inference.py:228-231); the greedy loop stays on the device.
"""
from __future__ import annotations

import ctypes
import time
from typing import Optional, Sequence, Union

import numpy as np

from . import _lib
from . import dfssm_format as fmt


class _DevArray:
    """Minimal __cuda_array_interface__ view of engine-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str, strides=None):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2, "strides": strides}


class LayerWeights:
    """Read-only device views of one layer's resident weights, named after the reference's
    LayerWeights (df_ssm_inference.py:32-44,68-106).  The scaffold stays bit-packed as in the file
    (`in_packed` / `out_packed`, int32 [N, K/32]); `in_w_T` / `out_w_T` unpack it on demand to the
    reference's int8 +-1 transpose [K, N] (a new tensor: the engine never holds it).  Norm weights
    are fp32 (the exporter's dtype)."""

    _FIELDS = {  # attribute: (engine name, dtype, shape from dims)
        "in_packed": ("in_bits", "<i4", lambda d: (d.n_in, d.d_model // 32)),
        "in_scale": ("in_scale", "<f2", lambda d: (d.n_in,)),
        "in_lora_A": ("in_lora_A", "<f2", lambda d: (d.n_in, 16)),
        "in_lora_B": ("in_lora_B", "<f2", lambda d: (16, d.d_model)),
        "out_packed": ("out_bits", "<i4", lambda d: (d.d_model, d.d_inner // 32)),
        "out_scale": ("out_scale", "<f2", lambda d: (d.d_model,)),
        "out_lora_A": ("out_lora_A", "<f2", lambda d: (d.d_model, 16)),
        "out_lora_B": ("out_lora_B", "<f2", lambda d: (16, d.d_inner)),
        "conv_weight": ("conv_w", "<f2", lambda d: (d.d_xbc, 4)),
        "conv_bias": ("conv_b", "<f2", lambda d: (d.d_xbc,)),
        "A_log": ("A_log", "<f4", lambda d: (d.nheads,)),
        "D": ("D", "<f4", lambda d: (d.nheads,)),
        "dt_bias": ("dt_bias", "<f4", lambda d: (d.nheads,)),
        "norm_weight": ("norm_w", "<f4", lambda d: (d.d_inner,)),
        "layer_norm_weight": ("ln_w", "<f4", lambda d: (d.d_model,)),
    }

    def __init__(self, model: "DFSSMModel", layer: int):
        for attr, (name, ts, shape) in self._FIELDS.items():
            setattr(self, attr, model._weight(layer, name, ts, shape(model.dims)))

    @staticmethod
    def _unpack_T(packed):
        """Packed signs [N, K/32] -> int8 +-1 [K, N] (bit b of word j is column 32j + b)."""
        import torch
        n, w = packed.shape
        bits = (packed.unsqueeze(-1) >> torch.arange(32, device=packed.device, dtype=torch.int32)) & 1
        return (2 * bits - 1).to(torch.int8).reshape(n, w * 32).T.contiguous()

    @property
    def in_w_T(self):
        return self._unpack_T(self.in_packed)

    @property
    def out_w_T(self):
        return self._unpack_T(self.out_packed)


class DFSSMModel:
    MODES = {"auto": 0, "graph": 1, "eager": 2, "persistent": 3}

    def __init__(self, path: Union[str, bytes, fmt.Weights], device="cuda", batch_size: int = 1,
                 max_batch: Optional[int] = None, mode: str = "auto", emb_kind: int = fmt.EMB_INT8):
        import torch
        self.torch = torch
        self.lib = _lib.load()
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DFSSMModel runs on CUDA devices only (there is no CPU fallback)")
        dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", dev_index)
        torch.cuda.set_device(dev_index)
        self.batch_size = batch_size
        self.max_batch = max(batch_size, max_batch or batch_size)
        h = ctypes.c_void_p()
        if isinstance(path, fmt.Weights):
            path = fmt.to_bytes(path, emb_kind)
        if isinstance(path, (bytes, bytearray, memoryview)):
            buf = bytes(path)
            _lib.check(self.lib.dfssm_create_from_memory(buf, len(buf), dev_index, self.max_batch, ctypes.byref(h)))
        else:
            _lib.check(self.lib.dfssm_create_from_file(str(path).encode(), dev_index, self.max_batch, ctypes.byref(h)))
        self._h = h
        dims = _lib.Dims()
        _lib.check(self.lib.dfssm_get_dims(self._h, ctypes.byref(dims)))
        self.dims = dims
        self.vocab = dims.vocab
        _lib.check(self.lib.dfssm_set_batch(self._h, batch_size))
        self.set_mode(mode)
        self.logits = torch.empty(self.max_batch, dims.vocab, dtype=torch.float32, device=self.device)
        self._tok_in = torch.zeros(self.max_batch, dtype=torch.int32, device=self.device)
        self._tok_out = torch.zeros(self.max_batch, dtype=torch.int32, device=self.device)
        self.h_states, self.conv_states = [], []
        B = self.max_batch
        for l in range(dims.n_layer):
            sp, cp = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(self.lib.dfssm_state_ptrs(self._h, l, ctypes.byref(sp), ctypes.byref(cp)))
            self.h_states.append(torch.as_tensor(
                _DevArray(sp.value, (B, dims.nheads, dims.headdim, dims.d_state), "<f4"), device=self.device))
            conv = torch.as_tensor(_DevArray(cp.value, (B, 3, dims.d_xbc), "<f4"), device=self.device)
            self.conv_states.append(conv.permute(0, 2, 1))  # [B, D_XBC, 3] view
        # resident weights as read-only device views (the reference's DFSSMModel.layers /
        # .embedding, df_ssm_inference.py:51,62-110)
        self.layers = [LayerWeights(self, l) for l in range(dims.n_layer)]
        self.embedding_q = self._weight(-1, "emb_q", "|i1", (dims.vocab, dims.d_model))
        self.embedding_scale = self._weight(-1, "emb_s", "<f4", (dims.vocab,))
        self.norm_f_weight = self._weight(-1, "norm_f", "<f4", (dims.d_model,))

    def _weight(self, layer: int, name: str, typestr: str, shape):
        p, n = ctypes.c_void_p(), ctypes.c_size_t()
        _lib.check(self.lib.dfssm_weight_ptr(self._h, layer, name.encode(), ctypes.byref(p), ctypes.byref(n)))
        return self.torch.as_tensor(_DevArray(p.value, shape, typestr), device=self.device)

    @property
    def embedding(self):
        """The tied embedding as fp16 [vocab, d_model] (df_ssm_inference.py:65), dequantised on demand
        from the resident int8 rows and their scales (fp16(q * s)); a new tensor each access."""
        return (self.embedding_q.float() * self.embedding_scale[:, None]).half()

    # ------------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "_h", None):
            self.lib.dfssm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream(self.device).cuda_stream)

    def set_mode(self, mode: str):
        _lib.check(self.lib.dfssm_set_mode(self._h, self.MODES[mode]))
        m = ctypes.c_int()
        _lib.check(self.lib.dfssm_get_mode(self._h, ctypes.byref(m)))
        self.mode = {v: k for k, v in self.MODES.items()}[m.value]

    def set_batch(self, batch_size: int):
        _lib.check(self.lib.dfssm_set_batch(self._h, batch_size))
        self.batch_size = batch_size

    def reset_state(self):
        _lib.check(self.lib.dfssm_reset(self._h, self._stream()))

    def reset_sequences(self, first: int, count: int = 1):
        """Zero the state of sequence slots [first, first + count) only (continuous batching)."""
        _lib.check(self.lib.dfssm_reset_slots(self._h, first, count, self._stream()))

    # ------------------------------------------------------------------ decode
    def step(self, token_ids=None, logits: bool = True):
        """One decode step.  token_ids: [B] ints (host or device) or None to continue from the
        previous step's greedy tokens.  Returns the greedy next tokens (int32 [B], device)."""
        torch = self.torch
        B = self.batch_size
        tin = None
        if token_ids is not None:
            t = torch.as_tensor(token_ids).reshape(-1)
            if t.numel() != B:
                raise ValueError(f"expected {B} token ids, got {t.numel()}")
            self._tok_in[:B].copy_(t.to(torch.int32), non_blocking=True)
            tin = ctypes.c_void_p(self._tok_in.data_ptr())
        lg = ctypes.c_void_p(self.logits.data_ptr()) if logits else None
        _lib.check(self.lib.dfssm_step(self._h, tin, lg, ctypes.c_void_p(self._tok_out.data_ptr()), self._stream()))
        return self._tok_out[:B]

    def step_host(self, tokens_host, next_host, logits_host=None):
        """One step through host buffers (numpy int32 [B], ideally pinned): copies the tokens in,
        runs the step, copies the next greedy tokens (and optionally fp32 logits) out and
        synchronises the stream (dfssm_step_host)."""
        _lib.check(self.lib.dfssm_step_host(
            self._h, ctypes.c_void_p(tokens_host.ctypes.data) if tokens_host is not None else None,
            ctypes.c_void_p(logits_host.ctypes.data) if logits_host is not None else None,
            ctypes.c_void_p(next_host.ctypes.data), self._stream()))
        return next_host

    def forward(self, token_ids):
        """Reference-compatible forward: logits [B, vocab] (fp32) for token_ids [B]."""
        self.step(token_ids, logits=True)
        return self.logits[:self.batch_size]

    __call__ = forward

    def prefill(self, prompt, chunked: bool = True, logits: bool = False) -> "object":
        """Consume prompt tokens [B, T] (dfssm_prefill: batched projections and a per-head scan
        over time; chunked=False feeds them one step at a time); returns the token chosen after
        the prompt (device int32 [B]) and fills self.logits if `logits`."""
        torch = self.torch
        prompt = torch.as_tensor(prompt)
        if prompt.dim() == 1:
            prompt = prompt.reshape(self.batch_size, -1)
        if not chunked:
            nxt = None
            for t in range(prompt.shape[1]):
                nxt = self.step(prompt[:, t], logits=logits)
            return nxt
        tok = prompt.to(device=self.device, dtype=torch.int32).contiguous()
        lg = ctypes.c_void_p(self.logits.data_ptr()) if logits else None
        _lib.check(self.lib.dfssm_prefill(self._h, ctypes.c_void_p(tok.data_ptr()), int(tok.shape[1]), lg,
                                          ctypes.c_void_p(self._tok_out.data_ptr()), self._stream()))
        return self._tok_out[: self.batch_size]

    def prefill_slots(self, first: int, prompt, logits: bool = False):
        """Consume prompt tokens [count, T] into sequence slots [first, first + count) only
        (dfssm_prefill_slots; continuous batching: reset_sequences() the slots first for new
        sequences).  Returns the next tokens of those slots (device int32 [count]); with `logits`
        their rows of self.logits are filled.  The other slots are untouched."""
        torch = self.torch
        prompt = torch.as_tensor(prompt)
        if prompt.dim() == 1:
            prompt = prompt.reshape(1, -1)
        count = int(prompt.shape[0])
        tok = prompt.to(device=self.device, dtype=torch.int32).contiguous()
        lg = ctypes.c_void_p(self.logits[first:].data_ptr()) if logits else None
        _lib.check(self.lib.dfssm_prefill_slots(self._h, int(first), count, ctypes.c_void_p(tok.data_ptr()),
                                                int(tok.shape[1]), lg, ctypes.c_void_p(self._tok_out[first:].data_ptr()),
                                                self._stream()))
        return self._tok_out[first:first + count]

    def set_sampling(self, temperature: float = 0.0, top_p: float = 1.0, rep_penalty: float = 1.0, seed: int = 0):
        """Token choice of later steps: greedy argmax for temperature <= 0 (the default, as the
        reference DFSSMModel.generate), else the sampling of eval/gen_test.py:54-95 (temperature,
        repetition penalty over the tokens already in each sequence, top-p nucleus, multinomial),
        on the device.  Draws are reproducible for a seed after reset_state()."""
        _lib.check(self.lib.dfssm_set_sampling(self._h, float(temperature), float(top_p), float(rep_penalty),
                                               int(seed) & (2**64 - 1)))

    def generate(self, n_tokens: int = 128, prompt=None, verbose: bool = True, logits: bool = False,
                 temperature: float = 0.0, top_p: float = 0.9, rep_penalty: float = 1.2, seed: int = 0):
        """Decode: reset, consume `prompt` ([B, T]; token 0 if None), then n_tokens steps.  Greedy
        by default; temperature > 0 samples as eval/gen_test.py's generate() (defaults 0.7 / 0.9 /
        1.2 there).  Returns int32 tokens [B, n_tokens] (host numpy)."""
        torch = self.torch
        B = self.batch_size
        self.set_sampling(temperature, top_p, rep_penalty, seed)
        self.reset_state()
        if prompt is None:
            prompt = torch.zeros(B, 1, dtype=torch.int64)
        self.prefill(prompt)
        out = torch.empty(n_tokens, B, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        start = time.perf_counter()
        stream = self._stream()
        lg = ctypes.c_void_p(self.logits.data_ptr()) if logits else None
        for s in range(n_tokens):
            # tokens_dev = NULL: the step consumes the previous step's greedy token on device
            _lib.check(self.lib.dfssm_step(self._h, None, lg, ctypes.c_void_p(out[s].data_ptr()), stream))
        torch.cuda.synchronize(self.device)
        elapsed = time.perf_counter() - start
        total = n_tokens * B
        if verbose:
            print(f"batch={B}  {n_tokens} steps  {total} total tokens")
            print(f"  {elapsed * 1000:.1f} ms  ({total / elapsed:.0f} tok/s total, "
                  f"{elapsed / n_tokens * 1e6:.0f} us/step, {total / elapsed / B:.0f} tok/s/seq)")
        self.last_elapsed = elapsed
        return out.t().contiguous().cpu().numpy()

    # ------------------------------------------------------------------ tools
    def buffer(self, name: str, dtype, shape):
        p, n = ctypes.c_void_p(), ctypes.c_size_t()
        _lib.check(self.lib.dfssm_get_buffer(self._h, name.encode(), ctypes.byref(p), ctypes.byref(n)))
        ts = {self.torch.float16: "<f2", self.torch.float32: "<f4", self.torch.int32: "<i4", self.torch.int8: "|i1"}[dtype]
        return self.torch.as_tensor(_DevArray(p.value, shape, ts), device=self.device)

    def layer_step(self, layer: int):
        _lib.check(self.lib.dfssm_layer_step(self._h, layer, self._stream()))

    def check_finite(self):
        _lib.check(self.lib.dfssm_check_finite(self._h, self._stream()))


def main(argv: Optional[Sequence[str]] = None):
    import argparse
    p = argparse.ArgumentParser(description="DF-SSM B200 greedy decode (drop-in for df_ssm_inference.py)")
    p.add_argument("model")
    p.add_argument("--batch_size", type=int, default=1)
    p.add_argument("--n_tokens", type=int, default=128)
    p.add_argument("--mode", default="auto", choices=list(DFSSMModel.MODES))
    p.add_argument("--temperature", type=float, default=0.0, help="> 0 samples (eval/gen_test.py); 0 = greedy")
    p.add_argument("--top_p", type=float, default=0.9)
    p.add_argument("--rep_penalty", type=float, default=1.2)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    DFSSMModel(a.model, batch_size=a.batch_size, mode=a.mode).generate(
        n_tokens=a.n_tokens, temperature=a.temperature, top_p=a.top_p, rep_penalty=a.rep_penalty, seed=a.seed)


if __name__ == "__main__":
    main()
