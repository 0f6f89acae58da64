"""The reference GPU decode driver restated op for op in torch — TEST INFRASTRUCTURE ONLY.

cs-cmyk/df-ssm's inference/gpu/df_ssm_inference.py (class DFSSMModel) is a short torch
program around two custom CUDA kernels.  It cannot travel to the GPU box, so this module
restates its decode path with the same torch calls in the same order, which on CUDA
tensors gives the reference GPU path itself: real `torch._int_mm` (cuBLAS int8), cuBLAS
fp16 LoRA / LM-head GEMMs and torch's CUDA elementwise rounding.  The conv / SSM steps are
either the reference kernels compiled from the checkout by oracle/build_ref.py
(oracle/_ref/ref_kernels/df_ssm_kernels_h64.so: fp16 state, 1.3B dims only) or the torch
restatement below (any state dtype), which tests/test_parity_ref_gpu.py pins to those
kernels.  On the CPU the same code reproduces the goldens that the reference module itself
produced (tests/golden/make_golden.py), which pins this restatement to the reference.

Only tests/ may import it; the product path never does.

Reference lines restated (df_ssm_inference.py unless noted):
  _unpack_to_int8          :23-29     (packed >> b) & 1 -> 2*bits - 1, columns b::32
  _load                    :62-110    in_w_T = unpack(...).T, LoRA (q * s).half(), fp16 norms
  _alloc_state             :112-135   per-layer h [B,H,P,N] / conv [B,D_XBC,3], B_pad = max(B, 32)
  _rms_norm                :141-145
  _quantize_to_int8        :147-152
  _scaffold_matmul         :154-158
  _run_layers              :160-210
  forward                  :219-224   x = embedding[tokens]; logits = norm_out @ embedding.T
  generate (greedy)        :236       tokens = logits.argmax(-1)
  conv_step_kernel         df_ssm_kernels.cu:27-47
  ssm_step_kernel          df_ssm_kernels.cu:53-103
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_KERNELS_SO = os.path.join(HERE, "_ref", "ref_kernels", "df_ssm_kernels_h64.so")
# compile-time dims of the reference kernel build (df_ssm_kernels.cu:15-21, HEADDIM patched to 64)
REF_KERNEL_DIMS = dict(d_inner=4096, d_xbc=4352, d_state=128, nheads=64, headdim=64)


def load_ref_kernels():
    """The reference's own conv/SSM CUDA kernels (pybind module), or None if not built."""
    if not os.path.exists(REF_KERNELS_SO):
        return None
    loader = importlib.machinery.ExtensionFileLoader("df_ssm_kernels_h64", REF_KERNELS_SO)
    spec = importlib.util.spec_from_loader("df_ssm_kernels_h64", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def conv_step_torch(conv_state, xBC, conv_weight, conv_bias, d_xBC):
    """df_ssm_kernels.cu:27-47 in torch: fp32 arithmetic, state and output stored in their dtypes."""
    s = conv_state.float()
    xv = xBC.float()
    w = conv_weight.float()
    out = s[..., 0] * w[:, 0] + s[..., 1] * w[:, 1] + s[..., 2] * w[:, 2] + xv * w[:, 3] + conv_bias.float()
    conv_state[..., 0] = s[..., 1].to(conv_state.dtype)
    conv_state[..., 1] = s[..., 2].to(conv_state.dtype)
    conv_state[..., 2] = xv.to(conv_state.dtype)
    xBC.copy_((out * (1.0 / (1.0 + torch.exp(-out)))).to(xBC.dtype))


def make_ssm_step_torch(d_inner, d_state, nheads, headdim):
    """df_ssm_kernels.cu:53-103 in torch (the state keeps its tensor's dtype; y from the fp32 state)."""
    def ssm_step(h_state, xBC, dt, dt_bias, A_log, D_param, y_out):
        B = h_state.shape[0]
        dtv = torch.log1p(torch.exp(dt.float() + dt_bias.float()))
        Abar = torch.exp(dtv * (-torch.exp(A_log.float())))
        x = xBC[:, :d_inner].float().reshape(B, nheads, headdim)
        Bp = xBC[:, d_inner:d_inner + d_state].float()
        Cp = xBC[:, d_inner + d_state:d_inner + 2 * d_state].float()
        X = x * dtv[:, :, None]
        h = Abar[:, :, None, None] * h_state.float() + X[..., None] * Bp[:, None, None, :]
        h_state.copy_(h.to(h_state.dtype))
        y = (h * Cp[:, None, None, :]).sum(-1) + x * D_param.float()[None, :, None]
        y_out.copy_(y.reshape(B, nheads * headdim).to(y_out.dtype))
    return ssm_step


def unpack_to_int8(packed, out_features, in_features):
    """df_ssm_inference.py:23-29."""
    w = torch.zeros(out_features, in_features, dtype=torch.int8, device=packed.device)
    for b in range(32):
        bits = (packed >> b) & 1
        w[:, b::32] = (2 * bits - 1).to(torch.int8)
    return w


class RefTorchModel:
    """DFSSMModel of df_ssm_inference.py:47-236 populated from in-memory weights.

    state_dtype: torch.float16 (the reference) or torch.float32 (the B200 engine's contract).
    kernels: "ref" (the compiled reference kernels; fp16 state and 1.3B dims only) or "torch".
    Norm weights are held in fp16 as `_load` reads them (:105-106,110)."""

    def __init__(self, w, batch: int, device="cuda", state_dtype=torch.float16, kernels: str = "torch"):
        d = w.dims
        self.d, self.B, self.device = d, batch, torch.device(device)
        dev = self.device
        if kernels == "ref":
            mod = load_ref_kernels()
            if mod is None:
                raise RuntimeError("reference kernels not built (python oracle/build_ref.py --gpu-kernels)")
            if state_dtype != torch.float16:
                raise ValueError("the reference kernels keep fp16 state")
            for k, v in REF_KERNEL_DIMS.items():
                if getattr(d, k) != v:
                    raise ValueError(f"the reference kernels are compiled for {k}={v}")
            self.conv_step, self.ssm_step = mod.conv_step, mod.ssm_step
        else:
            self.conv_step = conv_step_torch
            self.ssm_step = make_ssm_step_torch(d.d_inner, d.d_state, d.nheads, d.headdim)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        self.embedding = t(w.embedding_f16())
        self.layers = []
        for L in w.layers:
            lw = {}
            for name, p, k in (("in", L.in_proj, d.d_model), ("out", L.out_proj, d.d_inner)):
                n = p.packed.shape[0]
                lw[f"{name}_w_T"] = unpack_to_int8(t(p.packed), n, k).T.contiguous()
                lw[f"{name}_scale"] = t(p.scale)
                lw[f"{name}_lora_A"] = (t(p.lora_A).float() * t(p.lora_A_s).float().unsqueeze(1)).half()
                lw[f"{name}_lora_B"] = (t(p.lora_B).float() * t(p.lora_B_s).float().unsqueeze(1)).half()
            lw["conv_weight"], lw["conv_bias"] = t(L.conv_w), t(L.conv_b)
            lw["A_log"], lw["D"], lw["dt_bias"] = t(L.A_log), t(L.D), t(L.dt_bias)
            lw["norm_weight"], lw["layer_norm_weight"] = t(L.norm_w).half(), t(L.ln_w).half()
            self.layers.append(lw)
        self.norm_f_weight = t(w.norm_f).half()
        B, B_pad = batch, max(batch, 32)
        self.h_states = [torch.zeros(B, d.nheads, d.headdim, d.d_state, dtype=state_dtype, device=dev)
                         for _ in range(d.n_layer)]
        self.conv_states = [torch.zeros(B, d.d_xbc, 3, dtype=state_dtype, device=dev) for _ in range(d.n_layer)]
        f16 = dict(dtype=torch.float16, device=dev)
        self.x = torch.empty(B, d.d_model, **f16)
        self.x_norm = torch.empty(B, d.d_model, **f16)
        self.x_int8 = torch.zeros(B_pad, d.d_model, dtype=torch.int8, device=dev)
        self.proj = torch.empty(B, d.n_in, **f16)
        self.y_buf = torch.zeros(B, d.d_inner, **f16)
        self.y_norm = torch.empty(B, d.d_inner, **f16)
        self.y_int8 = torch.zeros(B_pad, d.d_inner, dtype=torch.int8, device=dev)
        self.out_buf = torch.empty(B, d.d_model, **f16)
        self.norm_out = torch.empty(B, d.d_model, **f16)
        self.x_scale = torch.empty(B, 1, **f16)
        self.spy = None  # optional callable(name, tensor) that sees intermediates

    def reset_state(self):
        for h in self.h_states:
            h.zero_()
        for c in self.conv_states:
            c.zero_()

    @staticmethod
    def rms_norm(x, weight):
        var = x.float().pow(2).mean(dim=-1, keepdim=True)
        return (x * torch.rsqrt(var + 1e-5)) * weight

    def quantize_to_int8(self, x, scale_buf, int8_buf):
        B = x.size(0)
        scale_buf.copy_(x.abs().amax(dim=-1, keepdim=True).clamp(min=1e-4) / 127.0)
        int8_buf[:B].copy_((x / scale_buf).round().clamp(-128, 127).to(torch.int8))
        return scale_buf, int8_buf

    def scaffold_matmul(self, x_int8_padded, x_scale, w_T, w_scale):
        out_int32 = torch._int_mm(x_int8_padded, w_T)
        if self.spy:
            self.spy("int_mm", x_int8_padded[:self.B], out_int32[:self.B])
        return (out_int32[:self.B].half() * x_scale) * w_scale.unsqueeze(0)

    def run_layers(self):
        d = self.d
        DI, DX, H, N = d.d_inner, d.d_xbc, d.nheads, d.d_state
        for l in range(d.n_layer):
            w = self.layers[l]
            self.x_norm.copy_(self.rms_norm(self.x, w["layer_norm_weight"]))
            self.quantize_to_int8(self.x_norm, self.x_scale, self.x_int8)
            self.proj.copy_(self.scaffold_matmul(self.x_int8, self.x_scale, w["in_w_T"], w["in_scale"]))
            self.proj.addmm_(self.x_norm @ w["in_lora_B"].T, w["in_lora_A"].T)
            z = self.proj[:, :DI]
            xBC = self.proj[:, DI:DI + DX].contiguous()
            dt = self.proj[:, DI + DX:DI + DX + H].contiguous()
            self.conv_step(self.conv_states[l], xBC, w["conv_weight"], w["conv_bias"], DX)
            self.y_buf.zero_()
            self.ssm_step(self.h_states[l], xBC, dt, w["dt_bias"], w["A_log"], w["D"], self.y_buf)
            silu_z = z * torch.sigmoid(z)
            gated = self.y_buf * silu_z
            self.y_norm.copy_(self.rms_norm(gated, w["norm_weight"]))
            self.quantize_to_int8(self.y_norm, self.x_scale, self.y_int8)
            self.out_buf.copy_(self.scaffold_matmul(self.y_int8, self.x_scale, w["out_w_T"], w["out_scale"]))
            self.out_buf.addmm_(self.y_norm @ w["out_lora_B"].T, w["out_lora_A"].T)
            self.x.add_(self.out_buf)
            if self.spy:
                self.spy(f"x{l}", self.x)
        self.norm_out.copy_(self.rms_norm(self.x, self.norm_f_weight))

    @torch.no_grad()
    def forward(self, token_ids):
        self.x.copy_(self.embedding[token_ids.to(self.device)])
        self.run_layers()
        return self.norm_out @ self.embedding.T

    @torch.no_grad()
    def generate(self, prompts, n_steps: int, teacher=None):
        """Feed prompts [B, T] one forward() per token, then n_steps greedy steps (argmax, :236).
        With `teacher` [n_steps, B] the decode inputs are forced.  Returns (tokens [n_steps, B]
        int64 numpy: the argmax fed/compared at each step, logits [n_steps, B, V] fp16 torch)."""
        prompts = torch.as_tensor(np.asarray(prompts), device=self.device)
        tok = None
        for t in range(prompts.shape[1]):
            tok = self.forward(prompts[:, t]).argmax(-1)
        toks, logs = [], []
        for s in range(n_steps):
            toks.append(tok.cpu().numpy())
            inp = tok if teacher is None else torch.as_tensor(np.asarray(teacher[s]), device=self.device)
            lg = self.forward(inp)
            logs.append(lg)
            tok = lg.argmax(-1)
        return np.stack(toks), torch.stack(logs)
