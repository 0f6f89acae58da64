"""ctypes binding of libdfssm.so (the C ABI declared in include/dfssm.h).

The library is built in-tree (df-ssm_b200/lib/libdfssm.so, see build.py).  There is
no fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int8, c_int32, c_size_t, c_uint32, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libdfssm.so")

DFSSM_OK = 0
STATUS = {1: "ERR_ARG", 2: "ERR_FORMAT", 3: "ERR_UNSUPPORTED", 4: "ERR_CUDA", 5: "ERR_OOM", 6: "ERR_STATE",
          7: "ERR_NUMERIC"}

# Every exported symbol with (restype, argtypes); the tests check this list against
# the declarations in include/dfssm.h.
SIGNATURES = {
    "dfssm_version": (c_char_p, []),
    "dfssm_last_error": (c_char_p, []),
    "dfssm_kernel_binary_version": (c_int, [c_int, POINTER(c_int)]),
    "dfssm_create_from_memory": (c_int, [c_void_p, c_size_t, c_int, c_int, POINTER(c_void_p)]),
    "dfssm_create_from_file": (c_int, [c_char_p, c_int, c_int, POINTER(c_void_p)]),
    "dfssm_destroy": (None, [c_void_p]),
    "dfssm_get_dims": (c_int, [c_void_p, c_void_p]),
    "dfssm_set_batch": (c_int, [c_void_p, c_int]),
    "dfssm_set_mode": (c_int, [c_void_p, c_int]),
    "dfssm_get_mode": (c_int, [c_void_p, POINTER(c_int)]),
    "dfssm_reset": (c_int, [c_void_p, c_void_p]),
    "dfssm_reset_slots": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "dfssm_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dfssm_step_host": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dfssm_check_finite": (c_int, [c_void_p, c_void_p]),
    "dfssm_selftest_division": (c_int, [c_int, c_void_p]),
    "dfssm_sample": (c_int, [c_void_p, c_int, c_int, c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                             ctypes.c_uint64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dfssm_set_sampling": (c_int, [c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_uint64]),
    "dfssm_prefill": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "dfssm_prefill_slots": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "dfssm_state_ptrs": (c_int, [c_void_p, c_int, POINTER(c_void_p), POINTER(c_void_p)]),
    "dfssm_get_buffer": (c_int, [c_void_p, c_char_p, POINTER(c_void_p), POINTER(c_size_t)]),
    "dfssm_weight_ptr": (c_int, [c_void_p, c_int, c_char_p, POINTER(c_void_p), POINTER(c_size_t)]),
    "dfssm_layer_step": (c_int, [c_void_p, c_int, c_void_p]),
    "dfssm_trace_entries": (c_size_t, [c_void_p]),
    "dfssm_trace_step": (c_int, [c_void_p, c_void_p, c_void_p]),
    "dfssm_debug_set_wait_limit": (c_int, [c_void_p, c_uint32]),
    "dfssm_debug_skew_next_step": (c_int, [c_void_p]),
    "dfssm_scaffold_gemm_workspace": (c_size_t, [c_int, c_int]),
    "dfssm_scaffold_gemm": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "dfssm_scaffold_gemm_noalloc": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "dfssm_conv_step": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "dfssm_ssm_step": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "dfssm_rmsnorm_quantize": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "dfssm_lm_head_workspace": (c_size_t, [c_int]),
    "dfssm_lm_head_argmax": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                     c_void_p, c_void_p]),
}


class DFSSMError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"dfssm {STATUS.get(code, code)}: {msg}")
        self.code = code


class Dims(ctypes.Structure):
    _fields_ = [(n, c_int32) for n in ("n_layer", "d_model", "d_inner", "d_state", "nheads", "headdim",
                                       "ngroups", "vocab", "d_xbc", "n_in")]


_lib = None


def load(path: str = None) -> ctypes.CDLL:
    """Load libdfssm.so (or the library named by DFSSM_LIB) and bind every entry point.
    Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("DFSSM_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is not built; run `python -m dfssm_b200.build` (no CPU fallback exists)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != DFSSM_OK:
        msg = _lib.dfssm_last_error().decode(errors="replace") if _lib is not None else ""
        raise DFSSMError(rc, msg)
