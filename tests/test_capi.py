"""CPU tests of the C ABI: the library loads, exports exactly what include/dfssm.h declares,
and rejects malformed .dfssm images before touching a GPU."""
import ctypes
import os
import re
import struct
import subprocess

import pytest

from dfssm_b200 import _lib
from dfssm_b200 import dfssm_format as fmt
from dfssm_b200 import synthetic

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dfssm.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dfssm_[a-z0-9_]+)\s*\(", src)))


def test_header_declarations_are_bound_and_exported():
    lib = _lib.load()
    decl = declared_functions()
    assert decl, "no declarations parsed"
    assert sorted(_lib.SIGNATURES) == decl
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(dfssm_[a-z0-9_]+)\b", out))
    for name in decl:
        assert name in exported, name
        assert getattr(lib, name) is not None
    assert lib.dfssm_version().startswith(b"dfssm-b200")


def test_library_is_built_for_sm100a_only():
    """The build compiles every kernel for sm_100a and nothing else (no PTX to JIT elsewhere)."""
    from dfssm_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


@pytest.mark.gpu
def test_kernels_run_as_sm100a_binaries():
    import ctypes
    lib = _lib.load()
    v = ctypes.c_int()
    _lib.check(lib.dfssm_kernel_binary_version(0, ctypes.byref(v)))
    assert v.value == 100


def _create(buf):
    lib = _lib.load()
    h = ctypes.c_void_p()
    rc = lib.dfssm_create_from_memory(buf, len(buf), 0, 1, ctypes.byref(h))
    return rc, lib.dfssm_last_error().decode()


def test_create_rejects_bad_images_without_gpu():
    w = synthetic.make_weights(synthetic.make_dims("tiny", 1), seed=0)
    good = fmt.to_bytes(w)
    rc, msg = _create(good[:-4])
    assert rc == 2 and "header implies" in msg
    bad = bytearray(good)
    bad[:8] = b"DFSSM999"
    rc, msg = _create(bytes(bad))
    assert rc == 2 and "magic" in msg
    bad = bytearray(good)
    struct.pack_into("<I", bad, 8 + 4 * 5, 32)  # headdim 32: nheads*headdim != d_inner
    rc, msg = _create(bytes(bad))
    assert rc == 2 and "d_inner" in msg
    bad = bytearray(good)
    struct.pack_into("<I", bad, 8 + 4 * 6, 2)  # ngroups 2
    rc, msg = _create(bytes(bad))
    assert rc == 3
    rc, msg = _create(good[:10])
    assert rc == 2
    lib = _lib.load()
    assert lib.dfssm_create_from_memory(good, len(good), 0, 0, ctypes.byref(ctypes.c_void_p())) == 1
    assert lib.dfssm_create_from_file(b"/nonexistent.dfssm", 0, 1, ctypes.byref(ctypes.c_void_p())) == 1
    assert lib.dfssm_step(None, None, None, None, None) == 1


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.dfssm_scaffold_gemm_workspace(1, 2048) >= 2048 + 4
    assert lib.dfssm_lm_head_workspace(8) >= 64
    assert lib.dfssm_scaffold_gemm_workspace(0, 2048) == 0
