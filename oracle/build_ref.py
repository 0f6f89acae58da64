"""Build the reference's own implementations into oracle/_ref/ (TEST INFRASTRUCTURE).

Compiled from the sources where they lie in the reference checkout (never copied into
this repository); outputs go only to oracle/_ref/ (git-ignored, travels to the GPU box):

  libcpu_inference_<shape>.so  inference/cpu/cpu_inference.c, compile-time dims patched
                               on the way into gcc through a pipe (HEADDIM 32 -> 64, the
                               value of the trained model; D_* for other shapes):
                               gcc -O3 -fopenmp -mavx512{f,bw,vl,dq,vnni} -mfma -shared -fPIC
  ref_kernels/                 inference/gpu/df_ssm_kernels.cu (HEADDIM 32 -> 64) as a torch
                               extension for sm_100a, used only by a GPU test that pins the
                               oracle's conv/SSM restatement to the real reference kernels.

Usage: python oracle/build_ref.py [--ref <checkout>] [--gpu-kernels]
"""
from __future__ import annotations

import argparse
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# the reference checkout: $DFSSM_REFERENCE, else a `reference` directory beside this repository
DEFAULT_REF = os.environ.get("DFSSM_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")

SHAPES = {
    "1p3b": dict(D_MODEL=2048, D_INNER=4096, D_XBC=4352, D_STATE=128, NHEADS=64, HEADDIM=64, IN_PROJ_OUT=8512),
    "2p7b": dict(D_MODEL=2560, D_INNER=5120, D_XBC=5376, D_STATE=128, NHEADS=80, HEADDIM=64, IN_PROJ_OUT=10576),
    "tiny": dict(D_MODEL=256, D_INNER=512, D_XBC=768, D_STATE=128, NHEADS=8, HEADDIM=64, IN_PROJ_OUT=1288),
}


def patch_defines(src: str, defs: dict) -> str:
    for k, v in defs.items():
        src, n = re.subn(rf"(#define\s+{k}\s+)\d+", rf"\g<1>{v}", src)
        if n != 1:
            raise RuntimeError(f"could not patch #define {k}")
    return src


def cpu_lib_path(shape: str) -> str:
    return os.path.join(OUT, f"libcpu_inference_{shape}.so")


def build_cpu(ref: str, shape: str) -> str:
    src_path = os.path.join(ref, "inference", "cpu", "cpu_inference.c")
    with open(src_path) as f:
        src = patch_defines(f.read(), SHAPES[shape])
    os.makedirs(OUT, exist_ok=True)
    out = cpu_lib_path(shape)
    cmd = ["gcc", "-O3", "-fopenmp", "-mavx512f", "-mavx512bw", "-mavx512vl", "-mavx512dq", "-mavx512vnni", "-mfma",
           "-shared", "-fPIC", "-x", "c", "-", "-o", out, "-lm"]
    subprocess.run(cmd, input=src.encode(), check=True)
    return out


def build_gpu_kernels(ref: str) -> str:
    """The reference pybind extension, HEADDIM patched, as a torch extension for sm_100a."""
    from torch.utils.cpp_extension import load
    src_path = os.path.join(ref, "inference", "gpu", "df_ssm_kernels.cu")
    with open(src_path) as f:
        src = patch_defines(f.read(), {"HEADDIM": 64})
    bdir = os.path.join(OUT, "ref_kernels")
    os.makedirs(bdir, exist_ok=True)
    tmp = os.path.join(bdir, "df_ssm_kernels_h64.cu")
    with open(tmp, "w") as f:
        f.write(src)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    try:
        load(name="df_ssm_kernels_h64", sources=[tmp], build_directory=bdir, verbose=False,
             extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"])
    finally:
        os.remove(tmp)  # keep only the built module, not the patched source
    return bdir


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=DEFAULT_REF)
    ap.add_argument("--shapes", default="1p3b,tiny")
    ap.add_argument("--gpu-kernels", action="store_true")
    a = ap.parse_args()
    if not os.path.isdir(a.ref):
        print(f"reference checkout {a.ref} not present; nothing built", file=sys.stderr)
        return
    for s in a.shapes.split(","):
        print(build_cpu(a.ref, s))
    if a.gpu_kernels:
        print(build_gpu_kernels(a.ref))


if __name__ == "__main__":
    main()
