"""dfssm_b200 — B200-native (sm_100a) per-token decode engine for DF-SSM's Mamba-2 layer.

Drop-in for cs-cmyk/df-ssm's inference/gpu path: same .dfssm layout, same DFSSMModel API,
compute in libdfssm.so (hand-written CUDA for sm_100a behind a C ABI, include/dfssm.h).
"""
from . import dfssm_format, synthetic  # noqa: F401
from .dfssm_format import Dims, Weights  # noqa: F401


def __getattr__(name):
    # DFSSMModel imports torch lazily so that format/synthetic tools stay light.
    if name == "DFSSMModel":
        from .model import DFSSMModel
        return DFSSMModel
    raise AttributeError(name)
