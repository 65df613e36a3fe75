"""eva_b200: B200-native (sm_100a) DeepSeek MoE hot path of the eva inference engine.

router -> token permutation -> fused EXL3 expert kernel (gate/up, SiLU*mul, down) -> routed
combine + shared expert, behind the reference's MoE operator interfaces. The compute is in
libeva_moe.so (C ABI, include/eva_moe.h); this package is the host side.
"""
from .config import CONFIGS, REF_NATIVE, V2_LITE, V3, MoEConfig

__all__ = ["MoEConfig", "CONFIGS", "V2_LITE", "V3", "REF_NATIVE", "EvaMoE", "EvaMoERunner", "make_layer"]


def __getattr__(name):
    if name in ("EvaMoE", "EvaMoERunner"):
        from . import runner
        return getattr(runner, name)
    if name == "make_layer":
        from .experts import make_layer
        return make_layer
    raise AttributeError(name)
