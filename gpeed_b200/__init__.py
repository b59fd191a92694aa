"""gpeed_b200: B200 (sm_100a) IQ3_XXS routed-expert MoE path.

The compute lives in libgpeed_moe.so (gpeed_b200/csrc, C ABI in
include/gpeed_moe.h); this package is the host-side mirror of the reference
engine's expert-op interface on top of it.
"""
from ._capi import GpeedError, load as load_library  # noqa: F401
from .moe import Context, MoeConfig, MoeLayer, WeightStore, dequantize  # noqa: F401
from .gguf import GgufModel  # noqa: F401

__all__ = ["Context", "MoeConfig", "MoeLayer", "WeightStore", "dequantize", "GpeedError", "load_library",
           "GgufModel"]
