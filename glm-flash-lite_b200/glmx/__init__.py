"""glmx: B200-native routed-expert MoE layer over EXL3 trellis-coded experts (drop-in for glm-flash-lite's expert
tier). The compute lives in libglmx.so (include/glmx.h); this package is the PyTorch-side host."""
from ._lib import GlmxError, load  # noqa: F401
from .layer import MoELayer, decode_tiles  # noqa: F401
from .router import Router  # noqa: F401

__all__ = ["MoELayer", "Router", "decode_tiles", "GlmxError", "load"]
