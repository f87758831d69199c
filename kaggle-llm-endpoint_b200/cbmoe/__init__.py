"""cbmoe: B200-native codebook-quantized MoE expert path (the GLM engine's ResidentFetch boundary) on hand-written
sm_100a CUDA kernels behind a C ABI (include/cbmoe.h, libcbmoe.so)."""
from ._lib import CbmoeError, device_errors, lib  # noqa: F401
from . import iq, ops  # noqa: F401
from .resident import ResidentFetch, moe_dense, moe_route, pack_layer  # noqa: F401
