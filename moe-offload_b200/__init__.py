"""moe_offload_b200 -- B200 (sm_100a) implementation of the routed-expert MoE block of
Jakevin/moe-offload: router softmax/top-k, per-layer LRU expert-slot cache, 2-bit affine
gate/up/down expert GEMVs with SwiGLU, routing-weighted combine.

Compute runs in libmoe_b200.so (hand-written CUDA behind a C ABI, include/moe_b200.h);
this package is the host side that mirrors the reference's Python surface
(CachedSwitchGLU, OffloadEngine, compute_layer_capacities)."""
from ._lib import MoeError, load as load_library  # noqa: F401

__all__ = ["MoeError", "load_library"]
