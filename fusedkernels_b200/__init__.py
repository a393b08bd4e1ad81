"""fusedkernels_b200: the fusedkernels training hot path on B200 (sm_100a).

Same public API as fusedkernels 0.2.0 (fusedkernels/__init__.py:1-15) for the
hot-path ops; every op runs hand-written CUDA kernels from libfkb200.so through the
C ABI in include/fkb200.h.  There is no CPU or Triton fallback.
"""
from .cross_entropy import fused_cross_entropy, fused_cross_entropy_global_mean
from .rmsnorm import FusedRMSNorm
from .swiglu import fused_swiglu
from .moe_routing import fused_moe_route
from .moe_routing_v2 import fused_moe_route_v2
from .moe_routing_v4 import fused_moe_route_v4
from .moe_layer import FusedMoEMLP
from .moe_layer_sorted import FusedMoEMLPSorted

__all__ = [
    "fused_cross_entropy", "FusedRMSNorm", "fused_swiglu",
    "fused_moe_route", "fused_moe_route_v2", "fused_moe_route_v4",
    "FusedMoEMLP", "FusedMoEMLPSorted",
    "fused_cross_entropy_global_mean",  # data-parallel form (no counterpart in the reference)
]
__version__ = "0.2.0+b200"
