"""v1 router API (``fused_moe_route``) on the B200 router kernel.

Mirrors fusedkernels/moe_routing.py (``_FusedMoERoute`` at moe_routing.py:84-125,
``fused_moe_route`` at moe_routing.py:128-130): same signature and outputs (fp32 weights
renormalised over the top k, int64 indices in descending order, dense fp32 dlogits in the
backward).  The reference selects with k sequential argmax passes over the softmax
probabilities; here the selection is the same bitonic kernel as ``fused_moe_route_v2``,
ranking by the exact logit (softmax is monotonic, so the order is the probability order;
exact ties go to the lower expert index, as an argmax that returns the first maximum
does).
"""
from .moe_routing_v2 import _FusedMoERouteV2


def fused_moe_route(router_logits, k: int):
    """v1 router API -- see module docstring.  Prefer fused_moe_route_v2."""
    return _FusedMoERouteV2.apply(router_logits, k)
