"""v4 router API (``fused_moe_route_v4``) on the B200 router kernel.

Mirrors fusedkernels/moe_routing_v4.py (``_FusedMoERouteV4`` at moe_routing_v4.py:120-154,
``fused_moe_route_v4`` at moe_routing_v4.py:157-170): same signature, the same warning
when k > n_experts // 2, and the same output order -- the top k in ASCENDING rank order
(moe_routing_v4.py:114-117 keeps the last k keys of an ascending sort), i.e. the reverse
of ``fused_moe_route_v2``.  The reference composes a grouped bitonic sort and pairwise
merges in several launches; the group-then-merge selection here runs inside the single
router kernel (runs of next_pow2(k) keys sorted and merged in registers).
"""
import warnings

import torch

from . import _lib
from .moe_routing_v2 import MAX_EXPERTS


class _FusedMoERouteV4(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits: torch.Tensor, k: int):
        assert logits.is_cuda and logits.ndim == 2
        n_rows, n_experts = logits.shape
        assert k <= n_experts
        assert n_experts <= MAX_EXPERTS, f"n_experts={n_experts} exceeds {MAX_EXPERTS}"
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        w = torch.empty((n_rows, k), dtype=torch.float32, device=logits.device)
        idx = torch.empty((n_rows, k), dtype=torch.int64, device=logits.device)
        _lib.call("fk_router_fwd", logits.data_ptr(), logits.stride(0),
                  _lib.dtype_code(logits.dtype), n_rows, n_experts, k, w.data_ptr(),
                  idx.data_ptr(), _lib.stream_of(logits))
        ctx.save_for_backward(w, idx)
        ctx.n_experts = n_experts
        w_asc, idx_asc = w.flip(-1), idx.flip(-1)
        ctx.mark_non_differentiable(idx_asc)
        return w_asc, idx_asc

    @staticmethod
    def backward(ctx, dweights, dindices_unused):
        w, idx = ctx.saved_tensors
        n_rows, k = w.shape
        dlogits = torch.empty((n_rows, ctx.n_experts), dtype=torch.float32, device=w.device)
        if dweights is None:
            return dlogits.zero_(), None
        dw = dweights.to(torch.float32).flip(-1).contiguous()
        _lib.call("fk_router_bwd", dw.data_ptr(), w.data_ptr(), idx.data_ptr(), dlogits.data_ptr(),
                  n_rows, ctx.n_experts, k, _lib.stream_of(w))
        return dlogits, None


def fused_moe_route_v4(router_logits: torch.Tensor, k: int):
    """v4 router API: same interface as fused_moe_route_v2, top k in ascending order."""
    n_experts = router_logits.shape[-1]
    if k > n_experts // 2:
        warnings.warn(
            f"fused_moe_route_v4: k={k} is a large fraction of n_experts={n_experts}.",
            stacklevel=2,
        )
    return _FusedMoERouteV4.apply(router_logits, k)
