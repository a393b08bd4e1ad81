"""Fused MoE router: softmax + top-k selection + renormalisation in one kernel.

Mirrors fusedkernels/moe_routing_v2.py (``_FusedMoERouteV2`` at moe_routing_v2.py:114-162,
``fused_moe_route_v2`` at moe_routing_v2.py:165-173): same signature, returns
(weights fp32 [N, k], indices int64 [N, k]) in descending rank order, same
AssertionError preconditions (CUDA, 2-D, k <= E, E <= 256), and a backward that
returns a dense fp32 dlogits (the index output has no gradient).

Selection differs from the reference's quantised tanh key on purpose: experts are
ranked by the exact logit value and ties go to the LOWER expert index (-0.0 == +0.0,
NaN ranks above +inf), i.e. ``torch.sort(logits, descending=True, stable=True)[:, :k]``.
"""
import torch

from . import _lib

MAX_EXPERTS = 256


class _FusedMoERouteV2(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits: torch.Tensor, k: int):
        assert logits.is_cuda and logits.ndim == 2
        n_rows, n_experts = logits.shape
        assert k <= n_experts
        assert n_experts <= MAX_EXPERTS, f"n_experts={n_experts} exceeds {MAX_EXPERTS}"
        assert k >= 1
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        w = torch.empty((n_rows, k), dtype=torch.float32, device=logits.device)
        idx = torch.empty((n_rows, k), dtype=torch.int64, device=logits.device)
        _lib.call("fk_router_fwd", logits.data_ptr(), logits.stride(0),
                  _lib.dtype_code(logits.dtype), n_rows, n_experts, k, w.data_ptr(),
                  idx.data_ptr(), _lib.stream_of(logits))
        ctx.save_for_backward(w, idx)
        ctx.n_experts = n_experts
        ctx.k = k
        ctx.mark_non_differentiable(idx)
        return w, idx

    @staticmethod
    def backward(ctx, dweights, dindices_unused):
        w, idx = ctx.saved_tensors
        n_rows, k = w.shape
        dlogits = torch.empty((n_rows, ctx.n_experts), dtype=torch.float32, device=w.device)
        if dweights is None:
            dlogits.zero_()
            return dlogits, None
        dw = dweights.to(torch.float32).contiguous()
        _lib.call("fk_router_bwd", dw.data_ptr(), w.data_ptr(), idx.data_ptr(),
                  dlogits.data_ptr(), n_rows, ctx.n_experts, k, _lib.stream_of(w))
        return dlogits, None


def fused_moe_route_v2(router_logits: torch.Tensor, k: int):
    """Fused MoE router: fuses softmax + top-k selection + renormalization into one
    kernel launch.  Drop-in replacement for:
        probs = F.softmax(router_logits, dim=-1)
        topk_weights, topk_idx = torch.topk(probs, k, dim=-1)
        topk_weights = topk_weights / topk_weights.sum(-1, keepdim=True)
    """
    return _FusedMoERouteV2.apply(router_logits, k)
