"""CPU restatement of the fusedkernels reference path (test infrastructure only).

Each function names the reference code it restates.  Citations are paths inside the
fusedkernels source tree (Siddhuuuu/fusedKernels v0.2.0).  Everything runs in fp64 (or
the stated precision) on the CPU with torch's CPU kernels.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# ------------------------------------------------------------------------ router -------
def route_oracle(logits: torch.Tensor, k: int, dtype=torch.float64):
    """Top-k router: softmax over E, top-k by logit, renormalise.

    Restates ``naive_route`` (tests/test_moe_routing_v2.py:11-15) -- softmax, topk,
    weights / weights.sum -- with the selection made explicit and deterministic: rank by
    the exact logit, ties toward the lower expert index (a stable descending sort; CPU
    torch.topk does not break exact ties toward the lower index).  -0.0 and +0.0 rank
    equal and NaN ranks above +inf, as torch.sort ranks them.  Weights are gathered from
    an fp64 softmax and renormalised (moe_routing_v2.py:48-94 computes the same
    quantities: probs, gather at the selected indices, divide by their sum).

    Returns (w float32 [N, k], idx int64 [N, k]) in descending rank order.  ``dtype`` is
    the arithmetic precision (fp64 for parity; fp32, the reference path's own, for the
    timed CPU baseline).
    """
    x = logits.detach().to(dtype).cpu()
    key = torch.where(x == 0, torch.zeros_like(x), x)  # fold -0.0 onto +0.0
    idx = torch.sort(key, dim=-1, descending=True, stable=True).indices[:, :k]
    probs = torch.softmax(x, dim=-1)
    w = torch.gather(probs, 1, idx)
    w = w / w.sum(dim=-1, keepdim=True)
    return w.to(torch.float32), idx


def route_bwd_oracle(logits: torch.Tensor, k: int, dw: torch.Tensor, dtype=torch.float64,
                     idx: torch.Tensor | None = None) -> torch.Tensor:
    """dlogits for upstream dw at fixed selection (moe_routing_v2.py:102-126).

    The selection is not differentiated (moe_routing_v2.py:109-112); the renormalised
    weights are a softmax over the selected logits, so autograd through
    softmax -> gather -> renormalise gives w_j (dw_j - sum_m w_m dw_m) at the selected
    columns and exactly 0 elsewhere.  fp64 by default, returned as fp32; ``idx`` reuses a
    selection already made by ``route_oracle``.
    """
    x = logits.detach().to(dtype).cpu().requires_grad_(True)
    if idx is None:
        _, idx = route_oracle(logits, k, dtype)
    probs = torch.softmax(x, dim=-1)
    w = torch.gather(probs, 1, idx)
    w = w / w.sum(dim=-1, keepdim=True)
    w.backward(dw.detach().to(dtype).cpu())
    return x.grad.to(torch.float32)


# ------------------------------------------------------------------------ RMSNorm ------
def rmsnorm_oracle(x: torch.Tensor, weight: torch.Tensor, eps: float, dy: torch.Tensor | None = None,
                   dtype=torch.float64):
    """``RefRMSNorm`` (tests/test_correctness.py:47-56; same in benchmarks/bench_all.py:60-69):
    y = x * rsqrt(mean(x^2) + eps) * w, evaluated in ``dtype`` (fp64 default).  With
    ``dy`` also returns (dx, dw) by autograd.  16-bit inputs are upcast first (the
    reference's fp32 accumulation, rmsnorm.py:33-40 and :60-70)."""
    xf = x.detach().to(dtype).cpu().requires_grad_(dy is not None)
    wf = weight.detach().to(dtype).cpu().requires_grad_(dy is not None)
    var = xf.pow(2).mean(-1, keepdim=True)
    y = xf * torch.rsqrt(var + eps) * wf
    if dy is None:
        return y.detach()
    y.backward(dy.detach().to(dtype).cpu())
    return y.detach(), xf.grad, wf.grad


# ------------------------------------------------------------------------ SwiGLU -------
def swiglu_oracle(gate: torch.Tensor, up: torch.Tensor, dout: torch.Tensor | None = None,
                  dtype=torch.float64):
    """``F.silu(gate) * up`` (tests/test_correctness.py:89; swiglu.py:84-86 docstring) in
    ``dtype``; with ``dout`` also (dgate, dup) by autograd."""
    g = gate.detach().to(dtype).cpu().requires_grad_(dout is not None)
    u = up.detach().to(dtype).cpu().requires_grad_(dout is not None)
    out = F.silu(g) * u
    if dout is None:
        return out.detach()
    out.backward(dout.detach().to(dtype).cpu())
    return out.detach(), g.grad, u.grad


# ------------------------------------------------------------------------ cross-entropy -
def cross_entropy_oracle(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                         label_smoothing: float = 0.0, dtype=torch.float64):
    """Loss and d(loss)/d(logits) of the reference's fused cross-entropy.

    Per row (cross_entropy.py:41-79): lse = logsumexp(x); loss = lse - x_t, blended with
    the smoothing term (1-ls)*loss + ls*(lse - mean x) when ls > 0; ignored rows give 0.
    The mean divides by n_valid = max(1, #targets != ignore_index) (cross_entropy.py:107,
    :110).  This equals ``F.cross_entropy(..., ignore_index, label_smoothing)`` (the
    reference's own test oracle, tests/test_correctness.py:21, :39) whenever one row is
    valid; the explicit form also covers the all-ignored batch, where the reference
    returns 0.  Gradient by autograd.  Returns (loss fp64 scalar, grad fp64 [N, V]).
    """
    x = logits.detach().to(dtype).cpu().requires_grad_(True)
    t = targets.detach().cpu().to(torch.int64)
    valid = t != ignore_index
    n_valid = max(int(valid.sum()), 1)
    lse = torch.logsumexp(x, dim=-1)
    t_safe = torch.where(valid, t, torch.zeros_like(t))
    xt = torch.gather(x, 1, t_safe[:, None])[:, 0]
    loss_rows = lse - xt
    if label_smoothing > 0.0:
        loss_rows = (1.0 - label_smoothing) * loss_rows + label_smoothing * (lse - x.mean(-1))
    loss_rows = torch.where(valid, loss_rows, torch.zeros_like(loss_rows))
    loss = loss_rows.sum() / n_valid
    loss.backward()
    return loss.detach(), x.grad


# ------------------------------------------------------------------------ MoE layer ----
def zipf_expert_bias(n_experts: int, s: float = 1.1) -> torch.Tensor:
    """Per-expert logit bias 2*ln(w_e), w_e proportional to (e+1)^-s and normalised: the
    imbalanced-load term the MoE-layer workload adds to the router logits."""
    ranks = torch.arange(1, n_experts + 1, dtype=torch.float64)
    w = ranks.pow(-s)
    w = w / w.sum()
    return (2.0 * torch.log(w)).to(torch.float32)


def moe_layer_oracle(x, router_logits, w_gate, w_up, w_down, k, dout=None, dtype=torch.float64):
    """``NaiveMoEMLP`` (tests/test_moe_sorted_dispatch.py:12-40) with ``Expert``
    (fusedkernels/moe_layer.py:22-31): route, run every expert's SwiGLU MLP
    w_down(silu(w_gate x) * w_up x) on its tokens, weight and sum per token.

    ``router_logits`` are given (the device's router GEMM output), so the oracle and the
    kernels see the same selection; routing follows ``route_oracle``.  Stacked weights:
    w_gate, w_up [E, H, D], w_down [E, D, H].  With ``dout`` also returns
    (dx_expert_path, dw_gate, dw_up, dw_down, d_router_logits) by autograd; dx excludes
    the router-GEMM path, which the caller adds through its own Linear.
    """
    req = dout is not None
    X = x.detach().to(dtype).cpu().requires_grad_(req)
    L = router_logits.detach().to(dtype).cpu().requires_grad_(req)
    E = w_gate.shape[0]
    # one leaf per expert matrix, as the reference's ModuleList of Linear layers holds them
    Wg = [w_gate[e].detach().to(dtype).cpu().requires_grad_(req) for e in range(E)]
    Wu = [w_up[e].detach().to(dtype).cpu().requires_grad_(req) for e in range(E)]
    Wd = [w_down[e].detach().to(dtype).cpu().requires_grad_(req) for e in range(E)]
    _, idx = route_oracle(router_logits, k)
    probs = torch.softmax(L, dim=-1)
    wsel = torch.gather(probs, 1, idx)
    wsel = wsel / wsel.sum(dim=-1, keepdim=True)
    out = torch.zeros_like(X)
    for e in range(E):
        match = idx == e
        tok = match.any(dim=-1)
        if not bool(tok.any()):
            continue
        we = (wsel * match).sum(dim=-1)[tok]
        xe = X[tok]
        h = F.silu(xe @ Wg[e].T) * (xe @ Wu[e].T)
        out = out.index_add(0, tok.nonzero()[:, 0], (h @ Wd[e].T) * we[:, None])
    if not req:
        return out.detach()
    out.backward(dout.detach().to(dtype).cpu())

    def stacked(ws):
        return torch.stack([w.grad if w.grad is not None else torch.zeros_like(w) for w in ws])

    return out.detach(), X.grad, stacked(Wg), stacked(Wu), stacked(Wd), L.grad


def relative_error(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-30))


__all__ = [
    "route_oracle", "route_bwd_oracle", "rmsnorm_oracle", "swiglu_oracle",
    "cross_entropy_oracle", "moe_layer_oracle", "zipf_expert_bias", "relative_error",
    "math",
]
