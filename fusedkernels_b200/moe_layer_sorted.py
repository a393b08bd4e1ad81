"""MoE MLP layer with sorted dispatch on B200.

Mirrors fusedkernels/moe_layer_sorted.py (``FusedMoEMLPSorted`` at moe_layer_sorted.py:28-87):
same constructor, same submodules (``router`` = nn.Linear(dim, E, bias=False), ``experts`` =
ModuleList of ``Expert``), same state_dict keys and the same forward semantics
(out[t] = sum_j w[t,j] * Expert_{idx[t,j]}(x[t])).  The body differs:

  router GEMM (nn.Linear) -> fused_moe_route_v2 -> fk_moe_route_meta (stable counting sort,
  128-row padded expert segments, all on the device) -> fk_moe_gather_by_token ->
  fk_moe_gemm_up_weighted
  (tcgen05 grouped GEMM, SwiGLU and routing-weight epilogue) -> fk_moe_gemm_down ->
  fk_moe_combine (per-token fp32 sum in slot order: deterministic, no index_add_ atomics).

There is no device->host synchronisation (the reference reads the expert counts back with
.tolist(), moe_layer_sorted.py:67-68): every buffer is sized for the worst case
N*k + E*127 rows.  Backward gathers dout's rows, runs the input-gradient GEMMs (the
down-projection's fuses the SwiGLU backward, the routing weight and the routing-weight
gradient into its epilogue) and the per-expert weight-gradient GEMMs.  fp16 and fp32
layers apply the routing weight in the combine kernels instead (fk_moe_combine_bwd in
backward).

Expert weights live in two stacked buffers, w13 [E, 2H, D] (gate rows then up rows) and
w2 [E, D, H]; every ``experts[e].w_*.weight`` Parameter is a view into them (re-pointed at
construction and after ``.to()``/``.cuda()``/dtype casts), so the parameters the reference
exposes stay the leaves that receive gradients.

Every GEMM runs on the tcgen05 tensor cores in the layer's dtype: bf16 and fp16 layers on
16-bit MMAs with fp32 accumulation; fp32 layers (the reference's default dtype) with the
3xTF32 split (each fp32 operand becomes a tf32 hi part plus a residual, and the kernel
sums hi*hi + hi*lo + lo*hi in fp32), which keeps fp32-class accuracy.
"""
import torch
import torch.nn as nn

from . import _lib
from .moe_layer import Expert
from .moe_routing import fused_moe_route
from .moe_routing_v2 import fused_moe_route_v2


class _Plan:
    """Device buffers of one routing (sized by shapes only)."""

    def __init__(self, n_tokens, k, n_experts, dev):
        self.max_rows, ws = _lib.moe_capacity(n_tokens, k, n_experts)
        i32 = dict(dtype=torch.int32, device=dev)
        self.counts = torch.empty(n_experts, **i32)
        self.seg_start = torch.empty(n_experts + 1, **i32)
        self.tile_expert = torch.empty(max(self.max_rows // 128, 1), **i32)
        self.n_mblk = torch.empty(1, **i32)
        self.sorted_assign = torch.empty(max(self.max_rows, 1), **i32)
        self.sorted_w = torch.empty(max(self.max_rows, 1), dtype=torch.float32, device=dev)
        self.slot_pos = torch.empty(max(n_tokens * k, 1), **i32)
        self.ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.err = torch.zeros(2, **i32)  # [routing error, GEMM error]


def _check_err(plan):
    """Raise if a kernel reported an error (reads a device flag: synchronises)."""
    e = plan.err.tolist()
    if e[0]:
        raise RuntimeError("fk_moe_route_meta: expert index outside [0, n_experts)")
    if e[1]:
        raise RuntimeError(f"fk_moe_gemm: a pipeline wait timed out (code {e[1]})")


def _split(t, st):
    """fp32 tensor -> (hi, lo) for the 3xTF32 GEMMs (fk_tf32_split)."""
    hi = torch.empty_like(t)
    lo = torch.empty_like(t)
    _lib.call("fk_tf32_split", t.data_ptr(), t.numel(), hi.data_ptr(), lo.data_ptr(), st)
    return hi, lo


def _operand(t, st):
    """GEMM operand pair (value, lo part): fp32 operands are split, 16-bit ones are not."""
    return _split(t, st) if t.dtype == torch.float32 else (t, None)


def _p(t):
    return None if t is None else t.data_ptr()


class _SortedMoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, idx, layer, *expert_params):
        n, d = x.shape
        k = idx.shape[1]
        E, H = layer.n_experts, layer.hidden_dim
        dev = x.device
        dt = x.dtype
        code = _lib.dtype_code(dt)
        st = _lib.stream_of(x)
        plan = _Plan(n, k, E, dev)
        R = plan.max_rows
        idx = idx.contiguous()
        w = w.to(torch.float32).contiguous()
        eptr = plan.err.data_ptr()
        _lib.call("fk_moe_route_meta", idx.data_ptr(), w.data_ptr(), n, k, E,
                  plan.counts.data_ptr(), plan.seg_start.data_ptr(), plan.tile_expert.data_ptr(),
                  plan.n_mblk.data_ptr(), plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(),
                  plan.slot_pos.data_ptr(), R, plan.ws.data_ptr(), plan.ws.numel(), eptr, st)
        td = dict(dtype=dt, device=dev)
        ctx.plan = plan
        ctx.layer = layer
        ctx.dims = (n, d, k, E, H)
        ctx.weighted = dt == torch.bfloat16
        if ctx.weighted:
            # The routing weight is applied in the up-projection's epilogue (act_w =
            # w * silu(g) * u), so the down-projection gives weighted rows that the combine
            # sums unweighted; the backward then needs no pass over the output rows.
            xs = torch.empty(R, d, **td)
            h1 = torch.empty(R, 2 * H, **td)
            act_w = torch.empty(R, H, **td)
            y = torch.empty(R, d, **td)
            out = torch.empty(n, d, **td)
            if R > 0:
                te, nm = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr()
                _lib.call("fk_moe_gather_by_token", x.data_ptr(), d, plan.slot_pos.data_ptr(), n,
                          k, plan.sorted_assign.data_ptr(), nm, R, xs.data_ptr(), code, st)
                _lib.call("fk_moe_gemm_up_weighted", xs.data_ptr(), R, d, layer.w13.data_ptr(),
                          H, E, te, nm, plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(),
                          h1.data_ptr(), act_w.data_ptr(), 0, eptr + 4, st)
                _lib.call("fk_moe_gemm_down", act_w.data_ptr(), R, H, layer.w2.data_ptr(), d, E,
                          te, nm, y.data_ptr(), 0, eptr + 4, st)
            _lib.call("fk_moe_combine", y.data_ptr(), d, plan.slot_pos.data_ptr(), None, n, k,
                      out.data_ptr(), code, st)
            if layer.check_errors:
                _check_err(plan)
            ctx.save_for_backward(xs, h1, act_w)
            return out
        xs = torch.empty(R, d, **td)
        h1 = torch.empty(R, 2 * H, **td)
        act = torch.empty(R, H, **td)
        y = torch.empty(R, d, **td)
        out = torch.empty(n, d, **td)
        xs_lo = act_lo = None
        if R > 0:
            _lib.call("fk_moe_gather", x.data_ptr(), d, plan.sorted_assign.data_ptr(), k,
                      plan.n_mblk.data_ptr(), R, xs.data_ptr(), code, st)
            te, nm = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr()
            if dt == torch.bfloat16:
                _lib.call("fk_moe_gemm_up", xs.data_ptr(), R, d, layer.w13.data_ptr(), H, E, te,
                          nm, h1.data_ptr(), act.data_ptr(), 0, eptr + 4, st)
                _lib.call("fk_moe_gemm_down", act.data_ptr(), R, H, layer.w2.data_ptr(), d, E,
                          te, nm, y.data_ptr(), 0, eptr + 4, st)
            else:
                xs, xs_lo = _operand(xs, st)
                w13, w13_lo = _operand(layer.w13, st)
                _lib.call("fk_moe_gemm_up_typed", xs.data_ptr(), _p(xs_lo), R, d, w13.data_ptr(),
                          _p(w13_lo), H, E, te, nm, h1.data_ptr(), act.data_ptr(), code,
                          eptr + 4, st)
                del w13, w13_lo
                act, act_lo = _operand(act, st)
                w2, w2_lo = _operand(layer.w2, st)
                _lib.call("fk_moe_gemm_down_typed", act.data_ptr(), _p(act_lo), R, H,
                          w2.data_ptr(), _p(w2_lo), d, E, te, nm, y.data_ptr(), code, eptr + 4, st)
        _lib.call("fk_moe_combine", y.data_ptr(), d, plan.slot_pos.data_ptr(), w.data_ptr(), n, k,
                  out.data_ptr(), code, st)
        if layer.check_errors:
            _check_err(plan)
        # fp32: xs / act are the hi parts and xs_lo / act_lo the lo parts
        ctx.save_for_backward(xs, h1, act, y, xs_lo, act_lo)
        return out

    @staticmethod
    def backward(ctx, dout):
        if ctx.weighted:
            return _SortedMoEFn._backward_weighted(ctx, dout)
        xs, h1, act, y, xs_lo, act_lo = ctx.saved_tensors
        plan, layer = ctx.plan, ctx.layer
        n, d, k, E, H = ctx.dims
        R = plan.max_rows
        dev = xs.device
        dt = xs.dtype
        code = _lib.dtype_code(dt)
        st = _lib.stream_of(xs)
        eptr = plan.err.data_ptr()
        dout = dout.to(dt).contiguous()
        td = dict(dtype=dt, device=dev)
        dy = torch.empty(R, d, **td)
        dw = torch.empty(n, k, dtype=torch.float32, device=dev)
        dh1 = torch.empty(R, 2 * H, **td)
        dxs = torch.empty(R, d, **td)
        dw13 = torch.empty(E, 2 * H, d, **td)
        dw2 = torch.empty(E, d, H, **td)
        dx = torch.empty(n, d, **td)
        if R > 0:
            te, nm, seg = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), plan.seg_start.data_ptr()
            _lib.call("fk_moe_combine_bwd", dout.data_ptr(), y.data_ptr(), d,
                      plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(), k,
                      plan.n_mblk.data_ptr(), R, dy.data_ptr(), dw.data_ptr(), code, st)
            if dt == torch.bfloat16:
                _lib.call("fk_moe_gemm_down_dgrad", dy.data_ptr(), R, d, layer.w2.data_ptr(), H, E,
                          te, nm, h1.data_ptr(), dh1.data_ptr(), 0, eptr + 4, st)
                _lib.call("fk_moe_gemm_wgrad", dy.data_ptr(), d, act.data_ptr(), H, R, seg, E,
                          dw2.data_ptr(), 0, eptr + 4, st)
                _lib.call("fk_moe_gemm_up_dgrad", dh1.data_ptr(), R, H, layer.w13.data_ptr(), d,
                          E, te, nm, dxs.data_ptr(), 0, eptr + 4, st)
                _lib.call("fk_moe_gemm_wgrad", dh1.data_ptr(), 2 * H, xs.data_ptr(), d, R, seg, E,
                          dw13.data_ptr(), 0, eptr + 4, st)
            else:
                dy, dy_lo = _operand(dy, st)
                w2, w2_lo = _operand(layer.w2, st)
                _lib.call("fk_moe_gemm_down_dgrad_typed", dy.data_ptr(), _p(dy_lo), R, d,
                          w2.data_ptr(), _p(w2_lo), H, E, te, nm, h1.data_ptr(), dh1.data_ptr(),
                          code, eptr + 4, st)
                del w2, w2_lo
                _lib.call("fk_moe_gemm_wgrad_typed", dy.data_ptr(), _p(dy_lo), d, act.data_ptr(),
                          _p(act_lo), H, R, seg, E, dw2.data_ptr(), code, eptr + 4, st)
                dh1, dh1_lo = _operand(dh1, st)
                w13, w13_lo = _operand(layer.w13, st)
                _lib.call("fk_moe_gemm_up_dgrad_typed", dh1.data_ptr(), _p(dh1_lo), R, H,
                          w13.data_ptr(), _p(w13_lo), d, E, te, nm, dxs.data_ptr(), code,
                          eptr + 4, st)
                del w13, w13_lo
                _lib.call("fk_moe_gemm_wgrad_typed", dh1.data_ptr(), _p(dh1_lo), 2 * H,
                          xs.data_ptr(), _p(xs_lo), d, R, seg, E, dw13.data_ptr(), code,
                          eptr + 4, st)
            _lib.call("fk_moe_combine", dxs.data_ptr(), d, plan.slot_pos.data_ptr(), None, n, k,
                      dx.data_ptr(), code, st)
        else:
            dw.zero_()
            dw13.zero_()
            dw2.zero_()
            dx.zero_()
        if layer.check_errors:
            _check_err(plan)
        grads = []
        for e in range(E):
            grads += [dw13[e, :H], dw13[e, H:], dw2[e]]
        return (dx, dw, None, None, *grads)


    @staticmethod
    def _backward_weighted(ctx, dout):
        """Backward of the row-weighted bf16 path: dout's rows are gathered unweighted; the
        down-projection's input-gradient epilogue applies the routing weight and forms the
        routing-weight gradient partials (fk_moe_dw_from_parts sums them)."""
        xs, h1, act_w = ctx.saved_tensors
        plan, layer = ctx.plan, ctx.layer
        n, d, k, E, H = ctx.dims
        R = plan.max_rows
        dev, dt = xs.device, xs.dtype
        code = _lib.dtype_code(dt)
        st = _lib.stream_of(xs)
        eptr = plan.err.data_ptr()
        dout = dout.to(dt).contiguous()
        td = dict(dtype=dt, device=dev)
        dw = torch.empty(n, k, dtype=torch.float32, device=dev)
        dw13 = torch.empty(E, 2 * H, d, **td)
        dw2 = torch.empty(E, d, H, **td)
        dx = torch.empty(n, d, **td)
        if R > 0:
            te, nm, seg = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), plan.seg_start.data_ptr()
            sa, sw = plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr()
            dy = torch.empty(R, d, **td)
            _lib.call("fk_moe_gather_by_token", dout.data_ptr(), d, plan.slot_pos.data_ptr(), n,
                      k, sa, nm, R, dy.data_ptr(), code, st)
            dh1 = torch.empty(R, 2 * H, **td)
            part = torch.empty(R, H // 64, dtype=torch.float32, device=dev)
            _lib.call("fk_moe_gemm_down_dgrad_weighted", dy.data_ptr(), R, d, layer.w2.data_ptr(),
                      H, E, te, nm, sa, sw, h1.data_ptr(), dh1.data_ptr(), part.data_ptr(), 0,
                      eptr + 4, st)
            _lib.call("fk_moe_dw_from_parts", part.data_ptr(), H, sa, nm, R, dw.data_ptr(), st)
            _lib.call("fk_moe_gemm_wgrad", dy.data_ptr(), d, act_w.data_ptr(), H, R, seg, E,
                      dw2.data_ptr(), 0, eptr + 4, st)
            del dy
            dxs = torch.empty(R, d, **td)
            _lib.call("fk_moe_gemm_up_dgrad", dh1.data_ptr(), R, H, layer.w13.data_ptr(), d, E,
                      te, nm, dxs.data_ptr(), 0, eptr + 4, st)
            _lib.call("fk_moe_gemm_wgrad", dh1.data_ptr(), 2 * H, xs.data_ptr(), d, R, seg, E,
                      dw13.data_ptr(), 0, eptr + 4, st)
            del dh1
            _lib.call("fk_moe_combine", dxs.data_ptr(), d, plan.slot_pos.data_ptr(), None, n, k,
                      dx.data_ptr(), code, st)
        else:
            dw.zero_()
            dw13.zero_()
            dw2.zero_()
            dx.zero_()
        if layer.check_errors:
            _check_err(plan)
        grads = []
        for e in range(E):
            grads += [dw13[e, :H], dw13[e, H:], dw2[e]]
        return (dx, dw, None, None, *grads)


class FusedMoEMLPSorted(nn.Module):
    def __init__(self, dim: int, hidden_dim: int, n_experts: int, k: int = 2,
                 router_version: str = "v2"):
        super().__init__()
        assert router_version in ("v1", "v2")
        self.dim = dim
        self.hidden_dim = hidden_dim
        self.n_experts = n_experts
        self.k = k
        self.router_version = router_version
        self.router = nn.Linear(dim, n_experts, bias=False)
        self.experts = nn.ModuleList([Expert(dim, hidden_dim) for _ in range(n_experts)])
        self.check_errors = False  # True: read the device error flags after each call (syncs)
        self._restack()

    # -- stacked expert storage ------------------------------------------------------
    def _expert_params(self):
        out = []
        for ex in self.experts:
            out += [ex.w_gate.weight, ex.w_up.weight, ex.w_down.weight]
        return out

    def _restack(self):
        """Copy the expert weights into w13 [E, 2H, D] / w2 [E, D, H] and make every
        expert Parameter a view of them (once; after device/dtype moves)."""
        E, H, D = self.n_experts, self.hidden_dim, self.dim
        p0 = self.experts[0].w_gate.weight
        with torch.no_grad():
            w13 = torch.empty(E, 2 * H, D, dtype=p0.dtype, device=p0.device)
            w2 = torch.empty(E, D, H, dtype=p0.dtype, device=p0.device)
            for e, ex in enumerate(self.experts):
                w13[e, :H].copy_(ex.w_gate.weight)
                w13[e, H:].copy_(ex.w_up.weight)
                w2[e].copy_(ex.w_down.weight)
                ex.w_gate.weight.data = w13[e, :H]
                ex.w_up.weight.data = w13[e, H:]
                ex.w_down.weight.data = w2[e]
        self.w13, self.w2 = w13, w2
        self._stack_ptrs = self._current_ptrs()

    def _current_ptrs(self):
        return tuple(p.data_ptr() for p in self._expert_params())

    def _apply(self, fn, *args, **kwargs):
        r = super()._apply(fn, *args, **kwargs)
        self._restack()
        return r

    def _ensure_stacked(self):
        p = self._expert_params()
        H, D = self.hidden_dim, self.dim
        base13, base2 = self.w13.data_ptr(), self.w2.data_ptr()
        es = self.w13.element_size()
        ok = all(p[3 * e].data_ptr() == base13 + (e * 2 * H * D) * es and
                 p[3 * e + 1].data_ptr() == base13 + (e * 2 * H * D + H * D) * es and
                 p[3 * e + 2].data_ptr() == base2 + (e * D * H) * es and
                 p[3 * e].dtype == self.w13.dtype
                 for e in range(self.n_experts))
        if not ok:
            self._restack()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        assert x.is_cuda
        orig_shape = x.shape
        x_flat = x.reshape(-1, self.dim)
        self._ensure_stacked()
        if x_flat.dtype != self.w13.dtype:
            raise TypeError(f"FusedMoEMLPSorted: input dtype {x_flat.dtype} does not match the "
                            f"layer's parameters ({self.w13.dtype})")
        if x_flat.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise TypeError(f"FusedMoEMLPSorted: unsupported dtype {x_flat.dtype}")
        x_flat = x_flat.contiguous()
        router_logits = self.router(x_flat)
        route_fn = fused_moe_route_v2 if self.router_version == "v2" else fused_moe_route
        topk_weights, topk_idx = route_fn(router_logits, self.k)
        out = _SortedMoEFn.apply(x_flat, topk_weights, topk_idx, self, *self._expert_params())
        return out.reshape(orig_shape)
