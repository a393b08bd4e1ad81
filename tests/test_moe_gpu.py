"""MoE sorted-dispatch kernels: routing metadata (bit-exact vs a numpy stable counting
sort), the tcgen05 grouped GEMMs (vs plain PyTorch fp32 on the GPU), and the whole
FusedMoEMLPSorted layer vs the CPU oracle (NaiveMoEMLP restated, fp64).
Tolerances: GEMM outputs (bf16) atol 2e-2 + rtol 2e-2 of the fp32 reference; layer out,
dx, dW atol = rtol = 2e-2 relative to the tensor's max magnitude, with identical routing."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import fusedkernels_b200 as fk
from fusedkernels_b200 import _lib
from fusedkernels_b200.moe_layer_sorted import FusedMoEMLPSorted, _Plan
from oracle import moe_layer_oracle, route_oracle, zipf_expert_bias
from conftest import gen

pytestmark = pytest.mark.gpu
DEV = "cuda"


def meta(idx, w, E):
    n, k = idx.shape
    plan = _Plan(n, k, E, torch.device(DEV))
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("fk_moe_route_meta", idx.data_ptr(), w.data_ptr(), n, k, E,
              plan.counts.data_ptr(), plan.seg_start.data_ptr(), plan.tile_expert.data_ptr(),
              plan.n_mblk.data_ptr(), plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(),
              plan.slot_pos.data_ptr(), plan.max_rows, plan.ws.data_ptr(), plan.ws.numel(),
              plan.err.data_ptr(), st)
    return plan


def meta_reference(idx, E):
    """numpy stable counting sort with 128-row padded segments."""
    idx = idx.reshape(-1)
    counts = np.bincount(idx, minlength=E)
    pad = (counts + 127) // 128 * 128
    seg = np.concatenate([[0], np.cumsum(pad)])
    order = np.argsort(idx, kind="stable")
    sorted_assign = np.full(seg[-1], -1, dtype=np.int64)
    slot_pos = np.zeros(idx.size, dtype=np.int64)
    fill = seg[:-1].copy()
    for a in order:
        e = idx[a]
        sorted_assign[fill[e]] = a
        slot_pos[a] = fill[e]
        fill[e] += 1
    return counts, seg, sorted_assign, slot_pos


def random_routing(n, k, E, seed, skew=0.0):
    G = gen(seed)
    logits = torch.randn(n, E, generator=G) + skew * torch.linspace(3, -3, E)
    w, idx = route_oracle(logits, k)
    return w, idx


@pytest.mark.parametrize("n,k,E,skew", [(1000, 2, 8, 0.0), (4096, 8, 128, 2.0), (5, 2, 64, 0.0),
                                        (32768, 8, 128, 4.0)])
def test_route_meta_matches_stable_counting_sort(n, k, E, skew):
    w, idx = random_routing(n, k, E, n + E, skew)
    plan = meta(idx.to(DEV), w.to(DEV), E)
    counts, seg, sa, sp = meta_reference(idx.numpy(), E)
    assert plan.err[0].item() == 0
    assert np.array_equal(plan.counts.cpu().numpy(), counts)
    assert np.array_equal(plan.seg_start.cpu().numpy(), seg)
    nm = plan.n_mblk.item()
    assert nm * 128 == seg[-1]
    assert np.array_equal(plan.sorted_assign[:seg[-1]].cpu().numpy(), sa)
    assert np.array_equal(plan.slot_pos[:n * k].cpu().numpy(), sp)
    te = plan.tile_expert.cpu().numpy()
    for e in range(E):
        assert (te[seg[e] // 128:seg[e + 1] // 128] == e).all()
    assert (te[nm:] == -1).all()
    sw = plan.sorted_w[:seg[-1]].cpu().numpy()
    wf = w.reshape(-1).numpy()
    valid = sa >= 0
    assert np.array_equal(sw[valid], wf[sa[valid]]) and (sw[~valid] == 0).all()


def make_problem(n, k, E, D, H, seed, skew=0.0):
    w, idx = random_routing(n, k, E, seed, skew)
    G = gen(seed + 1)
    x = (torch.randn(n, D, generator=G)).bfloat16().to(DEV)
    w13 = (torch.randn(E, 2 * H, D, generator=G) * D ** -0.5).bfloat16().to(DEV)
    w2 = (torch.randn(E, D, H, generator=G) * H ** -0.5).bfloat16().to(DEV)
    plan = meta(idx.to(DEV), w.to(DEV), E)
    R = plan.max_rows
    xs = torch.empty(R, D, dtype=torch.bfloat16, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("fk_moe_gather", x.data_ptr(), D, plan.sorted_assign.data_ptr(), k,
              plan.n_mblk.data_ptr(), R, xs.data_ptr(), _lib.FK_BF16, st)
    return dict(n=n, k=k, E=E, D=D, H=H, w=w.to(DEV), idx=idx.to(DEV), x=x, w13=w13, w2=w2,
                plan=plan, xs=xs, st=st)


def expert_of_rows(plan):
    te = plan.tile_expert.cpu()
    rows = plan.n_mblk.item() * 128
    return te.repeat_interleave(128)[:rows].to(DEV), rows


def close(got, ref, tol=2e-2):
    got = got.float()
    ref = ref.float()
    scale = max(ref.abs().max().item(), 1e-6)
    err = (got - ref).abs().max().item()
    assert err <= tol * scale + tol * 0.1, f"max abs err {err:.4g} vs scale {scale:.4g}"


SHAPES = [(512, 2, 8, 256, 128), (300, 4, 16, 64, 64), (2048, 4, 16, 1024, 512),
          (64, 8, 128, 128, 256)]


@pytest.mark.parametrize("n,k,E,D,H", SHAPES)
def test_gather_and_gemm_up_down(n, k, E, D, H):
    P = make_problem(n, k, E, D, H, seed=n + D)
    plan, R = P["plan"], P["plan"].max_rows
    xs = P["xs"]
    eor, rows = expert_of_rows(plan)
    sa = plan.sorted_assign[:rows].long()
    ref_xs = torch.where((sa >= 0)[:, None], P["x"][sa.clamp(min=0) // k], 0)
    assert torch.equal(xs[:rows], ref_xs)
    h1 = torch.empty(R, 2 * H, dtype=torch.bfloat16, device=DEV)
    act = torch.empty(R, H, dtype=torch.bfloat16, device=DEV)
    y = torch.empty(R, D, dtype=torch.bfloat16, device=DEV)
    eptr = plan.err.data_ptr() + 4
    _lib.call("fk_moe_gemm_up", xs.data_ptr(), R, D, P["w13"].data_ptr(), H, E,
              plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), h1.data_ptr(), act.data_ptr(),
              0, eptr, P["st"])
    _lib.call("fk_moe_gemm_down", act.data_ptr(), R, H, P["w2"].data_ptr(), D, E,
              plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), y.data_ptr(), 0, eptr,
              P["st"])
    torch.cuda.synchronize()
    assert plan.err[1].item() == 0
    xf = xs[:rows].float()
    ref_h1 = torch.einsum("rd,rjd->rj", xf, P["w13"].float()[eor])
    close(h1[:rows], ref_h1)
    g, u = ref_h1[:, :H], ref_h1[:, H:]
    ref_act = F.silu(g) * u
    close(act[:rows], ref_act)
    ref_y = torch.einsum("rh,rdh->rd", act[:rows].float(), P["w2"].float()[eor])
    close(y[:rows], ref_y)


@pytest.mark.parametrize("n,k,E,D,H", SHAPES)
def test_gemm_backward_pieces(n, k, E, D, H):
    P = make_problem(n, k, E, D, H, seed=2 * n + D)
    plan, R = P["plan"], P["plan"].max_rows
    eor, rows = expert_of_rows(plan)
    G = gen(99)
    sa = plan.sorted_assign[:rows]
    valid = (sa >= 0)[:, None]
    dy = torch.where(valid, torch.randn(rows, D, generator=G).bfloat16().to(DEV), 0)
    h1 = torch.where(valid, torch.randn(rows, 2 * H, generator=G).bfloat16().to(DEV), 0)
    dyb = torch.zeros(R, D, dtype=torch.bfloat16, device=DEV)
    dyb[:rows] = dy
    h1b = torch.zeros(R, 2 * H, dtype=torch.bfloat16, device=DEV)
    h1b[:rows] = h1
    dh1 = torch.empty(R, 2 * H, dtype=torch.bfloat16, device=DEV)
    dxs = torch.empty(R, D, dtype=torch.bfloat16, device=DEV)
    dw2 = torch.empty(E, D, H, dtype=torch.bfloat16, device=DEV)
    dw13 = torch.empty(E, 2 * H, D, dtype=torch.bfloat16, device=DEV)
    act = torch.where(valid, torch.randn(rows, H, generator=G).bfloat16().to(DEV), 0)
    actb = torch.zeros(R, H, dtype=torch.bfloat16, device=DEV)
    actb[:rows] = act
    eptr = plan.err.data_ptr() + 4
    st = P["st"]
    _lib.call("fk_moe_gemm_down_dgrad", dyb.data_ptr(), R, D, P["w2"].data_ptr(), H, E,
              plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), h1b.data_ptr(), dh1.data_ptr(),
              0, eptr, st)
    _lib.call("fk_moe_gemm_up_dgrad", dh1.data_ptr(), R, H, P["w13"].data_ptr(), D, E,
              plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), dxs.data_ptr(), 0, eptr, st)
    _lib.call("fk_moe_gemm_wgrad", dyb.data_ptr(), D, actb.data_ptr(), H, R,
              plan.seg_start.data_ptr(), E, dw2.data_ptr(), 0, eptr, st)
    _lib.call("fk_moe_gemm_wgrad", dh1.data_ptr(), 2 * H, P["xs"].data_ptr(), D, R,
              plan.seg_start.data_ptr(), E, dw13.data_ptr(), 0, eptr, st)
    torch.cuda.synchronize()
    assert plan.err[1].item() == 0
    dact = torch.einsum("rd,rdh->rh", dy.float(), P["w2"].float()[eor])
    g, u = h1[:, :H].float(), h1[:, H:].float()
    s = torch.sigmoid(g)
    ref_dh1 = torch.cat([dact * u * s * (1 + g * (1 - s)), dact * g * s], dim=1)
    close(dh1[:rows], ref_dh1)
    ref_dxs = torch.einsum("rj,rjd->rd", dh1[:rows].float(), P["w13"].float()[eor])
    close(dxs[:rows], ref_dxs)
    seg = plan.seg_start.cpu().tolist()
    for e in range(E):
        a, b = seg[e], seg[e + 1]
        ref2 = dy[a:b].float().t() @ act[a:b].float()
        ref13 = dh1[a:b].float().t() @ P["xs"][a:b].float()
        if b == a:
            assert torch.count_nonzero(dw2[e]) == 0 and torch.count_nonzero(dw13[e]) == 0
        else:
            close(dw2[e], ref2)
            close(dw13[e], ref13)


@pytest.mark.parametrize("n,k,E,D,H", SHAPES)
def test_gather_by_token_equals_row_gather(n, k, E, D, H):
    """The token-order gather writes the same sorted rows as the row-order gather, bit for
    bit (padding rows zero), and leaves the rows past the last valid block alone."""
    P = make_problem(n, k, E, D, H, seed=11 * n + D)
    plan, R, st = P["plan"], P["plan"].max_rows, P["st"]
    rows = plan.n_mblk.item() * 128
    xs = torch.full((R, D), float("nan"), dtype=torch.bfloat16, device=DEV)
    _lib.call("fk_moe_gather_by_token", P["x"].data_ptr(), D, plan.slot_pos.data_ptr(), n, k,
              plan.sorted_assign.data_ptr(), plan.n_mblk.data_ptr(), R, xs.data_ptr(),
              _lib.FK_BF16, st)
    torch.cuda.synchronize()
    assert torch.equal(xs[:rows], P["xs"][:rows])
    assert torch.isnan(xs[rows:].float()).all()


@pytest.mark.parametrize("n,k,E,D,H", SHAPES)
def test_row_weighted_epilogues(n, k, E, D, H):
    """The row-weighted GEMM variants against the plain ones and PyTorch fp32: h1
    bit-identical (same operands), act_w = w * act, zero padding rows; the weighted
    input-gradient GEMM on unweighted dout rows gives SwiGLU'(w * dy @ w2) and the
    routing-weight gradient <dout[token], y_row> through fk_moe_dw_from_parts."""
    P = make_problem(n, k, E, D, H, seed=3 * n + D)
    plan, R, st = P["plan"], P["plan"].max_rows, P["st"]
    te, nm = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr()
    sa, sw = plan.sorted_assign, plan.sorted_w
    eptr = plan.err.data_ptr() + 4
    eor, rows = expert_of_rows(plan)
    bf = dict(dtype=torch.bfloat16, device=DEV)
    h1, act = torch.empty(R, 2 * H, **bf), torch.empty(R, H, **bf)
    _lib.call("fk_moe_gemm_up", P["xs"].data_ptr(), R, D, P["w13"].data_ptr(), H, E, te, nm,
              h1.data_ptr(), act.data_ptr(), 0, eptr, st)
    h1w, actw = torch.full((R, 2 * H), 7.0, **bf), torch.full((R, H), 7.0, **bf)
    _lib.call("fk_moe_gemm_up_weighted", P["xs"].data_ptr(), R, D, P["w13"].data_ptr(), H, E, te,
              nm, sa.data_ptr(), sw.data_ptr(), h1w.data_ptr(), actw.data_ptr(), 0, eptr, st)
    torch.cuda.synchronize()
    assert plan.err[1].item() == 0
    valid = (sa[:rows] >= 0)
    assert torch.equal(h1w[:rows], h1[:rows])
    wrow = torch.where(valid, sw[:rows], 0.0)[:, None]
    close(actw[:rows], act[:rows].float() * wrow)
    assert torch.count_nonzero(actw[:rows][~valid]) == 0

    G = gen(11)
    dout = torch.randn(n, D, generator=G).bfloat16().to(DEV)
    dy = torch.empty(R, D, **bf)
    _lib.call("fk_moe_gather", dout.data_ptr(), D, sa.data_ptr(), k, nm, R, dy.data_ptr(),
              _lib.FK_BF16, st)
    dh1 = torch.full((R, 2 * H), 7.0, **bf)
    part = torch.full((R, H // 64), 7.0, dtype=torch.float32, device=DEV)
    _lib.call("fk_moe_gemm_down_dgrad_weighted", dy.data_ptr(), R, D, P["w2"].data_ptr(), H, E,
              te, nm, sa.data_ptr(), sw.data_ptr(), h1w.data_ptr(), dh1.data_ptr(),
              part.data_ptr(), 0, eptr, st)
    dw = torch.full((n * k,), 7.0, dtype=torch.float32, device=DEV)
    _lib.call("fk_moe_dw_from_parts", part.data_ptr(), H, sa.data_ptr(), nm, R, dw.data_ptr(), st)
    torch.cuda.synchronize()
    assert plan.err[1].item() == 0
    tok = torch.where(valid, sa[:rows] // k, 0).long()
    g, u = h1w[:rows, :H].float(), h1w[:rows, H:].float()
    dsum = torch.einsum("rd,rdh->rh", dout[tok].float(), P["w2"].float()[eor])
    dact = dsum * wrow
    sg = torch.sigmoid(g)
    ref_dh1 = torch.cat([dact * u * sg * (1 + g * (1 - sg)), dact * g * sg], dim=1)
    close(dh1[:rows], torch.where(valid[:, None], ref_dh1, 0.0))
    assert torch.count_nonzero(dh1[:rows][~valid]) == 0
    ref_dw_rows = (dsum * (F.silu(g) * u)).sum(1)
    ref_dw = torch.zeros(n * k, device=DEV)
    ref_dw[sa[:rows][valid].long()] = ref_dw_rows[valid]
    close(dw, ref_dw)
    with pytest.raises(RuntimeError):
        _lib.call("fk_moe_gemm_up_weighted", P["xs"].data_ptr(), R, D, P["w13"].data_ptr(), H, E,
                  te, nm, None, sw.data_ptr(), h1w.data_ptr(), actw.data_ptr(), 0, eptr, st)


@pytest.mark.parametrize("n,k,E,skew", [(700, 2, 4, 2.0), (96, 4, 8, 0.0)])
def test_wgrad_256_row_tiles(n, k, E, skew):
    """Weight gradients whose experts have more 128 x 256 tiles than the GPU has SMs
    (dW13 at dim 4096, hidden 1024: 256 tiles) run 256-row tiles (two TMEM accumulators per
    CTA); they match PyTorch fp32 per expert, including experts with no tokens."""
    D, H = 4096, 1024
    P = make_problem(n, k, E, D, H, seed=17 + n, skew=skew)
    plan, R, st = P["plan"], P["plan"].max_rows, P["st"]
    seg = plan.seg_start
    eptr = plan.err.data_ptr() + 4
    G = gen(3)
    rows = plan.n_mblk.item() * 128
    valid = (plan.sorted_assign[:rows] >= 0)[:, None]
    dh1 = torch.zeros(R, 2 * H, dtype=torch.bfloat16, device=DEV)
    dh1[:rows] = torch.where(valid, torch.randn(rows, 2 * H, generator=G).bfloat16().to(DEV), 0)
    dw13 = torch.empty(E, 2 * H, D, dtype=torch.bfloat16, device=DEV)
    _lib.call("fk_moe_gemm_wgrad", dh1.data_ptr(), 2 * H, P["xs"].data_ptr(), D, R,
              seg.data_ptr(), E, dw13.data_ptr(), 0, eptr, st)
    torch.cuda.synchronize()
    assert plan.err[1].item() == 0
    segs = seg.cpu().tolist()
    for e in range(E):
        a, b = segs[e], segs[e + 1]
        if b == a:
            assert torch.count_nonzero(dw13[e]) == 0
        else:
            close(dw13[e], dh1[a:b].float().t() @ P["xs"][a:b].float())


@pytest.mark.parametrize("cap", [1, 7, 100])
def test_gemm_grid_cap_is_bitwise_neutral(cap):
    """max_ctas only changes which CTA computes a tile, never the tile's arithmetic: every
    GEMM gives the same bits with the grid capped (the expert-parallel backward caps it to
    leave SMs to a concurrent all-reduce)."""
    n, k, E, D, H = 2048, 4, 16, 1024, 512
    P = make_problem(n, k, E, D, H, seed=5)
    plan, R = P["plan"], P["plan"].max_rows
    te, nm, seg = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), plan.seg_start.data_ptr()
    eptr = plan.err.data_ptr() + 4
    st = P["st"]
    bf = dict(dtype=torch.bfloat16, device=DEV)
    G = gen(7)
    dy = (torch.randn(R, D, generator=G) * 0.5).bfloat16().to(DEV)

    def run(c):
        h1 = torch.empty(R, 2 * H, **bf)
        act = torch.empty(R, H, **bf)
        y = torch.empty(R, D, **bf)
        dh1 = torch.empty(R, 2 * H, **bf)
        dxs = torch.empty(R, D, **bf)
        dw2 = torch.empty(E, D, H, **bf)
        dw13 = torch.empty(E, 2 * H, D, **bf)
        _lib.call("fk_moe_gemm_up", P["xs"].data_ptr(), R, D, P["w13"].data_ptr(), H, E, te, nm,
                  h1.data_ptr(), act.data_ptr(), c, eptr, st)
        _lib.call("fk_moe_gemm_down", act.data_ptr(), R, H, P["w2"].data_ptr(), D, E, te, nm,
                  y.data_ptr(), c, eptr, st)
        _lib.call("fk_moe_gemm_down_dgrad", dy.data_ptr(), R, D, P["w2"].data_ptr(), H, E, te, nm,
                  h1.data_ptr(), dh1.data_ptr(), c, eptr, st)
        _lib.call("fk_moe_gemm_up_dgrad", dh1.data_ptr(), R, H, P["w13"].data_ptr(), D, E, te,
                  nm, dxs.data_ptr(), c, eptr, st)
        _lib.call("fk_moe_gemm_wgrad", dy.data_ptr(), D, act.data_ptr(), H, R, seg, E,
                  dw2.data_ptr(), c, eptr, st)
        _lib.call("fk_moe_gemm_wgrad", dh1.data_ptr(), 2 * H, P["xs"].data_ptr(), D, R, seg, E,
                  dw13.data_ptr(), c, eptr, st)
        torch.cuda.synchronize()
        assert plan.err[1].item() == 0
        rows = plan.n_mblk.item() * 128
        return [t[:rows] for t in (h1, act, y, dh1, dxs)] + [dw2, dw13]

    for a, b in zip(run(0), run(cap)):
        assert torch.equal(a, b)
    with pytest.raises(RuntimeError):
        _lib.call("fk_moe_gemm_down", P["xs"].data_ptr(), R, H, P["w2"].data_ptr(), D, E, te,
                  nm, P["xs"].data_ptr(), -1, eptr, st)


def run_layer(layer, x, dout, bias=None):
    logits_box = {}

    def hook(mod, inp, out):
        if bias is not None:
            out = out + bias.to(out.dtype)
        logits_box["l"] = out.detach()
        return out

    h = layer.router.register_forward_hook(hook)
    xg = x.clone().requires_grad_(True)
    out = layer(xg)
    out.backward(dout)
    h.remove()
    return out.detach(), xg.grad, logits_box["l"]


def stacked_grads(layer):
    E = layer.n_experts
    g13 = torch.stack([torch.cat([ex.w_gate.weight.grad, ex.w_up.weight.grad]) for ex in layer.experts])
    g2 = torch.stack([ex.w_down.weight.grad for ex in layer.experts])
    return g13, g2


@pytest.mark.parametrize("E,k", [(8, 2), (32, 4), (64, 8), (128, 16)])
def test_layer_matches_oracle(E, k):
    """tests/test_moe_sorted_dispatch.py:43-69 shapes (B=2, T=128, D=256, H=512), bf16."""
    torch.manual_seed(0)
    D, H = 256, 512
    layer = FusedMoEMLPSorted(D, H, E, k).to(DEV).bfloat16()
    G = gen(E)
    x = torch.randn(2, 128, D, generator=G).bfloat16().to(DEV)
    dout = torch.randn(2, 128, D, generator=G).bfloat16().to(DEV)
    out, dx, logits = run_layer(layer, x, dout)
    H_ = H
    w13 = layer.w13.float().cpu()
    ro, rdx, rdwg, rdwu, rdwd, rdl = moe_layer_oracle(
        x.reshape(-1, D).cpu(), logits.cpu(), w13[:, :H_], w13[:, H_:], layer.w2.float().cpu(), k,
        dout.reshape(-1, D).cpu())
    close(out.reshape(-1, D).cpu(), ro)
    # dx: expert path + router path (logits = x @ Wr^T)
    rdx_total = rdx + rdl @ layer.router.weight.double().cpu()
    close(dx.reshape(-1, D).cpu(), rdx_total)
    g13, g2 = stacked_grads(layer)
    close(g13.cpu(), torch.cat([rdwg, rdwu], dim=1))
    close(g2.cpu(), rdwd)
    rdwr = rdl.t() @ x.reshape(-1, D).double().cpu()
    close(layer.router.weight.grad.cpu(), rdwr)


def test_layer_handles_empty_experts():
    """tests/test_moe_sorted_dispatch.py:72-82: 4 tokens, 64 experts."""
    torch.manual_seed(1)
    layer = FusedMoEMLPSorted(64, 128, 64, 2).to(DEV).bfloat16()
    x = torch.randn(1, 4, 64, device=DEV).bfloat16().requires_grad_(True)
    out = layer(x)
    assert out.shape == x.shape
    out.float().sum().backward()
    assert x.grad is not None
    g13, g2 = stacked_grads(layer)
    used = set()
    with torch.no_grad():
        _, idx = route_oracle(layer.router(x.detach().reshape(-1, 64)).float().cpu(), 2)
    used = set(idx.reshape(-1).tolist())
    for e in range(64):
        if e not in used:
            assert torch.count_nonzero(g13[e]) == 0 and torch.count_nonzero(g2[e]) == 0


def test_layer_deterministic():
    torch.manual_seed(2)
    layer = FusedMoEMLPSorted(256, 256, 32, 4).to(DEV).bfloat16()
    x = torch.randn(1024, 256, device=DEV).bfloat16()
    dout = torch.randn(1024, 256, device=DEV).bfloat16()
    res = []
    for _ in range(3):
        layer.zero_grad(set_to_none=True)
        out, dx, _ = run_layer(layer, x, dout)
        g13, g2 = stacked_grads(layer)
        res.append((out, dx, g13, g2, layer.router.weight.grad.clone()))
    for r in res[1:]:
        assert all(torch.equal(a, b) for a, b in zip(r, res[0]))


def test_layer_state_dict_keys_and_error_flags():
    layer = FusedMoEMLPSorted(128, 128, 8, 2).to(DEV).bfloat16()
    keys = list(layer.state_dict().keys())
    assert keys[0] == "router.weight" and "experts.7.w_down.weight" in keys and len(keys) == 25
    layer.check_errors = True
    x = torch.randn(64, 128, device=DEV).bfloat16().requires_grad_(True)
    layer(x).float().sum().backward()


def _token_reference(layer, x_t, dout_t, w, idx, H):
    """fp64 forward output and input gradient of one token (expert and router paths)."""
    ref = torch.zeros_like(x_t)
    dx = torch.zeros_like(x_t)
    ys, dacts = [], []
    for j in range(idx.numel()):
        e = int(idx[j])
        h = layer.w13[e].double() @ x_t
        g, u = h[:H], h[H:]
        a = F.silu(g) * u
        y = layer.w2[e].double() @ a
        ys.append(y)
        ref += float(w[j]) * y
        dact = float(w[j]) * (layer.w2[e].double().t() @ dout_t)
        s = torch.sigmoid(g)
        dg = dact * u * s * (1 + g * (1 - s))
        du = dact * g * s
        dx += layer.w13[e, :H].double().t() @ dg + layer.w13[e, H:].double().t() @ du
    # router path: d out / d w_j = dout . y_j; renormalised-softmax Jacobian at the selection
    dw = torch.stack([dout_t @ y for y in ys])
    wd = w.double().to(dout_t.device)
    dl = wd * (dw - (wd * dw).sum())
    dx += (dl[:, None] * layer.router.weight.double()[idx.to(dout_t.device)]).sum(0)
    return ref, dx


@pytest.mark.slow
def test_layer_workload_shape_sampled_tokens_and_expert_gradients():
    """x [32768, 4096] bf16, E=128, k=8, H=1024, Zipf(1.1) expert bias on the logits.
    Forward outputs and input gradients of 16 sampled tokens against a per-token fp64
    evaluation, and the weight gradients of the hottest expert (a ~30 K-token segment:
    the long-K weight-gradient path of the timed step) and of two cold experts against fp32
    matmuls over their token segments (bf16 inputs; 2e-2 of the tensor's max magnitude)."""
    torch.manual_seed(3)
    N, D, H, E, k = 32768, 4096, 1024, 128, 8
    layer = FusedMoEMLPSorted(D, H, E, k)
    with torch.no_grad():
        layer.router.weight.normal_(0, 0.02)
        for ex in layer.experts:
            for lin in (ex.w_gate, ex.w_up, ex.w_down):
                lin.weight.normal_(0, 0.02)
    layer = layer.to(DEV).bfloat16()
    G = gen(4)
    x = torch.randn(N, D, generator=G).bfloat16().to(DEV)
    dout = torch.randn(N, D, generator=G).bfloat16().to(DEV)
    bias = zipf_expert_bias(E).to(DEV)
    out, dx, logits = run_layer(layer, x, dout, bias=bias)
    w_all, idx_all = route_oracle(logits.float().cpu(), k)
    toks = torch.randint(0, N, (16,), generator=G)
    for t in toks.tolist():
        ref, rdx = _token_reference(layer, x[t].double(), dout[t].double(), w_all[t], idx_all[t], H)
        close(out[t], ref)
        close(dx[t], rdx)
    g13, g2 = stacked_grads(layer)
    load = torch.bincount(idx_all.reshape(-1), minlength=E)
    order = torch.argsort(load, descending=True, stable=True).tolist()
    hot = order[0]
    cold = [e for e in order[::-1] if load[e] > 0][:2]
    assert load[hot] > 20000, f"hottest expert has only {int(load[hot])} tokens"
    for e in [hot] + cold:
        sel = (idx_all == e)
        tok = sel.any(dim=1).nonzero()[:, 0]
        we = (w_all * sel).sum(dim=1)[tok].to(DEV)
        tok = tok.to(DEV)
        xe = x[tok].float()
        h = xe @ layer.w13[e].float().t()
        hb = h.bfloat16().float()  # the kernels keep h1 in bf16
        g, u = hb[:, :H], hb[:, H:]
        a = (F.silu(g) * u).bfloat16().float()
        dy = (dout[tok].float() * we[:, None]).bfloat16().float()
        close(g2[e], dy.t() @ a)
        dact = dy @ layer.w2[e].float()
        s = torch.sigmoid(g)
        dh1 = torch.cat([dact * u * s * (1 + g * (1 - s)), dact * g * s], dim=1).bfloat16().float()
        close(g13[e], dh1.t() @ xe)


def test_masked_dispatch_layer_api():
    """tests/test_moe_correctness.py:50-65: FusedMoEMLP(dim=256, hidden_dim=512,
    n_experts=8, k=2, router_version="v1") on x [2, 64, 256]: output shape, input and
    router gradients present, and values against the oracle (2e-2 of max magnitude)."""
    from fusedkernels_b200.moe_layer import FusedMoEMLP
    torch.manual_seed(2)
    B, T, D, H = 2, 64, 256, 512
    moe = FusedMoEMLP(dim=D, hidden_dim=H, n_experts=8, k=2, router_version="v1").to(DEV).bfloat16()
    x = torch.randn(B, T, D, generator=gen(5)).bfloat16().to(DEV)
    dout = torch.randn(B, T, D, generator=gen(6)).bfloat16().to(DEV)
    out, dx, logits = run_layer(moe, x, dout)
    assert out.shape == x.shape and dx.shape == x.shape
    assert moe.router.weight.grad is not None
    w13 = moe.w13.float().cpu()
    ro, rdx, _, _, _, rdl = moe_layer_oracle(x.reshape(-1, D).cpu(), logits.cpu(), w13[:, :H],
                                             w13[:, H:], moe.w2.float().cpu(), 2,
                                             dout.reshape(-1, D).cpu())
    close(out.reshape(-1, D).cpu(), ro)
    close(dx.reshape(-1, D).cpu(), rdx + rdl @ moe.router.weight.double().cpu())


# ----------------------------------------------------------------- fp16 / fp32 layers ---
def _typed_operand(t, st):
    if t.dtype != torch.float32:
        return t, None
    hi, lo = torch.empty_like(t), torch.empty_like(t)
    _lib.call("fk_tf32_split", t.data_ptr(), t.numel(), hi.data_ptr(), lo.data_ptr(), st)
    return hi, lo


def _pp(t):
    return None if t is None else t.data_ptr()


def test_tf32_split_is_exact():
    """hi has the 13 low mantissa bits cleared and hi + lo == x exactly (odd length: tail)."""
    x = torch.randn(1001, generator=gen(8)).to(DEV) * 1e3
    x[0], x[1], x[2] = 0.0, -0.0, 1e-40  # zeros and a denormal
    hi, lo = torch.empty_like(x), torch.empty_like(x)
    _lib.call("fk_tf32_split", x.data_ptr(), x.numel(), hi.data_ptr(), lo.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    assert torch.equal(hi + lo, x)
    assert (hi.view(torch.int32) & 0x1FFF).eq(0).all()
    normal = x.abs() >= torch.finfo(torch.float32).tiny
    assert (lo.abs() <= x.abs() * 2 ** -10)[normal].all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("n,k,E,D,H", [(512, 2, 8, 256, 128), (300, 4, 16, 64, 64),
                                       (64, 8, 128, 128, 256)])
def test_typed_gemms_match_fp64(dtype, n, k, E, D, H):
    """All five grouped GEMMs of the fp16 and fp32 (3xTF32) layers against fp64 matmuls of
    the same operands: fp32 within 1e-5 of the max magnitude, fp16 within 2e-2."""
    code = _lib.dtype_code(dtype)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    w, idx = random_routing(n, k, E, n + 3 * D, 0.5)
    G = gen(n + D)
    x = torch.randn(n, D, generator=G).to(dtype).to(DEV)
    w13 = (torch.randn(E, 2 * H, D, generator=G) * D ** -0.5).to(dtype).to(DEV)
    w2 = (torch.randn(E, D, H, generator=G) * H ** -0.5).to(dtype).to(DEV)
    plan = meta(idx.to(DEV), w.to(DEV), E)
    R = plan.max_rows
    st = torch.cuda.current_stream().cuda_stream
    te, nm, seg = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), plan.seg_start.data_ptr()
    eptr = plan.err.data_ptr() + 4
    xs = torch.empty(R, D, dtype=dtype, device=DEV)
    _lib.call("fk_moe_gather", x.data_ptr(), D, plan.sorted_assign.data_ptr(), k,
              plan.n_mblk.data_ptr(), R, xs.data_ptr(), code, st)
    eor, rows = expert_of_rows(plan)
    td = dict(dtype=dtype, device=DEV)
    h1, act, y = torch.empty(R, 2 * H, **td), torch.empty(R, H, **td), torch.empty(R, D, **td)
    xa, w13p, w2p = _typed_operand(xs, st), _typed_operand(w13, st), _typed_operand(w2, st)
    _lib.call("fk_moe_gemm_up_typed", xa[0].data_ptr(), _pp(xa[1]), R, D, w13p[0].data_ptr(),
              _pp(w13p[1]), H, E, te, nm, h1.data_ptr(), act.data_ptr(), code, eptr, st)
    aa = _typed_operand(act, st)
    _lib.call("fk_moe_gemm_down_typed", aa[0].data_ptr(), _pp(aa[1]), R, H, w2p[0].data_ptr(),
              _pp(w2p[1]), D, E, te, nm, y.data_ptr(), code, eptr, st)
    sa = plan.sorted_assign[:rows]
    valid = (sa >= 0)[:, None]
    dy = torch.where(valid, torch.randn(rows, D, generator=G).to(dtype).to(DEV), 0)
    dyb = torch.zeros(R, D, **td)
    dyb[:rows] = dy
    dh1, dxs = torch.empty(R, 2 * H, **td), torch.empty(R, D, **td)
    dw2, dw13 = torch.empty(E, D, H, **td), torch.empty(E, 2 * H, D, **td)
    da = _typed_operand(dyb, st)
    _lib.call("fk_moe_gemm_down_dgrad_typed", da[0].data_ptr(), _pp(da[1]), R, D,
              w2p[0].data_ptr(), _pp(w2p[1]), H, E, te, nm, h1.data_ptr(), dh1.data_ptr(), code,
              eptr, st)
    _lib.call("fk_moe_gemm_wgrad_typed", da[0].data_ptr(), _pp(da[1]), D, aa[0].data_ptr(),
              _pp(aa[1]), H, R, seg, E, dw2.data_ptr(), code, eptr, st)
    ha = _typed_operand(dh1, st)
    _lib.call("fk_moe_gemm_up_dgrad_typed", ha[0].data_ptr(), _pp(ha[1]), R, H,
              w13p[0].data_ptr(), _pp(w13p[1]), D, E, te, nm, dxs.data_ptr(), code, eptr, st)
    _lib.call("fk_moe_gemm_wgrad_typed", ha[0].data_ptr(), _pp(ha[1]), 2 * H, xa[0].data_ptr(),
              _pp(xa[1]), D, R, seg, E, dw13.data_ptr(), code, eptr, st)
    torch.cuda.synchronize()
    assert plan.err[1].item() == 0
    X = xs[:rows].double() if dtype != torch.float32 else (xa[0] + xa[1])[:rows].double()
    ref_h1 = torch.einsum("rd,rjd->rj", X, w13.double()[eor])
    close(h1[:rows], ref_h1, tol)
    g, u = ref_h1[:, :H], ref_h1[:, H:]
    close(act[:rows], F.silu(g) * u, tol)
    A = act[:rows].double() if dtype != torch.float32 else (aa[0] + aa[1])[:rows].double()
    close(y[:rows], torch.einsum("rh,rdh->rd", A, w2.double()[eor]), tol)
    H1 = h1[:rows].double()
    dact = torch.einsum("rd,rdh->rh", dy.double(), w2.double()[eor])
    g, u = H1[:, :H], H1[:, H:]
    s = torch.sigmoid(g)
    ref_dh1 = torch.cat([dact * u * s * (1 + g * (1 - s)), dact * g * s], dim=1)
    close(dh1[:rows], ref_dh1, tol)
    DH1 = dh1[:rows].double() if dtype != torch.float32 else (ha[0] + ha[1])[:rows].double()
    close(dxs[:rows], torch.einsum("rj,rjd->rd", DH1, w13.double()[eor]), tol)
    segl = plan.seg_start.cpu().tolist()
    for e in range(E):
        a, b = segl[e], segl[e + 1]
        if b == a:
            assert torch.count_nonzero(dw2[e]) == 0 and torch.count_nonzero(dw13[e]) == 0
            continue
        close(dw2[e], dy[a:b].double().t() @ A[a:b], tol)
        close(dw13[e], DH1[a:b].t() @ X[a:b], tol)


def _naive_check(layer, x, k, tol, dout):
    """Layer output, input gradient and router gradient against the fp64 oracle at the
    reference's tolerance form: |got - ref| <= atol + rtol * |ref| elementwise."""
    out, dx, logits = run_layer(layer, x, dout)
    D, H = layer.dim, layer.hidden_dim
    w13 = layer.w13.double().cpu()
    ro, rdx, rdwg, rdwu, rdwd, rdl = moe_layer_oracle(
        x.reshape(-1, D).cpu(), logits.cpu(), w13[:, :H], w13[:, H:], layer.w2.double().cpu(), k,
        dout.reshape(-1, D).cpu())
    wr = layer.router.weight.double().cpu()
    X = x.reshape(-1, D).double().cpu()
    torch.testing.assert_close(out.reshape(-1, D).double().cpu(), ro, atol=tol, rtol=tol)
    torch.testing.assert_close(dx.reshape(-1, D).double().cpu(), rdx + rdl @ wr, atol=tol, rtol=tol)
    torch.testing.assert_close(layer.router.weight.grad.double().cpu(), rdl.t() @ X, atol=tol, rtol=tol)
    g13, g2 = stacked_grads(layer)
    torch.testing.assert_close(g13.double().cpu(), torch.cat([rdwg, rdwu], dim=1), atol=tol, rtol=tol)
    torch.testing.assert_close(g2.double().cpu(), rdwd, atol=tol, rtol=tol)


@pytest.mark.parametrize("E,k", [(8, 2), (32, 4), (64, 8), (128, 16)])
def test_layer_fp32_reference_test_shapes(E, k):
    """tests/test_moe_sorted_dispatch.py:43-69 as the reference runs it: an fp32 layer with
    default nn.Linear init, x [2, 128, 256], H=512, router v2; out, x.grad and the router
    weight gradient within atol = rtol = 1e-3 (the reference test's tolerance), and the
    expert weight gradients too."""
    torch.manual_seed(0)
    B, T, D, H = 2, 128, 256, 512
    layer = FusedMoEMLPSorted(D, H, E, k, router_version="v2").cuda()
    x = torch.randn(B, T, D, device=DEV)
    dout = torch.randn(B, T, D, device=DEV)
    _naive_check(layer, x, k, 1e-3, dout)


def test_layer_fp32_matches_reference_golden(golden_moe):
    """The reference's NaiveMoEMLP outputs (fp64 on the CPU, tests/golden/make_moe_golden.py)
    for 64 tokens, D = H = 64, E = 8, k = 2, against the fp32 layer on the GPU: out, dx,
    router and expert weight gradients within atol 1e-4, rtol 1e-3."""
    g = {kk[len("moe_e8k2_"):]: torch.from_numpy(v) for kk, v in golden_moe.items()
         if kk.startswith("moe_e8k2_")}
    E, k = g["wg"].shape[0], int(g["k"])
    H, D = g["wg"].shape[1], g["wg"].shape[2]
    layer = FusedMoEMLPSorted(D, H, E, k).cuda()
    with torch.no_grad():
        layer.router.weight.copy_(g["wr"])
        for e, ex in enumerate(layer.experts):
            ex.w_gate.weight.copy_(g["wg"][e])
            ex.w_up.weight.copy_(g["wu"][e])
            ex.w_down.weight.copy_(g["wd"][e])
    x = g["x"].to(DEV).requires_grad_(True)
    out = layer(x)
    out.backward(g["dout"].to(DEV))
    tol = dict(atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(out.detach().cpu(), g["out"], **tol)
    torch.testing.assert_close(x.grad.cpu(), g["dx"], **tol)
    torch.testing.assert_close(layer.router.weight.grad.cpu(), g["dwr"], **tol)
    g13, g2 = stacked_grads(layer)
    torch.testing.assert_close(g13.cpu(), torch.cat([g["dwg"], g["dwu"]], dim=1), **tol)
    torch.testing.assert_close(g2.cpu(), g["dwd"], **tol)


def test_masked_dispatch_layer_fp32_reference_test():
    """tests/test_moe_correctness.py:50-65 exactly: FusedMoEMLP(dim=256, hidden_dim=512,
    n_experts=8, k=2, router_version="v1") in fp32, x [2, 64, 256]; plus values against
    the oracle at 1e-3."""
    from fusedkernels_b200.moe_layer import FusedMoEMLP
    torch.manual_seed(2)
    B, T, D = 2, 64, 256
    moe = FusedMoEMLP(dim=D, hidden_dim=512, n_experts=8, k=2, router_version="v1").cuda()
    x = torch.randn(B, T, D, device=DEV, requires_grad=True)
    out = moe(x)
    assert out.shape == x.shape
    out.sum().backward()
    assert x.grad is not None and x.grad.shape == x.shape
    assert moe.router.weight.grad is not None
    moe.zero_grad(set_to_none=True)
    _naive_check(moe, x.detach(), 2, 1e-3, torch.randn(B, T, D, device=DEV))


def test_layer_fp16_matches_oracle():
    """An fp16 layer (kind::f16 MMAs with fp16 operands): outputs and gradients within 2e-2
    of each tensor's max magnitude."""
    torch.manual_seed(4)
    D, H, E, k = 256, 512, 32, 4
    layer = FusedMoEMLPSorted(D, H, E, k).to(DEV).half()
    G = gen(9)
    x = torch.randn(256, D, generator=G).half().to(DEV)
    dout = torch.randn(256, D, generator=G).half().to(DEV)
    out, dx, logits = run_layer(layer, x, dout)
    w13 = layer.w13.float().cpu()
    ro, rdx, rdwg, rdwu, rdwd, rdl = moe_layer_oracle(x.cpu(), logits.cpu(), w13[:, :H],
                                                      w13[:, H:], layer.w2.float().cpu(), k,
                                                      dout.cpu())
    close(out.cpu(), ro)
    close(dx.cpu(), rdx + rdl @ layer.router.weight.double().cpu())
    g13, g2 = stacked_grads(layer)
    close(g13.cpu(), torch.cat([rdwg, rdwu], dim=1))
    close(g2.cpu(), rdwd)
