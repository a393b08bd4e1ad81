"""Expert-parallel kernels and layer on the GPU.  The plan/pack/unpack kernels are checked
bit-exactly (integers) and to fp32 rounding (sums) against tests/ep_reference.py for
2 and 8 simulated ranks; the EP layer on a one-rank NCCL group must reproduce the
single-GPU FusedMoEMLPSorted bit for bit; with two or more GPUs, a 2-rank run is checked
against the single-GPU layer (2e-2 of max magnitude, bf16)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist

from fusedkernels_b200 import _lib, fused_moe_route_v2
from fusedkernels_b200.moe_ep import ExpertParallelMoEMLP, lpt_placement
from fusedkernels_b200.moe_layer_sorted import FusedMoEMLPSorted
from oracle import route_oracle
from ep_reference import ep_plan, ep_unpack_dw, ep_unpack_sum
from conftest import gen

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("n_ranks,T,k,E", [(2, 300, 2, 8), (8, 1000, 8, 128), (8, 5, 2, 64),
                                             (4, 4096, 8, 128), (32, 777, 4, 64)])
def test_ep_plan_pack_unpack_match_reference(n_ranks, T, k, E):
    G = gen(T + E)
    w, idx = route_oracle(torch.randn(T, E, generator=G), k)
    placement = lpt_placement(torch.rand(E, generator=G).tolist(), n_ranks)
    er = torch.tensor(placement, dtype=torch.int32)
    el = torch.full((E,), -1, dtype=torch.int32)
    for d in range(n_ranks):
        for i, e in enumerate([e for e in range(E) if placement[e] == d]):
            el[e] = i
    ref = ep_plan(idx, w, er.long(), el.long(), n_ranks)
    i32 = dict(dtype=torch.int32, device=DEV)
    send_token = torch.empty(n_ranks * T, **i32)
    send_e = torch.empty(n_ranks * T, k, **i32)
    send_w = torch.empty(n_ranks * T, k, device=DEV)
    src_pos = torch.empty(T, n_ranks, **i32)
    count = torch.empty(n_ranks, **i32)
    err = torch.zeros(1, **i32)
    st = torch.cuda.current_stream().cuda_stream
    idx_d, w_d, er_d, el_d = idx.to(DEV), w.to(DEV), er.to(DEV), el.to(DEV)
    ws = torch.empty(_lib.ep_plan_workspace_bytes(T, n_ranks), dtype=torch.uint8, device=DEV)
    _lib.call("fk_ep_plan", idx_d.data_ptr(), w_d.data_ptr(), T, k, er_d.data_ptr(), el_d.data_ptr(),
              E, n_ranks, send_token.data_ptr(), send_e.data_ptr(), send_w.data_ptr(),
              src_pos.data_ptr(), count.data_ptr(), ws.data_ptr(), ws.numel(), err.data_ptr(), st)
    assert err.item() == 0
    for got, want in zip((send_token, send_e, send_w, src_pos, count), ref):
        assert torch.equal(got.cpu(), want.to(got.dtype)), "plan mismatch"
    D = 64
    x = torch.randn(T, D, generator=G).bfloat16().to(DEV)
    send_x = torch.zeros(n_ranks * T, D, dtype=torch.bfloat16, device=DEV)
    _lib.call("fk_ep_pack", x.data_ptr(), D, send_token.data_ptr(), n_ranks * T, send_x.data_ptr(),
              _lib.FK_BF16, st)
    ok = send_token.long() >= 0
    assert torch.equal(send_x[ok], x[send_token.long()[ok]])
    back = torch.randn(n_ranks * T, D, generator=G).bfloat16().to(DEV)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    _lib.call("fk_ep_unpack_sum", back.data_ptr(), D, src_pos.data_ptr(), T, n_ranks,
              out.data_ptr(), _lib.FK_BF16, st)
    torch.testing.assert_close(out.cpu().double(), ep_unpack_sum(back.cpu(), src_pos.cpu(), T).bfloat16().double(),
                               atol=1e-2, rtol=1e-2)
    back_dw = torch.randn(n_ranks * T, k, generator=G).to(DEV)
    dw = torch.empty(T, k, device=DEV)
    _lib.call("fk_ep_unpack_dw", back_dw.data_ptr(), idx_d.data_ptr(), er_d.data_ptr(),
              src_pos.data_ptr(), T, k, n_ranks, E, dw.data_ptr(), st)
    assert torch.equal(dw.cpu(), ep_unpack_dw(back_dw.cpu(), idx, er.long(), src_pos.cpu()))


def _make_weights(D, H, E, seed):
    G = gen(seed)
    return (torch.randn(E, D, generator=G) * 0.05, torch.randn(E, H, D, generator=G) * 0.05,
            torch.randn(E, H, D, generator=G) * 0.05, torch.randn(E, D, H, generator=G) * 0.05)


def _single_gpu(D, H, E, k, wts, x, dout):
    layer = FusedMoEMLPSorted(D, H, E, k)
    with torch.no_grad():
        layer.router.weight.copy_(wts[0])
        for e, ex in enumerate(layer.experts):
            ex.w_gate.weight.copy_(wts[1][e])
            ex.w_up.weight.copy_(wts[2][e])
            ex.w_down.weight.copy_(wts[3][e])
    layer = layer.to(DEV).bfloat16()
    xg = x.clone().requires_grad_(True)
    out = layer(xg)
    out.backward(dout)
    return layer, out.detach(), xg.grad


@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_ep_layer_one_rank_matches_single_gpu_bitwise(transport):
    D, H, E, k, T = 256, 256, 16, 4, 512
    wts = _make_weights(D, H, E, 1)
    G = gen(2)
    x = torch.randn(T, D, generator=G).bfloat16().to(DEV)
    dout = torch.randn(T, D, generator=G).bfloat16().to(DEV)
    ref_layer, ref_out, ref_dx = _single_gpu(D, H, E, k, wts, x, dout)
    store = dist.TCPStore("127.0.0.1", _free_port(), 1, True)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1)
    try:
        ep = ExpertParallelMoEMLP(D, H, E, k, transport=transport).to(DEV).bfloat16()
        ep.load_from_full(*(t.bfloat16().to(DEV) for t in wts))
        for _ in range(2):  # the second step reuses the exchange regions
            ep.zero_grad(set_to_none=True)
            xg = x.clone().requires_grad_(True)
            out = ep(xg)
            out.backward(dout)
        torch.cuda.synchronize()
        assert ep.peer_error() == 0
        assert torch.equal(out, ref_out)
        assert torch.equal(xg.grad, ref_dx)
        assert torch.equal(ep.router.weight.grad, ref_layer.router.weight.grad)
        for e in range(E):
            a, b = ep.experts[str(e)], ref_layer.experts[e]
            assert torch.equal(a.w_gate.weight.grad, b.w_gate.weight.grad)
            assert torch.equal(a.w_down.weight.grad, b.w_down.weight.grad)
        ep.close()
    finally:
        dist.destroy_process_group()


def test_ep_peer_layer_cuda_graph_replay():
    """The peer transport keeps its sequence numbers on the device: a captured step
    replays correctly (one rank)."""
    D, H, E, k, T = 256, 256, 16, 4, 512
    wts = _make_weights(D, H, E, 1)
    G = gen(4)
    x = torch.randn(T, D, generator=G).bfloat16().to(DEV)
    dout = torch.randn(T, D, generator=G).bfloat16().to(DEV)
    store = dist.TCPStore("127.0.0.1", _free_port(), 1, True)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1)
    try:
        ep = ExpertParallelMoEMLP(D, H, E, k, transport="peer").to(DEV).bfloat16()
        ep.load_from_full(*(t.bfloat16().to(DEV) for t in wts))
        xg = x.clone().requires_grad_(True)

        def step():
            xg.grad = None
            out = ep(xg)
            out.backward(dout)
            return out

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            eager = step().clone()
            eager_dx = xg.grad.clone()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = step()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        assert ep.peer_error() == 0
        assert torch.equal(out, eager)
        assert torch.equal(xg.grad, eager_dx)
        del g
        ep.close()
    finally:
        dist.destroy_process_group()


def test_ep_peer_wait_times_out_and_reports():
    """A phase that no rank publishes: the wait gives up after its bound (0.5 s), records
    16 + phase and leaves the context usable."""
    flags = torch.zeros(4, dtype=torch.int32, device=DEV)
    ctl = torch.zeros(24, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("fk_ep_peer_wait", flags.data_ptr(), 1, 2, ctl.data_ptr(), 500, err.data_ptr(), st)
    torch.cuda.synchronize()
    assert err.item() == 18
    assert ctl[16 + 2].item() == 1  # the expected sequence number moved on
    assert (torch.ones(4, device=DEV) * 2).sum().item() == 8.0


def _ep_worker(rank, world, port, q, transport="peer", replicated=()):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import datetime
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        D, H, E, k, T = 256, 256, 16, 4, 256
        wts = _make_weights(D, H, E, 1)
        G = torch.Generator().manual_seed(3)
        x_all = torch.randn(world * T, D, generator=G).bfloat16()
        d_all = torch.randn(world * T, D, generator=G).bfloat16()
        ep = ExpertParallelMoEMLP(D, H, E, k, placement=lpt_placement([1.0] * E, world),
                                  transport=transport, replicated=replicated).to(dev).bfloat16()
        ep.load_from_full(*(t.bfloat16().to(dev) for t in wts))
        x = x_all[rank * T:(rank + 1) * T].to(dev).requires_grad_(True)
        out = ep(x)
        out.backward(d_all[rank * T:(rank + 1) * T].to(dev))
        with torch.no_grad():
            _, idx = fused_moe_route_v2(ep.router(x.detach()), k)
        torch.cuda.synchronize()
        assert ep.peer_error() == 0, f"peer wait timed out: {ep.peer_error()}"
        grads = {e: tuple(getattr(ep.experts[str(e)], n).weight.grad.float().cpu()
                          for n in ("w_gate", "w_up", "w_down")) for e in ep.local_ids}
        ep.close()
        q.put((rank, out.detach().float().cpu(), x.grad.detach().float().cpu(), idx.cpu(), grads))
    except Exception as exc:
        q.put((rank, repr(exc), None, None, None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport,replicated", [("peer", ()), ("nccl", ()), ("peer", (0, 5))])
def test_ep_layer_two_ranks_matches_single_gpu(transport, replicated):
    import torch.multiprocessing as mp
    D, H, E, k, T, world = 256, 256, 16, 4, 256, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q, transport, replicated))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert not isinstance(r[1], str), f"rank {r[0]}: {r[1]}"
    wts = _make_weights(D, H, E, 1)
    G = torch.Generator().manual_seed(3)
    x_all = torch.randn(world * T, D, generator=G).bfloat16().to(DEV)
    d_all = torch.randn(world * T, D, generator=G).bfloat16().to(DEV)
    # Tokens are independent, so the single-GPU layer runs on each rank's T tokens: the
    # router GEMM then has the same shape on both sides and the bf16 logits (and with them
    # the expert selection, which a 1-ulp difference on a near-tie would flip) are equal.
    ref_grads = {}
    for r in res:
        sl = slice(r[0] * T, (r[0] + 1) * T)
        layer, ref_out, ref_dx = _single_gpu(D, H, E, k, wts, x_all[sl], d_all[sl])
        with torch.no_grad():
            _, ref_idx = fused_moe_route_v2(layer.router(x_all[sl]), k)
        assert torch.equal(r[3], ref_idx.cpu()), f"rank {r[0]}: routing differs"
        scale = ref_out.abs().max().item()
        assert (r[1] - ref_out.float().cpu()).abs().max().item() <= 2e-2 * scale, f"rank {r[0]} out"
        scale = ref_dx.abs().max().item()
        assert (r[2] - ref_dx.float().cpu()).abs().max().item() <= 2e-2 * scale, f"rank {r[0]} dx"
        for e in range(E):  # expert gradients: the sum of the chunks' gradients
            ex = layer.experts[e]
            g = tuple(getattr(ex, n).weight.grad.float().cpu() for n in ("w_gate", "w_up", "w_down"))
            ref_grads[e] = g if e not in ref_grads else tuple(a + b for a, b in zip(ref_grads[e], g))
    held = set()
    for r in res:
        for e, g in r[4].items():
            held.add(e)
            for a, b in zip(g, ref_grads[e]):
                scale = max(b.abs().max().item(), 1e-6)
                assert (a - b).abs().max().item() <= 3e-2 * scale, f"rank {r[0]} expert {e} grad"
    assert held == set(range(E))
