"""Cross-entropy kernel vs the oracle (fp64) and the reference kernel's golden vectors.
Tolerances: loss rtol 1e-5 (fp32) / 1e-4 (bf16); gradient x n_valid atol 1e-5 (fp32),
atol 1e-3 + rtol 1e-2 (bf16: rounding of the stored gradient)."""
import pytest
import torch

import fusedkernels_b200 as fk
from fusedkernels_b200.cross_entropy import last_target_error
from oracle import cross_entropy_oracle
from conftest import gen

pytestmark = pytest.mark.gpu


def run(logits, targets, ignore_index=-100, ls=0.0, inplace=False, go=None):
    x = logits.cuda().requires_grad_(True)
    leaf = x
    if inplace:
        x = x.detach().clone().requires_grad_(True)
        leaf = x
    loss = fk.fused_cross_entropy(x, targets.cuda(), ignore_index=ignore_index,
                                  label_smoothing=ls, inplace_grad=inplace)
    if go is None:
        loss.backward()
    else:
        loss.backward(torch.tensor(go, device="cuda"))
    return loss.detach().cpu(), leaf.grad.cpu()


def check(logits, targets, ls=0.0, inplace=False, go=None):
    loss, grad = run(logits, targets, ls=ls, inplace=inplace, go=go)
    rl, rg = cross_entropy_oracle(logits, targets, -100, ls)
    n_valid = max(int((targets != -100).sum()), 1)
    scale = 1.0 if go is None else go
    if logits.dtype == torch.float32:
        torch.testing.assert_close(loss.double(), rl, atol=1e-6, rtol=1e-5)
        torch.testing.assert_close(grad.double() * n_valid, rg * scale * n_valid, atol=1e-5, rtol=1e-5)
    else:
        torch.testing.assert_close(loss.double(), rl, atol=1e-5, rtol=1e-4)
        torch.testing.assert_close(grad.double() * n_valid, rg * scale * n_valid, atol=1e-3, rtol=1e-2)


def test_ce_reference_case_ignore_index():
    """tests/test_correctness.py:11-27: N=512, V=32000 fp32, every 37th target ignored."""
    G = gen(0)
    logits = torch.randn(512, 32000, generator=G)
    targets = torch.randint(0, 32000, (512,), generator=G)
    targets[::37] = -100
    check(logits, targets)


def test_ce_reference_case_label_smoothing():
    """tests/test_correctness.py:30-41: N=256, V=4096, label_smoothing=0.1 (grad too)."""
    G = gen(1)
    logits = torch.randn(256, 4096, generator=G)
    targets = torch.randint(0, 4096, (256,), generator=G)
    check(logits, targets, ls=0.1)


@pytest.mark.parametrize("V", [7, 128, 1000, 32001, 50257, 128256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ce_vocab_sizes(V, dtype):
    G = gen(V)
    N = 64
    logits = (torch.randn(N, V, generator=G) * 2).to(dtype)
    targets = torch.randint(0, V, (N,), generator=G)
    targets[::5] = -100
    check(logits, targets)


def test_ce_bf16_workload_vocab_inplace_and_smoothing():
    G = gen(3)
    logits = (torch.randn(96, 128256, generator=G) * 2).bfloat16()
    targets = torch.randint(0, 128256, (96,), generator=G)
    targets[torch.rand(96, generator=G) < 0.05] = -100
    check(logits, targets, inplace=True)
    check(logits, targets, ls=0.1)


def test_ce_grad_output_scaling():
    G = gen(4)
    logits = torch.randn(32, 1000, generator=G)
    targets = torch.randint(0, 1000, (32,), generator=G)
    check(logits, targets, go=2.5)


def test_ce_all_ignored_is_zero():
    logits = torch.randn(8, 100, generator=gen(5))
    targets = torch.full((8,), -100)
    loss, grad = run(logits, targets)
    assert loss.item() == 0.0 and torch.count_nonzero(grad) == 0


def test_ce_empty_batch():
    loss, grad = run(torch.zeros(0, 100), torch.zeros(0, dtype=torch.long))
    assert loss.item() == 0.0 and grad.shape == (0, 100)


def test_ce_out_of_range_target_flags_error():
    logits = torch.randn(4, 50, generator=gen(6))
    targets = torch.tensor([1, 2, 77, 3])  # 77 >= V: invalid, not ignore_index
    loss, grad = run(logits, targets)
    assert torch.isnan(loss).item()
    assert last_target_error() == 1
    assert torch.isnan(grad[2]).all() and torch.isfinite(grad[0]).all()
    run(logits, torch.tensor([1, 2, 3, 4]))
    assert last_target_error() == 0


def test_ce_very_long_rows_fallback():
    """Rows longer than the cluster path's shared-memory budget use the 3-sweep kernel."""
    G = gen(7)
    V = 500_000
    logits = torch.randn(4, V, generator=G)
    targets = torch.tensor([0, V - 1, -100, 12345])
    check(logits, targets)


def test_ce_misaligned_rows():
    G = gen(8)
    base = torch.randn(16, 1003, generator=G)
    logits = base[:, 1:1002]  # row stride 1003 fp32: rows not 16-byte aligned
    targets = torch.randint(0, 1001, (16,), generator=G)
    loss, grad = run(logits, targets)
    rl, rg = cross_entropy_oracle(logits, targets)
    torch.testing.assert_close(loss.double(), rl, atol=1e-6, rtol=1e-5)


def test_ce_matches_reference_golden(golden):
    for tag in ("a", "smooth", "wide"):
        p = f"ce_{tag}_"
        t = lambda k: torch.from_numpy(golden[p + k])
        loss, grad = run(t("logits"), t("targets"), ls=float(golden[p + "ls"]))
        torch.testing.assert_close(loss, t("loss"), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(grad, t("grad"), atol=1e-7, rtol=1e-4)


def test_ce_full_size_properties():
    """Workload [8192, 128256] bf16 ~N(0,2), 5% ignored, in-place: per-row loss and grad of
    64 sampled rows vs the oracle, ignored rows zero, valid grad rows sum to ~0."""
    G = gen(9)
    N, V = 8192, 128256
    logits = (torch.randn(N, V, generator=G) * 2).bfloat16()
    targets = torch.randint(0, V, (N,), generator=G)
    targets[torch.rand(N, generator=G) < 0.05] = -100
    x = logits.cuda().requires_grad_(True)
    loss = fk.fused_cross_entropy(x, targets.cuda(), inplace_grad=True)
    loss.backward()
    grad = x.grad
    n_valid = int((targets != -100).sum())
    # loss over all rows, fp64, in row blocks (no autograd on the full batch)
    tot = torch.zeros((), dtype=torch.float64)
    for r0 in range(0, N, 512):
        xb = logits[r0:r0 + 512].double()
        tb = targets[r0:r0 + 512]
        ok = tb != -100
        lse = torch.logsumexp(xb, -1)
        xt = xb.gather(1, torch.where(ok, tb, 0)[:, None])[:, 0]
        tot += torch.where(ok, lse - xt, torch.zeros_like(lse)).sum()
    torch.testing.assert_close(loss.double().cpu(), tot / n_valid, atol=1e-5, rtol=1e-4)
    rows = torch.randint(0, N, (64,), generator=G)
    _, rg = cross_entropy_oracle(logits[rows].float(), targets[rows])
    nv_sub = max(int((targets[rows] != -100).sum()), 1)
    torch.testing.assert_close(grad[rows.cuda()].double().cpu() * n_valid, rg * nv_sub,
                               atol=1e-3, rtol=1e-2)
    ign = (targets == -100).cuda()
    assert torch.count_nonzero(grad[ign]) == 0
    row_sums = grad[~ign].float().sum(-1) * n_valid
    assert row_sums.abs().max().item() < 0.05


def test_global_mean_single_process_equals_local_mean():
    """Without a process group the sharded-batch form is the plain fused loss."""
    from fusedkernels_b200.cross_entropy import fused_cross_entropy_global_mean
    G = gen(31)
    x = (torch.randn(64, 3000, generator=G) * 2).bfloat16()
    t = torch.randint(0, 3000, (64,), generator=G)
    t[::4] = -100
    a = x.cuda().requires_grad_(True)
    la = fk.fused_cross_entropy(a, t.cuda())
    la.backward(torch.tensor(0.5, device="cuda"))
    b = x.cuda().requires_grad_(True)
    lb = fused_cross_entropy_global_mean(b, t.cuda())
    lb.backward(torch.tensor(0.5, device="cuda"))
    torch.testing.assert_close(lb, la, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(b.grad.float(), a.grad.float(), atol=1e-6, rtol=1e-2)


def _ce_worker(rank, world, port, q):
    import datetime
    import os
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from fusedkernels_b200.cross_entropy import fused_cross_entropy_global_mean
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    try:
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        G = torch.Generator().manual_seed(41)
        x = (torch.randn(256, 4096, generator=G) * 2).bfloat16()
        t = torch.randint(0, 4096, (256,), generator=G)
        t[::3] = -100
        per = 256 // world
        xs = x[rank * per:(rank + 1) * per].to(dev).requires_grad_(True)
        loss = fused_cross_entropy_global_mean(xs, t[rank * per:(rank + 1) * per].to(dev))
        loss.backward()
        q.put((rank, float(loss), xs.grad.float().cpu()))
    except Exception as exc:
        q.put((rank, repr(exc), None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_global_mean_two_ranks_nccl():
    """Two ranks, one half of the rows each: both see the full-batch mean loss, and each
    rank's gradient equals its rows of the full-batch gradient."""
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ce_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    G = torch.Generator().manual_seed(41)
    x = (torch.randn(256, 4096, generator=G) * 2).bfloat16()
    t = torch.randint(0, 4096, (256,), generator=G)
    t[::3] = -100
    rl, rg = cross_entropy_oracle(x, t)
    for rank, loss, grad in res:
        assert not isinstance(loss, str), f"rank {rank}: {loss}"
        assert abs(loss - float(rl)) <= 1e-4 * abs(float(rl))
        ref = rg[rank * 128:(rank + 1) * 128].float()
        torch.testing.assert_close(grad, ref.bfloat16().float(), atol=1e-6, rtol=1e-2)
