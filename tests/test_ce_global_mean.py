"""Cross-entropy over a batch sharded by rows (data parallel): the all-reduce of
(sum of row losses, count of valid rows) and the per-rank gradient rescale
(``global_mean_scales``), run on 2 gloo ranks on the CPU against the single-process oracle
of the whole batch (the reference's mean, cross_entropy.py:107-110).  Each rank's local
loss and gradient come from the oracle, as the kernel would produce them: gradient scaled
by 1/max(1, local valid rows)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _batch(case):
    G = torch.Generator().manual_seed(7 + case)
    N, V = 24, 50
    x = torch.randn(N, V, generator=G) * 2
    t = torch.randint(0, V, (N,), generator=G)
    t[::5] = -100
    if case == 1:
        t[12:] = -100  # rank 1's whole shard is ignored
    return x, t


def _worker(rank, world, port, case, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from fusedkernels_b200.cross_entropy import global_mean_scales
    from oracle import cross_entropy_oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, t = _batch(case)
        per = x.shape[0] // world
        xs, ts = x[rank * per:(rank + 1) * per], t[rank * per:(rank + 1) * per]
        # what the row kernel gives this rank: mean over its own valid rows, gradient / n_local
        local_loss, local_grad = cross_entropy_oracle(xs, ts)
        count = (ts != -100).sum()
        n_local = count.clamp(min=1)
        loss_sum = local_loss * n_local
        gloss, factor = global_mean_scales(loss_sum, count, n_local)
        ref_loss, ref_grad = cross_entropy_oracle(x, t)
        err_loss = abs(float(gloss) - float(ref_loss))
        err_grad = float((local_grad * factor - ref_grad[rank * per:(rank + 1) * per]).abs().max())
        q.put((rank, err_loss, err_grad))
    except Exception as exc:  # report instead of hanging the peer
        q.put((rank, repr(exc), None))
    finally:
        dist.destroy_process_group()


def _run(case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, el, eg in res:
        assert isinstance(el, float), f"rank {rank}: {el}"
        assert el < 1e-6 and eg < 1e-7, f"rank {rank}: loss err {el}, grad err {eg}"


def test_global_mean_two_gloo_ranks():
    _run(0)


def test_global_mean_rank_with_only_ignored_rows():
    _run(1)


def test_global_mean_without_process_group_is_local_mean():
    from fusedkernels_b200.cross_entropy import global_mean_scales
    loss, f = global_mean_scales(torch.tensor(6.0), torch.tensor(3), torch.tensor(3))
    assert float(loss) == 2.0 and float(f) == 1.0
    loss, f = global_mean_scales(torch.tensor(0.0), torch.tensor(0), torch.tensor(1))
    assert float(loss) == 0.0 and float(f) == 1.0
