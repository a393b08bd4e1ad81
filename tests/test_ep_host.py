"""Expert-parallel host logic on CPU: the load-aware placement, and the exchange protocol
(plan, fixed-capacity all-to-all, expert-side pre-reduction, rank-ordered unpack) run with
real gloo collectives on 2 ranks against the single-process oracle."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fusedkernels_b200.moe_ep import lpt_placement, round_robin_placement


def test_lpt_placement_balances_zipf_load():
    from oracle import zipf_expert_bias
    E, N = 128, 8
    load = torch.exp(zipf_expert_bias(E) / 2)  # the Zipf weights themselves
    rr = round_robin_placement(E, N)
    lpt = lpt_placement(load.tolist(), N)
    for pl in (rr, lpt):
        assert all(sum(1 for p in pl if p == r) == E // N for r in range(N))

    def imbalance(pl):
        per = [sum(float(load[e]) for e in range(E) if pl[e] == r) for r in range(N)]
        return max(per) / (sum(per) / N)

    assert imbalance(lpt) <= imbalance(rr)
    contiguous = [e // (E // N) for e in range(E)]
    assert imbalance(lpt) < imbalance(contiguous)
    assert lpt == lpt_placement(load.tolist(), N)  # deterministic


def test_owner_local_index_matches_per_rank_order():
    """The destination rank of a slot stacks its experts in ascending global id; the
    planning table must give every expert's index there, for remote experts too."""
    from fusedkernels_b200.moe_ep import owner_local_index
    G = torch.Generator().manual_seed(5)
    for E, N in [(8, 2), (128, 8), (64, 4)]:
        pl = lpt_placement(torch.rand(E, generator=G).tolist(), N)
        table = owner_local_index(pl, N)
        for r in range(N):
            ids = [e for e in range(E) if pl[e] == r]
            assert [table[e] for e in ids] == list(range(len(ids)))


def test_replication_tables_are_consistent_across_ranks():
    """Every slot a rank plans for its own tokens lands on a rank whose stack holds that
    expert at the planned index; replicated experts stay on the token's rank."""
    from fusedkernels_b200.moe_ep import hot_experts, lpt_placement_excluding, plan_tables
    from oracle import zipf_expert_bias
    E = 128
    load = torch.exp(zipf_expert_bias(E) / 2).tolist()
    for N in (2, 4, 8):
        rep = hot_experts(load, N)
        pl = lpt_placement_excluding(load, N, rep)
        assert all((pl[e] == -1) == (e in rep) for e in range(E))
        stacks = {r: plan_tables(pl, rep, N, r)[0] for r in range(N)}
        assert sorted(e for r in range(N) for e in stacks[r] if e not in rep) == \
            [e for e in range(E) if e not in rep]
        for r in range(N):
            _, n_own, rank_tab, local_tab = plan_tables(pl, rep, N, r)
            for e in range(E):
                d = rank_tab[e]
                assert stacks[d][local_tab[e]] == e
                if e in rep:
                    assert d == r
        counts = [len(stacks[r]) - len(rep) for r in range(N)]
        assert max(counts) <= -(-(E - len(rep)) // N)
    assert hot_experts(load, 1) == []


def test_lpt_placement_rejects_uneven():
    with pytest.raises(ValueError):
        lpt_placement([1.0] * 10, 4)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from ep_reference import ep_pack, ep_plan, ep_unpack_sum, expert_side
    from fusedkernels_b200.moe_ep import Exchange
    from oracle import route_oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, k, T, D, H = 8, 3, 12, 16, 8
        G = torch.Generator().manual_seed(0)
        wg = torch.randn(E, H, D, generator=G) * 0.3
        wu = torch.randn(E, H, D, generator=G) * 0.3
        wd = torch.randn(E, D, H, generator=G) * 0.3
        x_all = torch.randn(world * T, D, generator=G)
        logits_all = torch.randn(world * T, E, generator=G)
        placement = lpt_placement(torch.rand(E, generator=G).tolist(), world)
        expert_rank = torch.tensor(placement)
        local_ids = [e for e in range(E) if placement[e] == rank]
        expert_local = torch.full((E,), -1, dtype=torch.long)
        for d in range(world):
            ids = [e for e in range(E) if placement[e] == d]
            for i, e in enumerate(ids):
                expert_local[e] = i
        x = x_all[rank * T:(rank + 1) * T]
        w, idx = route_oracle(logits_all[rank * T:(rank + 1) * T], k)
        send_token, send_e, send_w, src_pos, _ = ep_plan(idx, w, expert_rank, expert_local, world)
        ex = Exchange()
        recv_x = ex.all_to_all(ep_pack(x, send_token))
        recv_e = ex.all_to_all(send_e)
        recv_w = ex.all_to_all(send_w)
        lid = torch.tensor(local_ids)
        partial = expert_side(recv_x, recv_e, recv_w, wg[lid], wu[lid], wd[lid]).float()
        back = ex.all_to_all(partial)
        out = ep_unpack_sum(back, src_pos, T)
        # single-process reference for this rank's tokens
        ref = torch.zeros(T, D, dtype=torch.float64)
        F = torch.nn.functional
        for t in range(T):
            for j in range(k):
                e = int(idx[t, j])
                h = F.silu(wg[e].double() @ x[t].double()) * (wu[e].double() @ x[t].double())
                ref[t] += float(w[t, j]) * (wd[e].double() @ h)
        q.put((rank, float((out - ref).abs().max())))
    except Exception as exc:  # report instead of hanging the peer
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_protocol_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err in res:
        assert isinstance(err, float), f"rank {rank}: {err}"
        assert err < 1e-5, f"rank {rank}: max err {err}"
