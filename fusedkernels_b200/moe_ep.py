"""Expert-parallel sorted-dispatch MoE layer (one process per GPU on one node).

The reference runs every expert on one GPU (fusedkernels/moe_layer_sorted.py:37); this
module shards the experts of ``FusedMoEMLPSorted`` across the ranks of a process group
(16 experts per GPU for E=128 on 8 GPUs) and exchanges token rows between them:

  forward   route locally -> fk_ep_plan (which ranks need each token, deduplicated) ->
            rows and slot metadata to the expert ranks -> local grouped-GEMM experts on
            the received rows -> per-row pre-reduction of the local slots -> partial rows
            back -> fk_ep_unpack_sum (rank-ordered sum: deterministic)
  backward  the mirror image: dout rows out, per-slot routing gradients and partial input
            gradients back; the return exchange overlaps the weight-gradient GEMMs, and the
            replicated experts' gradient all-reduce overlaps the input-gradient GEMMs.

Every (source, destination) pair has a fixed capacity of T rows (a token is sent at most
once per destination), so no host synchronisation or split-size exchange is needed.

Transports: ``"peer"`` (default) -- put kernels store the rows straight into the other
ranks' memory over NVLink (``PeerExchange``, csrc/moe_ep_peer.cu); ``"nccl"`` --
fk_ep_pack + fixed-capacity ``all_to_all_single``.

Placement is static and load-aware: ``lpt_placement`` bin-packs experts, hottest first,
onto the least-loaded rank with a free slot.  Experts hot enough that nearly every token
picks them (``hot_experts``) can be replicated on every rank instead: their slots are
computed on the token's own rank and their weight gradients are summed over the group
inside backward (``lpt_placement_excluding`` places the rest).

``ExpertParallelMoEMLP`` keeps the reference's parameter naming for the experts it holds
(``experts.<global id>.w_gate.weight`` ...) and a replicated ``router``.  Gradients of the
replicated router weight are local; averaging them across data-parallel ranks is the
caller's job (``allreduce_router_grad``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib
from .moe_layer import Expert
from .moe_layer_sorted import _Plan
from .moe_routing_v2 import fused_moe_route_v2


def lpt_placement(load, n_ranks: int) -> list[int]:
    """Static expert -> rank map with exactly E/n_ranks experts per rank, balancing the
    given per-expert load: experts in descending load order go to the least-loaded rank
    that still has a free slot (longest-processing-time-first bin packing)."""
    load = [float(v) for v in load]
    E = len(load)
    if E % n_ranks:
        raise ValueError(f"n_experts={E} is not divisible by n_ranks={n_ranks}")
    cap = E // n_ranks
    tot = [0.0] * n_ranks
    used = [0] * n_ranks
    rank_of = [0] * E
    for e in sorted(range(E), key=lambda i: (-load[i], i)):
        r = min((r for r in range(n_ranks) if used[r] < cap), key=lambda r: (tot[r], r))
        rank_of[e] = r
        tot[r] += load[e]
        used[r] += 1
    return rank_of


def round_robin_placement(n_experts: int, n_ranks: int) -> list[int]:
    return [e % n_ranks for e in range(n_experts)]


def hot_experts(load, n_ranks: int, fraction: float = 0.25) -> list[int]:
    """Experts worth replicating on every rank: those whose load alone exceeds `fraction`
    of one rank's fair share of all assignments.  Such an expert is picked by a large
    share of all tokens, so owning it on one rank makes that rank receive nearly every
    token of every other rank; replicated, its slots are computed where the token lives
    and only its weight gradient (25 MB at D=4096, H=1024) is summed across ranks."""
    load = [float(v) for v in load]
    if n_ranks <= 1:
        return []
    share = sum(load) / n_ranks
    return sorted(e for e, v in enumerate(load) if v >= fraction * share)


def plan_tables(placement, replicated, n_ranks: int, rank: int):
    """Stack and planning tables of one rank.

    Returns (local_ids, n_owned, expert_rank, expert_local): the rank's stacked experts
    (owned ones by ascending id, then the replicated ones), how many it owns, and for every
    expert e the rank that computes e's slots for a token of this rank (the owner, or this
    rank for a replicated expert) with e's index inside that rank's stack."""
    E = len(placement)
    rep_set = set(replicated)
    rep_sorted = sorted(rep_set)
    owned = [e for e in range(E) if e not in rep_set and placement[e] == rank]
    cold_place = [placement[e] if e not in rep_set else n_ranks for e in range(E)]
    cold_index = owner_local_index(cold_place, n_ranks + 1)
    expert_rank = [rank if e in rep_set else placement[e] for e in range(E)]
    expert_local = [len(owned) + rep_sorted.index(e) if e in rep_set else cold_index[e]
                    for e in range(E)]
    return owned + rep_sorted, len(owned), expert_rank, expert_local


def lpt_placement_excluding(load, n_ranks: int, replicated) -> list[int]:
    """LPT placement of the experts that are not replicated, at most
    ceil(n_cold / n_ranks) per rank; replicated experts get -1."""
    load = [float(v) for v in load]
    rep = set(replicated)
    cold = [e for e in range(len(load)) if e not in rep]
    cap = -(-len(cold) // n_ranks)
    tot = [0.0] * n_ranks
    used = [0] * n_ranks
    rank_of = [-1] * len(load)
    for e in sorted(cold, key=lambda i: (-load[i], i)):
        r = min((r for r in range(n_ranks) if used[r] < cap), key=lambda r: (tot[r], r))
        rank_of[e] = r
        tot[r] += load[e]
        used[r] += 1
    return rank_of


def owner_local_index(placement, n_ranks: int) -> list[int]:
    """For every expert, its position among the experts of the rank that owns it (the
    order of that rank's stacked weights: ascending global id)."""
    seen = [0] * n_ranks
    out = []
    for r in placement:
        out.append(seen[r])
        seen[r] += 1
    return out


class Exchange:
    """Fixed-capacity all-to-all of [n_ranks * cap, ...] buffers over a process group
    (the NCCL transport)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_to_all(self, send: torch.Tensor, async_op: bool = False):
        recv = torch.empty_like(send)
        work = dist.all_to_all_single(recv, send, group=self.group, async_op=async_op)
        return (recv, work) if async_op else recv


class PeerExchange:
    """The NVLink transport: one exchange region per rank (allocated by the library, shared
    with CUDA IPC, mapped into every other rank of the group, which must sit on one node),
    written directly by the put kernels (see csrc/moe_ep_peer.cu for the protocol).

    Regions (fixed-capacity layout of fk_ep_plan, T tokens per rank): to_expert
    [N*T, dim] bf16, meta_e [N*T, k] int32, meta_w [N*T, k] fp32, to_source [N*T, dim]
    bf16, dw [N*T, k] fp32, flags [4, N] uint32.  Creating and closing are collective."""

    PHASE_FWD_DISPATCH, PHASE_FWD_COMBINE, PHASE_BWD_DISPATCH, PHASE_BWD_COMBINE = 0, 1, 2, 3

    def __init__(self, group, n_tokens: int, dim: int, k: int, device, timeout_ms: int = 2000):
        import ctypes as C
        self.timeout_ms = timeout_ms
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.key = (n_tokens, dim, k)
        N, T = self.world, n_tokens
        sizes = [("to_expert", N * T * dim * 2), ("meta_e", N * T * k * 4),
                 ("meta_w", N * T * k * 4), ("to_source", N * T * dim * 2),
                 ("dw", N * T * k * 4), ("flags", 4 * N * 4)]
        self.offset, total = {}, 0
        for name, nbytes in sizes:
            self.offset[name] = total
            total += (nbytes + 255) // 256 * 256
        own = C.c_void_p()
        handle = C.create_string_buffer(64)
        _lib.call("fk_ipc_alloc", total, C.byref(own), handle)
        self._own = own.value
        handles = [None] * N
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        self._opened = []
        bases = []
        for d in range(N):
            if d == self.rank:
                bases.append(self._own)
                continue
            p = C.c_void_p()
            _lib.call("fk_ipc_open", C.create_string_buffer(handles[d], 64), C.byref(p))
            self._opened.append(p.value)
            bases.append(p.value)
        self.tables = {name: torch.tensor([b + off for b in bases], dtype=torch.int64,
                                          device=device)
                       for name, off in self.offset.items()}
        self.ctl = torch.zeros(24, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        dist.barrier(group=group)  # every rank has mapped every region

    def local(self, name: str) -> int:
        return self._own + self.offset[name]

    def table(self, name: str) -> int:
        return self.tables[name].data_ptr()

    def wait(self, phase: int, stream) -> None:
        _lib.call("fk_ep_peer_wait", self.local("flags"), self.world, phase, self.ctl.data_ptr(),
                  self.timeout_ms, self.err.data_ptr(), stream)

    def close(self) -> None:
        """Collective: unmap the peers' regions, then free this rank's region."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.call("fk_ipc_close", p)
        self._opened = []
        dist.barrier(group=self.group)
        _lib.call("fk_ipc_free", self._own)
        self._own = None


def _pack_meta(e: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """[rows, k] int32 expert ids + [rows, k] fp32 weights -> one [rows, 2k] int32 tensor."""
    return torch.cat([e, w.view(torch.int32)], dim=1)


def _unpack_meta(m: torch.Tensor, k: int):
    return m[:, :k].contiguous(), m[:, k:].contiguous().view(torch.float32)


class _EPMoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, idx, layer, *expert_params):
        T, d = x.shape
        k = idx.shape[1]
        ex = layer.exchange
        N = ex.world
        El, H, E = len(layer.local_ids), layer.hidden_dim, layer.n_experts
        dev = x.device
        st = _lib.stream_of(x)
        i32 = dict(dtype=torch.int32, device=dev)
        idx = idx.contiguous()
        w = w.to(torch.float32).contiguous()
        send_token = torch.empty(N * T, **i32)
        send_e = torch.empty(N * T, k, **i32)
        send_w = torch.empty(N * T, k, dtype=torch.float32, device=dev)
        src_pos = torch.empty(T, N, **i32)
        send_count = torch.empty(N, **i32)
        perr = torch.zeros(1, **i32)
        pws = torch.empty(_lib.ep_plan_workspace_bytes(T, N), dtype=torch.uint8, device=dev)
        _lib.call("fk_ep_plan", idx.data_ptr(), w.data_ptr(), T, k, layer.expert_rank.data_ptr(),
                  layer.expert_local.data_ptr(), E, N, send_token.data_ptr(), send_e.data_ptr(),
                  send_w.data_ptr(), src_pos.data_ptr(), send_count.data_ptr(), pws.data_ptr(),
                  pws.numel(), perr.data_ptr(), st)
        px = layer._peer(T, d, k, dev) if layer.transport == "peer" else None
        if px is not None:
            _lib.call("fk_ep_peer_put_rows", x.data_ptr(), d, send_token.data_ptr(), T, N, ex.rank,
                      send_e.data_ptr(), send_w.data_ptr(), k, px.table("to_expert"),
                      px.table("meta_e"), px.table("meta_w"), px.table("flags"),
                      px.PHASE_FWD_DISPATCH, px.ctl.data_ptr(), _lib.FK_BF16, st)
            px.wait(px.PHASE_FWD_DISPATCH, st)
            recv_x_p, recv_e_p, recv_w_p = px.local("to_expert"), px.local("meta_e"), px.local("meta_w")
        else:
            send_x = torch.empty(N * T, d, dtype=torch.bfloat16, device=dev)
            _lib.call("fk_ep_pack", x.data_ptr(), d, send_token.data_ptr(), N * T,
                      send_x.data_ptr(), _lib.FK_BF16, st)
            recv_x = ex.all_to_all(send_x)
            recv_e, recv_w = _unpack_meta(ex.all_to_all(_pack_meta(send_e, send_w)), k)
            recv_x_p, recv_e_p, recv_w_p = recv_x.data_ptr(), recv_e.data_ptr(), recv_w.data_ptr()
        # local experts on the received rows (N*T "tokens" with k slots, -1 = not local)
        R_tok = N * T
        plan = _Plan(R_tok, k, El, dev)
        R = plan.max_rows
        eptr = plan.err.data_ptr()
        _lib.call("fk_moe_route_meta_skip", recv_e_p, recv_w_p, R_tok, k, El,
                  plan.counts.data_ptr(), plan.seg_start.data_ptr(), plan.tile_expert.data_ptr(),
                  plan.n_mblk.data_ptr(), plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(),
                  plan.slot_pos.data_ptr(), R, plan.ws.data_ptr(), plan.ws.numel(), eptr, st)
        bf = dict(dtype=torch.bfloat16, device=dev)
        xs = torch.empty(R, d, **bf)
        h1 = torch.empty(R, 2 * H, **bf)
        act = torch.empty(R, H, **bf)
        y = torch.empty(R, d, **bf)
        _lib.call("fk_moe_gather_by_token", recv_x_p, d, plan.slot_pos.data_ptr(), R_tok, k,
                  plan.sorted_assign.data_ptr(), plan.n_mblk.data_ptr(), R, xs.data_ptr(),
                  _lib.FK_BF16, st)
        # routing weights applied in the up-projection's epilogue (act = w * silu(g) * u):
        # the expert rows come out weighted and the local slots are summed unweighted
        _lib.call("fk_moe_gemm_up_weighted", xs.data_ptr(), R, d, layer.w13.data_ptr(), H, El,
                  plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(),
                  plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(), h1.data_ptr(),
                  act.data_ptr(), 0, eptr + 4, st)
        _lib.call("fk_moe_gemm_down", act.data_ptr(), R, H, layer.w2.data_ptr(), d, El,
                  plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr(), y.data_ptr(), 0, eptr + 4,
                  st)
        if px is not None:
            _lib.call("fk_ep_peer_combine_put", y.data_ptr(), d, plan.slot_pos.data_ptr(), None,
                      T, N, ex.rank, k, None, px.table("to_source"), None, px.table("flags"),
                      px.PHASE_FWD_COMBINE, px.ctl.data_ptr(), _lib.FK_BF16, st)
            px.wait(px.PHASE_FWD_COMBINE, st)
            back_p = px.local("to_source")
        else:
            partial = torch.empty(R_tok, d, **bf)
            _lib.call("fk_moe_combine", y.data_ptr(), d, plan.slot_pos.data_ptr(), None,
                      R_tok, k, partial.data_ptr(), _lib.FK_BF16, st)
            back = ex.all_to_all(partial)
            back_p = back.data_ptr()
        out = torch.empty(T, d, **bf)
        _lib.call("fk_ep_unpack_sum", back_p, d, src_pos.data_ptr(), T, N, out.data_ptr(),
                  _lib.FK_BF16, st)
        ctx.save_for_backward(xs, h1, act, idx, src_pos, send_token)
        ctx.plan = plan
        ctx.layer = layer
        ctx.dims = (T, d, k, N, El, H, E)
        return out

    @staticmethod
    def backward(ctx, dout):
        xs, h1, act, idx, src_pos, send_token = ctx.saved_tensors
        plan, layer = ctx.plan, ctx.layer
        T, d, k, N, El, H, E = ctx.dims
        ex = layer.exchange
        dev = xs.device
        st = _lib.stream_of(xs)
        R = plan.max_rows
        R_tok = N * T
        eptr = plan.err.data_ptr()
        bf = dict(dtype=torch.bfloat16, device=dev)
        dout = dout.to(torch.bfloat16).contiguous()
        px = layer._peer(T, d, k, dev) if layer.transport == "peer" else None
        if px is not None:
            _lib.call("fk_ep_peer_put_rows", dout.data_ptr(), d, send_token.data_ptr(), T, N,
                      ex.rank, None, None, k, px.table("to_expert"), None, None,
                      px.table("flags"), px.PHASE_BWD_DISPATCH, px.ctl.data_ptr(),
                      _lib.FK_BF16, st)
            px.wait(px.PHASE_BWD_DISPATCH, st)
            recv_d_p = px.local("to_expert")
        else:
            send_d = torch.empty(R_tok, d, **bf)
            _lib.call("fk_ep_pack", dout.data_ptr(), d, send_token.data_ptr(), R_tok,
                      send_d.data_ptr(), _lib.FK_BF16, st)
            recv_d = ex.all_to_all(send_d)
            recv_d_p = recv_d.data_ptr()
        dy = torch.empty(R, d, **bf)
        dw_recv = torch.zeros(R_tok, k, dtype=torch.float32, device=dev)
        dh1 = torch.empty(R, 2 * H, **bf)
        dxs = torch.empty(R, d, **bf)
        dw13 = torch.empty(El, 2 * H, d, **bf)
        dw2 = torch.empty(El, d, H, **bf)
        te, nm = plan.tile_expert.data_ptr(), plan.n_mblk.data_ptr()
        seg = plan.seg_start.data_ptr()
        # dy: the received output-gradient rows, unweighted; the down-projection's input
        # gradient applies the routing weight and forms the routing-weight gradient
        sa, sw = plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr()
        _lib.call("fk_moe_gather_by_token", recv_d_p, d, plan.slot_pos.data_ptr(), R_tok, k, sa,
                  nm, R, dy.data_ptr(), _lib.FK_BF16, st)
        part = torch.empty(R, H // 64, dtype=torch.float32, device=dev)

        def wgrad(lo, hi, cap, which):
            """Weight gradients of stacked experts lo..hi-1 (dW2 or dW13)."""
            if hi <= lo:
                return
            if which == 2:
                _lib.call("fk_moe_gemm_wgrad", dy.data_ptr(), d, act.data_ptr(), H, R,
                          seg + 4 * lo, hi - lo, dw2[lo].data_ptr(), cap, eptr + 4, st)
            else:
                _lib.call("fk_moe_gemm_wgrad", dh1.data_ptr(), 2 * H, xs.data_ptr(), d, R,
                          seg + 4 * lo, hi - lo, dw13[lo].data_ptr(), cap, eptr + 4, st)

        # Replicated experts sit at the end of the stack.  Their weight gradients are
        # computed as soon as their inputs exist (dW2 right after dy, dW13 right after dh1)
        # and summed over the group by NCCL on its own stream, while the remaining GEMMs
        # run on a grid that leaves layer.overlap_sms SMs free for the collective.
        n_own = layer.n_owned
        rep = bool(layer.replicated) and N > 1
        cap = max(_lib.num_sms() - layer.overlap_sms, 1) if rep and layer.overlap_sms > 0 else 0
        red = []
        if rep:
            wgrad(n_own, El, 0, 2)
            red.append(dist.all_reduce(dw2[n_own:], group=ex.group, async_op=True))
        _lib.call("fk_moe_gemm_down_dgrad_weighted", dy.data_ptr(), R, d, layer.w2.data_ptr(),
                  H, El, te, nm, sa, sw, h1.data_ptr(), dh1.data_ptr(), part.data_ptr(), cap,
                  eptr + 4, st)
        _lib.call("fk_moe_dw_from_parts", part.data_ptr(), H, sa, nm, R, dw_recv.data_ptr(), st)
        if rep:
            wgrad(n_own, El, cap, 13)
            red.append(dist.all_reduce(dw13[n_own:], group=ex.group, async_op=True))
        _lib.call("fk_moe_gemm_up_dgrad", dh1.data_ptr(), R, H, layer.w13.data_ptr(), d, El,
                  te, nm, dxs.data_ptr(), cap, eptr + 4, st)
        # The input-gradient and routing-gradient exchange overlaps the owned experts'
        # weight-gradient GEMMs.
        if px is not None:
            _lib.call("fk_ep_peer_combine_put", dxs.data_ptr(), d, plan.slot_pos.data_ptr(), None,
                      T, N, ex.rank, k, dw_recv.data_ptr(), px.table("to_source"),
                      px.table("dw"), px.table("flags"), px.PHASE_BWD_COMBINE,
                      px.ctl.data_ptr(), _lib.FK_BF16, st)
        else:
            dx_part = torch.empty(R_tok, d, **bf)
            _lib.call("fk_moe_combine", dxs.data_ptr(), d, plan.slot_pos.data_ptr(), None, R_tok,
                      k, dx_part.data_ptr(), _lib.FK_BF16, st)
            back_dx, w1 = ex.all_to_all(dx_part, async_op=True)
            back_dw, w2 = ex.all_to_all(dw_recv, async_op=True)
        own_hi = n_own if rep else El
        wgrad(0, own_hi, cap, 2)
        wgrad(0, own_hi, cap, 13)
        for wk in red:
            wk.wait()
        if px is not None:
            px.wait(px.PHASE_BWD_COMBINE, st)
            back_dx_p, back_dw_p = px.local("to_source"), px.local("dw")
        else:
            w1.wait()
            w2.wait()
            back_dx_p, back_dw_p = back_dx.data_ptr(), back_dw.data_ptr()
        dx = torch.empty(T, d, **bf)
        _lib.call("fk_ep_unpack_sum", back_dx_p, d, src_pos.data_ptr(), T, N,
                  dx.data_ptr(), _lib.FK_BF16, st)
        dw = torch.empty(T, k, dtype=torch.float32, device=dev)
        _lib.call("fk_ep_unpack_dw", back_dw_p, idx.data_ptr(),
                  layer.expert_rank.data_ptr(), src_pos.data_ptr(), T, k, N, E, dw.data_ptr(), st)
        grads = []
        for e in range(El):
            grads += [dw13[e, :H], dw13[e, H:], dw2[e]]
        return (dx, dw, None, None, *grads)


class ExpertParallelMoEMLP(nn.Module):
    """``FusedMoEMLPSorted`` with its experts sharded over a process group (see module doc).

    placement: expert -> rank list (default ``round_robin_placement``).  replicated:
    experts held by every rank (their slots are computed on the token's own rank; their
    weight gradients are summed over the group inside backward, so every copy receives
    the full-batch gradient); their placement entries are ignored.  Every rank must
    construct the layer with the same placement and replicated set.

    overlap_sms: SMs the backward GEMMs leave free while the replicated experts' gradient
    all-reduce runs beside them (0: the GEMMs take every SM and the collective waits)."""

    def __init__(self, dim: int, hidden_dim: int, n_experts: int, k: int = 2, group=None,
                 placement=None, router_version: str = "v2", transport: str = "peer",
                 replicated=(), overlap_sms: int = 32):
        super().__init__()
        assert overlap_sms >= 0
        self.overlap_sms = int(overlap_sms)
        assert router_version == "v2"
        assert transport in ("peer", "nccl")
        self.transport = transport
        self._peer_ex = None
        self.dim, self.hidden_dim, self.n_experts, self.k = dim, hidden_dim, n_experts, k
        self.exchange = Exchange(group)
        N, r = self.exchange.world, self.exchange.rank
        placement = list(placement) if placement is not None else round_robin_placement(n_experts, N)
        self.replicated = sorted(set(int(e) for e in replicated))
        rep_set = set(self.replicated)
        assert len(placement) == n_experts
        assert all(0 <= placement[e] < N for e in range(n_experts) if e not in rep_set)
        assert all(0 <= e < n_experts for e in self.replicated)
        self.placement = placement
        self.local_ids, self.n_owned, rank_tab, local_tab = plan_tables(
            placement, self.replicated, N, r)
        self.router = nn.Linear(dim, n_experts, bias=False)
        self.experts = nn.ModuleDict({str(e): Expert(dim, hidden_dim) for e in self.local_ids})
        self.register_buffer("expert_rank", torch.tensor(rank_tab, dtype=torch.int32),
                             persistent=False)
        self.register_buffer("expert_local", torch.tensor(local_tab, dtype=torch.int32),
                             persistent=False)
        self._restack()

    def _expert_params(self):
        out = []
        for e in self.local_ids:
            ex = self.experts[str(e)]
            out += [ex.w_gate.weight, ex.w_up.weight, ex.w_down.weight]
        return out

    def _restack(self):
        El, H, D = len(self.local_ids), self.hidden_dim, self.dim
        p0 = self.router.weight
        with torch.no_grad():
            w13 = torch.empty(El, 2 * H, D, dtype=p0.dtype, device=p0.device)
            w2 = torch.empty(El, D, H, dtype=p0.dtype, device=p0.device)
            for i, e in enumerate(self.local_ids):
                ex = self.experts[str(e)]
                w13[i, :H].copy_(ex.w_gate.weight)
                w13[i, H:].copy_(ex.w_up.weight)
                w2[i].copy_(ex.w_down.weight)
                ex.w_gate.weight.data = w13[i, :H]
                ex.w_up.weight.data = w13[i, H:]
                ex.w_down.weight.data = w2[i]
        self.w13, self.w2 = w13, w2

    def _apply(self, fn, *args, **kwargs):
        r = super()._apply(fn, *args, **kwargs)
        self._restack()
        return r

    @torch.no_grad()
    def load_from_full(self, router_weight, w_gate, w_up, w_down):
        """Copy the router and this rank's experts out of full stacked weights
        (w_gate, w_up [E, H, D], w_down [E, D, H])."""
        self.router.weight.copy_(router_weight)
        for i, e in enumerate(self.local_ids):
            self.w13[i, :self.hidden_dim].copy_(w_gate[e])
            self.w13[i, self.hidden_dim:].copy_(w_up[e])
            self.w2[i].copy_(w_down[e])

    def _peer(self, n_tokens: int, dim: int, k: int, device) -> PeerExchange:
        """The peer-memory exchange for T = n_tokens per rank (created on first use; every
        rank must call with the same T)."""
        px = self._peer_ex
        if px is not None and px.key == (n_tokens, dim, k):
            return px
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("ExpertParallelMoEMLP: run one step eagerly before capturing "
                               "a CUDA graph (the peer exchange is set up on first use)")
        if px is not None:
            px.close()
        self._peer_ex = PeerExchange(self.exchange.group, n_tokens, dim, k, device)
        return self._peer_ex

    def close(self) -> None:
        """Collective: release the peer-memory exchange (before destroy_process_group)."""
        if self._peer_ex is not None:
            self._peer_ex.close()
            self._peer_ex = None

    def peer_error(self) -> int:
        """Device error flag of the peer transport (16 + phase after a wait timed out)."""
        return 0 if self._peer_ex is None else int(self._peer_ex.err.item())

    def allreduce_router_grad(self):
        g = self.router.weight.grad
        if g is not None and self.exchange.world > 1:
            dist.all_reduce(g, group=self.exchange.group)
            g.div_(self.exchange.world)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        assert x.is_cuda
        orig_shape = x.shape
        x_flat = x.reshape(-1, self.dim).contiguous()
        if x_flat.dtype != torch.bfloat16 or self.w13.dtype != torch.bfloat16:
            raise TypeError("ExpertParallelMoEMLP runs on bf16 tensor cores: use bfloat16")
        logits = self.router(x_flat)
        w, idx = fused_moe_route_v2(logits, self.k)
        out = _EPMoEFn.apply(x_flat, w, idx, self, *self._expert_params())
        return out.reshape(orig_shape)
