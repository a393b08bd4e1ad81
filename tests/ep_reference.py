"""Python restatement of the expert-parallel exchange protocol (test helper).

Mirrors fk_ep_plan / fk_ep_pack / fk_ep_unpack_sum / fk_ep_unpack_dw and the expert-side
pre-reduction of fusedkernels_b200/moe_ep.py on CPU tensors, so the protocol can be
checked with real gloo collectives and the CUDA kernels can be checked against it."""
import torch


def ep_plan(idx, w, expert_rank, expert_local, n_ranks):
    T, k = idx.shape
    send_token = torch.full((n_ranks * T,), -1, dtype=torch.int32)
    send_e = torch.full((n_ranks * T, k), -1, dtype=torch.int32)
    send_w = torch.zeros(n_ranks * T, k)
    src_pos = torch.full((T, n_ranks), -1, dtype=torch.int32)
    count = torch.zeros(n_ranks, dtype=torch.int32)
    ranks = expert_rank[idx]  # [T, k]
    for d in range(n_ranks):
        pos = 0
        for t in range(T):
            mine = ranks[t] == d
            if not bool(mine.any()):
                continue
            r = d * T + pos
            send_token[r] = t
            send_e[r] = torch.where(mine, expert_local[idx[t]], torch.tensor(-1)).to(torch.int32)
            send_w[r] = w[t]
            src_pos[t, d] = pos
            pos += 1
        count[d] = pos
    return send_token, send_e, send_w, src_pos, count


def ep_pack(x, send_token):
    out = torch.zeros(send_token.numel(), x.shape[1], dtype=x.dtype)
    ok = send_token >= 0
    out[ok] = x[send_token[ok].long()]
    return out


def ep_unpack_sum(back, src_pos, T):
    n_ranks = src_pos.shape[1]
    out = torch.zeros(T, back.shape[1], dtype=torch.float64)
    for t in range(T):
        for d in range(n_ranks):
            p = int(src_pos[t, d])
            if p >= 0:
                out[t] += back[d * T + p].double()
    return out


def ep_unpack_dw(back_dw, idx, expert_rank, src_pos):
    T, k = idx.shape
    dw = torch.zeros(T, k)
    for t in range(T):
        for j in range(k):
            d = int(expert_rank[idx[t, j]])
            p = int(src_pos[t, d])
            if p >= 0:
                dw[t, j] = back_dw[d * T + p, j]
    return dw


def expert_side(recv_x, recv_e, recv_w, w_gate, w_up, w_down):
    """Pre-reduced partial rows: sum over a row's local slots of w * Expert(x), fp64."""
    F = torch.nn.functional
    out = torch.zeros(recv_x.shape[0], recv_x.shape[1], dtype=torch.float64)
    for r in range(recv_x.shape[0]):
        for j in range(recv_e.shape[1]):
            e = int(recv_e[r, j])
            if e < 0:
                continue
            xr = recv_x[r].double()
            h = F.silu(w_gate[e].double() @ xr) * (w_up[e].double() @ xr)
            out[r] += float(recv_w[r, j]) * (w_down[e].double() @ h)
    return out
