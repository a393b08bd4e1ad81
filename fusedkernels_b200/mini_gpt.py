"""Small GPT training harness wiring the fused ops into a model (end-to-end integration).

Mirrors fusedkernels' examples/train_mini_gpt.py (MiniGPT at train_mini_gpt.py:81-110 with
RMSNorm, a SwiGLU MLP and the cross-entropy loss, and the fused / native toggle of
train_mini_gpt.py:60-105): ``fused=True`` uses ``FusedRMSNorm``, ``fused_swiglu`` and
``fused_cross_entropy`` (gradient written in place over the logits); ``fused=False`` uses
the eager PyTorch formulation of the same ops.  Attention and the linear layers are
PyTorch's (SDPA / cuBLAS) in both modes.

``train_step`` runs forward, backward and an AdamW step; ``python -m
fusedkernels_b200.mini_gpt --mode fused`` prints tokens/s.  Under torchrun every rank trains
its own batch and DistributedDataParallel all-reduces the gradients of the replicated
parameters (data parallelism); tokens/s is then the sum over ranks.
"""
from __future__ import annotations

import argparse
import os
import time

import torch
import torch.nn as nn
import torch.nn.functional as F

from .cross_entropy import fused_cross_entropy
from .rmsnorm import FusedRMSNorm
from .swiglu import fused_swiglu


class RefRMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        var = x.float().pow(2).mean(-1, keepdim=True)
        return (x.float() * torch.rsqrt(var + self.eps) * self.weight.float()).to(x.dtype)


class CausalSelfAttention(nn.Module):
    def __init__(self, dim, n_heads):
        super().__init__()
        self.n_heads = n_heads
        self.head_dim = dim // n_heads
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.proj = nn.Linear(dim, dim, bias=False)

    def forward(self, x):
        B, T, D = x.shape
        qkv = self.qkv(x).view(B, T, 3, self.n_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        out = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], is_causal=True)
        return self.proj(out.transpose(1, 2).reshape(B, T, D))


class MLP(nn.Module):
    def __init__(self, dim, hidden_dim, fused: bool):
        super().__init__()
        self.fused = fused
        self.w_gate = nn.Linear(dim, hidden_dim, bias=False)
        self.w_up = nn.Linear(dim, hidden_dim, bias=False)
        self.w_down = nn.Linear(hidden_dim, dim, bias=False)

    def forward(self, x):
        g, u = self.w_gate(x), self.w_up(x)
        return self.w_down(fused_swiglu(g, u) if self.fused else F.silu(g) * u)


class Block(nn.Module):
    def __init__(self, dim, n_heads, hidden_dim, fused: bool):
        super().__init__()
        Norm = FusedRMSNorm if fused else RefRMSNorm
        self.norm1, self.norm2 = Norm(dim), Norm(dim)
        self.attn = CausalSelfAttention(dim, n_heads)
        self.mlp = MLP(dim, hidden_dim, fused)

    def forward(self, x):
        x = x + self.attn(self.norm1(x))
        return x + self.mlp(self.norm2(x))


class MiniGPT(nn.Module):
    def __init__(self, vocab_size=32000, dim=1024, n_layers=12, n_heads=16, hidden_dim=2752,
                 max_seq_len=1024, fused: bool = True):
        super().__init__()
        self.fused = fused
        self.tok_emb = nn.Embedding(vocab_size, dim)
        self.pos_emb = nn.Embedding(max_seq_len, dim)
        self.blocks = nn.ModuleList([Block(dim, n_heads, hidden_dim, fused) for _ in range(n_layers)])
        self.norm_f = (FusedRMSNorm if fused else RefRMSNorm)(dim)
        self.lm_head = nn.Linear(dim, vocab_size, bias=False)

    def forward(self, idx, targets):
        B, T = idx.shape
        x = self.tok_emb(idx) + self.pos_emb(torch.arange(T, device=idx.device))[None]
        for blk in self.blocks:
            x = blk(x)
        logits = self.lm_head(self.norm_f(x)).reshape(B * T, -1)
        t = targets.reshape(-1)
        if self.fused:
            return fused_cross_entropy(logits, t, inplace_grad=True)
        return F.cross_entropy(logits.float(), t)


def train_step(model, opt, x, y):
    loss = model(x, y)
    loss.backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return loss


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["fused", "native"], default="fused")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=1024)
    ap.add_argument("--dim", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=12)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=dev)
    torch.manual_seed(0)  # identical initial weights on every rank
    model = MiniGPT(dim=args.dim, n_layers=args.layers, hidden_dim=args.dim * 43 // 16,
                    max_seq_len=args.seq_len, fused=args.mode == "fused").to(dev, torch.bfloat16)
    V = model.lm_head.out_features
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[dev.index])
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4)
    torch.manual_seed(1000 + rank)  # each rank draws its own batches
    for _ in range(args.warmup):
        idx = torch.randint(0, V, (args.batch_size, args.seq_len + 1), device=dev)
        train_step(model, opt, idx[:, :-1], idx[:, 1:])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        idx = torch.randint(0, V, (args.batch_size, args.seq_len + 1), device=dev)
        loss = train_step(model, opt, idx[:, :-1], idx[:, 1:])
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt = float(t.item())
    if rank == 0:
        tok = world * args.steps * args.batch_size * args.seq_len
        print(f"mode={args.mode} ranks={world} tokens/s={tok / dt:,.0f} loss={loss.item():.4f}")
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
