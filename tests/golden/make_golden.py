"""Generate golden vectors by running the reference's own Triton kernels on the CPU.

The fusedkernels reference (Siddhuuuu/fusedKernels v0.2.0) is pure Python + Triton.  Its
autograd wrappers assert ``is_cuda``, so this script calls the ``@triton.jit`` kernels
directly, with the launch arguments the wrappers use, under ``TRITON_INTERPRET=1``
(Triton's CPU interpreter).  Outputs are stored with their inputs in ``golden.npz``.

    python tests/golden/make_golden.py <path-to-reference-checkout>

Only this generator reads the reference checkout; the tests read ``golden.npz``.
"""
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_golden.py <path-to-reference-checkout>")
REF = sys.argv[1]
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402

from fusedkernels import cross_entropy, moe_routing_v2, rmsnorm, swiglu  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
g = torch.Generator().manual_seed(1234)
data = {}


def randn(*shape, scale=1.0):
    return torch.randn(*shape, generator=g) * scale


# --- SwiGLU (swiglu.py:56-81 launch arguments) -------------------------------------
def gold_swiglu(tag, shape):
    gate, up, dout = randn(*shape), randn(*shape), randn(*shape)
    n = gate.numel()
    out, dgate, dup = torch.empty_like(gate), torch.empty_like(gate), torch.empty_like(gate)
    grid = (triton.cdiv(n, 1024),)
    swiglu._swiglu_fwd_kernel[grid](gate, up, out, n, BLOCK_SIZE=1024)
    swiglu._swiglu_bwd_kernel[grid](dout, gate, up, dgate, dup, n, BLOCK_SIZE=1024)
    for k, v in dict(gate=gate, up=up, dout=dout, out=out, dgate=dgate, dup=dup).items():
        data[f"swiglu_{tag}_{k}"] = v.numpy()


# --- RMSNorm (rmsnorm.py:76-113 launch arguments) -----------------------------------
def gold_rmsnorm(tag, rows, cols, eps=1e-6):
    x, dy = randn(rows, cols), randn(rows, cols)
    w = 1.0 + randn(cols, scale=0.02)
    y, rstd = torch.empty_like(x), torch.empty(rows)
    block = triton.next_power_of_2(cols)
    rmsnorm._rmsnorm_fwd_kernel[(rows,)](x, w, y, rstd, x.stride(0), y.stride(0), cols, eps,
                                         BLOCK_SIZE=block)
    dx, dwp = torch.empty_like(x), torch.empty(rows, cols)
    rmsnorm._rmsnorm_bwd_kernel[(rows,)](dy, x, w, rstd, dx, dwp, dy.stride(0), x.stride(0),
                                         dx.stride(0), dwp.stride(0), cols, BLOCK_SIZE=block)
    dw = dwp.sum(0)
    for k, v in dict(x=x, w=w, dy=dy, y=y, rstd=rstd, dx=dx, dw=dw).items():
        data[f"rmsnorm_{tag}_{k}"] = v.numpy()
    data[f"rmsnorm_{tag}_eps"] = np.float32(eps)


# --- Cross-entropy (cross_entropy.py:83-116 launch + the backward scale) ------------
def gold_ce(tag, rows, cols, ls=0.0, ignore_every=0, scale=1.0):
    logits = randn(rows, cols, scale=scale)
    targets = torch.randint(0, cols, (rows,), generator=g)
    if ignore_every:
        targets[::ignore_every] = -100
    loss_rows, grad = torch.empty(rows), torch.empty_like(logits)
    block = min(triton.next_power_of_2(cols), 16384)
    cross_entropy._cross_entropy_fwd_bwd_kernel[(rows,)](
        logits, targets, loss_rows, grad, logits.stride(0), grad.stride(0), cols, -100, ls,
        BLOCK_SIZE=block)
    n_valid = (targets != -100).sum().clamp(min=1)
    loss = loss_rows.sum() / n_valid
    grad_final = grad * (torch.ones(()) / n_valid)  # backward with grad_output = 1
    for k, v in dict(logits=logits, targets=targets, loss=loss, grad=grad_final).items():
        data[f"ce_{tag}_{k}"] = v.numpy()
    data[f"ce_{tag}_ls"] = np.float32(ls)


# --- Router v2 (moe_routing_v2.py:131-177 launch arguments) -------------------------
def gold_router(E, k, rows=48):
    logits, dw = randn(rows, E), randn(rows, k)
    block, block_k = triton.next_power_of_2(E), triton.next_power_of_2(k)
    w = torch.empty(rows, k)
    idx = torch.empty(rows, k, dtype=torch.int32)
    moe_routing_v2._moe_route_fwd_kernel_v2[(rows,)](
        logits, w, idx, logits.stride(0), E, SCALE=moe_routing_v2._SCALE,
        TANH_TEMP=moe_routing_v2._TANH_TEMP, K=k, BLOCK_SIZE=block, BLOCK_K=block_k)
    dlogits = torch.zeros(rows, E)
    moe_routing_v2._moe_route_bwd_kernel_v2[(rows,)](dw, w, idx, dlogits, E, K=k,
                                                     BLOCK_K=block_k)
    tag = f"E{E}_k{k}"
    for kk, v in dict(logits=logits, dw=dw, w=w, idx=idx, dlogits=dlogits).items():
        data[f"router_{tag}_{kk}"] = v.numpy()


if __name__ == "__main__":
    gold_swiglu("a", (37, 211))
    gold_swiglu("b", (2, 4096))
    gold_rmsnorm("a", 24, 320)
    gold_rmsnorm("b", 4, 4096)
    gold_ce("a", 48, 1500, ignore_every=7)
    gold_ce("smooth", 32, 777, ls=0.1)
    gold_ce("wide", 3, 20000, ignore_every=3, scale=2.0)
    for E, k in [(8, 2), (64, 2), (64, 8), (128, 8), (128, 16)]:
        gold_router(E, k)
    data["meta_triton_version"] = np.array(triton.__version__)
    data["meta_torch_version"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(data)} arrays, {os.path.getsize(OUT)} bytes")
