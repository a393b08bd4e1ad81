"""Generate MoE-layer golden vectors by running the reference's own layer oracle on the CPU.

The reference checks its sorted-dispatch layer against ``NaiveMoEMLP``
(tests/test_moe_sorted_dispatch.py:12-40), a plain PyTorch module built around the
reference's ``Expert`` (fusedkernels/moe_layer.py:22-31).  Neither needs a GPU, so this
script imports both from the reference checkout, runs them forward and backward in fp64 on
seeded inputs, and stores inputs, outputs and every gradient in ``golden_moe.npz``:

  x [N, D], router weight [E, D], stacked expert weights w_gate/w_up [E, H, D] and
  w_down [E, D, H] (fp32 values, computed in fp64), upstream gradient dout [N, D];
  out, dx (router path included), router weight gradient, stacked expert gradients
  (fp64 results stored rounded to fp32).

Inputs are continuous random values, so no two logits of a row tie and the reference's
``torch.topk`` selects the same experts as a stable descending sort.  Expert weights are
drawn at the reference's ``nn.Linear`` default scale (U(-1/sqrt(fan_in), 1/sqrt(fan_in))).

    python tests/golden/make_moe_golden.py <path-to-reference-checkout>

Only this generator reads the reference checkout; the tests read ``golden_moe.npz``.
"""
import importlib.util
import os
import sys

if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_moe_golden.py <path-to-reference-checkout>")
REF = sys.argv[1]
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from fusedkernels.moe_layer import Expert  # noqa: E402

_spec = importlib.util.spec_from_file_location(
    "ref_test_moe_sorted_dispatch", os.path.join(REF, "tests", "test_moe_sorted_dispatch.py"))
_mod = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_mod)
NaiveMoEMLP = _mod.NaiveMoEMLP

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_moe.npz")
data = {}


def uniform(g, shape, fan_in):
    b = fan_in ** -0.5
    return (torch.rand(*shape, generator=g) * 2 - 1) * b


def gold_moe(tag, n, D, H, E, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, D, generator=g)
    wr = uniform(g, (E, D), D)
    wg = uniform(g, (E, H, D), D)
    wu = uniform(g, (E, H, D), D)
    wd = uniform(g, (E, D, H), H)
    dout = torch.randn(n, D, generator=g)
    experts = torch.nn.ModuleList([Expert(D, H) for _ in range(E)]).double()
    with torch.no_grad():
        for e, ex in enumerate(experts):
            ex.w_gate.weight.copy_(wg[e])
            ex.w_up.weight.copy_(wu[e])
            ex.w_down.weight.copy_(wd[e])
    layer = NaiveMoEMLP(D, H, E, k, experts).double()
    with torch.no_grad():
        layer.router.weight.copy_(wr)
    xx = x.double().requires_grad_(True)
    out = layer(xx)
    out.backward(dout.double())

    def grad(p):
        return p.grad if p.grad is not None else torch.zeros_like(p)

    res = dict(x=x, wr=wr, wg=wg, wu=wu, wd=wd, dout=dout, out=out.detach(), dx=xx.grad,
               dwr=layer.router.weight.grad,
               dwg=torch.stack([grad(ex.w_gate.weight) for ex in experts]),
               dwu=torch.stack([grad(ex.w_up.weight) for ex in experts]),
               dwd=torch.stack([grad(ex.w_down.weight) for ex in experts]))
    for key, v in res.items():  # inputs are fp32 values; fp64 results are rounded to fp32
        data[f"moe_{tag}_{key}"] = v.detach().float().numpy()
    data[f"moe_{tag}_k"] = np.int64(k)


if __name__ == "__main__":
    # (E, k) pairs of the reference's layer test (tests/test_moe_sorted_dispatch.py:43) at
    # small dims, plus the many-empty-experts case of its second test (:72-82).
    # e8k2 has tile-aligned dims (multiples of 64), so the GPU layer runs on it directly.
    gold_moe("e8k2", n=64, D=64, H=64, E=8, k=2, seed=10)
    gold_moe("e32k4", n=96, D=16, H=16, E=32, k=4, seed=11)
    gold_moe("e64k8", n=64, D=16, H=8, E=64, k=8, seed=12)
    gold_moe("e128k16", n=32, D=8, H=8, E=128, k=16, seed=13)
    gold_moe("empty", n=4, D=16, H=8, E=64, k=2, seed=14)
    data["meta_torch_version"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(data)} arrays, {os.path.getsize(OUT)} bytes")
