"""SwiGLU kernels vs the oracle (F.silu(g)*u in fp64) and vs the reference kernels' golden
vectors.  Tolerances: fp32 atol=rtol=1e-5; bf16/fp16 outputs atol=rtol=1e-2 (rounding of
the 16-bit result)."""
import pytest
import torch

import fusedkernels_b200 as fk
from oracle import swiglu_oracle
from conftest import gen

pytestmark = pytest.mark.gpu
TOL = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (1e-2, 1e-2), torch.float16: (1e-2, 1e-2)}


def run(gate, up, dout):
    g = gate.cuda().requires_grad_(True)
    u = up.cuda().requires_grad_(True)
    out = fk.fused_swiglu(g, u)
    out.backward(dout.cuda())
    return out.detach().cpu(), g.grad.cpu(), u.grad.cpu()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2048, 4096), (37, 211), (1,), (3, 5, 7)])
def test_swiglu_matches_oracle(dtype, shape):
    G = gen(3)
    gate, up, dout = (torch.randn(*shape, generator=G).to(dtype) for _ in range(3))
    out, dg, du = run(gate, up, dout)
    ro, rdg, rdu = swiglu_oracle(gate, up, dout)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(out.double(), ro.to(dtype).double(), atol=atol, rtol=rtol)
    torch.testing.assert_close(dg.double(), rdg.to(dtype).double(), atol=atol, rtol=rtol)
    torch.testing.assert_close(du.double(), rdu.to(dtype).double(), atol=atol, rtol=rtol)


def test_swiglu_unaligned_views():
    G = gen(4)
    base = torch.randn(3, 1003, generator=G).cuda()
    gate, up = base[0, 1:1000], base[1, 3:1002]  # offsets break 16-byte alignment
    out = fk.fused_swiglu(gate, up)
    ref = swiglu_oracle(gate.cpu(), up.cpu())
    torch.testing.assert_close(out.cpu().double(), ref, atol=1e-5, rtol=1e-5)


def test_swiglu_matches_reference_golden(golden):
    for tag in ("a", "b"):
        p = f"swiglu_{tag}_"
        out, dg, du = run(*(torch.from_numpy(golden[p + k]) for k in ("gate", "up", "dout")))
        torch.testing.assert_close(out, torch.from_numpy(golden[p + "out"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dg, torch.from_numpy(golden[p + "dgate"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(du, torch.from_numpy(golden[p + "dup"]), atol=1e-5, rtol=1e-5)


def test_swiglu_full_size_sampled():
    """Workload shape [16384, 14336] bf16: every element computed, 2^16 sampled checked."""
    G = gen(5)
    shape = (16384, 14336)
    gate = torch.randn(*shape, generator=G, dtype=torch.bfloat16).cuda()
    up = torch.randn(*shape, generator=G, dtype=torch.bfloat16).cuda()
    dout = torch.randn(*shape, generator=G, dtype=torch.bfloat16).cuda()
    g = gate.requires_grad_(True)
    u = up.requires_grad_(True)
    out = fk.fused_swiglu(g, u)
    out.backward(dout)
    sel = torch.randint(0, gate.numel(), (1 << 16,), generator=G).cuda()
    flat = lambda t: t.detach().reshape(-1)[sel].cpu()
    ro, rdg, rdu = swiglu_oracle(flat(gate), flat(up), flat(dout))
    for got, ref in [(flat(out), ro), (flat(g.grad), rdg), (flat(u.grad), rdu)]:
        torch.testing.assert_close(got.double(), ref.to(torch.bfloat16).double(), atol=1e-2, rtol=1e-2)
    assert torch.isfinite(out).all()
