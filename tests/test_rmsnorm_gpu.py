"""RMSNorm kernels vs the oracle (RefRMSNorm in fp64) and the reference kernels' golden
vectors.  Tolerances: fp32 y/dx atol=rtol=1e-5, dw atol 1e-4 rtol 1e-5; bf16 y/dx
atol=rtol=1e-2 against the fp64 oracle rounded to bf16, dw rtol 1e-3."""
import pytest
import torch

import fusedkernels_b200 as fk
from oracle import rmsnorm_oracle
from conftest import gen

pytestmark = pytest.mark.gpu


def run(x, w, dy, eps=1e-6):
    norm = fk.FusedRMSNorm(x.shape[-1], eps=eps).cuda()
    with torch.no_grad():
        norm.weight.data = w.cuda()
    xg = x.cuda().requires_grad_(True)
    y = norm(xg)
    y.backward(dy.cuda())
    return y.detach().cpu(), xg.grad.cpu(), norm.weight.grad.cpu()


@pytest.mark.parametrize("shape", [(4, 128, 4096), (24, 320), (7, 301), (3, 8192), (5, 40000)])
def test_rmsnorm_fp32_matches_oracle(shape):
    G = gen(2)
    x = torch.randn(*shape, generator=G)
    w = 1.0 + 0.02 * torch.randn(shape[-1], generator=G)
    dy = torch.randn(*shape, generator=G)
    y, dx, dw = run(x, w, dy)
    ry, rdx, rdw = rmsnorm_oracle(x, w, 1e-6, dy)
    torch.testing.assert_close(y.double(), ry, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(dx.double(), rdx, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(dw.double(), rdw, atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cols", [4096, 1024, 8192, 200])
def test_rmsnorm_16bit_matches_oracle(dtype, cols):
    G = gen(7)
    x = torch.randn(256, cols, generator=G).to(dtype)
    w = 1.0 + 0.02 * torch.randn(cols, generator=G)
    dy = torch.randn(256, cols, generator=G).to(dtype)
    y, dx, dw = run(x, w, dy)
    assert y.dtype == dtype and dx.dtype == dtype and dw.dtype == torch.float32
    ry, rdx, rdw = rmsnorm_oracle(x, w, 1e-6, dy)
    torch.testing.assert_close(y.double(), ry.to(dtype).double(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(dx.double(), rdx.to(dtype).double(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(dw.double(), rdw, atol=1e-3, rtol=1e-3)


def test_rmsnorm_bf16_weight_dtype():
    G = gen(8)
    x = torch.randn(64, 512, generator=G).bfloat16()
    w = (1.0 + 0.02 * torch.randn(512, generator=G)).bfloat16()
    dy = torch.randn(64, 512, generator=G).bfloat16()
    y, dx, dw = run(x, w, dy)
    assert dw.dtype == torch.bfloat16
    ry, rdx, rdw = rmsnorm_oracle(x, w, 1e-6, dy)
    torch.testing.assert_close(dw.double(), rdw.bfloat16().double(), atol=2e-2, rtol=1e-2)


def test_rmsnorm_matches_reference_golden(golden):
    for tag in ("a", "b"):
        p = f"rmsnorm_{tag}_"
        t = lambda k: torch.from_numpy(golden[p + k])
        y, dx, dw = run(t("x"), t("w"), t("dy"), float(golden[p + "eps"]))
        torch.testing.assert_close(y, t("y"), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dx, t("dx"), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dw, t("dw"), atol=1e-4, rtol=1e-5)


def test_rmsnorm_dw_deterministic():
    G = gen(9)
    x = torch.randn(4096, 4096, generator=G).bfloat16()
    w = torch.ones(4096)
    dy = torch.randn(4096, 4096, generator=G).bfloat16()
    outs = [run(x, w, dy) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o[2], outs[0][2]) and torch.equal(o[1], outs[0][1])


def test_rmsnorm_full_size_sampled_rows():
    """Workload [16384, 4096] bf16, weight 1+N(0,0.02): 128 sampled rows vs the oracle, dw
    against the fp64 oracle over all rows."""
    G = gen(10)
    x = torch.randn(16384, 4096, generator=G).bfloat16()
    w = 1.0 + 0.02 * torch.randn(4096, generator=G)
    dy = torch.randn(16384, 4096, generator=G).bfloat16()
    y, dx, dw = run(x, w, dy)
    rows = torch.randint(0, 16384, (128,), generator=G)
    ry, rdx, _ = rmsnorm_oracle(x[rows], w, 1e-6, dy[rows])
    torch.testing.assert_close(y[rows].double(), ry.bfloat16().double(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(dx[rows].double(), rdx.bfloat16().double(), atol=1e-2, rtol=1e-2)
    rstd = torch.rsqrt(x.double().pow(2).mean(-1, keepdim=True) + 1e-6)
    rdw = (dy.double() * x.double() * rstd).sum(0)
    torch.testing.assert_close(dw.double(), rdw, atol=1e-3, rtol=1e-3)
