"""fk_rmsnorm_bwd_noalloc: the RMSNorm backward for callers that cannot allocate device
memory (they only hold tensors handed to them, or run under a fixed memory budget), so
they cannot give fk_rmsnorm_bwd its workspace.  This file is collected last on purpose.

Called through the C ABI twice in a row; each result is compared with fk_rmsnorm_bwd
(with a torch-allocated workspace) on the same inputs: dx exactly, dw within the RMSNorm
weight-gradient tolerance of the other tests (atol 1e-4 / rtol 1e-5 fp32 weights from
fp32 inputs, atol = rtol = 1e-3 from 16-bit inputs)."""
import pytest
import torch

from fusedkernels_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(rows, cols, dtype, seed):
    G = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=G).to(dtype).to(DEV)
    dy = torch.randn(rows, cols, generator=G).to(dtype).to(DEV)
    w = (1.0 + 0.02 * torch.randn(cols, generator=G)).to(DEV)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    return x, dy, w, rstd


def _with_workspace(x, dy, w, rstd):
    rows, cols = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    ws = torch.empty(max(_lib.rmsnorm_bwd_workspace_bytes(rows, cols, x.device), 16),
                     dtype=torch.uint8, device=DEV)
    _lib.call("fk_rmsnorm_bwd", dy.data_ptr(), x.data_ptr(), w.data_ptr(), _lib.FK_F32,
              rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), ws.data_ptr(), ws.numel(), rows, cols,
              _lib.dtype_code(x.dtype), torch.cuda.current_stream().cuda_stream)
    return dx, dw


def _no_alloc(x, dy, w, rstd):
    rows, cols = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    _lib.call("fk_rmsnorm_bwd_noalloc", dy.data_ptr(), x.data_ptr(), w.data_ptr(), _lib.FK_F32,
              rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows, cols,
              _lib.dtype_code(x.dtype), torch.cuda.current_stream().cuda_stream)
    return dx, dw


# 4096 x 16384 bf16 and 1024 x 65536 fp32 need more partial rows than the fixed scratch
# holds (128 and 32 fit), so the grid is capped below one CTA per SM there.
@pytest.mark.parametrize("rows,cols,dtype", [(4096, 4096, torch.bfloat16), (1000, 1024, torch.float16),
                                             (300, 301, torch.float32), (7, 40000, torch.float32),
                                             (4096, 16384, torch.bfloat16),
                                             (1024, 65536, torch.float32)])
def test_no_alloc_matches_workspace_entry_point_twice(rows, cols, dtype):
    x, dy, w, rstd = _inputs(rows, cols, dtype, rows + cols)
    ref_dx, ref_dw = _with_workspace(x, dy, w, rstd)
    tol = dict(atol=1e-4, rtol=1e-5) if dtype == torch.float32 else dict(atol=1e-3, rtol=1e-3)
    for _ in range(2):  # the fixed scratch keeps the previous call's contents
        dx, dw = _no_alloc(x, dy, w, rstd)
        torch.cuda.synchronize()
        assert torch.equal(dx, ref_dx)
        torch.testing.assert_close(dw, ref_dw, **tol)


def test_no_alloc_rejects_too_many_columns():
    lib = _lib.load()
    st = lib.fk_rmsnorm_bwd_noalloc(None, None, 1, 0, None, None, 1, 4, (8 << 20) // 4 + 1, 0, None)
    assert st == 2 and b"fixed scratch" in lib.fk_last_error()
