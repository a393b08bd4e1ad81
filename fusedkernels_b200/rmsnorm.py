"""Fused RMSNorm forward + backward.

Mirrors fusedkernels/rmsnorm.py (``_FusedRMSNormFn`` at rmsnorm.py:74-113,
``FusedRMSNorm`` at rmsnorm.py:116-125): y = x * rsqrt(mean(x^2) + eps) * weight with
fp32 accumulation, output in x's dtype, weight an fp32 ``ones`` parameter by default and
its gradient returned in the weight's dtype.  The weight gradient is reduced on the
device in a fixed order (per-CTA partial rows + a column reduce), replacing the
[rows, cols] fp32 partial and torch ``.sum(0)`` of rmsnorm.py:104 and :112.
"""
import torch
import torch.nn as nn

from . import _lib


class _FusedRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        assert x.is_cuda and weight.is_cuda
        orig_shape = x.shape
        x2 = x.reshape(-1, orig_shape[-1]).contiguous()
        n_rows, n_cols = x2.shape
        assert weight.numel() == n_cols
        w = weight.contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(n_rows, dtype=torch.float32, device=x.device)
        _lib.call("fk_rmsnorm_fwd", x2.data_ptr(), n_cols, w.data_ptr(),
                  _lib.dtype_code(w.dtype), y.data_ptr(), n_cols, rstd.data_ptr(), n_rows,
                  n_cols, float(eps), _lib.dtype_code(x2.dtype), _lib.stream_of(x2))
        ctx.save_for_backward(x2, w, rstd)
        ctx.orig_shape = orig_shape
        ctx.weight_shape = weight.shape
        return y.reshape(orig_shape)

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        n_rows, n_cols = x.shape
        dy2 = dy.reshape(-1, n_cols).to(x.dtype).contiguous()
        dx = torch.empty_like(x)
        dw = torch.empty(n_cols, dtype=w.dtype, device=x.device)
        ws_bytes = _lib.rmsnorm_bwd_workspace_bytes(n_rows, n_cols, x.device)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
        _lib.call("fk_rmsnorm_bwd", dy2.data_ptr(), x.data_ptr(), w.data_ptr(),
                  _lib.dtype_code(w.dtype), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                  ws.data_ptr(), ws.numel(), n_rows, n_cols, _lib.dtype_code(x.dtype),
                  _lib.stream_of(x))
        return dx.reshape(ctx.orig_shape), dw.reshape(ctx.weight_shape), None


class FusedRMSNorm(nn.Module):
    """Drop-in replacement for LlamaRMSNorm / nn.RMSNorm."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _FusedRMSNormFn.apply(x, self.weight, self.eps)
