"""Fused cross-entropy loss (mean over non-ignored rows) with its gradient.

Mirrors fusedkernels/cross_entropy.py (``_FusedCrossEntropy`` at cross_entropy.py:82-116,
``fused_cross_entropy`` at cross_entropy.py:119-123): same arguments, same AssertionError
preconditions, loss = sum of per-row losses / max(1, #non-ignored targets), optional
label smoothing, ignored rows contribute 0 loss and a zero gradient row.

The forward pass already produces the gradient (one HBM read of the logits, one write
of the gradient, with 1/n_valid folded in); backward only rescales it when the incoming
grad_output differs from 1, which the device decides without a host sync.

``inplace_grad=True`` writes the gradient over the logits buffer (no second
[N, V] allocation); the logits tensor must not be read again after the call.
An out-of-range target (not ignore_index) makes the loss NaN; ``last_target_error()``
reads the device error flag of the most recent call (this synchronises).

``fused_cross_entropy_global_mean`` is the data-parallel form: every rank holds a shard of
the batch's rows, and the loss is the mean over the non-ignored rows of ALL ranks.  The
reference's mean is loss_rows.sum() / n_valid (cross_entropy.py:107-110); sharded, that
needs one all-reduce of the two scalars (sum of row losses, count of valid rows), after
which each rank's gradient is rescaled from its local 1/n_valid to the global one.
"""
import torch
import torch.distributed as dist

from . import _lib

_last_err = None


class _FusedCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index=-100, label_smoothing=0.0, inplace_grad=False):
        global _last_err
        assert logits.is_cuda and logits.ndim == 2
        n_rows, n_cols = logits.shape
        assert targets.shape == (n_rows,)
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        targets = targets.to(device=logits.device, dtype=torch.int64).contiguous()
        dev = logits.device
        grad = logits if inplace_grad else torch.empty_like(logits)
        loss_rows = torch.empty(n_rows, dtype=torch.float32, device=dev)
        loss = torch.empty((), dtype=torch.float32, device=dev)
        flags = torch.empty(2, dtype=torch.int32, device=dev)  # [n_valid, error flag]
        _lib.call("fk_ce_fwd", logits.data_ptr(), logits.stride(0), grad.data_ptr(),
                  grad.stride(0), targets.data_ptr(), n_rows, n_cols, int(ignore_index),
                  float(label_smoothing), _lib.dtype_code(logits.dtype), loss_rows.data_ptr(),
                  loss.data_ptr(), flags.data_ptr(), flags.data_ptr() + 4,
                  _lib.stream_of(logits))
        _last_err = flags
        ctx.grad = grad
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        grad = ctx.grad
        ctx.grad = None
        go = grad_output.to(device=grad.device, dtype=torch.float32).contiguous()
        _lib.call("fk_ce_bwd_scale", grad.data_ptr(), grad.stride(0), grad.shape[0],
                  grad.shape[1], go.data_ptr(), _lib.dtype_code(grad.dtype),
                  _lib.stream_of(grad))
        return grad.detach(), None, None, None, None


def fused_cross_entropy(logits: torch.Tensor, targets: torch.Tensor,
                        ignore_index: int = -100, label_smoothing: float = 0.0,
                        inplace_grad: bool = False) -> torch.Tensor:
    """Drop-in fused replacement for F.cross_entropy(logits, targets).
    logits: [N, V], targets: [N] long. Returns scalar mean loss."""
    return _FusedCrossEntropy.apply(logits, targets, ignore_index, label_smoothing, inplace_grad)


def global_mean_scales(loss_sum: torch.Tensor, n_count: torch.Tensor, n_valid_local: torch.Tensor,
                       group=None):
    """All-reduce [sum of this rank's row losses, its count of non-ignored rows] over
    ``group`` (one 2-element collective) and return (global mean loss, factor that turns
    this rank's gradient -- written with 1/n_valid_local folded in -- into the gradient of
    the global mean).  The global count is clamped to >= 1 as the reference clamps it
    (cross_entropy.py:107)."""
    stats = torch.stack([loss_sum.float(), n_count.float()])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(stats, group=group)
    nv = stats[1].clamp(min=1.0)
    return stats[0] / nv, n_valid_local.float() / nv


class _FusedCrossEntropyGlobalMean(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index, label_smoothing, inplace_grad, group):
        assert logits.is_cuda and logits.ndim == 2
        n_rows, n_cols = logits.shape
        assert targets.shape == (n_rows,)
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        targets = targets.to(device=logits.device, dtype=torch.int64).contiguous()
        dev = logits.device
        grad = logits if inplace_grad else torch.empty_like(logits)
        loss_rows = torch.empty(n_rows, dtype=torch.float32, device=dev)
        loss = torch.empty((), dtype=torch.float32, device=dev)
        flags = torch.empty(2, dtype=torch.int32, device=dev)  # [local n_valid >= 1, error]
        _lib.call("fk_ce_fwd", logits.data_ptr(), logits.stride(0), grad.data_ptr(),
                  grad.stride(0), targets.data_ptr(), n_rows, n_cols, int(ignore_index),
                  float(label_smoothing), _lib.dtype_code(logits.dtype), loss_rows.data_ptr(),
                  loss.data_ptr(), flags.data_ptr(), flags.data_ptr() + 4,
                  _lib.stream_of(logits))
        global _last_err
        _last_err = flags
        count = (targets != ignore_index).sum()
        gloss, factor = global_mean_scales(loss_rows.sum(), count, flags[0], group)
        ctx.grad = grad
        ctx.save_for_backward(factor)
        return gloss

    @staticmethod
    def backward(ctx, grad_output):
        (factor,) = ctx.saved_tensors
        grad = ctx.grad
        ctx.grad = None
        go = (grad_output.to(device=grad.device, dtype=torch.float32) * factor).contiguous()
        _lib.call("fk_ce_bwd_scale", grad.data_ptr(), grad.stride(0), grad.shape[0],
                  grad.shape[1], go.data_ptr(), _lib.dtype_code(grad.dtype),
                  _lib.stream_of(grad))
        return grad.detach(), None, None, None, None, None


def fused_cross_entropy_global_mean(logits: torch.Tensor, targets: torch.Tensor,
                                    ignore_index: int = -100, label_smoothing: float = 0.0,
                                    inplace_grad: bool = False, group=None) -> torch.Tensor:
    """Cross-entropy of a batch sharded by rows over the ranks of ``group`` (default: the
    world): returns the mean over every rank's non-ignored rows (the same value on every
    rank) and gives each rank the gradient of that global mean for its own rows.  Costs
    one all-reduce of two scalars; without an initialised process group it equals
    ``fused_cross_entropy``."""
    return _FusedCrossEntropyGlobalMean.apply(logits, targets, ignore_index, label_smoothing,
                                              inplace_grad, group)


def last_target_error() -> int:
    """Device error flag of the last fused_cross_entropy call: 0 ok, 1 target out of range."""
    return 0 if _last_err is None else int(_last_err[1].item())
