"""Bitonic sorting utilities on int32 rows (the reference's verification utilities for its
v4 router, fusedkernels/_bitonic_primitive.py): same function names, arguments, padding
values and output shapes, one CTA per row sorting in shared memory (fk_bitonic_sort_i32,
fk_bitonic_sort_bounded_i32)."""
import torch

from . import _lib


def _next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p <<= 1
    return p


def bitonic_sort_ascending(x: torch.Tensor) -> torch.Tensor:
    """Sort each row of x ascending.  x: [n_rows, n_elements] int32
    (reference _bitonic_primitive.py:59-76)."""
    assert x.is_cuda and x.ndim == 2 and x.dtype == torch.int32
    x = x.contiguous()
    n_rows, n = x.shape
    out = torch.empty_like(x)
    _lib.call("fk_bitonic_sort_i32", x.data_ptr(), n_rows, n, x.stride(0), out.data_ptr(),
              out.stride(0), _lib.stream_of(x))
    return out


def bitonic_sort_bounded(x: torch.Tensor, stop_k: int) -> torch.Tensor:
    """Independently ascending-sort every contiguous stop_k-sized chunk of each row, after
    padding the row to the next power of two with -2^30 (reference
    _bitonic_primitive.py:137-164).  Returns [n_rows, next_pow2(n)] int32."""
    assert x.is_cuda and x.ndim == 2 and x.dtype == torch.int32
    n_rows, n = x.shape
    N = _next_pow2(n)
    assert N % stop_k == 0, "padded width must be a multiple of stop_k"
    x = x.contiguous()
    out = torch.empty((n_rows, N), dtype=torch.int32, device=x.device)
    _lib.call("fk_bitonic_sort_bounded_i32", x.data_ptr(), n_rows, n, x.stride(0), stop_k,
              out.data_ptr(), _lib.stream_of(x))
    return out
