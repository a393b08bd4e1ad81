"""Top-KP merge of two ascending-sorted int32 lists (reference
fusedkernels/_bitonic_merge_primitive.py:65-85), on fk_bitonic_merge_topk_i32."""
import torch

from . import _lib


def bitonic_merge_topk(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a, b: [n_rows, KP] int32, each ascending-sorted, KP a power of two.  Returns the top
    KP values of each row's union, ascending."""
    assert a.is_cuda and b.is_cuda and a.shape == b.shape and a.dtype == torch.int32
    n_rows, kp = a.shape
    assert (kp & (kp - 1)) == 0, "KP must be a power of 2"
    a, b = a.contiguous(), b.to(torch.int32).contiguous()
    out = torch.empty((n_rows, kp), dtype=torch.int32, device=a.device)
    _lib.call("fk_bitonic_merge_topk_i32", a.data_ptr(), b.data_ptr(), n_rows, kp, out.data_ptr(),
              _lib.stream_of(a))
    return out
