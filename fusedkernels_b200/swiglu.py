"""Fused SwiGLU activation: out = silu(gate) * up, forward and backward.

Mirrors fusedkernels/swiglu.py (``_FusedSwiGLUFn`` at swiglu.py:54-81, ``fused_swiglu``
at swiglu.py:84-86): same signature, same AssertionError preconditions, outputs in the
input dtype with fp32 arithmetic.  The bodies are the sm_100a streaming kernels
``fk_swiglu_fwd`` / ``fk_swiglu_bwd`` (16-byte packets, evict-first hints).
"""
import torch

from . import _lib


class _FusedSwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        assert gate.shape == up.shape and gate.is_cuda
        if up.dtype != gate.dtype:
            up = up.to(gate.dtype)
        gate_c = gate.contiguous()
        up_c = up.contiguous()
        out = torch.empty_like(gate_c)
        _lib.call("fk_swiglu_fwd", gate_c.data_ptr(), up_c.data_ptr(), out.data_ptr(),
                  gate_c.numel(), _lib.dtype_code(gate_c.dtype), _lib.stream_of(gate_c))
        ctx.save_for_backward(gate_c, up_c)
        ctx.shape = gate.shape
        return out.view(gate.shape)

    @staticmethod
    def backward(ctx, dout):
        gate, up = ctx.saved_tensors
        dout_c = dout.to(gate.dtype).contiguous()
        dgate = torch.empty_like(gate)
        dup = torch.empty_like(up)
        _lib.call("fk_swiglu_bwd", dout_c.data_ptr(), gate.data_ptr(), up.data_ptr(),
                  dgate.data_ptr(), dup.data_ptr(), gate.numel(), _lib.dtype_code(gate.dtype),
                  _lib.stream_of(gate))
        return dgate.view(ctx.shape), dup.view(ctx.shape)


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Fused equivalent of F.silu(gate) * up."""
    return _FusedSwiGLUFn.apply(gate, up)
