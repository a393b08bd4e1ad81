"""Expert MLP module of the MoE layers.

``Expert`` keeps the parameter layout of fusedkernels/moe_layer.py:22-31 (three
``nn.Linear(bias=False)``: w_gate, w_up [hidden, dim] and w_down [dim, hidden]), so
state_dict keys and optimizers see exactly the reference's parameters.  The sorted-dispatch
layer stores these parameters in stacked per-expert buffers (see moe_layer_sorted.py) and
runs them on the tensor-core grouped GEMM; ``Expert.forward`` itself is the reference's
eager SwiGLU MLP and is not on the fused path.
"""
import torch.nn as nn
import torch.nn.functional as F


class Expert(nn.Module):
    """A single expert MLP (SwiGLU-style)."""

    def __init__(self, dim, hidden_dim):
        super().__init__()
        self.w_gate = nn.Linear(dim, hidden_dim, bias=False)
        self.w_up = nn.Linear(dim, hidden_dim, bias=False)
        self.w_down = nn.Linear(hidden_dim, dim, bias=False)

    def forward(self, x):
        return self.w_down(F.silu(self.w_gate(x)) * self.w_up(x))



# Imported after Expert is defined: moe_layer_sorted imports Expert from this module.
from .moe_layer_sorted import FusedMoEMLPSorted  # noqa: E402


class FusedMoEMLP(FusedMoEMLPSorted):
    """Masked-dispatch MoE layer API (fusedkernels/moe_layer.py:34-64).

    The reference loops over experts with boolean masks; its output is the same function
    of the inputs as the sorted-dispatch layer (out[t] = sum_j w[t,j] Expert_{idx[t,j]}(x[t])),
    so this class keeps the constructor, submodules and state_dict keys and runs the
    sorted-dispatch tensor-core path."""
