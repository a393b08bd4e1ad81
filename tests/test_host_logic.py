"""Host-side preconditions of the Python API (mirror the reference's AssertionErrors)."""
import pytest
import torch

import fusedkernels_b200 as fk


def test_ops_require_cuda_tensors():
    x = torch.randn(4, 8)
    with pytest.raises(AssertionError):
        fk.fused_swiglu(x, x)
    with pytest.raises(AssertionError):
        fk.fused_moe_route_v2(x, 2)
    with pytest.raises(AssertionError):
        fk.fused_cross_entropy(x, torch.zeros(4, dtype=torch.long))
    with pytest.raises(AssertionError):
        fk.FusedRMSNorm(8)(x)


def test_public_names():
    for name in ["fused_cross_entropy", "FusedRMSNorm", "fused_swiglu", "fused_moe_route_v2"]:
        assert hasattr(fk, name)
