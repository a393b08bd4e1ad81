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


def test_full_public_api_names():
    """fusedkernels/__init__.py:10-14 exports."""
    for name in ["fused_cross_entropy", "FusedRMSNorm", "fused_swiglu", "fused_moe_route",
                 "fused_moe_route_v2", "fused_moe_route_v4", "FusedMoEMLP", "FusedMoEMLPSorted"]:
        assert name in fk.__all__ and hasattr(fk, name)


def test_moe_layers_keep_reference_parameters():
    m = fk.FusedMoEMLPSorted(64, 128, 4, 2)
    keys = list(m.state_dict().keys())
    assert keys == ["router.weight"] + [f"experts.{e}.{n}.weight" for e in range(4)
                                        for n in ("w_gate", "w_up", "w_down")]
    assert m.experts[1].w_up.weight.data_ptr() == m.w13[1, 128:].data_ptr()
    masked = fk.FusedMoEMLP(64, 128, 4, 2, router_version="v1")
    assert isinstance(masked, fk.FusedMoEMLPSorted) and masked.router_version == "v1"
    sd = m.state_dict()
    masked.load_state_dict(sd)
    assert masked.w13.data_ptr() == masked.experts[0].w_gate.weight.data_ptr()
    assert all(p.is_leaf for p in masked.parameters())


def test_mini_gpt_builds_both_modes():
    from fusedkernels_b200.mini_gpt import MiniGPT
    for fused in (True, False):
        m = MiniGPT(vocab_size=64, dim=32, n_layers=2, n_heads=4, hidden_dim=48, max_seq_len=16,
                    fused=fused)
        assert sum(p.numel() for p in m.parameters()) > 0
