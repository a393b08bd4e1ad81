"""CPU oracle for the fusedkernels training hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the PyTorch reference path that the fusedkernels
repository checks its fused ops against.  It is imported only by tests/, by
``__graft_entry__.smoke()`` (to verify the kernels' results) and by bench.py's CPU-baseline and
``--impl reference`` legs.  The product (fusedkernels_b200) never imports it and has no
CPU fallback.

Parity is pinned: tests/golden/ holds input/output vectors produced by running the
reference's own Triton kernels (fusedkernels/*.py) through Triton's CPU interpreter, and
tests/test_oracle_golden.py checks this oracle against them.
"""
from .reference_path import (  # noqa: F401
    route_oracle, route_bwd_oracle, rmsnorm_oracle, swiglu_oracle, cross_entropy_oracle,
    moe_layer_oracle, zipf_expert_bias,
)
