"""The CPU oracle against golden vectors produced by the reference's own Triton kernels
(tests/golden/make_golden.py runs them under Triton's CPU interpreter)."""
import torch

from oracle import (cross_entropy_oracle, rmsnorm_oracle, route_bwd_oracle, route_oracle,
                    swiglu_oracle)


def T(a):
    return torch.from_numpy(a)


def test_swiglu_oracle_matches_reference_kernels(golden):
    for tag in ("a", "b"):
        p = f"swiglu_{tag}_"
        out, dg, du = swiglu_oracle(T(golden[p + "gate"]), T(golden[p + "up"]), T(golden[p + "dout"]))
        torch.testing.assert_close(out.float(), T(golden[p + "out"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dg.float(), T(golden[p + "dgate"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(du.float(), T(golden[p + "dup"]), atol=1e-5, rtol=1e-5)


def test_rmsnorm_oracle_matches_reference_kernels(golden):
    for tag in ("a", "b"):
        p = f"rmsnorm_{tag}_"
        y, dx, dw = rmsnorm_oracle(T(golden[p + "x"]), T(golden[p + "w"]), float(golden[p + "eps"]),
                                   T(golden[p + "dy"]))
        torch.testing.assert_close(y.float(), T(golden[p + "y"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dx.float(), T(golden[p + "dx"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dw.float(), T(golden[p + "dw"]), atol=1e-4, rtol=1e-5)


def test_cross_entropy_oracle_matches_reference_kernel(golden):
    for tag in ("a", "smooth", "wide"):
        p = f"ce_{tag}_"
        loss, grad = cross_entropy_oracle(T(golden[p + "logits"]), T(golden[p + "targets"]),
                                          -100, float(golden[p + "ls"]))
        torch.testing.assert_close(loss.float(), T(golden[p + "loss"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(grad.float(), T(golden[p + "grad"]), atol=1e-7, rtol=1e-4)


def test_router_oracle_matches_reference_kernels(golden):
    for E, k in [(8, 2), (64, 2), (64, 8), (128, 8), (128, 16)]:
        p = f"router_E{E}_k{k}_"
        logits = T(golden[p + "logits"])
        w, idx = route_oracle(logits, k)
        ref_idx = T(golden[p + "idx"]).long()
        # The reference ranks by a quantised key; on these tie-free inputs it selects the
        # same experts in the same order as the exact-logit ranking.
        assert torch.equal(idx, ref_idx), f"E={E} k={k}"
        torch.testing.assert_close(w, T(golden[p + "w"]), atol=1e-6, rtol=1e-5)
        dl = route_bwd_oracle(logits, k, T(golden[p + "dw"]))
        torch.testing.assert_close(dl, T(golden[p + "dlogits"]), atol=1e-6, rtol=1e-5)


def test_router_oracle_tie_break_lower_index():
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.0, 3.0], [-0.0, 0.0, -1.0, 0.0, 2.0]])
    _, idx = route_oracle(logits, 2)
    assert idx.tolist() == [[1, 2], [4, 0]]
    nan_row = torch.tensor([[0.5, float("nan"), float("inf"), 1.0]])
    _, idx = route_oracle(nan_row, 3)
    assert idx.tolist() == [[1, 2, 3]]


MOE_TAGS = ("e8k2", "e32k4", "e64k8", "e128k16", "empty")


def test_moe_layer_oracle_matches_reference_naive_layer(golden_moe):
    """moe_layer_oracle against the reference's own NaiveMoEMLP (fp64 on the CPU, stored as
    fp32): forward output, input gradient (expert and router paths), router weight
    gradient and every expert's weight gradients; atol 1e-6 / rtol 1e-5."""
    from oracle import moe_layer_oracle
    tol = dict(atol=1e-6, rtol=1e-5)
    for tag in MOE_TAGS:
        g = {k[len(f"moe_{tag}_"):]: v for k, v in golden_moe.items() if k.startswith(f"moe_{tag}_")}
        x, wr = T(g["x"]).double(), T(g["wr"]).double()
        logits = x @ wr.t()
        out, dx, dwg, dwu, dwd, dl = moe_layer_oracle(x, logits, T(g["wg"]), T(g["wu"]), T(g["wd"]),
                                                      int(g["k"]), T(g["dout"]))
        torch.testing.assert_close(out.float(), T(g["out"]), **tol, msg=tag)
        torch.testing.assert_close((dx + dl @ wr).float(), T(g["dx"]), **tol, msg=tag)
        torch.testing.assert_close((dl.t() @ x).float(), T(g["dwr"]), **tol, msg=tag)
        torch.testing.assert_close(dwg.float(), T(g["dwg"]), **tol, msg=tag)
        torch.testing.assert_close(dwu.float(), T(g["dwu"]), **tol, msg=tag)
        torch.testing.assert_close(dwd.float(), T(g["dwd"]), **tol, msg=tag)
    # the many-experts case leaves experts without tokens: their gradients are exactly 0
    assert (T(golden_moe["moe_empty_dwg"]).flatten(1).abs().sum(1) == 0).sum() >= 56
