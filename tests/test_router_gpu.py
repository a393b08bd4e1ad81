"""Router kernels vs the oracle: indices bit-exact and in rank order (exact logit, ties to
the lower expert index), weights atol 1e-6 rtol 1e-5, dlogits atol 1e-5 rtol 1e-4.
Cases follow the reference's router tests (tests/test_moe_routing_v2.py,
tests/test_moe_imbalance.py) plus ties, signed zeros and NaN."""
import pytest
import torch

import fusedkernels_b200 as fk
from oracle import route_bwd_oracle, route_oracle
from conftest import gen

pytestmark = pytest.mark.gpu


def run(logits, k, dw=None):
    lg = logits.cuda().requires_grad_(dw is not None)
    w, idx = fk.fused_moe_route_v2(lg, k)
    dl = None
    if dw is not None:
        w.backward(dw.cuda())
        dl = lg.grad.float().cpu()
    return w.detach().cpu(), idx.cpu(), dl


def check(logits, k, with_bwd=True, seed=0):
    dw = torch.randn(logits.shape[0], k, generator=gen(seed + 100)) if with_bwd else None
    w, idx, dl = run(logits, k, dw)
    rw, ridx = route_oracle(logits, k)
    assert idx.dtype == torch.int64
    bad = (idx != ridx).any(dim=1).nonzero()
    assert bad.numel() == 0, f"{bad.numel()} rows differ, first {bad[:3].tolist()}"
    torch.testing.assert_close(w, rw, atol=1e-6, rtol=1e-5, equal_nan=True)
    if with_bwd:
        rdl = route_bwd_oracle(logits, k, dw)
        if logits.dtype == torch.float32:
            torch.testing.assert_close(dl, rdl, atol=1e-5, rtol=1e-4)
        else:
            # 16-bit logits: the kernel's fp32 dlogits are cast to the logits dtype by
            # autograd, so compare with the oracle rounded the same way (one ulp apart at most)
            ref = rdl.to(logits.dtype).float()
            torch.testing.assert_close(dl, ref, atol=1e-5, rtol=2 ** -7)
        # the gradient of every unselected logit is exactly zero
        sel = torch.zeros_like(dl, dtype=torch.bool).scatter_(1, idx, True)
        assert torch.count_nonzero(dl[~sel]) == 0
    return w, idx


CASES = [(8, 2), (16, 4), (64, 8), (128, 16), (64, 2), (128, 8), (32, 4), (256, 8), (128, 32),
         (4, 4), (1, 1), (3, 2), (100, 7), (200, 40), (128, 128), (64, 64), (256, 256)]


@pytest.mark.parametrize("E,k", CASES)
def test_router_fp32_matches_oracle(E, k):
    logits = torch.randn(1024, E, generator=gen(E * 1000 + k))
    check(logits, k)


@pytest.mark.parametrize("E,k", [(8, 2), (64, 8), (128, 8), (128, 16)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_router_16bit_ties_bit_exact(E, k, dtype):
    """16-bit logits tie often; the lower expert index must win every tie.  The backward
    (the path the MoE layer takes with its bf16 router logits) is checked too."""
    logits = torch.randn(4096, E, generator=gen(11)).to(dtype)
    w, idx = check(logits, k)
    assert idx.shape == (4096, k)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_router_16bit_layer_shape_backward(dtype):
    """The MoE layer's routing shape: [32768, 128] 16-bit logits, k = 8, with the Zipf
    expert bias of the workload (skewed, many cross-boundary ties in bf16)."""
    from oracle import zipf_expert_bias
    logits = (torch.randn(32768, 128, generator=gen(21)) * 0.3 + zipf_expert_bias(128)).to(dtype)
    check(logits, 8, seed=21)


@pytest.mark.parametrize("n", [1, 3, 1001])
@pytest.mark.parametrize("E,k", [(8, 1), (9, 2), (64, 2), (128, 8), (256, 4)])
def test_router_ragged_row_counts(n, E, k):
    """Row counts that leave part of the last warp's rows empty."""
    check(torch.randn(n, E, generator=gen(n * 7 + E + k)), k)


def test_router_integer_logits_many_ties():
    logits = torch.randint(-2, 3, (2048, 64), generator=gen(12)).float()
    check(logits, 8)


def test_router_signed_zero_and_nan():
    logits = torch.zeros(4, 8)
    logits[0, 3] = -0.0
    logits[1] = torch.tensor([-0.0, 0.0, -0.0, 0.0, -1.0, -1.0, 1.0, -0.0])
    logits[2, 5] = float("nan")
    logits[3] = torch.tensor([float("-inf")] * 6 + [0.5, float("inf")])
    w, idx, _ = run(logits, 3)
    rw, ridx = route_oracle(logits, 3)
    assert torch.equal(idx, ridx)
    torch.testing.assert_close(w, rw, equal_nan=True)
    assert idx[1].tolist() == [6, 0, 1] and idx[2, 0].item() == 5


@pytest.mark.parametrize("E,k,skew", [(64, 8, 8.0), (128, 16, 8.0), (128, 32, 12.0)])
def test_router_skewed_logits(E, k, skew):
    """tests/test_moe_imbalance.py:22-53: per-expert bias of +-skew."""
    G = gen(0)
    bias = (torch.rand(E, generator=G) - 0.5) * 2 * skew
    logits = torch.randn(2048, E, generator=G) + bias
    check(logits, k)


def test_router_saturated_logits():
    """tests/test_moe_imbalance.py:56-77: two saturated columns (+-50)."""
    logits = torch.randn(1024, 64, generator=gen(0)) * 2.0
    logits[:, 0] = 50.0
    logits[:, 1] = -50.0
    check(logits, 8)


def test_router_weights_sum_to_one():
    w, _, _ = run(torch.randn(512, 32, generator=gen(1)), 4)
    torch.testing.assert_close(w.sum(-1), torch.ones(512), atol=1e-6, rtol=0)


def test_router_strided_rows():
    base = torch.randn(300, 80, generator=gen(13))
    logits = base[:, 3:67]  # row stride 80, 64 experts
    w, idx, _ = run(logits, 8)
    rw, ridx = route_oracle(logits.contiguous(), 8)
    assert torch.equal(idx, ridx)


def test_router_matches_reference_golden(golden):
    for E, k in [(8, 2), (64, 2), (64, 8), (128, 8), (128, 16)]:
        p = f"router_E{E}_k{k}_"
        w, idx, dl = run(torch.from_numpy(golden[p + "logits"]), k,
                         torch.from_numpy(golden[p + "dw"]))
        assert torch.equal(idx, torch.from_numpy(golden[p + "idx"]).long())
        torch.testing.assert_close(w, torch.from_numpy(golden[p + "w"]), atol=1e-6, rtol=1e-5)
        torch.testing.assert_close(dl, torch.from_numpy(golden[p + "dlogits"]), atol=1e-6, rtol=1e-5)


def test_router_large_batch_bit_exact():
    """N=131072 rows (examples/moe_router_sweep_n.py's largest N), E=128, k=8, bf16."""
    logits = torch.randn(131072, 128, generator=gen(14)).bfloat16()
    _, idx, _ = run(logits, 8)
    _, ridx = route_oracle(logits, 8)
    assert torch.equal(idx, ridx)


def test_router_deterministic():
    logits = torch.randn(1024, 128, generator=gen(15))
    outs = [run(logits, 32, torch.ones(1024, 32)) for _ in range(5)]
    for o in outs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(o, outs[0]))


# ------------------------------------------------------------------ v1 / v4 router APIs
@pytest.mark.parametrize("E,k", [(8, 2), (16, 4), (64, 8), (128, 1)])
def test_v1_api_matches_oracle(E, k):
    """tests/test_moe_correctness.py:18-49 cases, exact ordered indices."""
    logits = torch.randn(1024, E, generator=gen(E + k))
    lg = logits.cuda().requires_grad_(True)
    w, idx = fk.fused_moe_route(lg, k)
    rw, ridx = route_oracle(logits, k)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.detach().cpu(), rw, atol=1e-6, rtol=1e-5)
    w.sum().backward()
    assert lg.grad.shape == logits.shape


@pytest.mark.parametrize("E,k", [(8, 2), (16, 4), (16, 8), (32, 4), (32, 8), (32, 16), (64, 8),
                                 (64, 16), (64, 32), (128, 8), (128, 16), (128, 32), (32, 3),
                                 (64, 5), (128, 7), (64, 11)])
def test_v4_api_ascending_order_and_grad(E, k):
    """tests/test_moe_routing_v4.py:22-94 cases: v4 returns the top k in ascending order."""
    import warnings
    logits = torch.randn(1024, E, generator=gen(100 + E + k))
    dw = torch.randn(1024, k, generator=gen(7))
    lg = logits.cuda().requires_grad_(True)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        w, idx = fk.fused_moe_route_v4(lg, k)
    rw, ridx = route_oracle(logits, k)
    assert torch.equal(idx.cpu(), ridx.flip(-1))
    torch.testing.assert_close(w.detach().cpu(), rw.flip(-1), atol=1e-6, rtol=1e-5)
    w.backward(dw.cuda())
    torch.testing.assert_close(lg.grad.cpu(), route_bwd_oracle(logits, k, dw.flip(-1)),
                               atol=1e-5, rtol=1e-4)


def test_v4_warns_for_large_k_and_is_deterministic():
    logits = torch.randn(1024, 128, generator=gen(4)).cuda()
    with pytest.warns(UserWarning):
        _, first = fk.fused_moe_route_v4(logits, 80)
    for _ in range(4):
        _, again = fk.fused_moe_route_v4(logits, 32)
        assert torch.equal(again, fk.fused_moe_route_v4(logits, 32)[1])
