"""End-to-end integration (examples/train_mini_gpt.py of the reference): a small GPT with
the fused ops trains like the eager PyTorch formulation -- same initial loss (bf16, 2e-2
relative) and both decrease over a few AdamW steps on a fixed batch."""
import pytest
import torch

from fusedkernels_b200.mini_gpt import MiniGPT, train_step

pytestmark = pytest.mark.gpu


def test_fused_and_native_mini_gpt_agree_and_train():
    cfg = dict(vocab_size=512, dim=128, n_layers=2, n_heads=4, hidden_dim=256, max_seq_len=64)
    torch.manual_seed(0)
    fused = MiniGPT(fused=True, **cfg).cuda().bfloat16()
    native = MiniGPT(fused=False, **cfg).cuda().bfloat16()
    native.load_state_dict(fused.state_dict())
    G = torch.Generator().manual_seed(1)
    idx = torch.randint(0, 512, (4, 65), generator=G).cuda()
    x, y = idx[:, :-1], idx[:, 1:]
    with torch.no_grad():
        lf, ln = fused(x, y).float(), native(x, y).float()
    assert abs(lf.item() - ln.item()) <= 2e-2 * abs(ln.item())
    losses = {}
    for name, m in (("fused", fused), ("native", native)):
        opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
        ls = [train_step(m, opt, x, y).item() for _ in range(8)]
        losses[name] = ls
        assert ls[-1] < ls[0]
    assert abs(losses["fused"][-1] - losses["native"][-1]) <= 0.1 * losses["native"][-1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_mini_gpt_data_parallel_two_ranks():
    """The training harness under torchrun: two ranks, DistributedDataParallel over NCCL,
    fused ops on each rank; the run finishes and rank 0 reports tokens/s and a finite loss."""
    import os
    import re
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29617", "-m",
           "fusedkernels_b200.mini_gpt", "--mode", "fused", "--steps", "3", "--warmup", "1",
           "--batch-size", "2", "--seq-len", "128", "--dim", "256", "--layers", "2"]
    r = subprocess.run(cmd, cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    m = re.search(r"ranks=2 tokens/s=([\d,]+) loss=([\d.]+)", r.stdout)
    assert m, r.stdout[-1000:]
    assert float(m.group(2)) > 0
