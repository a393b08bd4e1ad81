"""bench.py's contract pieces that need no GPU: the committed ncu traffic table covers the
dominant kernel of every default workload, every entry names a committed summary, and the
reference arm (the CPU reference path) prints its JSON line for every workload."""
import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_traffic_table_covers_default_workloads():
    cases = [("rmsnorm_bwd", bench.RMSNorm()), ("swiglu_bwd", bench.SwiGLU()),
             ("ce_fwd", bench.CrossEntropy()), ("router_bwd", bench.Router(131072)),
             ("moe_gemm_up", bench.MoELayer())]
    for kernel, wl in cases:
        t = bench.ncu_traffic(kernel, wl.size_key())
        assert isinstance(t, int) and t > 0, (kernel, wl.size_key())


def test_traffic_entries_name_committed_summaries():
    table = json.loads((ROOT / "profiles" / "traffic.json").read_text())
    for key, entry in table.items():
        assert (ROOT / entry["summary"]).is_file(), key
        assert entry["dram_bytes_per_launch"] == entry["dram_read_per_launch"] + \
            entry["dram_write_per_launch"] or abs(entry["dram_bytes_per_launch"] - (
                entry["dram_read_per_launch"] + entry["dram_write_per_launch"])) <= 1


def test_l2_note_states_size():
    assert "exceed" in bench.l2_note(200e6, "x")
    assert "fit" in bench.l2_note(10e6, "x")


@pytest.mark.parametrize("workload", ["moe", "rmsnorm", "swiglu", "ce", "router"])
def test_reference_arm_prints_its_line_without_a_gpu(workload):
    """`bench.py --impl reference` runs on the host alone and prints the contract's line
    (the driver launches it exactly like the GPU arm)."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env["CUDA_VISIBLE_DEVICES"] = ""
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--workload", workload, "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    wl = bench.make_workload(argparse.Namespace(workload=workload, router_rows=4096,
                                                router_experts=64, router_k=2))
    assert line["metric"] == wl.metric and line["unit"] == wl.unit
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"]
