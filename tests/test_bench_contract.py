"""bench.py's contract pieces that need no GPU: the committed ncu traffic table covers the
dominant kernel of every default workload, and every entry names a committed summary."""
import json
import sys
from pathlib import Path

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
