"""Benchmark of the fusedkernels hot path on B200.

    python bench.py [--workload moe|rmsnorm|swiglu|ce|router] [--gpus N] [--steps K]
                    [--warmup W] [--impl ours|reference]

The default workload is the sorted-dispatch MoE layer (x [32768, 4096] bf16, E=128, k=8,
hidden 1024): one GPU runs the whole layer, N GPUs run it expert-parallel over NVLink.

One JSON line on rank 0.  A step is one forward+backward pass of the workload's op over
one batch of seeded synthetic input at the workload's full shape.  ``value`` is timed on
the device (CUDA events, inputs resident in HBM, outputs preallocated, the kernels called
through the C ABI); ``e2e`` times the same step through the public Python API with the
step's inputs copied from pinned host memory and every result (outputs and all gradients)
copied back to pinned host memory inside the timed region.  With N ranks (torchrun) the
MoE layer splits its 32768 tokens over the ranks and shards the experts (strong scaling,
token rows exchanged over NVLink); the row ops run one batch per rank (weak scaling: rows
shard with no exchange).  ``value`` aggregates all ranks over the slowest rank's time.

``--impl reference`` times the reference path's CPU implementation (the oracle in
oracle/, all host threads) on a bounded sample of the same workload; only rank 0 runs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_PATH = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_PATH = ROOT / "profiles" / "traffic.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# ----------------------------------------------------------------------------- helpers --
def peaks():
    try:
        p = json.loads(PEAKS_PATH.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
                "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def ncu_traffic(kernel_key, size_key):
    """Per-launch DRAM bytes (read+write) of a kernel at one workload size, from the
    committed ncu summary (keys "<kernel>@<size>"); None when that size was not captured."""
    try:
        t = json.loads(TRAFFIC_PATH.read_text())
        return t[f"{kernel_key}@{size_key}"]["dram_bytes_per_launch"]
    except Exception:
        return None


def l2_note(nbytes, what):
    mb = nbytes / 1e6
    if nbytes > 126e6:
        return f"inputs exceed L2 ({what} {mb:.0f} MB > 126 MB)"
    return f"inputs fit in L2 ({what} {mb:.0f} MB): repeated steps may be served from L2"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.th.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gen(seed):
    return torch.Generator().manual_seed(seed)


class PinnedSink:
    """Pinned host destinations for a step's device results.  ``put`` enqueues an async
    device-to-host copy on the current stream (so it is inside the CUDA-event timed region)
    and counts its bytes; buffers are allocated on first use and reused."""

    def __init__(self):
        self.bufs = {}
        self.nbytes = 0

    def start(self):
        self.nbytes = 0

    def put(self, key, t):
        t = t.detach()
        b = self.bufs.get(key)
        if b is None or b.shape != t.shape or b.dtype != t.dtype:
            b = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            self.bufs[key] = b
        b.copy_(t, non_blocking=True)
        self.nbytes += t.numel() * t.element_size()


def cur_stream():
    return torch.cuda.current_stream().cuda_stream


def make_graph(fn, inner, warm=1):
    """Capture `inner` back-to-back calls of fn in a CUDA graph (after `warm` eager calls
    on a side stream, which also initialise any NCCL communicator fn uses)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(inner):
            fn()
    torch.cuda.synchronize()
    return g


# ----------------------------------------------------------------------------- workloads --
class Workload:
    graph_inner = 1
    use_graph = True
    name = ""
    metric = ""
    unit = ""
    dtype = "bf16"
    higher_is_better = True

    def config(self):
        return {}


class RMSNorm(Workload):
    """RMSNorm fwd+bwd, x [16384, 4096] bf16 ~N(0,1), weight fp32 1+N(0,0.02), eps 1e-6,
    upstream grad bf16 ~N(0,1).  Algorithmic bytes: fwd reads x, writes y; bwd reads dy
    and x, writes dx (the 16 KB weight, rstd and dw are counted too)."""
    name = "rmsnorm"
    metric = "RMSNorm fwd+bwd HBM throughput (algorithmic bytes)"
    unit = "GB/s"
    rows, cols = 16384, 4096

    def setup(self, dev):
        from fusedkernels_b200 import _lib
        self.lib = _lib
        G = gen(0)
        R, C = self.rows, self.cols
        self.x_h = torch.randn(R, C, generator=G).bfloat16().pin_memory()
        self.w_h = (1.0 + 0.02 * torch.randn(C, generator=G)).pin_memory()
        self.dy_h = torch.randn(R, C, generator=G).bfloat16().pin_memory()
        self.x = self.x_h.to(dev)
        self.w = self.w_h.to(dev)
        self.dy = self.dy_h.to(dev)
        self.y = torch.empty_like(self.x)
        self.dx = torch.empty_like(self.x)
        self.dw = torch.empty_like(self.w)
        self.rstd = torch.empty(R, dtype=torch.float32, device=dev)
        wsb = _lib.rmsnorm_bwd_workspace_bytes(R, C, dev)
        self.ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        e = 2
        self.fwd_bytes = R * C * e * 2 + C * 4 + R * 4
        self.bwd_bytes = R * C * e * 3 + C * 4 * 2 + R * 4
        self.dev = dev

    def fwd(self):
        self.lib.call("fk_rmsnorm_fwd", self.x.data_ptr(), self.cols, self.w.data_ptr(), 0,
                      self.y.data_ptr(), self.cols, self.rstd.data_ptr(), self.rows, self.cols,
                      1e-6, 2, cur_stream())

    def bwd(self):
        self.lib.call("fk_rmsnorm_bwd", self.dy.data_ptr(), self.x.data_ptr(), self.w.data_ptr(),
                      0, self.rstd.data_ptr(), self.dx.data_ptr(), self.dw.data_ptr(),
                      self.ws.data_ptr(), self.ws.numel(), self.rows, self.cols, 2, cur_stream())

    def step(self):
        self.fwd()
        self.bwd()

    launches_per_step = 3  # fwd, bwd, dw column reduce

    def units_per_step(self):
        return (self.fwd_bytes + self.bwd_bytes) / 1e9

    def kernels(self):
        return [("rmsnorm_bwd", self.bwd, self.bwd_bytes), ("rmsnorm_fwd", self.fwd, self.fwd_bytes)]

    def e2e_setup(self):
        import fusedkernels_b200 as fk
        self.norm = fk.FusedRMSNorm(self.cols, eps=1e-6).to(self.dev)
        with torch.no_grad():
            self.norm.weight.copy_(self.w)
        self.sink = PinnedSink()

    def e2e_step(self):
        """x, dy in; every result (y, dx, dw) back to pinned host memory."""
        self.sink.start()
        x = self.x_h.to(self.dev, non_blocking=True).requires_grad_(True)
        dy = self.dy_h.to(self.dev, non_blocking=True)
        self.norm.weight.grad = None
        y = self.norm(x)
        y.backward(dy)
        self.sink.put("y", y)
        self.sink.put("dx", x.grad)
        self.sink.put("dw", self.norm.weight.grad)

    def e2e_bytes(self):
        return self.x_h.numel() * 2 * 2, self.sink.nbytes

    def cpu_sample(self):
        """Oracle (RefRMSNorm, fp32) on 512 rows x 4096; returns (seconds, GB of work)."""
        from oracle import rmsnorm_oracle
        R = 512
        x = self.x_h[:R].float()
        dy = self.dy_h[:R].float()
        w = self.w_h
        rmsnorm_oracle(x, w, 1e-6, dy, dtype=torch.float32)
        reps, t0 = 0, time.perf_counter()
        while True:
            rmsnorm_oracle(x, w, 1e-6, dy, dtype=torch.float32)
            reps += 1
            if time.perf_counter() - t0 > 8.0:
                break
        dt = (time.perf_counter() - t0) / reps
        gb = (R * self.cols * 2 * 5) / 1e9  # same algorithmic bytes per row as the GPU step
        return dt, gb, f"{R} of {self.rows} rows x {self.cols}, fp32 RefRMSNorm fwd+bwd, {reps} reps"

    def config(self):
        return {"workload": "rmsnorm_fwd_bwd", "shape": [self.rows, self.cols], "x_dtype": "bf16",
                "weight_dtype": "fp32", "eps": 1e-6,
                "l2": l2_note(self.rows * self.cols * 2, "x, dy each")}

    def size_key(self):
        return f"{self.rows}x{self.cols}"


class SwiGLU(Workload):
    """SwiGLU fwd+bwd, gate/up [16384, 14336] bf16 ~N(0,1), upstream bf16 ~N(0,1).
    Algorithmic bytes: fwd 3 tensors, bwd 5 tensors of 469.8 MB."""
    name = "swiglu"
    metric = "SwiGLU fwd+bwd HBM throughput (algorithmic bytes)"
    unit = "GB/s"
    rows, cols = 16384, 14336

    def setup(self, dev):
        from fusedkernels_b200 import _lib
        self.lib = _lib
        G = gen(0)
        shape = (self.rows, self.cols)
        self.g_h = torch.randn(*shape, generator=G).bfloat16().pin_memory()
        self.u_h = torch.randn(*shape, generator=G).bfloat16().pin_memory()
        self.d_h = torch.randn(*shape, generator=G).bfloat16().pin_memory()
        self.g, self.u, self.d = (t.to(dev) for t in (self.g_h, self.u_h, self.d_h))
        self.out = torch.empty_like(self.g)
        self.dg = torch.empty_like(self.g)
        self.du = torch.empty_like(self.g)
        self.n = self.g.numel()
        self.fwd_bytes = self.n * 2 * 3
        self.bwd_bytes = self.n * 2 * 5
        self.dev = dev

    def fwd(self):
        self.lib.call("fk_swiglu_fwd", self.g.data_ptr(), self.u.data_ptr(), self.out.data_ptr(),
                      self.n, 2, cur_stream())

    def bwd(self):
        self.lib.call("fk_swiglu_bwd", self.d.data_ptr(), self.g.data_ptr(), self.u.data_ptr(),
                      self.dg.data_ptr(), self.du.data_ptr(), self.n, 2, cur_stream())

    def step(self):
        self.fwd()
        self.bwd()

    launches_per_step = 2

    def units_per_step(self):
        return (self.fwd_bytes + self.bwd_bytes) / 1e9

    def kernels(self):
        return [("swiglu_bwd", self.bwd, self.bwd_bytes), ("swiglu_fwd", self.fwd, self.fwd_bytes)]

    def e2e_setup(self):
        self.sink = PinnedSink()

    def e2e_step(self):
        """gate, up, dout in; out, dgate, dup back to pinned host memory."""
        import fusedkernels_b200 as fk
        self.sink.start()
        g = self.g_h.to(self.dev, non_blocking=True).requires_grad_(True)
        u = self.u_h.to(self.dev, non_blocking=True).requires_grad_(True)
        d = self.d_h.to(self.dev, non_blocking=True)
        out = fk.fused_swiglu(g, u)
        out.backward(d)
        self.sink.put("out", out)
        self.sink.put("dg", g.grad)
        self.sink.put("du", u.grad)

    def e2e_bytes(self):
        return self.n * 2 * 3, self.sink.nbytes

    def cpu_sample(self):
        from oracle import swiglu_oracle
        R = 256
        g, u, d = (t[:R].float() for t in (self.g_h, self.u_h, self.d_h))
        swiglu_oracle(g, u, d, dtype=torch.float32)
        reps, t0 = 0, time.perf_counter()
        while True:
            swiglu_oracle(g, u, d, dtype=torch.float32)
            reps += 1
            if time.perf_counter() - t0 > 8.0:
                break
        dt = (time.perf_counter() - t0) / reps
        gb = R * self.cols * 2 * 8 / 1e9
        return dt, gb, f"{R} of {self.rows} rows x {self.cols}, fp32 silu(g)*u fwd+bwd, {reps} reps"

    def config(self):
        return {"workload": "swiglu_fwd_bwd", "shape": [self.rows, self.cols], "dtype": "bf16",
                "l2": l2_note(self.rows * self.cols * 2, "per tensor")}

    def size_key(self):
        return f"{self.rows}x{self.cols}"


class CrossEntropy(Workload):
    """Cross-entropy fwd+bwd, logits [8192, 128256] bf16 ~N(0,2), targets uniform with 5%
    ignore_index=-100, mean reduction, gradient written in place over the logits.
    Algorithmic bytes: read logits once + write the gradient once (+ targets)."""
    name = "ce"
    metric = "cross-entropy fwd+bwd HBM throughput (algorithmic bytes)"
    unit = "GB/s"
    rows, cols = 8192, 128256

    def setup(self, dev):
        from fusedkernels_b200 import _lib
        self.lib = _lib
        G = gen(0)
        self.x_h = (torch.randn(self.rows, self.cols, generator=G) * 2).bfloat16().pin_memory()
        t = torch.randint(0, self.cols, (self.rows,), generator=G)
        t[torch.rand(self.rows, generator=G) < 0.05] = -100
        self.t_h = t.pin_memory()
        self.x = self.x_h.to(dev)
        self.t = self.t_h.to(dev)
        self.loss_rows = torch.empty(self.rows, dtype=torch.float32, device=dev)
        self.loss = torch.empty((), dtype=torch.float32, device=dev)
        self.flags = torch.zeros(2, dtype=torch.int32, device=dev)
        self.go = torch.ones((), dtype=torch.float32, device=dev)
        self.bytes = self.rows * self.cols * 2 * 2 + self.rows * 8
        self.dev = dev

    def fwd(self):
        self.lib.call("fk_ce_fwd", self.x.data_ptr(), self.cols, self.x.data_ptr(), self.cols,
                      self.t.data_ptr(), self.rows, self.cols, -100, 0.0, 2,
                      self.loss_rows.data_ptr(), self.loss.data_ptr(), self.flags.data_ptr(),
                      self.flags.data_ptr() + 4, cur_stream())

    def bwd(self):
        self.lib.call("fk_ce_bwd_scale", self.x.data_ptr(), self.cols, self.rows, self.cols,
                      self.go.data_ptr(), 2, cur_stream())

    def step(self):
        self.fwd()
        self.bwd()

    launches_per_step = 4  # prologue, row kernel, finalize, backward scale (early exit)

    def units_per_step(self):
        return self.bytes / 1e9

    def kernels(self):
        return [("ce_fwd", self.fwd, self.bytes)]

    def e2e_setup(self):
        self.sink = PinnedSink()

    def e2e_step(self):
        """logits, targets in; the loss and the full logits gradient back to pinned host."""
        import fusedkernels_b200 as fk
        self.sink.start()
        x = self.x_h.to(self.dev, non_blocking=True).requires_grad_(True)
        t = self.t_h.to(self.dev, non_blocking=True)
        loss = fk.fused_cross_entropy(x, t, inplace_grad=True)
        loss.backward()
        self.sink.put("loss", loss)
        self.sink.put("grad", x.grad)

    def e2e_bytes(self):
        return self.rows * self.cols * 2 + self.rows * 8, self.sink.nbytes

    def cpu_sample(self):
        from oracle import cross_entropy_oracle
        R = 64
        x = self.x_h[:R].float()
        t = self.t_h[:R]
        cross_entropy_oracle(x, t, dtype=torch.float32)
        reps, t0 = 0, time.perf_counter()
        while True:
            cross_entropy_oracle(x, t, dtype=torch.float32)
            reps += 1
            if time.perf_counter() - t0 > 8.0:
                break
        dt = (time.perf_counter() - t0) / reps
        gb = (R * self.cols * 2 * 2 + R * 8) / 1e9
        return dt, gb, f"{R} of {self.rows} rows x {self.cols}, fp32 cross-entropy fwd+bwd, {reps} reps"

    def config(self):
        return {"workload": "cross_entropy_fwd_bwd", "shape": [self.rows, self.cols],
                "dtype": "bf16", "ignore_fraction": 0.05, "inplace_grad": True,
                "l2": l2_note(self.rows * self.cols * 2, "logits")}

    def size_key(self):
        return f"{self.rows}x{self.cols}"


class Router(Workload):
    """Router fwd+bwd, logits [4096, 64] fp32 ~N(0,1), k=2, upstream dw ~N(0,1).
    ``--router-rows`` changes N (e.g. 131072 for a bandwidth-meaningful size)."""
    name = "router"
    metric = "MoE router fwd+bwd throughput"
    unit = "tokens/s"
    dtype = "f32"
    E, k = 64, 2
    graph_inner = 20

    def __init__(self, rows=4096, experts=64, k=2):
        self.rows, self.E, self.k = rows, experts, k

    def setup(self, dev):
        from fusedkernels_b200 import _lib
        self.lib = _lib
        G = gen(0)
        self.l_h = torch.randn(self.rows, self.E, generator=G).pin_memory()
        self.dw_h = torch.randn(self.rows, self.k, generator=G).pin_memory()
        self.l = self.l_h.to(dev)
        self.dwt = self.dw_h.to(dev)
        self.w = torch.empty(self.rows, self.k, device=dev)
        self.idx = torch.empty(self.rows, self.k, dtype=torch.int64, device=dev)
        self.dl = torch.empty(self.rows, self.E, device=dev)
        self.fwd_bytes = self.rows * (self.E * 4 + self.k * 12)
        self.bwd_bytes = self.rows * (self.k * 16 + self.E * 4)
        self.dev = dev

    def fwd(self):
        self.lib.call("fk_router_fwd", self.l.data_ptr(), self.E, 0, self.rows, self.E, self.k,
                      self.w.data_ptr(), self.idx.data_ptr(), cur_stream())

    def bwd(self):
        self.lib.call("fk_router_bwd", self.dwt.data_ptr(), self.w.data_ptr(), self.idx.data_ptr(),
                      self.dl.data_ptr(), self.rows, self.E, self.k, cur_stream())

    def step(self):
        self.fwd()
        self.bwd()

    launches_per_step = 2

    def units_per_step(self):
        return self.rows

    def kernels(self):
        return [("router_fwd", self.fwd, self.fwd_bytes), ("router_bwd", self.bwd, self.bwd_bytes)]

    def e2e_setup(self):
        self.sink = PinnedSink()

    def e2e_step(self):
        """logits, dw in; weights, indices and dlogits back to pinned host memory."""
        import fusedkernels_b200 as fk
        self.sink.start()
        lg = self.l_h.to(self.dev, non_blocking=True).requires_grad_(True)
        dw = self.dw_h.to(self.dev, non_blocking=True)
        w, idx = fk.fused_moe_route_v2(lg, self.k)
        w.backward(dw)
        self.sink.put("w", w)
        self.sink.put("idx", idx)
        self.sink.put("dl", lg.grad)

    def e2e_bytes(self):
        return self.rows * (self.E + self.k) * 4, self.sink.nbytes

    def cpu_sample(self):
        from oracle import route_bwd_oracle, route_oracle
        lg = self.l_h
        dw = self.dw_h
        reps, t0 = 0, time.perf_counter()
        while True:
            _, idx = route_oracle(lg, self.k, torch.float32)
            route_bwd_oracle(lg, self.k, dw, torch.float32, idx)
            reps += 1
            if time.perf_counter() - t0 > 8.0:
                break
        dt = (time.perf_counter() - t0) / reps
        return dt, self.rows, f"all {self.rows} rows, fp32 stable-sort router fwd+bwd, {reps} reps"

    def config(self):
        return {"workload": "moe_router_fwd_bwd", "shape": [self.rows, self.E], "k": self.k,
                "dtype": "fp32",
                "l2": (f"inputs {self.rows * self.E * 4 / 1e6:.0f} MB: "
                       + ("fit in L2; launch-latency bound" if self.rows * self.E * 4 < 16e6
                          else "HBM/L2 streaming"))}

    def size_key(self):
        return f"{self.rows}x{self.E}k{self.k}"


class MoELayer(Workload):
    """Sorted-dispatch MoE layer fwd+bwd: x [32768, 4096] bf16 ~N(0,1); router
    Linear(4096 -> 128) weights ~N(0, 0.02) plus a per-expert logit bias 2*ln(w_e),
    w_e ~ (e+1)^-1.1 normalised (added to the router output by a forward hook, as the
    workload specifies); k = 8; experts SwiGLU with hidden 1024, weights ~N(0, 0.02) bf16;
    upstream gradient ~N(0,1).  Algorithmic FLOPs: 6 GEMM passes over the 262144 real
    (token, expert) assignments (2*M*K*N each) plus the router GEMM fwd+bwd."""
    name = "moe"
    metric = "MoE layer fwd+bwd throughput"
    ep_transport = "peer"
    ep_replicate = "auto"
    ep_overlap_sms = 32
    unit = "tokens/s"
    strong = True  # the 32768 global tokens are split across ranks
    tokens, dim, hidden, E, k = 32768, 4096, 1024, 128, 8
    use_graph = True  # the whole fwd+bwd step (NCCL calls included) replays as one graph

    def setup(self, dev):
        import fusedkernels_b200 as fk
        from fusedkernels_b200 import _lib
        from oracle import zipf_expert_bias
        self.lib = _lib
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        D, H, E = self.dim, self.hidden, self.E
        # Full weights from one seed on every rank (device RNG): identical everywhere.
        torch.manual_seed(0)
        wr = torch.empty(E, D, device=dev).normal_(0, 0.02).bfloat16()
        wg = torch.empty(E, H, D, device=dev).normal_(0, 0.02).bfloat16()
        wu = torch.empty(E, H, D, device=dev).normal_(0, 0.02).bfloat16()
        wd = torch.empty(E, D, H, device=dev).normal_(0, 0.02).bfloat16()
        bias = zipf_expert_bias(E).to(dev).bfloat16()
        G = gen(0)
        x_all = torch.randn(self.tokens, D, generator=G).bfloat16()
        d_all = torch.randn(self.tokens, D, generator=G).bfloat16()
        if self.world == 1:
            layer = fk.FusedMoEMLPSorted(D, H, E, self.k).to(dev).bfloat16()
            with torch.no_grad():
                layer.router.weight.copy_(wr)
                layer.w13[:, :H].copy_(wg)
                layer.w13[:, H:].copy_(wu)
                layer.w2.copy_(wd)
            self.placement = None
            self.replicated = []
            T0, T1 = 0, self.tokens
        else:
            from fusedkernels_b200.moe_ep import (ExpertParallelMoEMLP, hot_experts,
                                                  lpt_placement_excluding)
            # Load-aware static placement from the expert loads of a calibration batch
            # (seed 1; the timed batch is seed 0), computed identically on every rank: no
            # communication.
            with torch.no_grad():
                x_cal = torch.randn(self.tokens, D, generator=gen(1)).bfloat16().to(dev)
                logits = x_cal @ wr.t() + bias
                _, idx = fk.fused_moe_route_v2(logits, self.k)
                load = torch.bincount(idx.reshape(-1), minlength=E).float().cpu()
                del x_cal, logits
            self.replicated = (hot_experts(load.tolist(), self.world)
                               if self.ep_replicate == "auto" else [])
            self.placement = lpt_placement_excluding(load.tolist(), self.world, self.replicated)
            layer = ExpertParallelMoEMLP(D, H, E, self.k, placement=self.placement,
                                         transport=self.ep_transport,
                                         replicated=self.replicated,
                                         overlap_sms=self.ep_overlap_sms).to(dev).bfloat16()
            layer.load_from_full(wr, wg, wu, wd)
            per = self.tokens // self.world
            T0, T1 = self.rank * per, (self.rank + 1) * per
        self.layer = layer
        self.layer.router.register_forward_hook(lambda m, i, o: o + bias)
        self.x_h = x_all[T0:T1].contiguous().pin_memory()
        self.d_h = d_all[T0:T1].contiguous().pin_memory()
        self.x = self.x_h.to(dev)
        self.dout = self.d_h.to(dev)
        self.dev = dev
        A = self.tokens * self.k
        self.flops = 3 * (2 * A * 2 * H * D + 2 * A * D * H) + 3 * 2 * self.tokens * D * E
        self.up_flops = 2 * (T1 - T0) * self.k * 2 * H * D
        del wg, wu, wd
        if self.world == 1:
            # one routing for the kernel-level timing of the expert GEMMs
            self._prep_kernel()

    def _prep_kernel(self):
        from fusedkernels_b200.moe_layer_sorted import _Plan
        with torch.no_grad():
            logits = self.layer.router(self.x)
            import fusedkernels_b200 as fk
            w, idx = fk.fused_moe_route_v2(logits, self.k)
        plan = _Plan(self.tokens, self.k, self.E, self.dev)
        st = cur_stream()
        L = self.lib
        L.call("fk_moe_route_meta", idx.data_ptr(), w.data_ptr(), self.tokens, self.k, self.E,
               plan.counts.data_ptr(), plan.seg_start.data_ptr(), plan.tile_expert.data_ptr(),
               plan.n_mblk.data_ptr(), plan.sorted_assign.data_ptr(), plan.sorted_w.data_ptr(),
               plan.slot_pos.data_ptr(), plan.max_rows, plan.ws.data_ptr(), plan.ws.numel(),
               plan.err.data_ptr(), st)
        R = plan.max_rows
        bf = dict(dtype=torch.bfloat16, device=self.dev)
        self.kp = plan
        self.kxs = torch.empty(R, self.dim, **bf)
        L.call("fk_moe_gather", self.x.data_ptr(), self.dim, plan.sorted_assign.data_ptr(), self.k,
               plan.n_mblk.data_ptr(), R, self.kxs.data_ptr(), L.FK_BF16, st)
        self.kh1 = torch.empty(R, 2 * self.hidden, **bf)
        self.kact = torch.empty(R, self.hidden, **bf)
        self.ky = torch.empty(R, self.dim, **bf)

    def gemm_up(self):
        """The up-projection of the layer step (SwiGLU and routing-weight epilogue)."""
        p = self.kp
        self.lib.call("fk_moe_gemm_up_weighted", self.kxs.data_ptr(), p.max_rows, self.dim,
                      self.layer.w13.data_ptr(), self.hidden, self.E, p.tile_expert.data_ptr(),
                      p.n_mblk.data_ptr(), p.sorted_assign.data_ptr(), p.sorted_w.data_ptr(),
                      self.kh1.data_ptr(), self.kact.data_ptr(), 0, p.err.data_ptr() + 4,
                      cur_stream())

    def gemm_down(self):
        p = self.kp
        self.lib.call("fk_moe_gemm_down", self.kact.data_ptr(), p.max_rows, self.hidden,
                      self.layer.w2.data_ptr(), self.dim, self.E, p.tile_expert.data_ptr(),
                      p.n_mblk.data_ptr(), self.ky.data_ptr(), 0, p.err.data_ptr() + 4,
                      cur_stream())

    def step(self):
        self.layer.zero_grad(set_to_none=True)
        x = self.x.detach().requires_grad_(True)
        out = self.layer(x)
        out.backward(self.dout)
        if self.world > 1:
            self.layer.allreduce_router_grad()  # data-parallel replicated router weight

    @property
    def launches_per_step(self):
        """Kernels of this library per step.  One GPU: router fwd/bwd 2, metadata 2,
        gather, up, down, combine | gather of dout, down dgrad, dw from parts, up dgrad,
        2 wgrad, combine = 15.
        Expert parallel (peer transport): router 2, plan 2, 2 puts, 4 waits, metadata 2,
        gather, up, down, 2 combine-puts, 2 unpack sums, unpack dw, gather of dout, dw from
        parts, 2 dgrad, 2 wgrad (4 when experts are replicated) = 26 (28); NCCL transport:
        2 packs and the local combines instead of the puts, waits and combine-puts = 22 (24)."""
        if self.world == 1:
            return 15
        base = 26 if self.ep_transport == "peer" else 22
        return base + (2 if self.replicated else 0)

    def units_per_step(self):
        return self.tokens

    def kernels(self):
        if self.world > 1:
            return []
        A = self.tokens * self.k
        return [("moe_gemm_up", self.gemm_up, self.up_flops),
                ("moe_gemm_down", self.gemm_down, 2 * A * self.dim * self.hidden)]

    def e2e_setup(self):
        self.sink = PinnedSink()
        self.copy_stream = torch.cuda.Stream(self.dev)

    def e2e_step(self):
        """x, dout in; out, dx, the router gradient and the gradient of every expert weight
        this GPU holds back to pinned host memory.  The upload of dout overlaps the forward
        and the download of out overlaps the backward (a side stream for the copies)."""
        self.sink.start()
        self.layer.zero_grad(set_to_none=True)
        main, cs = torch.cuda.current_stream(self.dev), self.copy_stream
        cs.wait_stream(main)  # the previous step's work on these buffers is done
        x = self.x_h.to(self.dev, non_blocking=True).requires_grad_(True)
        with torch.cuda.stream(cs):
            d = self.d_h.to(self.dev, non_blocking=True)
            d_ready = torch.cuda.Event()
            d_ready.record(cs)
        out = self.layer(x)
        fwd_done = torch.cuda.Event()
        fwd_done.record(main)
        with torch.cuda.stream(cs):
            cs.wait_event(fwd_done)
            self.sink.put("out", out)
        out.record_stream(cs)
        main.wait_event(d_ready)
        d.record_stream(main)
        out.backward(d)
        if self.world > 1:
            self.layer.allreduce_router_grad()
        self.sink.put("dx", x.grad)
        for name, prm in self.layer.named_parameters():
            if prm.grad is not None:
                self.sink.put(name, prm.grad)
        main.wait_stream(cs)  # the step ends when every copy has landed

    def e2e_bytes(self):
        return self.x_h.numel() * 2 * 2, self.sink.nbytes

    def cpu_sample(self):
        return moe_cpu_sample(self, 256)

    def config(self):
        if getattr(self, "host_only", False):
            # reference arm: the oracle on the host cores, whatever the GPU count
            par = "host CPU cores (reference path; no GPU, no expert sharding)"
        elif self.world == 1:
            par = "single GPU"
        else:
            par = (
                f"ep{self.world}: {len(self.replicated)} hot experts replicated on every GPU "
                f"(gradients all-reduced beside the input-gradient GEMMs, which leave "
                f"{self.ep_overlap_sms} SMs to it), the other {self.E - len(self.replicated)} "
                f"placed by "
                f"load-aware LPT bin packing (placement and replicated set from a calibration "
                f"batch, seed 1; the timed batch is seed 0), dispatch/combine "
                + ("by put kernels into peer memory over NVLink" if self.ep_transport == "peer"
                   else "by NCCL all-to-all") + f"; {self.tokens // self.world} tokens per GPU")
        return {"workload": "moe_sorted_dispatch_fwd_bwd", "tokens": self.tokens, "dim": self.dim,
                "hidden": self.hidden, "n_experts": self.E, "k": self.k, "dtype": "bf16",
                "router_bias": "2*ln(zipf(1.1) rank weights)", "parallelism": par,
                "l2": "inputs exceed L2 (x 268 MB, expert weights 3.2 GB)"}

    def size_key(self):
        return f"{self.tokens}x{self.dim}e{self.E}k{self.k}"


def moe_cpu_sample(wl, n_tok):
    """Oracle (NaiveMoEMLP restated, fp32 on the host) on n_tok tokens of the workload with
    full-size weight shapes (one random matrix per role shared by all experts: the values
    do not change the work); returns (seconds, tokens, description)."""
    from oracle import moe_layer_oracle, zipf_expert_bias
    G = gen(1)
    D, H, E, k = wl.dim, wl.hidden, wl.E, wl.k
    if not hasattr(wl, "_cpu_w"):
        wl._cpu_w = (torch.randn(E, D, generator=G) * 0.02,
                     (torch.randn(2 * H, D, generator=G) * 0.02).expand(E, 2 * H, D),
                     (torch.randn(D, H, generator=G) * 0.02).expand(E, D, H))
    wr, w13, w2 = wl._cpu_w
    x = torch.randn(n_tok, D, generator=G)
    dout = torch.randn(n_tok, D, generator=G)
    t0 = time.perf_counter()
    logits = x @ wr.t() + zipf_expert_bias(E)
    moe_layer_oracle(x, logits, w13[:, :H], w13[:, H:], w2, k, dout, dtype=torch.float32)
    dt = time.perf_counter() - t0
    return dt, n_tok, f"{n_tok} of {wl.tokens} tokens, full dims, fp32 NaiveMoEMLP fwd+bwd"


WORKLOADS = {"rmsnorm": RMSNorm, "swiglu": SwiGLU, "ce": CrossEntropy, "router": Router,
             "moe": MoELayer}


# ----------------------------------------------------------------------------- timing --
def time_device(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)  # ms


def barrier():
    if torch.distributed.is_initialized():
        torch.distributed.barrier()


def max_over_ranks(v, dev):
    if not torch.distributed.is_initialized():
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def make_workload(args):
    if args.workload == "router":
        return Router(args.router_rows, args.router_experts, args.router_k)
    return WORKLOADS[args.workload]()


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    wl = make_workload(args)
    if args.rows and hasattr(wl, "rows") and args.workload != "router":
        wl.rows = args.rows
    if args.workload == "moe":
        wl.ep_transport = args.ep_transport
        wl.ep_replicate = args.ep_replicate
        wl.ep_overlap_sms = args.ep_overlap_sms
        if args.moe_tokens:
            wl.tokens = args.moe_tokens
        if args.moe_experts:
            wl.E = args.moe_experts
    wl.setup(dev)
    stream = torch.cuda.current_stream(dev)
    pk = peaks()

    # The timed steps replay a CUDA graph of the step's C-ABI launches (`inner` steps per
    # graph for launch-latency-bound workloads), so the number is device time.
    inner = wl.graph_inner
    if wl.use_graph:
        graph = make_graph(wl.step, inner, warm=2 if wl.name == "moe" else 1)
        run_step = graph.replay
    else:
        inner = 1
        run_step = wl.step
    reps = max(1, args.steps // inner) if inner > 1 else args.steps
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize(dev)
    barrier()
    with ClockSampler(dev.index) as clk:
        ms = time_device(run_step, reps, stream)
        ms = max_over_ranks(ms, dev)
        # keep the GPU loaded for ~1 s so the clock record has samples under load; the
        # count comes from the max over ranks, so every rank runs the same steps (a step
        # may hold collectives, which every rank must enter equally often)
        extra = min(20000, max(0, int(1000.0 / max(ms / reps, 1e-3)) - reps))
        for _ in range(extra):
            run_step()
        torch.cuda.synchronize(dev)
    barrier()
    n_steps = reps * inner
    ms_per_step = ms / n_steps
    scale_units = 1 if getattr(wl, "strong", False) else world
    value = wl.units_per_step() * scale_units / (ms_per_step / 1e3)

    # Dominant kernel: per-launch duration with CUDA events on the launching stream.
    kern = []
    for name, fn, nbytes in wl.kernels():
        kg = make_graph(fn, inner)
        for _ in range(3):
            kg.replay()
        torch.cuda.synchronize(dev)
        kreps = max(args.steps, 10)
        kms = time_device(kg.replay, kreps, stream) / (kreps * inner)
        kern.append({"kernel": name, "ms": round(kms, 5), "bytes": nbytes,
                     "gbs": round(nbytes / (kms / 1e3) / 1e9, 1)})
    dom = max(kern, key=lambda k: k["ms"] if wl.name != "router" else k["bytes"]) if kern else None
    if wl.name == "moe" and dom is None:
        # multi-GPU: the whole layer step per GPU against the sustained GEMM peak
        per_gpu = wl.flops / world / (ms_per_step / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(per_gpu, 1), "peak": pk["bf16_tflops_sustained"],
                "unit": "TFLOP/s", "frac": round(per_gpu / pk["bf16_tflops_sustained"], 4),
                "traffic": None, "kernel": "whole layer step per GPU",
                "peak_source": pk["source"] + " (sustained: long step)"}
    elif wl.name == "moe":
        for kk in kern:
            kk["tflops"] = round(kk.pop("gbs") / 1e3, 1)  # bytes field holds FLOPs here
            kk["flops"] = kk.pop("bytes")
        roof = {"bound": "tensor", "achieved": dom["tflops"], "peak": pk["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(dom["tflops"] / pk["bf16_tflops"], 4),
                "traffic": ncu_traffic(dom["kernel"], wl.size_key()), "kernel": dom["kernel"],
                "peak_source": pk["source"] + " (burst: kernel timed alone)"}
    else:
        roof = {"bound": "hbm", "achieved": dom["gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(dom["gbs"] / pk["hbm_gbs"], 4), "traffic": ncu_traffic(dom["kernel"], wl.size_key()),
                "kernel": dom["kernel"], "peak_source": pk["source"]}

    # End to end through the public API with host buffers.
    wl.e2e_setup()
    for _ in range(max(args.warmup, 1)):
        wl.e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = time_device(wl.e2e_step, args.steps, stream) / args.steps
    e2e_ms = max_over_ranks(e2e_ms, dev)
    hb, db = wl.e2e_bytes()
    e2e = {"value": wl.units_per_step() * scale_units / (e2e_ms / 1e3), "unit": wl.unit,
           "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": hb, "d2h_bytes_per_step": db}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = len(os.sched_getaffinity(0))
        torch.set_num_threads(cores)
        dt, units, sample = wl.cpu_sample()
        cpu = {"value": units / dt, "unit": wl.unit, "cores": cores, "kind": "port",
               "sample": sample}

    if rank == 0:
        out = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
               "steps": n_steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
               "higher_is_better": True,
               "scaling": "strong" if getattr(wl, "strong", False) else "weak", "vs_baseline": None,
               "dtype": wl.dtype, "data": "synthetic (seeded torch.randn, shapes of the workload)",
               "config": wl.config(), "roofline": roof, "kernels": kern, "cpu_baseline": cpu,
               "e2e": e2e, "gpu_launches": wl.launches_per_step * n_steps,
               "step_tflops": (round(wl.flops / (ms_per_step / 1e3) / 1e12, 1)
                               if hasattr(wl, "flops") else None),
               "timing": (f"CUDA graph of {inner} step(s) replayed {reps}x, CUDA events" if wl.use_graph
                          else f"{reps} eager steps through the public API, CUDA events"),
               "clocks": clk.summary()}
        print(json.dumps(out), flush=True)
    # Graphs that hold NCCL calls must be released before the process group.
    graph = run_step = None
    torch.cuda.synchronize(dev)
    import gc
    gc.collect()
    if torch.distributed.is_initialized():
        layer = getattr(wl, "layer", None)
        if hasattr(layer, "close"):
            layer.close()  # collective: unmaps the peer-memory exchange regions
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = make_workload(args)
    # Host-only setup: the CPU reference never touches the GPU.
    wl_setup_host(wl)
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    times = []
    units = None
    sample = ""
    for i in range(args.warmup + args.steps):
        dt, units, sample = wl.cpu_sample_once()
        if i >= args.warmup:
            times.append(dt)
    dt = sum(times) / len(times)
    value = units / dt
    out = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
           "higher_is_better": True,
           "scaling": "strong" if getattr(wl, "strong", False) else "weak", "vs_baseline": None,
           "dtype": "f32",
           "data": "synthetic (seeded torch.randn, shapes of the workload)", "impl": "reference",
           "config": wl.config(),
           "cpu_baseline": {"value": value, "unit": wl.unit, "cores": cores, "kind": "port",
                            "sample": sample},
           "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_breakdown(args, reps=5):
    """Per-call device time of one step: every C-ABI call of the step is bracketed by CUDA
    events (eager launches), averaged over `reps` steps."""
    import collections
    from fusedkernels_b200 import _lib, moe_ep
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    wl = make_workload(args)
    if args.workload == "moe":
        wl.ep_transport = args.ep_transport
        wl.ep_replicate = args.ep_replicate
        wl.ep_overlap_sms = args.ep_overlap_sms
    wl.setup(dev)
    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()
    orig = _lib.call
    orig_a2a = moe_ep.Exchange.all_to_all
    rec = []

    def timed(name, *a):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        orig(name, *a)
        s1.record()
        rec.append((name, s0, s1))

    def timed_a2a(self, send, async_op=False):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        r = orig_a2a(self, send, async_op)
        s1.record()
        rec.append(("nccl all_to_all" + (" (async launch)" if async_op else ""), s0, s1))
        return r

    _lib.call = timed
    moe_ep.Exchange.all_to_all = timed_a2a
    tot, cnt, step_ms = collections.defaultdict(float), collections.Counter(), 0.0
    try:
        for _ in range(reps):
            rec.clear()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            wl.step()
            b.record()
            torch.cuda.synchronize()
            step_ms += a.elapsed_time(b) / reps
            for n, s0, s1 in rec:
                tot[n] += s0.elapsed_time(s1) / reps
                cnt[n] += 1
    finally:
        _lib.call = orig
        moe_ep.Exchange.all_to_all = orig_a2a
    if int(os.environ.get("RANK", "0")) == 0:
        print(f"| call | launches | ms / step |\n|---|---|---|")
        for n, t in sorted(tot.items(), key=lambda kv: -kv[1]):
            print(f"| {n} | {cnt[n] // reps} | {t:.3f} |")
        print(f"| sum of timed calls | | {sum(tot.values()):.3f} |")
        print(f"| whole eager step | | {step_ms:.3f} |")
    if world > 1:
        torch.cuda.synchronize()
        layer = getattr(wl, "layer", None)
        if hasattr(layer, "close"):
            layer.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def wl_setup_host(wl):
    """Build the workload's host tensors without a GPU (for the CPU reference arm)."""
    G = gen(0)
    if isinstance(wl, RMSNorm):
        R, C = 1024, wl.cols
        x = torch.randn(R, C, generator=G).bfloat16().float()
        w = 1.0 + 0.02 * torch.randn(C, generator=G)
        dy = torch.randn(R, C, generator=G).bfloat16().float()

        def once():
            from oracle import rmsnorm_oracle
            t0 = time.perf_counter()
            rmsnorm_oracle(x, w, 1e-6, dy, dtype=torch.float32)
            return time.perf_counter() - t0, R * C * 2 * 5 / 1e9, \
                f"{R} of {wl.rows} rows x {C} per step, fp32 RefRMSNorm fwd+bwd"
    elif isinstance(wl, SwiGLU):
        R, C = 512, wl.cols
        g, u, d = (torch.randn(R, C, generator=G).bfloat16().float() for _ in range(3))

        def once():
            from oracle import swiglu_oracle
            t0 = time.perf_counter()
            swiglu_oracle(g, u, d, dtype=torch.float32)
            return time.perf_counter() - t0, R * C * 2 * 8 / 1e9, \
                f"{R} of {wl.rows} rows x {C} per step, fp32 silu(g)*u fwd+bwd"
    elif isinstance(wl, CrossEntropy):
        R, C = 128, wl.cols
        x = (torch.randn(R, C, generator=G) * 2).bfloat16().float()
        t = torch.randint(0, C, (R,), generator=G)

        def once():
            from oracle import cross_entropy_oracle
            t0 = time.perf_counter()
            cross_entropy_oracle(x, t, dtype=torch.float32)
            return time.perf_counter() - t0, (R * C * 2 * 2 + R * 8) / 1e9, \
                f"{R} of {wl.rows} rows x {C} per step, fp32 cross-entropy fwd+bwd"
    elif isinstance(wl, MoELayer):
        wl.host_only = True

        def once():
            return moe_cpu_sample(wl, 128)
    elif isinstance(wl, Router):
        lg = torch.randn(wl.rows, wl.E, generator=G)
        dw = torch.randn(wl.rows, wl.k, generator=G)

        def once():
            from oracle import route_bwd_oracle, route_oracle
            t0 = time.perf_counter()
            _, idx = route_oracle(lg, wl.k, torch.float32)
            route_bwd_oracle(lg, wl.k, dw, torch.float32, idx)
            return time.perf_counter() - t0, wl.rows, \
                f"all {wl.rows} rows per step, fp32 stable-sort router fwd+bwd"
    else:
        raise ValueError(wl)
    wl.cpu_sample_once = once


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="moe")
    ap.add_argument("--router-rows", type=int, default=4096)
    ap.add_argument("--router-experts", type=int, default=64, help="profiling runs only")
    ap.add_argument("--router-k", type=int, default=2, help="profiling runs only")
    ap.add_argument("--moe-tokens", type=int, default=0, help="profiling runs only")
    ap.add_argument("--moe-experts", type=int, default=0, help="profiling runs only")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the row count of rmsnorm/swiglu/ce (profiling runs only)")
    ap.add_argument("--ep-transport", choices=["peer", "nccl"], default="peer",
                    help="token exchange of the expert-parallel MoE layer (N > 1)")
    ap.add_argument("--ep-replicate", choices=["auto", "none"], default="auto",
                    help="auto: replicate the experts hot enough that nearly every token picks "
                         "them on every GPU; none: exactly E/N experts per GPU")
    ap.add_argument("--ep-overlap-sms", type=int, default=32,
                    help="SMs the expert-parallel backward GEMMs leave free for the replicated "
                         "experts' gradient all-reduce running beside them (N > 1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--breakdown", action="store_true",
                    help="print the device time of every C-ABI call in one step (eager, CUDA "
                         "events around each call) instead of the JSON line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.breakdown:
        run_breakdown(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
