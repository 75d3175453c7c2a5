"""Benchmark of the row-reduction hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--no-suite] [--no-e2e] [--no-graph] [--only NAME ...]

A step is one pass of the headline workload -- RMSNorm forward + backward, bf16 [32768, 8192] with
a residual (weight bf16, eps 1e-6) -- on every rank (weak scaling: each GPU owns its own 32768
rows; ranks exchange only the dw all-reduce).  The reported value is the reference's "model
memory throughput": algorithmic bytes of forward + backward (benchmarks/benchmark_rmsnorm.py:107-111,
219-229) divided by the step time, summed over ranks.  Blocks of K steps, each bracketed by a
barrier + synchronize, are repeated until two seconds have passed; the median block is reported.
Rank 0 prints ONE JSON line.  The ``kernels`` object of that line carries every other kernel of
the path at its benchmark shape (LayerNorm [65536, 4096], the softmax sweep at 2^31 elements,
cross-entropy [16384, 128256]) with a CPU figure beside it, and, on more than one GPU, the
row-sharded LayerNorm and the vocabulary-sharded cross-entropy with their collectives.

``--impl reference`` times the reference's own CPU path (its PyTorch reference functions, restated
in oracle/) on the host cores, on all 32768 rows of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

M_ROWS, N_COLS = 32768, 8192
EPS = 1e-6
METRIC = "RMSNorm/LN/softmax/CE fwd+bwd HBM GB/s"
WORKLOAD = "RMSNorm fwd+bwd bf16 [32768,8192] + residual (weight bf16, eps 1e-6), per GPU"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_PEAK_GBS = 6650.0
MIN_TIMED_SECONDS = 2.0
# Nsight Compute summary of the forward kernel that carries the measured DRAM traffic per launch.
FWD_PROFILE = ROOT / "profiles" / "norm_fwd_kernel_rmsnorm_12288x8192.md"


def fwd_bytes(M, N, s=2):
    # x, residual in; out, residual_out back; weight; rstd
    return 4 * M * N * s + N * s + M * 4


def bwd_bytes(M, N, s=2):
    # x, dout in; dx out; weight in; rstd in; dw out
    return 3 * M * N * s + N * s + M * 4 + N * s


def ln_fwd_bytes(M, N, s=2):
    return 2 * M * N * s + 2 * N * s + 2 * M * 4


def ln_bwd_bytes(M, N, s=2):
    return 3 * M * N * s + 2 * M * 4 + N * s + 2 * N * s


def config_dict():
    """Identical for both arms, so that the two JSON lines describe the same workload."""
    return {"workload": WORKLOAD, "rows_per_gpu": M_ROWS, "N": N_COLS,
            "bytes_per_step_per_gpu": fwd_bytes(M_ROWS, N_COLS) + bwd_bytes(M_ROWS, N_COLS),
            "l2": "inputs exceed L2: every streamed tensor is 512 MiB (L2 is 126 MB)"}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return FALLBACK_PEAK_GBS, "fallback (6.65 TB/s)"


def profile_facts(path: Path) -> dict:
    """``key: value`` lines of a profile summary (kernel, traffic_bytes_per_launch, rows, ...)."""
    facts = {}
    try:
        for line in path.read_text().splitlines():
            m = re.match(r"^([a-z_]+):\s+(.*\S)\s*$", line)
            if m:
                facts.setdefault(m.group(1), m.group(2))
    except OSError:
        pass
    return facts


# ------------------------------------------------------------------------------------------------
# clocks
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        try:
            for line in open(self.path):
                f = [c.strip() for c in line.split(",")]
                if len(f) < 9:
                    continue
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                try:
                    power.append(float(f[3]))
                except ValueError:
                    pass
                for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                      "sw_power_cap"), f[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
            os.unlink(self.path)
        except Exception:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "sm_mhz_min": min(sm), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------------------------------------
# CPU arm (the reference's PyTorch CPU path, restated in oracle/)
# ------------------------------------------------------------------------------------------------
def cpu_step(d):
    import oracle

    out, h = oracle.rmsnorm_ref(d["x"], d["weight"], residual=d["residual"], eps=EPS)
    rstd = oracle.rmsnorm_rstd_ref(h, eps=EPS)
    dx, dw, _ = oracle.rmsnorm_bwd_ref(h, d["weight"], d["dout"], rstd)
    return out, h, rstd, dx.to(torch.bfloat16), dw.to(torch.bfloat16)


def _best_of(fn, repeats, warmup=1):
    for _ in range(warmup):
        fn()
    best = float("inf")
    for _ in range(repeats):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def cpu_model() -> str:
    """Model name of the host CPU (first entry of /proc/cpuinfo), or the platform's answer."""
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.lower().startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or platform.machine()


def cpu_baselines() -> dict:
    """The oracle on the host cores for every benchmark configuration: C1 and the headline C2 at
    full size, the others on a stated row slice (their fp32 upcasts need 4 - 17 GB per tensor at
    full size).  GB/s uses the same byte formulas as the GPU figures."""
    import oracle

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    used = torch.get_num_threads()
    model = cpu_model()
    out = {}

    def rec(name, seconds, nbytes, sample):
        out[name] = {"value": round(nbytes / seconds / 1e9, 3), "unit": "GB/s", "cores": used,
                     "kind": "port", "ms": round(seconds * 1e3, 2), "sample": sample, "cpu": model}

    # C1: RMSNorm forward fp32 [4096, 4096], exactly as stated
    d = oracle.make_config_inputs("c1")
    t = _best_of(lambda: (oracle.rmsnorm_ref(d["x"], d["weight"], eps=d["eps"]),
                          oracle.rmsnorm_rstd_ref(d["x"], eps=d["eps"])), 5, 2)
    rec("c1_rmsnorm_fwd_fp32_4096x4096", t, 2 * 4096 * 4096 * 4 + 2 * 4096 * 4, "full size, best of 5")
    # C2 headline, all rows
    d = oracle.make_config_inputs("c2")
    t = _best_of(lambda: cpu_step(d), 2, 1)
    rec("headline", t, fwd_bytes(M_ROWS, N_COLS) + bwd_bytes(M_ROWS, N_COLS),
        f"all {M_ROWS} rows, fwd + bwd, best of 2")
    del d
    # C3 LayerNorm, 8192-row slice
    rows = 8192
    d = oracle.make_config_inputs("c3", rows=rows)
    t = _best_of(lambda: oracle.layernorm_ref(d["x"], d["weight"], d["bias"], eps=d["eps"]), 3)
    rec("layernorm_fwd", t, ln_fwd_bytes(rows, 4096), f"first {rows} of 65536 rows, best of 3")
    rstd, mean = oracle.layernorm_rstd_ref(d["x"], eps=d["eps"]), oracle.layernorm_mean_ref(d["x"])
    t = _best_of(lambda: oracle.layernorm_bwd_ref(d["x"], d["weight"], d["dout"], rstd, mean), 3)
    rec("layernorm_bwd", t, ln_bwd_bytes(rows, 4096), f"first {rows} of 65536 rows, best of 3")
    # C4 softmax, one N
    N, rows = 16384, 2048
    d = oracle.make_config_inputs(f"c4:{N}", rows=rows)
    t = _best_of(lambda: oracle.softmax_ref(d["x"]), 3)
    rec("softmax_fwd_N16384", t, 2 * rows * N * 2, f"first {rows} of 131072 rows, best of 3")
    y = oracle.softmax_ref(d["x"])
    t = _best_of(lambda: oracle.softmax_bwd_ref(d["dy"], y), 3)
    rec("softmax_bwd_N16384", t, 3 * rows * N * 2, f"first {rows} of 131072 rows, best of 3")
    # C5 cross-entropy
    rows = 512
    d = oracle.make_config_inputs("c5", rows=rows)
    t = _best_of(lambda: oracle.cross_entropy_ref(d["x"], d["target"]), 3)
    rec("ce_fwd", t, rows * 128256 * 2 + 16 * rows, f"first {rows} of 16384 rows, best of 3")
    _, lse = oracle.cross_entropy_ref(d["x"], d["target"])
    dl = torch.full((rows,), 1.0 / rows)
    t = _best_of(lambda: oracle.cross_entropy_bwd_ref(d["x"].float(), d["target"], dl, lse).to(torch.bfloat16), 3)
    rec("ce_bwd", t, 2 * rows * 128256 * 2 + 16 * rows, f"first {rows} of 16384 rows, best of 3")
    return out


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    d = oracle.make_config_inputs("c2")
    for _ in range(min(max(args.warmup, 1), 2)):
        cpu_step(d)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(d)
    dt = (time.perf_counter() - t0) / args.steps
    nbytes = fwd_bytes(M_ROWS, N_COLS) + bwd_bytes(M_ROWS, N_COLS)
    val = nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": config_dict(),
        "arm": "the reference's PyTorch CPU reference functions (rmsnorm_ref / rmsnorm_bwd_ref, "
               "restated in oracle/) on the host cores; one rank's workload (the CPU arm does not shard)",
        "cpu_baseline": {"value": val, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"each step = all {M_ROWS} rows, full N={N_COLS}", "cpu": cpu_model()},
        "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------
class Timeline:
    """CUDA-event pairs around individual launches on the current stream."""

    def __init__(self):
        self.spans = {}

    def run(self, name, fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        self.spans.setdefault(name, []).append((a, b))

    def median_ms(self):
        return {k: statistics.median(a.elapsed_time(b) for a, b in v) for k, v in self.spans.items()}

    def counts(self):
        return {k: len(v) for k, v in self.spans.items()}


def time_kernel(fn, iters=20, warmup=3):
    """Median device time of fn() in ms over ``iters`` launches, one CUDA-event pair per launch
    (inputs exceed L2).  Warm-up: at least ``warmup`` launches and at least 100 ms of them, so that
    a kernel measured right after its inputs were generated does not carry that phase's clocks."""
    t0 = time.perf_counter()
    n = 0
    while n < warmup or time.perf_counter() - t0 < 0.1:
        fn()
        n += 1
        if n % 8 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    # Queue the launches behind ~15 ms of GPU-side sleep: several of these kernels are shorter than
    # the host-side launch path, and an event pair around a launch on an idle stream would time
    # the host, not the kernel.
    torch.cuda._sleep(int(3e7))
    pairs = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        pairs.append((a, b))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in pairs)


def time_kernel_graph(fn, launches=20, replays=7):
    """Median device time of fn() in ms with `launches` back-to-back launches captured in one CUDA
    graph and the graph replayed `replays` times (the timing protocol of the reference's
    quack/bench/bench_utils.py:69-155: no host launch path between the kernels; the tensors exceed
    L2, so every launch starts L2-cold with respect to its own inputs).  None if capture fails."""
    try:
        for _ in range(3):
            fn()  # fills every lazy host-side cache (occupancy, kernel attributes) before the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(launches):
                fn()
        graph.replay()  # warm
        torch.cuda.synchronize()
        times = []
        for _ in range(replays):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) / launches)
        del graph
        return statistics.median(times)
    except Exception:
        torch.cuda.synchronize()
        return None


def copy_canary(dev) -> float:
    """The measurement behind MEASURED_PEAKS.json (b.copy_(a) over 1 Gi bf16 elements, read + write
    bytes, best of 10), repeated in this run: a contention / clock canary."""
    n = 1 << 30
    a = torch.empty(n, device=dev, dtype=torch.bfloat16).normal_()
    b = torch.empty_like(a)
    best = float("inf")
    for _ in range(2):
        b.copy_(a)
    torch.cuda.synchronize()
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        b.copy_(a)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2 * n * 2 / best / 1e6


def host_overhead(dev) -> dict:
    """Host time per eager op call with the GPU kept busy (1000 back-to-back calls / 1000)."""
    import importlib

    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    sm = importlib.import_module("quack_flydsl_b200.softmax")
    bf = torch.bfloat16
    res = {}
    x = torch.randn(1024, 4096, device=dev).to(bf)
    w = torch.randn(4096, device=dev).to(bf)
    out = torch.empty_like(x)
    xs = torch.randn(4096, 4096, device=dev).to(bf)
    ys = torch.empty_like(xs)
    for name, fn in (("rmsnorm_fwd_1024x4096", lambda: rn._rmsnorm_fwd(x, w, out, None, None, None, None, None, EPS)),
                     ("softmax_fwd_4096x4096", lambda: sm._softmax_fwd(xs, ys))):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        torch.cuda._sleep(int(2e8))  # keep the stream busy so that the calls never wait for the GPU
        t0 = time.perf_counter()
        for _ in range(1000):
            fn()
        res[name] = round((time.perf_counter() - t0) * 1e3, 3)  # us per call
        torch.cuda.synchronize()
    return res


def suite(dev, peak, cpu, no_graph=False) -> dict:
    """Every other kernel of the hot path at its benchmark configuration: median device ms of 20
    launches, GB/s of algorithmic bytes, the fraction of the measured copy peak, the kernel that
    ran, and the CPU oracle's figure where one was taken.  Outside the timed region."""
    import importlib

    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    sm = importlib.import_module("quack_flydsl_b200.softmax")
    ce = importlib.import_module("quack_flydsl_b200.cross_entropy")
    from quack_flydsl_b200 import _C
    from quack_flydsl_b200.rmsnorm_config import get_sm_count

    res = {}

    def rec(name, ms, nbytes, kernel=None):
        gbs = nbytes / ms / 1e6
        res[name] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac_of_measured_peak": round(gbs / peak, 4),
                     "pct_of_8TBs": round(100 * gbs / NOMINAL_HBM_GBS, 2), "bytes": nbytes}
        if kernel:
            res[name]["kernel"] = kernel
        if cpu and name in cpu:
            res[name]["cpu_baseline"] = cpu[name]

    def timed(name, fn, nbytes, iters=20):
        ms = time_kernel(fn, iters=iters)
        rec(name, ms, nbytes, _C.last_kernel())
        ms_g = None if no_graph else time_kernel_graph(fn)
        if ms_g is not None:
            res[name]["cuda_graph"] = {"ms": round(ms_g, 4), "gbs": round(nbytes / ms_g / 1e6, 1),
                                       "protocol": "20 launches in one CUDA graph, median of 7 replays"}

    g = torch.Generator(device=dev).manual_seed(1)
    bf = torch.bfloat16
    # LayerNorm bf16 [65536, 4096]
    M, N = 65536, 4096
    x = (0.5 + torch.randn(M, N, device=dev, generator=g)).to(bf)
    w = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(bf)
    b = (0.1 * torch.randn(N, device=dev, generator=g)).to(bf)
    dout = torch.randn(M, N, device=dev, generator=g).to(bf)
    out, dx = torch.empty_like(x), torch.empty_like(x)
    rstd, mean = torch.empty(M, device=dev), torch.empty(M, device=dev)
    P = get_sm_count(N, dev, bf)
    dwp, dbp = torch.empty(P, N, device=dev), torch.empty(P, N, device=dev)
    dw, db = torch.empty(N, device=dev, dtype=bf), torch.empty(N, device=dev, dtype=bf)
    timed("layernorm_fwd", lambda: rn._rmsnorm_fwd(x, w, out, b, rstd, mean, None, None, 1e-5, True),
          ln_fwd_bytes(M, N))
    timed("layernorm_bwd", lambda: rn._rmsnorm_bwd(x, w, dout, rstd, dx, dwp, dbp, None, None, P, mean, True),
          ln_bwd_bytes(M, N))

    def ln_bwd_total():
        rn._rmsnorm_bwd(x, w, dout, rstd, dx, dwp, dbp, None, None, P, mean, True)
        rn._norm_bwd_colsum(dwp, dw)
        rn._norm_bwd_colsum(dbp, db)
    rec("layernorm_bwd_with_stage2", time_kernel(ln_bwd_total), ln_bwd_bytes(M, N))
    del x, dout, out, dx
    # softmax bf16, M * N = 2^31
    for N in (4096, 16384, 65536, 131072):
        M = (1 << 31) // N
        x = (3 * torch.randn(M, N, device=dev, generator=g)).to(bf)
        y = torch.empty_like(x)
        timed(f"softmax_fwd_N{N}", lambda: sm._softmax_fwd(x, y), 2 * M * N * 2)
        dy = torch.randn(M, N, device=dev, generator=g).to(bf)
        timed(f"softmax_bwd_N{N}", lambda: sm._softmax_backward(dy, y, x), 3 * M * N * 2)
        del x, y, dy
    # cross-entropy bf16 [16384, 128256], int64 targets, 5 % ignored
    M, N = 16384, 128256
    x = (2 * torch.randn(M, N, device=dev, generator=g)).to(bf)
    t = torch.randint(0, N, (M,), device=dev, generator=g)
    t[torch.rand(M, device=dev, generator=g) < 0.05] = -100
    loss, lse = torch.empty(M, device=dev), torch.empty(M, device=dev)
    dxl = torch.empty_like(x)
    dloss = torch.full((M,), 1.0 / M, device=dev)
    timed("ce_fwd", lambda: ce.cross_entropy_fwd_out(x, t, None, loss, lse, None, None, -100), M * N * 2 + 16 * M)
    timed("ce_bwd", lambda: ce.cross_entropy_bwd_out(x, t, dloss, lse, dxl, None, -100), 2 * M * N * 2 + 16 * M)
    # loss + lse + dx in one call (the form chunked linear cross-entropy uses)
    timed("ce_fwd_with_dx", lambda: ce.cross_entropy_fwd_out(x, t, None, loss, lse, dxl, None, -100),
          2 * M * N * 2 + 16 * M)
    return res


def sharded_suite(dev, rank, world, peak) -> dict:
    """The two sharded paths with a collective, on `world` GPUs: LayerNorm [65536, 4096] with rows
    split over the ranks and ONE all-reduce of fp32 [dw | db]; cross-entropy [16384, 128256] with
    the vocabulary split over the ranks and one all-gather of the per-row (max, sum-exp, target
    logit).  Each is checked against the unsharded kernels on the same data before it is timed.
    Times are device times, max over ranks; GB/s is the aggregate over all ranks."""
    import importlib

    import torch.distributed as dist

    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    ce = importlib.import_module("quack_flydsl_b200.cross_entropy")
    from quack_flydsl_b200 import sharded
    from quack_flydsl_b200.rmsnorm_config import get_sm_count

    bf = torch.bfloat16
    res = {}

    def max_ms(v):
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    # ---- LayerNorm, rows sharded ----
    M, N = 65536, 4096
    g = torch.Generator(device=dev).manual_seed(7)  # the same full tensors on every rank
    x = (0.5 + torch.randn(M, N, device=dev, generator=g)).to(bf)
    w = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(bf)
    b = (0.1 * torch.randn(N, device=dev, generator=g)).to(bf)
    dout = torch.randn(M, N, device=dev, generator=g).to(bf)
    r0, r1 = sharded.row_shard(M, rank, world)
    xs, ds = x[r0:r1], dout[r0:r1]
    Ms = r1 - r0
    out, dxs = torch.empty_like(xs), torch.empty_like(xs)
    rstd, mean = torch.empty(Ms, device=dev), torch.empty(Ms, device=dev)
    P = get_sm_count(N, dev, bf)
    dwp, dbp = torch.empty(P, N, device=dev), torch.empty(P, N, device=dev)
    grads32 = torch.empty(2, N, device=dev)
    grads = torch.empty(2, N, device=dev, dtype=bf)

    peer = sharded.PeerAllReduce(dev, cap_cols=2 * N)

    def ln_step(tl=None, fused=True):
        run = tl.run if tl is not None else (lambda _n, f: f())
        run("fwd", lambda: rn._rmsnorm_fwd(xs, w, out, b, rstd, mean, None, None, 1e-5, True))
        run("bwd", lambda: rn._rmsnorm_bwd(xs, w, ds, rstd, dxs, dwp, dbp, None, None, P, mean, True))
        if fused:
            run("colsum_allreduce", lambda: peer.reduce([dwp, dbp], outs=[grads[0], grads[1]],
                                                        outs_f32=[grads32[0], grads32[1]]))
        else:
            run("colsum", lambda: (rn._norm_bwd_colsum(dwp, grads32[0]), rn._norm_bwd_colsum(dbp, grads32[1])))
            run("allreduce", lambda: dist.all_reduce(grads32))
            run("round", lambda: grads.copy_(grads32))

    ln_step()
    # check: rank 0 recomputes dw / db on all rows, unsharded
    ok_ln = True
    if rank == 0:
        o2, dx2 = torch.empty_like(x), torch.empty_like(x)
        rs2, mn2 = torch.empty(M, device=dev), torch.empty(M, device=dev)
        rn._rmsnorm_fwd(x, w, o2, b, rs2, mn2, None, None, 1e-5, True)
        dwp2, dbp2 = torch.empty(P, N, device=dev), torch.empty(P, N, device=dev)
        rn._rmsnorm_bwd(x, w, dout, rs2, dx2, dwp2, dbp2, None, None, P, mn2, True)
        ref = torch.stack([dwp2.sum(0), dbp2.sum(0)])
        scale = float(ref.abs().max())
        ok_ln = bool((grads32 - ref).abs().max() <= 2e-5 * scale + 1e-3) and \
            bool(torch.equal(dxs[:256], dx2[r0:r0 + 256]))
        del o2, dx2
    tl = Timeline()
    for _ in range(3):
        ln_step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        ln_step(tl)
    e1.record()
    torch.cuda.synchronize()
    ms = max_ms(e0.elapsed_time(e1) / 20)
    phases = {k: round(max_ms(v), 4) for k, v in tl.median_ms().items()}
    # the same step with the two-step exchange (column sums, NCCL all-reduce, rounding), for comparison
    tl2 = Timeline()
    for _ in range(3):
        ln_step(fused=False)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        ln_step(tl2, fused=False)
    e1.record()
    torch.cuda.synchronize()
    ms_nccl = max_ms(e0.elapsed_time(e1) / 20)
    phases_nccl = {k: round(max_ms(v), 4) for k, v in tl2.median_ms().items()}
    nbytes = ln_fwd_bytes(M, N) + ln_bwd_bytes(M, N)
    res["layernorm_row_sharded"] = {
        "shape": [M, N], "rows_per_rank": Ms, "ms": round(ms, 4), "gbs_aggregate": round(nbytes / ms / 1e6, 1),
        "frac_of_measured_peak": round(nbytes / ms / 1e6 / (peak * world), 4), "phases_ms": phases,
        "collective": "fp32 [dw | db] summed over the GPUs inside the stage-2 kernel (peer stores + flags)",
        "collective_timeouts": peer.timeouts(),
        "with_nccl_allreduce": {"ms": round(ms_nccl, 4), "phases_ms": phases_nccl},
        "self_check": ok_ln}
    peer.close()
    del x, dout, xs, ds, out, dxs

    # ---- cross-entropy, vocabulary sharded ----
    M, V = 16384, 128256
    c0, c1 = sharded.vocab_shard(V, rank, world)
    Ns = c1 - c0
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    xsh = (2 * torch.randn(M, Ns, device=dev, generator=g)).to(bf)
    gc = torch.Generator(device=dev).manual_seed(9)  # common: targets and the checked rows
    target = torch.randint(0, V, (M,), device=dev, generator=gc)
    target[torch.rand(M, device=dev, generator=gc) < 0.05] = -100
    chk = 256
    xfull = (2 * torch.randn(chk, V, device=dev, generator=gc)).to(bf)
    xsh[:chk] = xfull[:, c0:c1]
    dxsh = torch.empty_like(xsh)
    count = max(int((target != -100).sum()), 1)
    dloss = torch.full((M,), 1.0 / count, device=dev)
    state = {}

    peer_ce = sharded.PeerAllReduce(dev, cap_cols=3 * M)

    def ce_step(tl=None, fused=True):
        run = tl.run if tl is not None else (lambda _n, f: f())
        run("stats", lambda: state.__setitem__("stats", sharded.ce_shard_stats(xsh, target, c0)))
        if fused:
            run("exchange_combine", lambda: state.__setitem__("ll", peer_ce.ce_combine(state["stats"], target)))
        else:
            run("allgather", lambda: state.__setitem__("all", sharded.gather_ce_stats(state["stats"])))
            run("combine", lambda: state.__setitem__("ll", sharded.ce_combine(state["all"], target)))
        run("bwd", lambda: state.__setitem__("dx", sharded.ce_shard_bwd(xsh, target, dloss, state["ll"][1], c0)))

    ce_step()
    loss_s, lse_s = state["ll"]
    loss_u, lse_u = ce.cross_entropy_fwd(xfull, target[:chk], return_lse=True)
    dx_u = ce.cross_entropy_bwd(xfull, target[:chk], dloss[:chk], lse_u)
    ok_ce = bool(torch.allclose(loss_s[:chk], loss_u, rtol=1e-5, atol=1e-5)) and \
        bool(torch.allclose(lse_s[:chk], lse_u, rtol=1e-5, atol=1e-6)) and \
        bool((state["dx"][:chk].float() - dx_u[:, c0:c1].float()).abs().max() <= 2.0**-8 * float(dx_u.abs().max()))
    tl = Timeline()
    for _ in range(2):
        ce_step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        ce_step(tl)
    e1.record()
    torch.cuda.synchronize()
    ms = max_ms(e0.elapsed_time(e1) / 10)
    phases = {k: round(max_ms(v), 4) for k, v in tl.median_ms().items()}
    tl2 = Timeline()
    for _ in range(2):
        ce_step(fused=False)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        ce_step(tl2, fused=False)
    e1.record()
    torch.cuda.synchronize()
    ms_nccl = max_ms(e0.elapsed_time(e1) / 10)
    phases_nccl = {k: round(max_ms(v), 4) for k, v in tl2.median_ms().items()}
    ce_timeouts = peer_ce.timeouts()
    peer_ce.close()
    nbytes = (M * V * 2 + 16 * M) + (2 * M * V * 2 + 16 * M)  # forward + backward of the whole problem
    oks = torch.tensor([int(ok_ce), int(ok_ln)], device=dev)
    dist.all_reduce(oks, op=dist.ReduceOp.MIN)
    res["ce_vocab_sharded"] = {
        "shape": [M, V], "cols_per_rank": Ns, "ms": round(ms, 4), "gbs_aggregate": round(nbytes / ms / 1e6, 1),
        "frac_of_measured_peak": round(nbytes / ms / 1e6 / (peak * world), 4), "phases_ms": phases,
        "collective": f"the (3, {M}) fp32 row statistics ({3 * M * 4 // 1024} KiB per rank) exchanged and folded by one "
                      "kernel (peer stores + flags)",
        "collective_timeouts": ce_timeouts,
        "with_nccl_allgather": {"ms": round(ms_nccl, 4), "phases_ms": phases_nccl},
        "self_check": bool(oks[0])}
    res["layernorm_row_sharded"]["self_check"] = bool(oks[1]) if rank != 0 else (ok_ln and bool(oks[1]))
    return res


def run_only(args) -> None:
    """One kernel on a (small) case: ``--only NAME [--rows M] [--cols N] [--iters I]``.  Used for
    Nsight Compute captures and quick checks; prints one JSON line with the median device time and
    the name of the kernel that ran."""
    import importlib

    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    sm = importlib.import_module("quack_flydsl_b200.softmax")
    ce = importlib.import_module("quack_flydsl_b200.cross_entropy")
    from quack_flydsl_b200 import _C
    from quack_flydsl_b200.rmsnorm_config import get_sm_count

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    name = args.only
    defaults = {"rms_fwd": (12288, 8192), "rms_bwd": (12288, 8192), "ln_fwd": (24576, 4096),
                "ln_bwd": (24576, 4096), "softmax_fwd": (24576, 4096), "softmax_bwd": (24576, 4096),
                "ce_fwd": (2048, 128256), "ce_bwd": (1024, 128256),
                "ce_fwd_dx": (2048, 128256)}
    if name not in defaults:
        raise SystemExit(f"--only must be one of {sorted(defaults)}")
    M = args.rows or defaults[name][0]
    N = args.cols or defaults[name][1]

    def randn(*shape, scale=1.0, shift=0.0):
        return (shift + scale * torch.randn(*shape, device=dev, generator=g)).to(bf)

    if name in ("rms_fwd", "rms_bwd"):
        x, res, w = randn(M, N), randn(M, N), randn(N, scale=0.1, shift=1.0)
        out, ro = torch.empty_like(x), torch.empty_like(x)
        rstd = torch.empty(M, device=dev)
        fwd = lambda: rn._rmsnorm_fwd(x, w, out, None, rstd, None, res, ro, EPS)  # noqa: E731
        fwd()
        if name == "rms_fwd":
            fn, nbytes = fwd, fwd_bytes(M, N)
        else:
            dout, dx = randn(M, N), torch.empty_like(x)
            P = get_sm_count(N, dev, bf)
            dwp = torch.empty(P, N, device=dev)
            fn = lambda: rn._rmsnorm_bwd(ro, w, dout, rstd, dx, dwp, None, None, None, P)  # noqa: E731
            nbytes = bwd_bytes(M, N)
    elif name in ("ln_fwd", "ln_bwd"):
        x, w, b = randn(M, N, shift=0.5), randn(N, scale=0.1, shift=1.0), randn(N, scale=0.1)
        out = torch.empty_like(x)
        rstd, mean = torch.empty(M, device=dev), torch.empty(M, device=dev)
        fwd = lambda: rn._rmsnorm_fwd(x, w, out, b, rstd, mean, None, None, 1e-5, True)  # noqa: E731
        fwd()
        if name == "ln_fwd":
            fn, nbytes = fwd, ln_fwd_bytes(M, N)
        else:
            dout, dx = randn(M, N), torch.empty_like(x)
            P = get_sm_count(N, dev, bf)
            dwp, dbp = torch.empty(P, N, device=dev), torch.empty(P, N, device=dev)
            fn = lambda: rn._rmsnorm_bwd(x, w, dout, rstd, dx, dwp, dbp, None, None, P, mean, True)  # noqa: E731
            nbytes = ln_bwd_bytes(M, N)
    elif name in ("softmax_fwd", "softmax_bwd"):
        x, y = randn(M, N, scale=3.0), torch.empty(M, N, device=dev, dtype=bf)
        sm._softmax_fwd(x, y)
        if name == "softmax_fwd":
            fn, nbytes = (lambda: sm._softmax_fwd(x, y)), 2 * M * N * 2
        else:
            dy, dx = randn(M, N), torch.empty_like(x)
            fn, nbytes = (lambda: sm._softmax_backward(dy, y, dx)), 3 * M * N * 2
    else:
        x = randn(M, N, scale=2.0)
        t = torch.randint(0, N, (M,), device=dev, generator=g)
        t[torch.rand(M, device=dev, generator=g) < 0.05] = -100
        loss, lse = torch.empty(M, device=dev), torch.empty(M, device=dev)
        if name == "ce_bwd":
            ce.cross_entropy_fwd_out(x, t, None, loss, lse, None, None, -100)
        if name == "ce_fwd":
            fn = lambda: ce.cross_entropy_fwd_out(x, t, None, loss, lse, None, None, -100)  # noqa: E731
            nbytes = M * N * 2 + 16 * M
        elif name == "ce_fwd_dx":
            dx = torch.empty_like(x)
            fn = lambda: ce.cross_entropy_fwd_out(x, t, None, loss, lse, dx, None, -100)  # noqa: E731
            nbytes = 2 * M * N * 2 + 16 * M
        else:
            dx, dloss = torch.empty_like(x), torch.full((M,), 1.0 / M, device=dev)
            fn = lambda: ce.cross_entropy_bwd_out(x, t, dloss, lse, dx, None, -100)  # noqa: E731
            nbytes = 2 * M * N * 2 + 16 * M
    ms = time_kernel(fn, iters=args.iters, warmup=1)
    print(json.dumps({"only": name, "rows": M, "cols": N, "iters": args.iters, "ms": ms,
                      "gbs": nbytes / ms / 1e6, "bytes": nbytes, "kernel": _C.last_kernel()}), flush=True)


def run_ours(args) -> None:
    import importlib

    import torch.distributed as dist

    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    from quack_flydsl_b200 import _C
    from quack_flydsl_b200.rmsnorm_config import get_sm_count

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA device; there is no CPU path (use --impl reference "
                           "for the CPU arm)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    _C.lib()
    peak, peak_src = measured_peak()

    M, N = M_ROWS, N_COLS
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(M, N, device=dev, generator=g).to(bf)
    res = torch.randn(M, N, device=dev, generator=g).to(bf)
    w = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(bf)
    dout = torch.randn(M, N, device=dev, generator=g).to(bf)
    out, res_out, dx = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    rstd = torch.empty(M, device=dev)
    P = get_sm_count(N, dev, bf)
    # Two sets of buffers alternate so that the cross-GPU sum of step i (side stream) overlaps the
    # forward of step i + 1: the partial slices (read by the fused kernel) and the fp32 column sums
    # (which go straight into the NCCL all-reduce in the two-step form).
    dw_partials = [torch.empty(P, N, device=dev) for _ in range(2 if world > 1 else 1)]
    dw_partial = dw_partials[0]
    dw32 = [torch.empty(N, device=dev) for _ in range(2)]
    dw = torch.empty(N, device=dev, dtype=bf)
    tl = Timeline()
    # N > 1: stage 2 and the cross-GPU sum of dw run as ONE kernel over peer-mapped exchange buffers
    # (qb_colsum_allreduce); --collective nccl selects the two-step form instead (column sum, then an
    # NCCL all-reduce on a side stream that overlaps the next step's forward).
    use_peer = world > 1 and args.collective == "peer"
    peer = None
    peer_error = None
    if use_peer:
        from quack_flydsl_b200 import sharded as _sharded
        try:
            peer = _sharded.PeerAllReduce(dev, cap_cols=N)
        except RuntimeError as exc:  # raised on every rank together: all take the NCCL form instead
            peer_error, use_peer = repr(exc), False
            args.collective = "nccl"
    s_ar = torch.cuda.Stream(device=dev) if (world > 1 and args.collective != "none") else None
    ar_done = [None, None]
    counter = {"i": 0}

    def step(record: bool, rows: int = M):
        run = tl.run if record else (lambda _n, f: f())
        xs, rs, os_, ros, dxs, dos = x[:rows], res[:rows], out[:rows], res_out[:rows], dx[:rows], dout[:rows]
        run("rmsnorm_fwd", lambda: rn._rmsnorm_fwd(xs, w, os_, None, rstd[:rows], None, rs, ros, EPS))
        if use_peer:
            i = counter["i"] & 1
            counter["i"] += 1
            cur = torch.cuda.current_stream(dev)
            if ar_done[i] is not None:
                cur.wait_event(ar_done[i])  # this set's previous reduction (two steps ago)
            run("rmsnorm_bwd", lambda: rn._rmsnorm_bwd(ros, w, dos, rstd[:rows], dxs, dw_partials[i], None, None, None, P))
            ev = torch.cuda.Event()
            ev.record(cur)
            with torch.cuda.stream(s_ar):
                s_ar.wait_event(ev)
                run("dw_colsum_allreduce", lambda: peer.reduce([dw_partials[i]], outs=[dw]))
                done = torch.cuda.Event()
                done.record(s_ar)
            ar_done[i] = done
            return
        run("rmsnorm_bwd", lambda: rn._rmsnorm_bwd(ros, w, dos, rstd[:rows], dxs, dw_partial, None, None, None, P))
        if world > 1 and args.collective != "none":
            i = counter["i"] & 1
            counter["i"] += 1
            cur = torch.cuda.current_stream(dev)
            if ar_done[i] is not None:
                cur.wait_event(ar_done[i])  # the buffer's previous all-reduce (two steps ago)
            run("dw_colsum", lambda: rn._norm_bwd_colsum(dw_partial, dw32[i]))
            ev = torch.cuda.Event()
            ev.record(cur)
            with torch.cuda.stream(s_ar):
                s_ar.wait_event(ev)
                dist.all_reduce(dw32[i])
                dw.copy_(dw32[i])  # rounded once, after the reduction: every rank holds the same bits
                done = torch.cuda.Event()
                done.record(s_ar)
            ar_done[i] = done
        else:
            run("dw_colsum", lambda: rn._norm_bwd_colsum(dw_partial, dw))

    def join():
        if s_ar is not None:
            torch.cuda.current_stream(dev).wait_stream(s_ar)

    def sync_all():
        join()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step(False)
    sync_all()
    fwd_kernel = None
    rn._rmsnorm_fwd(x, w, out, None, rstd, None, res, res_out, EPS)
    fwd_kernel = _C.last_kernel()
    sync_all()
    sampler = ClockSampler(local)
    if rank == 0:
        sampler.start()
    blocks = []
    t_begin = time.perf_counter()
    while True:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sync_all()
        t0.record()
        for _ in range(args.steps):
            step(False)  # no per-kernel events inside the timed blocks: an event costs 3-5 us of GPU time
        join()
        t1.record()
        sync_all()
        ms_total = torch.tensor([t0.elapsed_time(t1)], device=dev)
        if world > 1:
            dist.all_reduce(ms_total, op=dist.ReduceOp.MAX)
        blocks.append(float(ms_total))
        enough = torch.tensor([int(time.perf_counter() - t_begin >= MIN_TIMED_SECONDS and len(blocks) >= 3)],
                              device=dev)
        if world > 1:
            dist.all_reduce(enough, op=dist.ReduceOp.MIN)
        if int(enough) or len(blocks) >= 400:
            break
    clocks = sampler.stop() if rank == 0 else None
    # per-kernel medians: the same steps once more, with an event pair around every kernel
    for _ in range(3):
        sync_all()
        for _ in range(args.steps):
            step(True)
        join()
    sync_all()
    ms_block = statistics.median(blocks)
    ms_step = ms_block / args.steps
    step_bytes = fwd_bytes(M, N) + bwd_bytes(M, N)
    value = world * step_bytes / ms_step / 1e6
    kms = tl.median_ms()
    launches_per_step = 3  # forward, backward stage 1, column sum (the all-reduce is NCCL's)

    # the same step and its two main kernels with the host launch path taken out (one GPU only)
    graph_ms = None
    if world == 1 and not args.no_graph:
        graph_ms = {
            "step": time_kernel_graph(lambda: step(False), launches=20),
            "rmsnorm_fwd": time_kernel_graph(
                lambda: rn._rmsnorm_fwd(x, w, out, None, rstd, None, res, res_out, EPS)),
            "rmsnorm_bwd": time_kernel_graph(
                lambda: rn._rmsnorm_bwd(res_out, w, dout, rstd, dx, dw_partial, None, None, None, P)),
        }

    # ---- strong scaling: the same [32768, 8192] problem split over the ranks ----
    strong = None
    if world > 1:
        rows = M // world
        for _ in range(3):
            step(False, rows)
        sync_all()
        sb = []
        for _ in range(5):
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            sync_all()
            t0.record()
            for _ in range(args.steps):
                step(False, rows)
            join()
            t1.record()
            sync_all()
            t = torch.tensor([t0.elapsed_time(t1)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sb.append(float(t) / args.steps)
        # one GPU alone on the whole problem, no collective: rank 0 measures, the others wait
        t1gpu = torch.zeros(1, device=dev)
        if rank == 0:
            def solo():
                rn._rmsnorm_fwd(x, w, out, None, rstd, None, res, res_out, EPS)
                rn._rmsnorm_bwd(res_out, w, dout, rstd, dx, dw_partial, None, None, None, P)
                rn._norm_bwd_colsum(dw_partial, dw)
            t1gpu[0] = time_kernel(solo, iters=20)
        dist.broadcast(t1gpu, 0)
        ms_strong = statistics.median(sb)
        strong = {"problem": [M, N], "rows_per_rank": rows, "ms_per_step": round(ms_strong, 4),
                  "ms_per_step_1gpu": round(float(t1gpu), 4),
                  "gbs_aggregate": round(step_bytes / ms_strong / 1e6, 1),
                  "speedup": round(float(t1gpu) / ms_strong, 3),
                  "efficiency": round(float(t1gpu) / ms_strong / world, 4)}

    e2e = None
    if not args.no_e2e:
        # ---- end to end through the public API with host buffers (rank-local, then max over ranks) ----
        quack_rmsnorm = rn.rmsnorm
        hx, hres, hdout = (t.cpu().pin_memory() for t in (x, res, dout))
        hw = w.cpu().pin_memory()
        h_out, h_dx = (torch.empty(M, N, dtype=bf).pin_memory() for _ in range(2))
        h_dw = torch.empty(N, dtype=bf).pin_memory()
        dxg, dresg, dwg = (torch.empty_like(x), torch.empty_like(x), torch.empty_like(w))

        # The user-level loop: row blocks travel host -> device on one stream, go through
        # quack.rmsnorm + autograd backward on a second, and the results return on a third, so that
        # the two PCIe directions and the kernels overlap.  The weight gradient accumulates in
        # weight.grad over the blocks, as autograd does for any micro-batched loop.
        E2E_BLOCKS = args.e2e_blocks
        rows_blk = M // E2E_BLOCKS
        s_in, s_cmp, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))

        def e2e_step():
            cur = torch.cuda.current_stream(dev)
            for s in (s_in, s_cmp, s_out):
                s.wait_stream(cur)
            with torch.cuda.stream(s_in):
                wd = dwg.copy_(hw, non_blocking=True)
            wd.requires_grad_()
            ev_in = []
            for b in range(E2E_BLOCKS):
                sl = slice(b * rows_blk, (b + 1) * rows_blk)
                with torch.cuda.stream(s_in):
                    dxg[sl].copy_(hx[sl], non_blocking=True)
                    dresg[sl].copy_(hres[sl], non_blocking=True)
                    dout[sl].copy_(hdout[sl], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s_in)
                    ev_in.append(ev)
            for b in range(E2E_BLOCKS):
                sl = slice(b * rows_blk, (b + 1) * rows_blk)
                with torch.cuda.stream(s_cmp):
                    s_cmp.wait_event(ev_in[b])
                    xb = dxg[sl].detach().requires_grad_()
                    rb = dresg[sl].detach().requires_grad_()
                    o = quack_rmsnorm(xb, wd, residual=rb, eps=EPS)
                    o.backward(dout[sl])
                    ev = torch.cuda.Event()
                    ev.record(s_cmp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev)
                    o.record_stream(s_out)
                    xb.grad.record_stream(s_out)
                    h_out[sl].copy_(o.detach(), non_blocking=True)
                    h_dx[sl].copy_(xb.grad, non_blocking=True)  # dresidual is the same tensor
            with torch.cuda.stream(s_cmp):
                dwv = wd.grad
                if world > 1:
                    d32 = dwv.float()
                    dist.all_reduce(d32)
                    dwv = d32.to(bf)
                dwv.record_stream(s_out)
                ev = torch.cuda.Event()
                ev.record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                h_dw.copy_(dwv, non_blocking=True)
            for s in (s_in, s_cmp, s_out):
                cur.wait_stream(s)
            dwg.grad = None
            dwg.requires_grad_(False)

        e2e_steps = max(3, min(args.steps, 5))
        for _ in range(2):
            e2e_step()
        sync_all()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        sync_all()
        e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev)
        if world > 1:
            dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": world * step_bytes / float(e2e_ms) / 1e6, "unit": "GB/s",
               "h2d_bytes_per_step": 3 * M * N * 2 + N * 2, "d2h_bytes_per_step": 2 * M * N * 2 + N * 2,
               "ms_per_step": float(e2e_ms),
               "api": f"quack.rmsnorm(x, w, residual=res) + backward through autograd on {E2E_BLOCKS} row blocks; "
                      "pinned host buffers; x, residual, dout, weight copied in on one stream, out, "
                      "dx (= dresidual), dw copied back on another, kernels on a third"}
        del hx, hres, hdout, h_out, h_dx

    sharded_res = None
    if world > 1 and not args.no_suite:
        try:
            del x, res, dout, out, res_out, dx
            torch.cuda.empty_cache()
            sharded_res = sharded_suite(dev, rank, world, peak)
        except Exception as exc:  # the headline line must still be printed
            sharded_res = {"sharded_suite_error": repr(exc)}

    if rank == 0:
        fwd_ms = kms["rmsnorm_fwd"]
        fwd_gbs = fwd_bytes(M, N) / fwd_ms / 1e6
        counts = tl.counts()
        kernels = {
            "rmsnorm_fwd": {"ms": round(fwd_ms, 4), "gbs": round(fwd_gbs, 1),
                            "frac_of_measured_peak": round(fwd_gbs / peak, 4), "bytes": fwd_bytes(M, N),
                            "launches_timed": counts["rmsnorm_fwd"], "kernel": fwd_kernel},
            "rmsnorm_bwd": {"ms": round(kms["rmsnorm_bwd"], 4),
                            "gbs": round(bwd_bytes(M, N) / kms["rmsnorm_bwd"] / 1e6, 1),
                            "frac_of_measured_peak": round(bwd_bytes(M, N) / kms["rmsnorm_bwd"] / 1e6 / peak, 4),
                            "bytes": bwd_bytes(M, N), "launches_timed": counts["rmsnorm_bwd"]},
        }
        if "dw_colsum" in kms:
            kernels["dw_colsum"] = {"ms": round(kms["dw_colsum"], 4)}
        if "dw_colsum_allreduce" in kms:
            kernels["dw_colsum_allreduce"] = {
                "ms_on_side_stream": round(kms["dw_colsum_allreduce"], 4),
                "note": "event pair on the side stream: includes the time the kernel's blocks wait for SM "
                        "slots behind the next step's forward and for the slowest rank; it is off the critical "
                        "path (compare ms_per_step with --collective none)"}
        cpu = None
        if world == 1:
            try:
                cpu = cpu_baselines()
            except Exception as exc:
                cpu = {"error": repr(exc)}
        if world == 1 and not args.no_suite:
            try:
                del x, res, dout, out, res_out, dx
                torch.cuda.empty_cache()
                kernels.update(suite(dev, peak, cpu, args.no_graph))
                kernels["host_us_per_call"] = host_overhead(dev)
            except Exception as exc:  # the headline line must still be printed
                kernels["suite_error"] = repr(exc)
        if sharded_res:
            kernels.update(sharded_res)
        canary = None
        try:
            torch.cuda.empty_cache()
            canary = round(copy_canary(dev), 1)
        except Exception:
            pass
        # DRAM traffic of the forward kernel: from the committed Nsight Compute summary, if that
        # summary is about the very instantiation that ran here; scaled by rows (one pass per row).
        facts = profile_facts(FWD_PROFILE)
        traffic, traffic_note = None, "no profile summary for the kernel that ran"
        if facts.get("kernel") and facts.get("traffic_bytes_per_launch") and facts.get("rows"):
            if facts["kernel"] == fwd_kernel:
                traffic = round(float(facts["traffic_bytes_per_launch"]) / float(facts["rows"]) * M)
                traffic_note = (f"dram read+write of one ncu capture of {facts['kernel']} at {facts['rows']} rows "
                                f"(commit {facts.get('commit', '?')}), scaled by rows")
            else:
                traffic_note = (f"profile summary is about {facts['kernel']}, the step ran {fwd_kernel}: "
                                f"traffic not reported")
        # `config` is the same object in both arms (ours and --impl reference); what is specific to
        # this arm's step goes into `step_detail`.
        cfg = config_dict()
        detail = {"kernels": "rmsnorm_fwd kernel + rmsnorm_bwd kernel + dw column-sum kernel", "num_partials": P}
        if use_peer:
            detail["kernels"] = ("rmsnorm_fwd kernel + rmsnorm_bwd kernel + one kernel that sums dw over the partial "
                                 "slices and over the GPUs (plain stores into peer-mapped buffers, flags, bounded "
                                 "waits) on a side stream, overlapping the next step's forward")
            detail["collective"] = "peer stores (qb_colsum_allreduce)"
            detail["collective_timeouts"] = peer.timeouts()
        elif world > 1 and args.collective == "nccl":
            detail["kernels"] += (" + NCCL all-reduce of fp32 dw on a side stream, overlapping the next step's forward")
            detail["collective"] = "NCCL all-reduce"
            if peer_error:
                detail["collective_fallback_reason"] = peer_error
        elif world > 1:
            detail["collective"] = "none (diagnostic run)"
        mhz = clocks.get("sm_mhz") if clocks else None
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "pct_of_8TBs": round(100 * value / (world * NOMINAL_HBM_GBS), 2),
            "config": cfg,
            "step_detail": detail,
            "timing": {"blocks": len(blocks), "block_ms_median": round(ms_block, 4),
                       "block_ms_min": round(min(blocks), 4), "block_ms_max": round(max(blocks), 4),
                       "rule": f"blocks of {args.steps} steps repeated for >= {MIN_TIMED_SECONDS} s; median block",
                       "per_kernel": f"event pairs around every launch of 3 further blocks of {args.steps} steps, "
                                     "directly after the timed blocks (an event pair per kernel inside them "
                                     "costs the step 5-7 %)",
                       "ms_per_step_x_sm_mhz": round(ms_step * mhz, 2) if mhz else None,
                       "cuda_graph": None if not graph_ms or graph_ms["step"] is None else {
                           "protocol": "20 steps (fwd + bwd + column sum) or 20 launches of one kernel captured "
                                       "in one CUDA graph, median of 7 replays",
                           "ms_per_step": round(graph_ms["step"], 4),
                           "value": round(step_bytes / graph_ms["step"] / 1e6, 1),
                           "rmsnorm_fwd_ms": graph_ms["rmsnorm_fwd"] and round(graph_ms["rmsnorm_fwd"], 4),
                           "rmsnorm_fwd_gbs": graph_ms["rmsnorm_fwd"] and round(
                               fwd_bytes(M, N) / graph_ms["rmsnorm_fwd"] / 1e6, 1),
                           "rmsnorm_bwd_ms": graph_ms["rmsnorm_bwd"] and round(graph_ms["rmsnorm_bwd"], 4),
                           "rmsnorm_bwd_gbs": graph_ms["rmsnorm_bwd"] and round(
                               bwd_bytes(M, N) / graph_ms["rmsnorm_bwd"] / 1e6, 1)}},
            "roofline": {"bound": "hbm", "kernel": fwd_kernel,
                         "achieved": round(fwd_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(fwd_gbs / peak, 4), "peak_source": peak_src,
                         "traffic": traffic, "traffic_note": traffic_note},
            "copy_canary_gbs": canary,
            "cpu_baseline": (cpu or {}).get("headline") if cpu and "error" not in cpu else cpu,
            "cpu_baselines": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps * len(blocks),
            "clocks": clocks,
            "strong_scaling": strong,
            "kernels": kernels,
        }
        print(json.dumps(line), flush=True)
    if peer is not None:
        peer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-suite", action="store_true", help="skip the per-kernel sweep of the other configurations")
    ap.add_argument("--e2e-blocks", type=int, default=16,
                    help="row blocks of the end-to-end leg (copies and kernels of different blocks overlap)")
    ap.add_argument("--no-graph", action="store_true",
                    help="skip the CUDA-graph timings (keeps a profiler's launch list short)")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (for profiler launch lists of the timed step alone)")
    ap.add_argument("--collective", default="peer", choices=["peer", "nccl", "none"],
                    help="N > 1: how dw is summed over the GPUs (fused peer-store kernel, or column sum + NCCL)")
    ap.add_argument("--only", default=None, help="run one kernel on a small case (for ncu captures)")
    ap.add_argument("--rows", type=int, default=0)
    ap.add_argument("--cols", type=int, default=0)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
