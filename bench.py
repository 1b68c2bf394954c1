"""Benchmark of the fused all-gather GEMM (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mlp70b|qkv8b|smoke]

Launched as one process per GPU (torchrun for N > 1).  A "step" is one launch
of C_r = AllGather(A_r) . B_r^T over the workload's shapes on every rank:

  mlp70b (default)  Llama-3-70B MLP gate+up projection: M = 16384 tokens
                    (M/N per rank), K = 8192, 57344 output columns in total
                    (57344/N per rank), bf16, fp32 accumulate, bf16 output;
  qkv8b             Llama-3-8B QKV projection: M = 8192, K = 4096, N = 6144;
  smoke             M = 1024, K = 1024, N = 1024.

--op rs times the row-parallel twin instead (GEMM + reduce-scatter):
  mlp70b_down       Llama-3-70B MLP down projection: M = 16384, K = 28672
                    (28672/N per rank), N = 8192; rank r keeps rows r of the sum.

Inputs are synthetic, seeded per rank on the device: activations ~ N(0, 1),
weights ~ N(0, 0.02).  They are larger than L2 at mlp70b/qkv8b, so no flush
is inserted between timed steps (smoke flushes L2 with a 256 MiB write).

value   whole-job TFLOP/s = 2*M*K*N_total / (max over ranks of the device time
        per step), inputs resident in HBM;
e2e     the same through the public API with host buffers: each step copies
        A_r from pinned host memory to the GPU, launches, and copies C_r back;
unfused the baseline of an NCCL all-gather followed by a cuBLAS GEMM (torch);
cpu_baseline  the CPU oracle's fp32 GEMM on a bounded sample (rank 0, N = 1).

--impl reference times the reference's CPU path for this workload: the
reference has no CPU GEMM of its own, so this is the oracle's restatement of
its fp32 check (include/reference_matmul.cuh:17-32), multithreaded, on a
bounded sample per step; only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def delta(before, after):
    if before is None or after is None:
        return None
    return after[0] - before[0], after[1] - before[1]


def NvlinkCounters(device):
    """This GPU's NVLink byte counters (the package's NVML reader)."""
    import __graft_entry__ as ge

    pkg = ge.load_package()
    import importlib

    return importlib.import_module(pkg.__name__ + ".nvlink_counters").NvlinkCounters(device)

WORKLOADS = {
    "mlp70b": dict(name="llama3-70b-mlp-gate-up", M=16384, K=8192, N=57344),
    "qkv8b": dict(name="llama3-8b-qkv", M=8192, K=4096, N=6144),
    "smoke": dict(name="smoke-1024", M=1024, K=1024, N=1024),
    # a 4096-row x 8192-column slice of mlp70b (256 MB of operands): the case
    # the ncu captures run on
    "mlp70b_slice": dict(name="llama3-70b-mlp-slice", M=4096, K=8192, N=8192),
    # a 9472-row x 2048-column block of mlp70b: exactly two waves of 256 x 512
    # tiles on 148 SMs (A 155 MB + B 34 MB + C 39 MB, more than L2)
    "mlp70b_block": dict(name="llama3-70b-mlp-block", M=9472, K=8192, N=2048),
    # the row-parallel twin (--op rs): Llama-3-70B MLP down projection, K split over ranks
    "mlp70b_down": dict(name="llama3-70b-mlp-down", M=16384, K=28672, N=8192),
}
NVLINK_GBS = 770.0        # measured peer copy per direction on this pool
NVLINK_NOMINAL_GBS = 900.0  # NVLink 5, per direction per GPU (the north-star roofline's figure)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# Parity bar after each timed run (the reference's check_close defaults,
# include/reference_matmul.cuh:103-104, plus a normwise bound per dtype).
CHECK_ATOL, CHECK_RTOL = 0.1, 0.02
MAX_REL = {"bf16": 1e-2, "e4m3": 3e-2}


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return dict(bf16=float(d["bf16_tflops"]), bf16_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                    hbm=float(d["hbm_gbs"]), source="measured")
    except Exception:
        return dict(bf16=FALLBACK_BF16_TFLOPS, bf16_sustained=1400.0, hbm=FALLBACK_HBM_GBS, source="fallback")


def measure_e4m3_peak(dev, n=8192, reps=10):
    """Dense e4m3 tensor throughput of this GPU, measured the way the bf16 peak
    is: cuBLASLt (torch._scaled_mm, tensor-wise scales, bf16 out) on an n^3
    GEMM, best of `reps` CUDA-event-timed launches after warm-up (burst)."""
    import torch

    g = torch.Generator(device=dev).manual_seed(3)
    a = (torch.randn(n, n, device=dev, generator=g) * 0.5).to(torch.float8_e4m3fn)
    b = (torch.randn(n, n, device=dev, generator=g) * 0.5).to(torch.float8_e4m3fn)
    one = torch.ones((), device=dev, dtype=torch.float32)
    out = torch.empty(n, n, device=dev, dtype=torch.bfloat16)

    def run():
        return torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16, out=out)

    for _ in range(3):
        run()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b, out
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def compare_rows(got, want_rows, rows, chunk=2048, extra_tol=None):
    """The reference's check_close on the device, chunked over rows:
    |got - want| <= atol + rtol * |want| (+ extra_tol(r0, r1)) for every element
    (a NaN counts as a mismatch), plus the normwise max|got - want| / max|want|.
    `want_rows(r0, r1)` returns the fp32 reference rows [r0, r1)."""
    import torch

    bad, max_diff, max_ref = 0, 0.0, 0.0
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        w = want_rows(r0, r1)
        d = (got[r0:r1].float() - w).abs()
        tol = CHECK_ATOL + CHECK_RTOL * w.abs()
        if extra_tol is not None:
            tol = tol + extra_tol(r0, r1)
        bad += int((~(d <= tol)).sum().item())
        max_diff = max(max_diff, float(torch.nan_to_num(d, nan=float("inf")).max().item()))
        max_ref = max(max_ref, float(w.abs().max().item()))
        del w, d, tol
    return bad, (max_diff / max_ref if max_ref > 0 else max_diff)


def reduce_parity(local, world, group):
    """Combine per-rank parity results: worst error, total mismatches, and every
    rank's gather verdict."""
    if world == 1:
        return local
    import torch
    import torch.distributed as dist

    worst = torch.tensor([local["max_rel_err"]], dtype=torch.float64)
    counts = torch.tensor([float(local["check_close_bad"]),
                           0.0 if local.get("gather_bitexact", True) in (True, None) else 1.0], dtype=torch.float64)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
    out = dict(local)
    out["max_rel_err"] = float(worst[0])
    out["check_close_bad"] = int(counts[0])
    if "gather_bitexact" in local and local["gather_bitexact"] is not None:
        out["gather_bitexact"] = counts[1].item() == 0.0
    out["ranks_checked"] = world
    return out


def wire_summary(wire, steps, ms, expected_bytes, world, group):
    """Per-rank NVLink bytes of one step from the hardware counters read around
    the timed region, beside the bytes the exchange must move per rank."""
    import torch.distributed as dist

    mine = None if wire.last is None else (wire.last[0] / steps, wire.last[1] / steps)
    ranks = [None] * world
    dist.all_gather_object(ranks, mine, group=group)
    out = wire.describe()
    if all(r is not None for r in ranks):
        out.update({"tx_bytes_per_step": [r[0] for r in ranks], "rx_bytes_per_step": [r[1] for r in ranks],
                    "expected_bytes_per_rank": expected_bytes,
                    "rx_gbs_over_step": [r[1] / (ms * 1e-3) / 1e9 for r in ranks],
                    "tx_gbs_over_step": [r[0] / (ms * 1e-3) / 1e9 for r in ranks]})
    return out


def ncu_traffic(workload):
    """DRAM bytes per launch of the fused kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"ag_gemm_wide_kernel_{workload}.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


class NvmlClockSampler:
    """Clock, power and clock-event-reason samples every 5 ms from NVML in a
    background thread (reads only), so that even a timed region of a few tens of
    milliseconds is covered by several samples."""

    # nvmlClocksEventReason* bits
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, index):
        import threading

        import pynvml
        import torch

        self.nv = pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(index).uuid)
        self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        self.rows = []
        self.stop_evt = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nv
        while not self.stop_evt.is_set():
            try:
                self.rows.append((float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)),
                                  nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0,
                                  int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))))
            except nv.NVMLError:
                pass
            self.stop_evt.wait(0.005)

    def start(self):
        self.thread.start()
        while not self.rows and self.thread.is_alive():
            time.sleep(0.001)

    def stop(self):
        self.stop_evt.set()
        self.thread.join(timeout=5)
        if not self.rows:
            return None
        mhz = sorted(r[0] for r in self.rows)
        watts = sorted(r[1] for r in self.rows)
        reasons = sorted({name for r in self.rows for bit, name in self.REASONS.items() if r[2] & bit})
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "power_w": watts[len(watts) // 2], "samples": len(self.rows), "source": "NVML, 5 ms"}


class ClockSampler:
    """Clock / throttle sampling during the timed region: NVML every 5 ms where
    it answers, else nvidia-smi every 50 ms."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None
        try:
            self.nvml = NvmlClockSampler(index)
        except Exception:
            self.nvml = None

    def start(self):
        if self.nvml is not None:
            self.nvml.start()
            return
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # wait until the sampler is producing lines, so the timed region is covered
        t0 = time.time()
        while time.time() - t0 < 5.0 and os.path.getsize(self.path) == 0:
            time.sleep(0.05)

    def stop(self):
        if self.nvml is not None:
            return self.nvml.stop()
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        mhz = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        max_mhz = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        watts = sorted(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": max_mhz, "reasons": reasons,
                "power_w": watts[len(watts) // 2] if watts else None, "samples": len(rows),
                "source": "nvidia-smi, 50 ms"}


# ------------------------------------------------------------------ reference arm
def run_reference(args, rank, emit):
    if rank != 0:
        return
    import numpy as np

    import __graft_entry__ as ge

    oracle = ge.load_oracle()
    w = WORKLOADS[args.workload]
    world = args.gpus
    K = w["K"]
    n_r = w["N"] // world
    rows, cols = 256, min(2048, n_r)
    rng = np.random.default_rng(0)
    A = rng.standard_normal((rows, K), dtype=np.float32)
    B = (rng.standard_normal((cols, K), dtype=np.float32) * 0.02).astype(np.float32)
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        oracle.gemm_f32(A, B, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.gemm_f32(A, B, threads)
    dt = (time.perf_counter() - t0) / args.steps
    tflops = 2.0 * rows * cols * K / dt / 1e12
    sample = f"{rows} rows x {cols} cols x K={K} of the {w['name']} GEMM per step (fp32, {threads} threads)"
    line = {
        "impl": "reference", "metric": RS_METRIC if args.op == "rs" else METRIC, "value": tflops,
        "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args.workload, world),
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


METRIC = "all-gather GEMM TFLOP/s per GPU at 1/2/4/8 B200; % of roofline; vs NCCL+cuBLAS"


def config_of(workload, world, dtype="bf16"):
    w = WORKLOADS[workload]
    return {"workload": w["name"] + ("-e4m3" if dtype == "e4m3" else ""), "M": w["M"], "K": w["K"],
            "N_total": w["N"], "N_per_rank": w["N"] // world,
            "M_per_rank": w["M"] // world, "P": world,
            "l2": "inputs larger than L2, no flush" if workload != "smoke" else "256 MiB L2 flush between steps",
            "parallelism": f"ag-tp{world}"}


# ------------------------------------------------------------------ NVLink probe
def run_nvlink_probe(args, emit):
    """One process, GPUs 0 and 1 (the reference's thread-per-GPU set-up,
    minfer_spmm_init, done here from one thread): GPU 0 broadcasts `size` bytes
    once into the multicast slab with 16-byte multimem.st (agg_mc_broadcast),
    then both GPUs' copies are checked byte for byte.  The broadcast waits on
    nothing, so it can be profiled on its own (the NVLink tx/rx byte counters
    of the sending GPU)."""
    import ctypes

    import torch

    import __graft_entry__ as ge

    pkg = ge.load_package()
    agg = pkg.agg
    L = agg.lib()
    if torch.cuda.device_count() < 2:
        raise SystemExit("--nvlink-probe needs two GPUs")
    size = args.nvlink_probe
    world = 2
    for r in range(world):
        agg.spmm_init(r, world, r, world * size)
    infos = [agg.spmm_init(r, world, r, world * size) for r in range(world)]
    try:
        torch.cuda.set_device(0)
        g = torch.Generator(device="cuda:0").manual_seed(5)
        src = (torch.rand(size // 2, device="cuda:0", generator=g) * 2 - 1).bfloat16()
        stream = torch.cuda.current_stream(0)
        sp = ctypes.c_void_p(stream.cuda_stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        agg.check(L.agg_mc_broadcast(ctypes.c_void_p(src.data_ptr()), infos[0].mc, size, None, 0, sp),
                  "agg_mc_broadcast")
        e1.record(stream)
        torch.cuda.synchronize(0)
        ms = e0.elapsed_time(e1)
        bad = 0
        for r in range(world):
            with torch.cuda.device(r):
                st = torch.cuda.current_stream(r)
                rp = ctypes.c_void_p(st.cuda_stream)
                exp = src.to(f"cuda:{r}")
                cnt = torch.zeros(1, dtype=torch.int64, device=f"cuda:{r}")
                agg.check(L.agg_alias_fence(rp))
                agg.check(L.agg_verify_bytes(ctypes.c_void_p(infos[r].uc), ctypes.c_void_p(exp.data_ptr()), size,
                                             ctypes.c_void_p(cnt.data_ptr()), rp))
                torch.cuda.synchronize(r)
                bad += int(cnt.item())
    finally:
        for r in range(world):
            torch.cuda.synchronize(r)
            L.agg_spmm_finalize(r)
    emit({"probe": "multimem.st broadcast from GPU 0 to GPUs 0 and 1 (one launch)", "bytes": size, "ms": ms,
          "sender_gbs": size / (ms * 1e-3) / 1e9, "mismatched_words": bad})
    if bad:
        sys.exit(1)


# ------------------------------------------------------------------ our arm
def cpu_baseline(workload):
    import numpy as np

    import __graft_entry__ as ge

    oracle = ge.load_oracle()
    w = WORKLOADS[workload]
    K = w["K"]
    rows, cols = 512, 2048
    rng = np.random.default_rng(1)
    A = rng.standard_normal((rows, K), dtype=np.float32)
    B = rng.standard_normal((cols, K), dtype=np.float32)
    threads = os.cpu_count() or 1
    oracle.gemm_f32(A[:64], B[:256], threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.gemm_f32(A, B, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el > 10.0 or reps >= 50:
            break
    tflops = 2.0 * rows * cols * K * reps / el / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x ({rows} x {cols} x K={K}) slices of the {w['name']} GEMM, fp32, {el:.1f} s"}


RS_METRIC = "GEMM + reduce-scatter TFLOP/s per GPU at 1/2/4/8 B200; % of roofline; vs cuBLAS+NCCL"


def run_rs(args, pkg, rank, world, dev, host_group, emit):
    """The row-parallel twin: Y_r = rows r of sum_s X_s . W_s^T, K split over the
    ranks.  A step is one launch on every rank; the unfused baseline is a cuBLAS
    GEMM to a full [M, N] bf16 partial followed by an NCCL reduce-scatter."""
    import torch
    import torch.distributed as dist

    w = WORKLOADS[args.workload]
    M, Ktot, N = w["M"], w["K"], w["N"]
    k_r, m_local = Ktot // world, M // world
    g = torch.Generator(device=dev).manual_seed(1000 * rank + 9)
    X_r = torch.randn(M, k_r, device=dev, generator=g).bfloat16()
    W_r = (torch.randn(N, k_r, device=dev, generator=g) * 0.02).bfloat16()
    Y_r = torch.empty(m_local, N, device=dev, dtype=torch.bfloat16)
    if args.ce_streams:  # read by the library at each launch
        os.environ["AGG_RS_CE_STREAMS"] = str(args.ce_streams)
    else:
        os.environ.pop("AGG_RS_CE_STREAMS", None)
    op = pkg.GemmReduceScatter(M, N, k_r, host_group=host_group, exchange=args.exchange)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(group=host_group)

    def timed(step_fn, steps, wire=None):
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0 = wire.read() if wire is not None else None
        e0.record(stream)
        for _ in range(steps):
            step_fn()
        e1.record(stream)
        torch.cuda.synchronize()
        if wire is not None:
            wire.last = delta(c0, wire.read())
        barrier()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=host_group)
        return float(t.item())

    for _ in range(args.warmup):
        op(X_r, W_r, out=Y_r)
    torch.cuda.synchronize()
    op.check_status()
    wire = NvlinkCounters(dev.index) if world > 1 else None
    clocks = ClockSampler(dev.index)
    clocks.start()
    ms = timed(lambda: op(X_r, W_r, out=Y_r), args.steps, wire)
    clk = clocks.stop()
    op.check_status()

    flops_rank = 2.0 * M * N * k_r
    value = flops_rank * world / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    t_tc = flops_rank / (peaks["bf16"] * 1e12)
    nvl_bytes = (world - 1) / world * M * N * 2 if world > 1 else 0.0   # partials leaving each GPU
    t_nvl = nvl_bytes / (NVLINK_GBS * 1e9)
    t_nvl9 = nvl_bytes / (NVLINK_NOMINAL_GBS * 1e9)
    t_roof = max(t_tc, t_nvl)
    roofline = {"bound": "tensor" if t_tc >= t_nvl else "nvlink", "achieved": flops_rank / (ms * 1e-3) / 1e12,
                "peak": peaks["bf16"], "unit": "TFLOP/s", "frac": t_roof / (ms * 1e-3),
                "peak_source": f"{peaks['source']} bf16 burst (cuBLAS)", "traffic": None,
                "t_roof_ms": t_roof * 1e3, "t_tensor_ms": t_tc * 1e3, "t_nvlink_ms": t_nvl * 1e3,
                "nvlink_bytes_per_rank": nvl_bytes, "nvlink_gbs": NVLINK_GBS,
                "frac_at_900gbs": max(t_tc, t_nvl9) / (ms * 1e-3), "t_nvlink_ms_at_900gbs": t_nvl9 * 1e3}
    out = {"metric": RS_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic (X~N(0,1), W~N(0,0.02), seeded per rank)",
           "config": {"workload": w["name"], "M": M, "K_total": Ktot, "K_per_rank": k_r, "N": N,
                      "M_out_per_rank": m_local, "P": world, "l2": "inputs larger than L2, no flush",
                      "parallelism": f"rs-tp{world}", "exchange": op.exchange if world > 1 else None,
                      "copy_streams": int(os.environ.get("AGG_RS_CE_STREAMS", "1"))
                      if world > 1 and op.exchange == "ce" else None},
           "tflops_per_gpu": value / world, "gpu_launches": args.steps, "roofline": roofline, "clocks": clk}
    if wire is not None:
        out["nvlink_counters"] = wire_summary(wire, args.steps, ms, nvl_bytes, world, host_group)

    if not args.no_unfused:
        P_full = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        Y_u = torch.empty(m_local, N, device=dev, dtype=torch.bfloat16)

        def step_unfused():
            torch.matmul(X_r, W_r.t(), out=P_full)
            if world > 1:
                dist.reduce_scatter_tensor(Y_u, P_full)
            else:
                Y_u.copy_(P_full)

        for _ in range(args.warmup):
            step_unfused()
        ums = timed(step_unfused, args.steps)
        out["unfused_nccl_cublas"] = {"value": flops_rank * world / (ums * 1e-3) / 1e12, "unit": "TFLOP/s",
                                      "ms_per_step": ums, "speedup_fused": ums / ms}
        if world > 1:
            # same inputs, same reduction: the fused rows against NCCL's (bf16 partials both ways)
            ref = Y_u.float()
            out["unfused_max_rel_diff"] = float(((Y_r.float() - ref).abs().max() / ref.abs().max()).item())
        del P_full, Y_u

    if not args.no_e2e:
        X_host = torch.empty(M, k_r, dtype=torch.bfloat16, pin_memory=True)
        X_host.copy_(X_r)
        Y_host = torch.empty(m_local, N, dtype=torch.bfloat16, pin_memory=True)
        X_dev = torch.empty_like(X_r)

        def step_e2e():
            X_dev.copy_(X_host, non_blocking=True)
            op(X_dev, W_r, out=Y_r)
            Y_host.copy_(Y_r, non_blocking=True)

        step_e2e()
        e2e_steps = args.steps
        ems = timed(step_e2e, e2e_steps)
        out["e2e"] = {"value": flops_rank * world / (ems * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "h2d_bytes_per_step": X_host.numel() * 2, "d2h_bytes_per_step": Y_host.numel() * 2,
                      "ms_per_step": ems, "steps": e2e_steps, "gpu_launches": e2e_steps}
        op.check_status()
        del X_host, Y_host, X_dev

    # ---- parity of one more launch against an independent result: the fp32
    # partial X_r . W_r^T of every rank (cuBLAS SGEMM, no TF32), summed by an
    # fp32 NCCL reduce-scatter.  Each rank's partial is rounded to bf16 before
    # the fused sum (as in a bf16 reduce-scatter), so the element check is the
    # reference's check_close widened by 2^-8 x sum_s |partial_s|.
    torch.backends.cuda.matmul.allow_tf32 = False
    op(X_r, W_r, out=Y_r)
    torch.cuda.synchronize()
    op.check_status()
    part = X_r.float() @ W_r.float().t()
    if world > 1:
        want = torch.empty(m_local, N, device=dev, dtype=torch.float32)
        absum = torch.empty_like(want)
        dist.reduce_scatter_tensor(want, part)
        dist.reduce_scatter_tensor(absum, part.abs_())
    else:
        want, absum = part, part.abs()
    del part
    bad, rel = compare_rows(Y_r, lambda r0, r1: want[r0:r1], m_local,
                            extra_tol=lambda r0, r1: absum[r0:r1] * 2.0 ** -8)
    del want, absum
    par = reduce_parity({"max_rel_err": rel, "check_close_bad": bad}, world, host_group)
    par["ok"] = par["check_close_bad"] == 0 and par["max_rel_err"] <= MAX_REL["bf16"]
    par["reference"] = ("sum over ranks of fp32 X_s . W_s^T (cuBLAS SGEMM, TF32 off) reduce-scattered in fp32; "
                        "check_close atol 0.1 rtol 0.02 + 2^-8 sum|partial| on every element, "
                        f"max|Y - ref| / max|ref| <= {MAX_REL['bf16']}")
    out["parity"] = par

    if args.trace and world > 1:
        tr = op.new_trace()
        torch.cuda.synchronize()
        barrier()
        op(X_r, W_r, out=Y_r, trace=tr)
        torch.cuda.synchronize()
        op.check_status()
        per_rank = [None] * world
        dist.all_gather_object(per_rank, tr.cpu().numpy(), group=host_group)
        if rank == 0:
            with open(args.trace, "w") as f:
                json.dump({"workload": out["config"], "ranks": [pkg.agg.trace_summary(r) for r in per_rank]}, f,
                          indent=1)

    op.close()
    if rank == 0:
        emit(out)
    barrier()
    return out["parity"]["ok"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mlp70b", choices=sorted(WORKLOADS))
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "e4m3"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-unfused", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="multicast write bandwidth sweep (1 MiB .. --sweep-max) instead of the GEMM")
    ap.add_argument("--sweep-max", type=int, default=1 << 30)
    ap.add_argument("--sweep-ce", action="store_true",
                    help="add the copy-engine all-gathers (multicast push, push ring, pull ring) to the sweep")
    ap.add_argument("--producer", default="auto", choices=["auto", "sm", "ce_mc", "ce_push", "sm_peer"],
                    help="who moves the shards in the fused kernel: its producer warps by one multicast "
                         "store (sm) or by a store per peer (sm_peer), or the copy engines; auto: sm_peer for "
                         "bf16 on 2-4 GPUs, sm otherwise")
    ap.add_argument("--trace", default=None, metavar="PATH",
                    help="after timing, trace one launch per rank and write the per-event summary to PATH")
    ap.add_argument("--exchange", default="auto", choices=["auto", "sm", "ce"],
                    help="--op rs: who moves the partials, the epilogue's TMA stores into the owners' inboxes "
                         "(sm) or the copy engines from a local stage (ce); auto: ce")
    ap.add_argument("--ce-streams", type=int, default=0,
                    help="--op rs --exchange ce: internal copy streams per block (1-4; 0: the library default)")
    ap.add_argument("--also", default="", metavar="RUNS",
                    help="comma-separated further runs in the same process group after the first, each "
                         "WORKLOAD[:e4m3][:sm|sm_peer|ce_mc|ce_push] or rs[:WORKLOAD][:sm|ce][:sN] (N copy "
                         "streams); one result line each")
    ap.add_argument("--nvlink-probe", type=int, default=0, metavar="BYTES",
                    help="one process on GPUs 0-1: a single multicast broadcast of BYTES from GPU 0, checked on "
                         "both GPUs (for a profiler capture of its NVLink counters)")
    ap.add_argument("--op", default="ag", choices=["ag", "rs"],
                    help="ag: the all-gather GEMM (default); rs: its GEMM + reduce-scatter twin "
                         "(default workload mlp70b_down)")
    args = ap.parse_args()
    if args.op == "rs" and args.workload == "mlp70b":
        args.workload = "mlp70b_down"
    args.warmup = max(args.warmup, 3)
    # Library banners (NCCL, ...) go to stderr: stdout carries only the result line.
    sys.stdout.flush()
    result_fd = os.dup(1)
    os.dup2(2, 1)

    def emit(obj):
        sys.stdout.flush()
        os.write(result_fd, (json.dumps(obj) + "\n").encode())

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        args.gpus = world

    if args.impl == "reference":
        run_reference(args, rank, emit)
        return
    if args.nvlink_probe:
        run_nvlink_probe(args, emit)
        return

    import datetime

    import torch
    import torch.distributed as dist

    import __graft_entry__ as ge

    pkg = ge.load_package()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    host_group = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))

    if args.sweep:
        if world < 2:
            raise SystemExit("--sweep needs torchrun with 2 or more ranks")
        import importlib

        sweep = importlib.import_module(pkg.__name__ + ".sweep")
        sizes = []
        s = 1 << 20
        while s <= args.sweep_max:
            sizes.append(s)
            s <<= 1
        slab = pkg.agg.MulticastSlab(rank, world, local_rank, world * sizes[-1], pkg.agg.make_job_id(host_group),
                                     lambda: dist.barrier(group=host_group))
        try:
            rows, wire = sweep.run(slab, sizes, reps=args.steps, warmup=args.warmup, group=host_group,
                                   copy_engines=args.sweep_ce)
        finally:
            torch.cuda.synchronize()
            dist.barrier(group=host_group)
            slab.close()
            dist.barrier(group=host_group)
        if rank == 0:
            emit({"sweep": "multicast multimem.st write bandwidth", "n_gpus": world, "unit": "GB/s",
                  "nvlink_counters": wire, "nvlink_nominal_gbs_per_direction": NVLINK_NOMINAL_GBS,
                  "rows": rows})
        dist.destroy_process_group()
        return

    # The run named on the command line, then any --also runs in the same
    # process group (one line each; the driver's runs use the first only).
    runs = [args]
    for spec in [x for x in args.also.split(",") if x]:
        r = argparse.Namespace(**vars(args))
        r.also = ""
        parts = spec.split(":")
        r.op = "rs" if parts[0] == "rs" else "ag"
        if r.op == "rs":
            r.workload = next((x for x in parts[1:] if x in WORKLOADS), "mlp70b_down")
            r.exchange = next((x for x in parts[1:] if x in ("sm", "ce")), "auto")
            r.ce_streams = next((int(x[1:]) for x in parts[1:] if x[:1] == "s" and x[1:].isdigit()), 0)
        else:
            r.workload = parts[0]
        r.dtype = next((x for x in parts[1:] if x in ("bf16", "e4m3")), "bf16")
        r.producer = next((x for x in parts[1:] if x in ("sm", "ce_mc", "ce_push", "sm_peer")), "auto")
        runs.append(r)
    ok = True
    for r in runs:
        if r.trace and "{}" in r.trace:
            mode = f"{r.exchange}{r.ce_streams or ''}" if r.op == "rs" else r.producer
            r.trace = r.trace.format(f"{r.op}_{r.workload}_{r.dtype}_{mode}")
        if r.op == "rs":
            ok = run_rs(r, pkg, rank, world, dev, host_group, emit) and ok
        else:
            ok = run_ag(r, pkg, rank, world, local_rank, dev, host_group, emit) and ok
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier(group=host_group)
        dist.destroy_process_group()
    if not ok:
        sys.exit(1)


def run_ag(args, pkg, rank, world, local_rank, dev, host_group, emit):
    """The fused all-gather GEMM on one workload; returns the parity verdict."""
    import torch
    import torch.distributed as dist

    w = WORKLOADS[args.workload]
    M, K, Ntot = w["M"], w["K"], w["N"]
    m_local, n_r = M // world, Ntot // world
    g = torch.Generator(device=dev).manual_seed(1000 * rank + 7)
    A_r = torch.randn(m_local, K, device=dev, generator=g).bfloat16()
    B_r = (torch.randn(n_r, K, device=dev, generator=g) * 0.02).bfloat16()
    C_r = torch.empty(M, n_r, device=dev, dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if args.workload == "smoke" else None
    f8 = args.dtype == "e4m3"
    if f8:
        # per-row amax e4m3 of A_r, per-output-column (= per row of B_r [N_r, K]) e4m3 of B_r
        A_in, S_a = pkg.agg.quantize_rows_e4m3(A_r)
        B_in, S_b = pkg.agg.quantize_rows_e4m3(B_r)
        del A_r, B_r
    else:
        A_in, B_in, S_a, S_b = A_r, B_r, None, None
    elem = 1 if f8 else 2

    op = pkg.AllGatherGemm(m_local, K, dtype=args.dtype, host_group=host_group, producer=args.producer)
    stream = torch.cuda.current_stream()

    def launch(A, out, trace=None):
        return op(A, B_in, out=out, scale_a=S_a, scale_b=S_b, trace=trace)

    def barrier():
        if world > 1:
            dist.barrier(group=host_group)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=host_group)
        return float(t.item())

    def timed(step_fn, steps, wire=None):
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        c0 = wire.read() if wire is not None else None
        e0.record(stream)
        for _ in range(steps):
            step_fn()
        e1.record(stream)
        torch.cuda.synchronize()
        if wire is not None:
            wire.last = delta(c0, wire.read())
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps)

    def step_ours():
        if flush is not None:
            flush.fill_(1)
        launch(A_in, C_r)

    for _ in range(args.warmup):
        step_ours()
    torch.cuda.synchronize()
    op.check_status()

    wire = NvlinkCounters(local_rank) if world > 1 else None
    clocks = ClockSampler(local_rank)
    clocks.start()
    ms = timed(step_ours, args.steps, wire)
    clk = clocks.stop()
    op.check_status()
    # kernel-only time of the same launches (the flush is excluded for smoke)
    kernel_ms = ms if flush is None else timed(lambda: launch(A_in, C_r), args.steps)

    flops_step = 2.0 * M * K * Ntot
    value = flops_step / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    flops_rank = 2.0 * M * K * n_r
    achieved = flops_rank / (kernel_ms * 1e-3) / 1e12
    nvl_bytes = (world - 1) / world * M * K * elem if world > 1 else 0.0
    # the committed DRAM capture is of the bf16 kernel at world 1
    traffic = ncu_traffic(args.workload) if (not f8 and world == 1 and not os.environ.get("AGG_KERNEL")) else None

    def roofline_for(peak_tc, source):
        t_tc = flops_rank / (peak_tc * 1e12)
        t_nvl = nvl_bytes / (NVLINK_GBS * 1e9)
        t_nvl9 = nvl_bytes / (NVLINK_NOMINAL_GBS * 1e9)
        t_roof = max(t_tc, t_nvl)
        return {"bound": "tensor" if t_tc >= t_nvl else "nvlink", "achieved": achieved, "peak": peak_tc,
                "unit": "TFLOP/s", "frac": t_roof / (kernel_ms * 1e-3), "peak_source": source,
                "traffic": traffic, "t_roof_ms": t_roof * 1e3, "t_tensor_ms": t_tc * 1e3,
                "t_nvlink_ms": t_nvl * 1e3, "nvlink_bytes_per_rank": nvl_bytes, "nvlink_gbs": NVLINK_GBS,
                "frac_at_900gbs": max(t_tc, t_nvl9) / (kernel_ms * 1e-3), "t_nvlink_ms_at_900gbs": t_nvl9 * 1e3}

    # e4m3: replaced below by the e4m3 peak measured on this GPU after the timed runs
    roofline = roofline_for(peaks["bf16"] * (2.0 if f8 else 1.0),
                            f"{peaks['source']} bf16 burst (cuBLAS)" + (" x 2 for e4m3 (nominal)" if f8 else ""))

    out = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": args.dtype,
           "data": "synthetic (A~N(0,1), B~N(0,0.02), seeded per rank)" + (", per-row amax e4m3" if f8 else ""),
           "config": dict(config_of(args.workload, world, args.dtype), producer=op.producer),
           "tflops_per_gpu": value / world,
           "gpu_launches": args.steps, "roofline": roofline, "clocks": clk}
    if wire is not None:
        out["nvlink_counters"] = wire_summary(wire, args.steps, ms, nvl_bytes, world, host_group)

    # ---- unfused baseline: NCCL all-gather + cuBLAS GEMM (cuBLASLt fp8 for e4m3)
    if not args.no_unfused:
        A_full = torch.empty(M, K, device=dev, dtype=A_in.dtype)
        S_full = torch.empty(M, device=dev, dtype=torch.float32) if f8 else None
        C_u = torch.empty(M, n_r, device=dev, dtype=torch.bfloat16)

        def step_unfused():
            if flush is not None:
                flush.fill_(1)
            if world > 1:
                dist.all_gather_into_tensor(A_full, A_in)
                if f8:
                    dist.all_gather_into_tensor(S_full, S_a)
                a, sa = A_full, S_full
            else:
                a, sa = A_in, S_a
            if f8:
                C_u.copy_(torch._scaled_mm(a.view(torch.float8_e4m3fn), B_in.view(torch.float8_e4m3fn).t(),
                                           scale_a=sa[:, None], scale_b=S_b[None, :], out_dtype=torch.bfloat16))
            else:
                torch.matmul(a, B_in.t(), out=C_u)

        try:
            for _ in range(args.warmup):
                step_unfused()
            ums = timed(step_unfused, args.steps)
            out["unfused_nccl_cublas"] = {"value": flops_step / (ums * 1e-3) / 1e12, "unit": "TFLOP/s",
                                          "ms_per_step": ums, "speedup_fused": ums / ms}
        except RuntimeError as e:  # e.g. no rowwise-scaled fp8 GEMM in this torch build
            out["unfused_nccl_cublas"] = {"unavailable": str(e).splitlines()[0][:200]}
        del A_full, C_u

    # ---- end to end through the public API with host buffers
    if not args.no_e2e:
        A_host = torch.empty(m_local, K, dtype=A_in.dtype, pin_memory=True)
        A_host.copy_(A_in)
        C_host = torch.empty(M, n_r, dtype=torch.bfloat16, pin_memory=True)
        A_dev = torch.empty_like(A_in)

        def step_e2e():
            A_dev.copy_(A_host, non_blocking=True)
            launch(A_dev, C_r)
            C_host.copy_(C_r, non_blocking=True)

        for _ in range(max(1, args.warmup // 2)):
            step_e2e()
        e2e_steps = args.steps
        ems = timed(step_e2e, e2e_steps)
        out["e2e"] = {"value": flops_step / (ems * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "h2d_bytes_per_step": A_host.numel() * elem, "d2h_bytes_per_step": C_host.numel() * 2,
                      "ms_per_step": ems, "steps": e2e_steps, "gpu_launches": e2e_steps}
        op.check_status()
        del A_host, C_host, A_dev

    if f8:
        pk = measure_e4m3_peak(dev)
        out["roofline"] = roofline_for(pk, "measured e4m3 burst on this GPU: cuBLASLt (torch._scaled_mm, "
                                           "tensor-wise scales, bf16 out) 8192^3, best of 10")

    # ---- parity of one more launch against an independent result: the gathered
    # A must equal NCCL's all-gather of the shards byte for byte, and every
    # element of C_r must pass the reference's check_close against an fp32
    # product of that gathered A and B_r (cuBLAS SGEMM, TF32 off; e4m3 operands
    # dequantised exactly with their scales first).
    torch.backends.cuda.matmul.allow_tf32 = False
    launch(A_in, C_r)
    torch.cuda.synchronize()
    op.check_status()
    if world > 1:
        A_full = torch.empty(M, K, device=dev, dtype=A_in.dtype)
        dist.all_gather_into_tensor(A_full, A_in)
        S_full = None
        if f8:
            S_full = torch.empty(M, device=dev, dtype=torch.float32)
            dist.all_gather_into_tensor(S_full, S_a)
        gather_ok = bool(torch.equal(op.gathered().view(torch.uint8), A_full.view(torch.uint8)))
    else:
        A_full, S_full, gather_ok = A_in, S_a, None
    if f8:
        Bf = B_in.view(torch.float8_e4m3fn).float() * S_b[:, None]

        def want_rows(r0, r1):
            return (A_full[r0:r1].view(torch.float8_e4m3fn).float() * S_full[r0:r1, None]) @ Bf.t()
    else:
        Bf = B_in.float()

        def want_rows(r0, r1):
            return A_full[r0:r1].float() @ Bf.t()
    bad, rel = compare_rows(C_r, want_rows, M)
    del Bf
    par = reduce_parity({"gather_bitexact": gather_ok, "max_rel_err": rel, "check_close_bad": bad}, world,
                        host_group)
    par["ok"] = (par["gather_bitexact"] in (True, None) and par["check_close_bad"] == 0
                 and par["max_rel_err"] <= MAX_REL[args.dtype])
    par["reference"] = ("gathered A vs NCCL all_gather_into_tensor of the shards (bytes); C_r vs fp32 "
                        "gathered A . B_r^T (cuBLAS SGEMM, TF32 off" + (", e4m3 dequantised" if f8 else "") +
                        f"): check_close atol 0.1 rtol 0.02 on every element, max|C - ref| / max|ref| <= "
                        f"{MAX_REL[args.dtype]}")
    out["parity"] = par

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.workload)

    if args.trace:
        # one more launch, outside every timed region, with the event trace on
        tr = op.new_trace()
        torch.cuda.synchronize()
        barrier()
        launch(A_in, C_r, trace=tr)
        torch.cuda.synchronize()
        op.check_status()
        rows = tr.cpu().numpy()
        per_rank = [rows]
        if world > 1:
            per_rank = [None] * world
            dist.all_gather_object(per_rank, rows, group=host_group)
        if rank == 0:
            with open(args.trace, "w") as f:
                json.dump({"workload": config_of(args.workload, world, args.dtype),
                           "ranks": [pkg.agg.trace_summary(r) for r in per_rank]}, f, indent=1)

    op.close()
    if rank == 0:
        emit(out)
    barrier()
    return out["parity"]["ok"]


if __name__ == "__main__":
    main()
