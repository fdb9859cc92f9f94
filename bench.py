"""Benchmark of the RNS8 hot path on B200: effective exact int64 GOPS.

Workload: C = A x B over int64, M = N = K = 8192, inputs
uniform in [-2^24, 2^24] from a seed, declared bound 2^61, RNS8_BOUNDED_I64
with the prefix forced to 9 (RNS8_PLAN_FORCE_FIXED_PREFIX; the default plan
would select 8). One step = pack A + pack B into 9 centered int8 planes, nine
int8 plane GEMMs (one persistent tcgen05 launch), Garner export to int64.

  value  device-resident: inputs already in HBM, output left in HBM, timed
         with CUDA events on the launching stream (max over ranks).
  e2e    the same step through the public C ABI (rns8_gemm_i64_oneshot) from
         pinned host buffers: H2D of A and B and D2H of C inside the timing.

Multi-GPU (torchrun, one rank per GPU): rows are sharded, each rank owns an
8192-row slab of A and C and a full B (weak scaling, no collective on the
data path); value = all ranks' 2*M*N*K / max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M = N = K = 8192
PREFIX = 9
BOUND = 2**61
LO, HI = -(2**24), 2**24
METRIC = "effective exact int64 GOPS (2MNK/t) at 1/2/4/8 B200; int8 tensor-pipe % of peak"
WORKLOAD = "RNS8_BOUNDED_I64 8192^3 prefix-9 forced, U[-2^24,2^24], bound 2^61 (BASELINE config 3)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=128, help="rows of the CPU baseline slab sample")
    ap.add_argument("--size", type=int, default=8192,
                    help="M = N = K of the run (8192 is the benchmark; smaller sizes are for ncu captures)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "power_w_max": max(power) if power else None, "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------------- peaks
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def int8_peak_tops(torch, peaks) -> tuple[float, str]:
    """Dense int8 denominator: the larger of 2 x measured bf16 (int8 issues at
    twice the bf16 rate) and a cuBLASLt int8 GEMM timed here (torch._int_mm)."""
    derived = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    source = "2x measured bf16 burst" if not peaks.get("fallback") else "2x fallback bf16"
    try:
        a = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch._int_mm(a, b)
            e.record()
            e.synchronize()
            t = s.elapsed_time(e) * 1e-3
            best = t if best is None else min(best, t)
        cublas = 2 * 8192**3 / best / 1e12
        del a, b
        if cublas > derived:
            return cublas, f"cuBLASLt int8 8192^3 measured here (best of 10): {cublas:.0f} TOPS"
        return derived, f"{source} ({derived:.0f}); cuBLASLt int8 measured here {cublas:.0f} TOPS"
    except Exception as exc:  # torch build without int8 GEMM for this arch
        return derived, f"{source} ({derived:.0f}); cuBLASLt int8 unavailable: {type(exc).__name__}"


def profile_traffic() -> int | None:
    """dram bytes per GEMM launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "tc_plane_gemm_c3.json"
    if p.exists():
        try:
            return int(json.loads(p.read_text())["traffic_bytes_per_launch"])
        except Exception:
            return None
    return None


# ----------------------------------------------------------------- CPU baseline
def cpu_baseline(rows: int) -> dict:
    """The CPU oracle (a restatement of the reference's src/cpu path, OpenMP over
    all host cores) on a row slab of the workload: rows x 8192 by 8192 x 8192,
    pack + 9 plane GEMMs + export."""
    import numpy as np

    from oracle import bridge

    lib = bridge.lib()
    threads = lib.oracle_max_threads()
    rng = np.random.default_rng(123)
    A = rng.integers(LO, HI, (rows, K), dtype=np.int64, endpoint=True)
    B = rng.integers(LO, HI, (K, N), dtype=np.int64, endpoint=True)
    Cout = np.zeros((rows, N), np.int64)
    t0 = time.perf_counter()
    st, _, used = bridge.gemm_bounded_oneshot(A, B, BOUND, max_prefix=PREFIX, flags=1, out=Cout)
    dt = time.perf_counter() - t0
    assert st == 0 and used == PREFIX
    return {"value": 2.0 * rows * N * K / dt / 1e9, "unit": "GOPS", "cores": threads, "kind": "port",
            "sample": f"oracle oneshot on a {rows}x{K} by {K}x{N} row slab of the workload "
                      f"(pack A and B, {PREFIX} plane GEMMs, export), {dt:.1f} s, {threads} threads",
            "seconds": dt}


def reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    rows = max(8, args.cpu_rows // 4)
    for _ in range(args.warmup):
        cpu_baseline(rows)
    vals = [cpu_baseline(rows) for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in vals)
    sec = sum(x["seconds"] for x in vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sec / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample_rows": rows, "note": "reference CPU path (oracle port; the "
                       "reference's own src/cpu needs Boost.Multiprecision, absent here)"},
            "cpu_baseline": {**{k: vals[0][k] for k in ("unit", "cores", "kind", "sample")}, "value": v},
            "e2e": {"value": v, "unit": "GOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- our arm
def main():
    args = parse()
    global M, N, K
    M = N = K = args.size
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    import rns8_b200 as r8

    lib = r8.lib()
    dev = local
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)

    # Inputs: this rank's 8192-row slab of A and all of B, generated on device.
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    A = torch.randint(LO, HI + 1, (M, K), dtype=torch.int64, device="cuda", generator=g)
    gb = torch.Generator(device="cuda").manual_seed(999)
    B = torch.randint(LO, HI + 1, (K, N), dtype=torch.int64, device="cuda", generator=gb)
    ra = torch.empty((PREFIX, M, K), dtype=torch.int8, device="cuda")
    rb = torch.empty((PREFIX, K, N), dtype=torch.int8, device="cuda")
    rc = torch.empty((PREFIX, M, N), dtype=torch.int8, device="cuda")
    out = torch.empty((M, N), dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sbytes = lib.rns8_cuda_gemm_rns_scratch_bytes(dev, M, N, K, PREFIX)
    scratch = torch.empty(max(1, sbytes), dtype=torch.uint8, device="cuda")

    ev = {k: [torch.cuda.Event(enable_timing=True) for _ in range(5)] for k in ("s",)}

    def check(st, what):
        if st != 0:
            raise RuntimeError(f"{what} failed with status {st}")

    def step(record=None):
        if record:
            record[0].record(stream)
        check(lib.rns8_cuda_pack_i64_device(dev, A.data_ptr(), M, K, K, PREFIX, ra.data_ptr(), sptr), "pack A")
        check(lib.rns8_cuda_pack_i64_device(dev, B.data_ptr(), K, N, N, PREFIX, rb.data_ptr(), sptr), "pack B")
        if record:
            record[1].record(stream)
        check(lib.rns8_cuda_gemm_rns_device(dev, ra.data_ptr(), rb.data_ptr(), rc.data_ptr(), M, N, K, PREFIX, 0,
                                            scratch.data_ptr(), sbytes, status.data_ptr(), sptr), "gemm")
        if record:
            record[2].record(stream)
        check(lib.rns8_cuda_export_i64_device(dev, rc.data_ptr(), M, N, PREFIX, BOUND, out.data_ptr(), N,
                                              status.data_ptr(), sptr), "export")
        if record:
            record[3].record(stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if int(status[0].item()) != 0:
        raise RuntimeError(f"device status {int(status[0].item()):#x} after warm-up")

    peaks = measured_peaks()
    peak_int8, peak_note = int8_peak_tops(torch, peaks)
    torch.cuda.synchronize()

    clocks = ClockSampler(dev)
    records = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        step(records[i])
    stop.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = start.elapsed_time(stop)
    pack_ms = statistics.mean(r[0].elapsed_time(r[1]) for r in records)
    gemm_ms = statistics.mean(r[1].elapsed_time(r[2]) for r in records)
    exp_ms = statistics.mean(r[2].elapsed_time(r[3]) for r in records)
    if int(status[0].item()) != 0:
        raise RuntimeError(f"device status {int(status[0].item()):#x} in the timed region")

    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    value = world * 2.0 * M * N * K / (ms_per_step * 1e-3) / 1e9

    # ---- e2e through the public C ABI from pinned host memory -------------------
    e2e = None
    if not args.no_e2e:
        hA = A.cpu().pin_memory()
        hB = B.cpu().pin_memory()
        hC = torch.empty((M, N), dtype=torch.int64).pin_memory()
        ctx = r8.Context(dev)
        desc = r8.gemm_desc(r8.Semantics.BOUNDED_I64, r8.BoundKind.GLOBAL_MAX_ABS, M, N, K, bound=BOUND,
                            max_prefix=PREFIX, flags=r8.PLAN_FORCE_FIXED_PREFIX)

        def oneshot():
            st = lib.rns8_gemm_i64_oneshot(ctx.handle, C.byref(desc), hA.data_ptr(), K, hB.data_ptr(), N,
                                           hC.data_ptr(), N)
            check(st, "rns8_gemm_i64_oneshot")

        for _ in range(max(3, args.warmup)):
            oneshot()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            oneshot()  # synchronous: ends with a device sync and the result in host memory
        el = torch.tensor([(time.perf_counter() - t0) * 1e3], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(el, op=dist.ReduceOp.MAX)
        e2e_ms = float(el.item()) / args.steps
        assert torch.equal(hC, out.cpu()), "e2e result differs from the device-resident result"
        e2e = {"value": world * 2.0 * M * N * K / (e2e_ms * 1e-3) / 1e9, "unit": "GOPS",
               "h2d_bytes_per_step": 8 * (M * K + K * N), "d2h_bytes_per_step": 8 * M * N, "ms_per_step": e2e_ms,
               "api": "rns8_gemm_i64_oneshot (pinned host buffers)"}
        ctx.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_rows)

    gemm_ops = PREFIX * 2.0 * M * N * K
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
    pack_bytes = 2 * (8 * M * K) + 2 * PREFIX * M * K
    exp_bytes = PREFIX * M * N + 8 * M * N
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GOPS", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "m_per_rank": M, "n": N, "k": K, "prefix": PREFIX, "bound": "2^61",
                       "parallelism": f"row-slab x{world}", "l2": "inputs larger than L2 (512 MiB each)"},
            "roofline": {"kernel": "tc_plane_gemm_kernel", "bound": "tensor", "achieved": achieved,
                         "peak": peak_int8, "unit": "TOPS (int8)", "frac": achieved / peak_int8,
                         "peak_source": peak_note, "traffic": profile_traffic(),
                         "algorithmic_ops_per_launch": gemm_ops},
            "stages_ms": {"pack_a_b": pack_ms, "plane_gemm": gemm_ms, "export": exp_ms},
            "stage_hbm_frac": {"pack": pack_bytes / (pack_ms * 1e-3) / 1e9 / hbm,
                               "export": exp_bytes / (exp_ms * 1e-3) / 1e9 / hbm, "peak_gbs": hbm,
                               "peak_source": "MEASURED_PEAKS.json hbm_gbs" if not peaks.get("fallback") else "fallback"},
            "e2e": e2e, "cpu_baseline": cpu, "clocks": clock_info,
            "gpu_launches": 4 * args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
