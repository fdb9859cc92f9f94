"""Benchmark of the RNS8 hot path on B200: effective exact int64 GOPS.

Default workload: C = A x B over int64, M = N = K = 8192,
inputs uniform in [-2^24, 2^24] from a seed, declared bound 2^61,
RNS8_BOUNDED_I64 with the prefix forced to 9 (RNS8_PLAN_FORCE_FIXED_PREFIX;
the default plan would select 8). One step = pack A + pack B into 9 centered
int8 planes, nine int8 plane GEMMs (one persistent tcgen05 launch), export to
int64 (fractional CRT, exact Garner for undecided cells).

The other BASELINE configs run with --config C1|C2|C4|C5 (same metric, same
JSON line; they are measurements for the record, the driver runs C3), and
--config W runs the WRAP_U64_MOD_2_64 path at the C3 shape:
  C1  int64 512^3, U[-2^20, 2^20], bound 2^49, prefix 7 (default plan)
  C2  finite field 251, 64 independent 2048^3 pairs, grouped GEMM
  C4  uint64 256 x 256 x 262144, U[0, 2^22), bound 2^62, prefix 8 (split-K)
  C5  exact-wide signed int64 4096^3, full int64 range, 3 limbs, prefix 20 forced
  W   uint64 8192^3 modulo 2^64, full uint64 range

  value  device-resident: inputs already in HBM, output left in HBM, timed
         with CUDA events on the launching stream (max over ranks).
  e2e    the same work through the public C ABI from pinned host buffers
         (the oneshot call for C1/C3/C4, the matrix API for C2/C5): H2D of
         the inputs and D2H of the result inside the timing.

Multi-GPU (torchrun, one rank per GPU): rows are sharded, each rank owns a
slab of A and C of the config's size and a full B (weak scaling, no collective
on the data path); value = all ranks' work / max-over-ranks time. With several
ranks the line also carries `strong_scaling`: the config's one product split
into 2-D output blocks (rank (i, j) packs row slab i of A and column slab j of
B), its max-over-ranks step time and rank 0's per-stage times.

Inputs are the reference benchmark's: one std::mt19937_64(1) draws A, then B
(uniform_int_distribution), so the CPU oracle checks the GPU's output on a
sample of rows (`parity`) and times the same sample (`cpu_baseline`).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config C1..C5|W] [--size S (C3 only: M = N = K = S)]
"""

from __future__ import annotations

import argparse
import ctypes as C
import dataclasses
import datetime
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

METRIC = "effective exact int64 GOPS (2MNK/t) at 1/2/4/8 B200; int8 tensor-pipe % of peak"


@dataclasses.dataclass
class Config:
    name: str
    kind: str            # "i64" | "u64" | "finite" | "exact"
    m: int
    n: int
    k: int
    lo: int
    hi: int
    prefix: int          # residue planes per matrix (1 for finite, 8 byte planes for wrap)
    forced: bool         # RNS8_PLAN_FORCE_FIXED_PREFIX
    workload: str
    bound: int = 0
    batch: int = 1
    modulus: int = 0
    limbs: int = 0
    sample: int = 128    # CPU sample: rows of A (whole tasks for the batched finite config)

    @property
    def ops(self) -> float:
        """Effective exact ops of one step: 2*M*N*K per product."""
        return self.batch * 2.0 * self.m * self.n * self.k


CONFIGS = {
    "C1": Config("C1", "i64", 512, 512, 512, -(2**20), 2**20, 7, False,
                 "RNS8_BOUNDED_I64 512^3, U[-2^20,2^20], bound 2^49, prefix 7 default (BASELINE config 1)",
                 bound=2**49, sample=512),
    "C2": Config("C2", "finite", 2048, 2048, 2048, 0, 250, 1, False,
                 "RNS8_FINITE_FIELD_U8 modulus 251, 64 x 2048^3 grouped, U[0,250] (BASELINE config 2)",
                 batch=64, modulus=251, sample=8),
    "C3": Config("C3", "i64", 8192, 8192, 8192, -(2**24), 2**24, 9, True,
                 "RNS8_BOUNDED_I64 8192^3 prefix-9 forced, U[-2^24,2^24], bound 2^61 (BASELINE config 3)",
                 bound=2**61, sample=1024),
    "C4": Config("C4", "u64", 256, 256, 262144, 0, 2**22 - 1, 8, False,
                 "RNS8_BOUNDED_U64 256x256x262144, U[0,2^22), bound 2^62, prefix 8 default (BASELINE config 4)",
                 bound=2**62, sample=256),
    "C5": Config("C5", "exact", 4096, 4096, 4096, -(2**63), 2**63 - 1, 20, True,
                 "RNS8_EXACT_WIDE_SIGNED 4096^3, U[INT64_MIN,INT64_MAX], 3 limbs, prefix 20 forced "
                 "(BASELINE config 5)", limbs=3, sample=512),
    # Not a BASELINE config: the WRAP_U64_MOD_2_64 path at the C3 shape.
    "W": Config("W", "wrap", 8192, 8192, 8192, 0, 2**64 - 1, 8, False,
                "RNS8_WRAP_U64_MOD_2_64 8192^3, U[0,2^64) (36 byte-pair products on the tensor cores)",
                sample=1024),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="C3")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sample", type=int, default=0,
                    help="CPU sample (rows of A; tasks for C2) for the oracle parity check, the CPU baseline and the "
                         "reference arm (0: the config's)")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle comparison (and the CPU baseline)")
    ap.add_argument("--no-strong", action="store_true",
                    help="with several GPUs, skip the strong-scaling measurement attached to the weak line")
    ap.add_argument("--size", type=int, default=0,
                    help="C3 only: M = N = K = size (8192 is the benchmark; smaller sizes are for ncu captures)")
    ap.add_argument("--shard", choices=["weak-rows", "rows", "grid", "planes"], default="weak-rows",
                    help="weak-rows: each rank owns an M-row slab (the benchmark line); rows / grid / planes: the "
                         "config's one product split across ranks by row slabs / by 2-D output blocks / by residue "
                         "planes with the fused NVLink exchange (strong scaling, device-resident)")
    ap.add_argument("--exchange", choices=["fused", "copy"], default="fused",
                    help="--shard planes: epilogue stores into the slab owners' buffers, or local planes + copies")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every step's kernels from the host instead of replaying a captured CUDA graph")
    args = ap.parse_args()
    if args.shard != "weak-rows" and cfg_kind(args.config) not in ("i64", "u64", "exact"):
        ap.error("--shard rows|grid|planes applies to the int64/uint64/exact-wide configs")
    cfg = CONFIGS[args.config]
    if args.size:
        if cfg.name != "C3":
            ap.error("--size applies to C3 only")
        cfg = dataclasses.replace(cfg, m=args.size, n=args.size, k=args.size)
    if args.sample:
        cfg = dataclasses.replace(cfg, sample=args.sample)
    cfg = dataclasses.replace(cfg, sample=min(cfg.sample, cfg.batch if cfg.kind == "finite" else cfg.m))
    return args, cfg


def cfg_kind(name: str) -> str:
    return CONFIGS[name].kind


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region.

    Each sample carries nvidia-smi's own timestamp: its output reaches a pipe
    in buffered chunks, so the time a line is read says little about when
    the sample was taken."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            line = line.strip()
            try:  # "YYYY/MM/DD HH:MM:SS.mmm", local time
                t = datetime.datetime.strptime(line.split(",")[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                t = time.time()
            self.lines.append((t, line))

    def mark(self, t0: float, t1: float):
        """The timed region on the host's wall clock (time.time() seconds)."""
        self.window = (t0, t1)

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
        lines = self.lines
        in_window = [l for t, l in lines if self.window and self.window[0] - 0.02 <= t <= self.window[1] + 0.02]
        use = in_window if in_window else [l for _, l in lines]
        for line in use:
            parts = [p.strip() for p in line.split(",")][1:]  # drop the timestamp
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
                "power_w_max": max(power) if power else None, "samples": len(sm),
                "samples_in_timed_region": len(in_window), "interval_ms": 20, "reasons": sorted(reasons)}


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


def profile_traffic(cfg: Config, kernel: str) -> int | None:
    """dram bytes per launch of `kernel` on this config, from the committed ncu
    summary (profiles/traffic.json), if it holds that pair."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return int(json.loads(p.read_text())[cfg.name][kernel]["dram_bytes_per_launch"])
    except Exception:
        return None


# ------------------------------------------------------------- seeded inputs
# The reference benchmark's generator (rns8_bench_types.hpp:72 seed = 1;
# rns8_bench_bounded_i64_lane.inc:11-16): one std::mt19937_64 draws all of A,
# then all of B, row-major, each value from std::uniform_int_distribution over
# the config's range (uint32_t per byte for the finite lanes,
# rns8_bench_finite_lanes.inc:28-31). The generator is the CPU checker's
# (libstdc++ through the oracle library), so the GPU arm, the oracle parity
# check, the CPU baseline and the reference arm all see the same inputs.
SEED = 1


def seeded_inputs(cfg: Config, rank: int = 0):
    """Host A and B of this rank. Rank 0's are exactly the reference bench's
    draws; rank r > 0 (weak scaling) draws its own A slab from seed 1 + r and
    shares rank 0's B (the engine of seed 1 skips rank 0's A)."""
    import numpy as np

    from oracle import bridge

    m, n, k, bt = cfg.m, cfg.n, cfg.k, cfg.batch
    if cfg.kind == "finite":  # batched: A_t then B_t for each task t
        rng = bridge.Rng(SEED + rank)
        A = np.empty((bt, m, k), np.uint8)
        B = np.empty((bt, k, n), np.uint8)
        for t in range(bt):
            A[t] = rng.u8(cfg.hi, (m, k))
            B[t] = rng.u8(cfg.hi, (k, n))
        return A, B
    unsigned = cfg.kind in ("u64", "wrap")
    draw = (lambda r, shape: r.u64(cfg.lo, cfg.hi, shape)) if unsigned else (lambda r, shape: r.i64(cfg.lo, cfg.hi,
                                                                                                      shape))
    rng = bridge.Rng(SEED)
    if rank == 0:
        A = draw(rng, (m, k))
    else:
        (rng.skip_u64 if unsigned else rng.skip_i64)(cfg.lo, cfg.hi, m * k)
        A = draw(bridge.Rng(SEED + rank), (m, k))
    B = draw(rng, (k, n))
    return A, B


def fnv_checksum(values) -> int:
    """The reference benchmark's output checksum (rns8_bench_support.cpp:96-99):
    h = 1469598103934665603; h ^= v; h *= 1099511628211 over the outputs in
    memory order, each widened to uint64."""
    import numpy as np

    from oracle import bridge

    v = np.ascontiguousarray(values)
    if v.dtype.itemsize == 8:
        return bridge.checksum(v.reshape(v.shape[0], -1))
    h = 1469598103934665603
    flat = v.reshape(-1)
    step = 1 << 22
    # FNV is sequential: chain the chunks through the running hash.
    for i in range(0, flat.size, step):
        chunk = flat[i:i + step].astype(np.uint64)
        h = int(bridge.lib().oracle_checksum_u64_from(h, bridge._p(chunk), chunk.size))
    return h


# ----------------------------------------------------------------- CPU sample
def cpu_sample(cfg: Config, A, B, sample: int):
    """The CPU oracle (a restatement of the reference's src/cpu path, OpenMP
    over all host threads) on a bounded sample of the workload: rows [0,
    sample) of A against all of B (whole tasks for the batched finite config).

    Returns (info, out): out is the oracle's output for the sample, which the
    GPU's must equal bit for bit. B's pack serves all M rows in the full
    workload, so a sample step is charged t_slab + (sample / M) * t_pack_B;
    value = the sample's effective ops over that time. `wall_s` is what the
    sample actually took."""
    import numpy as np

    from oracle import bridge

    lib = bridge.lib()
    threads = lib.oracle_max_threads()
    m, n, k, P = cfg.m, cfg.n, cfg.k, cfg.prefix
    if cfg.kind == "finite":  # whole tasks: pack A_t and B_t, GEMM mod m, export
        t0 = time.perf_counter()
        out = np.empty((sample, m, n), np.uint8)
        for t in range(sample):
            a = bridge.pack_finite_u8(A[t], cfg.modulus)
            b = bridge.pack_finite_u8(B[t], cfg.modulus)
            c = bridge.ring_gemm(a, b, cfg.modulus)
            out[t] = (c.astype(np.int16) % cfg.modulus).astype(np.uint8)  # centered -> canonical (a15)
        wall = step = time.perf_counter() - t0
        ops = sample * 2.0 * m * n * k
        what = f"oracle pack, GEMM mod {cfg.modulus}, export of {sample} of {cfg.batch} tasks"
    elif cfg.kind == "wrap":  # wrap64_reference.cpp:254-290 on the slab; packing is a byte copy
        t0 = time.perf_counter()
        out = bridge.wrap64_gemm(A[:sample], B)
        wall = step = time.perf_counter() - t0
        ops = 2.0 * sample * n * k
        what = f"oracle wrap64 GEMM (native uint64 multiply-add) on rows [0, {sample}) of A"
    else:
        t0 = time.perf_counter()
        b = bridge.pack(B, P)
        t_b = time.perf_counter() - t0
        t0 = time.perf_counter()
        c = bridge.gemm_rns(bridge.pack(np.ascontiguousarray(A[:sample]), P), b, P)
        if cfg.kind == "i64":
            st, out = bridge.export_i64(c, P, cfg.bound)
        elif cfg.kind == "u64":
            st, out = bridge.export_u64(c, P, cfg.bound)
        else:
            st, out = bridge.export_limbs(c, P, cfg.limbs, True)
        t_slab = time.perf_counter() - t0
        if st != 0:
            raise RuntimeError(f"oracle export status {st} on the sample")
        wall = t_b + t_slab
        step = t_slab + sample / m * t_b
        ops = 2.0 * sample * n * k
        what = (f"oracle pack, {P} plane GEMMs, " + (f"{cfg.limbs}-limb export" if cfg.kind == "exact" else "export") +
                f" of rows [0, {sample}) of A against all of B; B packed in {t_b:.2f} s, charged {sample}/{m} of it")
    info = {"value": ops / step / 1e9, "unit": "GOPS", "cores": threads, "kind": "port",
            "sample": f"{what}; step {step:.2f} s ({wall:.2f} s wall); {threads} threads",
            "sample_ops": ops, "step_s": step, "wall_s": wall,
            "full_step_s_extrapolated": cfg.ops / (ops / step)}
    return info, out


def reference_arm(args, cfg: Config) -> None:
    """The reference's CPU path (the oracle port: the reference's own src/cpu
    needs Boost.Multiprecision, absent here) on every host thread, on the same
    seeded inputs and the same bounded sample as this arm's CPU baseline."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # Every host thread, also under torchrun (whose default is one thread per
    # process); set before the oracle library, and its OpenMP runtime, load.
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    A, B = seeded_inputs(cfg, 0)
    wall0 = time.perf_counter()
    for _ in range(args.warmup):
        cpu_sample(cfg, A, B, cfg.sample)
    vals = [cpu_sample(cfg, A, B, cfg.sample)[0] for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in vals)
    step_ms = 1e3 * statistics.median(x["step_s"] for x in vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": {"finite": "uint8", "wrap": "uint64"}.get(cfg.kind, "int64"), "data": "synthetic",
            "config": {"workload": cfg.workload, "name": cfg.name, "m_per_rank": cfg.m, "n": cfg.n, "k": cfg.k,
                       "batch": cfg.batch, "prefix": cfg.prefix, "seed": SEED,
                       "sample": (f"{cfg.sample} of {cfg.batch} tasks" if cfg.kind == "finite"
                                  else f"rows [0, {cfg.sample}) of {cfg.m}"),
                       "note": "reference CPU path (oracle port; the reference's own src/cpu needs "
                               "Boost.Multiprecision, absent here); each step is the bounded sample"},
            "measured_wall_s": time.perf_counter() - wall0,
            "full_step_s_extrapolated": statistics.median(x["full_step_s_extrapolated"] for x in vals),
            "cpu_baseline": {**{k: vals[0][k] for k in ("unit", "cores", "kind", "sample")}, "value": v},
            "e2e": {"value": v, "unit": "GOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- our arm
class DevicePipeline:
    """Device-resident buffers and the three stages of one step (pack, plane
    GEMM, export), launched through the C-ABI device seam on one stream."""

    def __init__(self, torch, lib, cfg: Config, dev: int, hostA, hostB):
        self.torch, self.lib, self.cfg, self.dev = torch, lib, cfg, dev
        m, n, k, P, bt = cfg.m, cfg.n, cfg.k, cfg.prefix, cfg.batch
        # The seeded host inputs, uploaded once (uint64 travels as int64 bits).
        as_t = (lambda a: torch.from_numpy(a.view("int64")) if a.dtype.itemsize == 8 else torch.from_numpy(a))
        self.A = as_t(hostA).to("cuda")
        self.B = as_t(hostB).to("cuda")
        if cfg.kind == "finite":
            self.ra = torch.empty((bt, m, k), dtype=torch.int8, device="cuda")
            self.rb = torch.empty((bt, k, n), dtype=torch.int8, device="cuda")
            self.rc = torch.empty((bt, m, n), dtype=torch.int8, device="cuda")
            self.out = torch.empty((bt, m, n), dtype=torch.uint8, device="cuda")
            vp = C.c_void_p * bt
            self.pa = vp(*[self.ra[t].data_ptr() for t in range(bt)])
            self.pb = vp(*[self.rb[t].data_ptr() for t in range(bt)])
            self.pc = vp(*[self.rc[t].data_ptr() for t in range(bt)])
            self.sbytes = lib.rns8_cuda_gemm_finite_u8_scratch_bytes(dev, m, n, k, bt)
        elif cfg.kind == "wrap":
            self.ra = torch.empty((8, m, k), dtype=torch.uint8, device="cuda")
            self.rb = torch.empty((8, k, n), dtype=torch.uint8, device="cuda")
            self.rc = torch.empty((1,), dtype=torch.uint8, device="cuda")
            self.out = torch.empty((m, n), dtype=torch.int64, device="cuda")
            self.sbytes = 0
        else:
            self.ra = torch.empty((P, m, k), dtype=torch.int8, device="cuda")
            self.rb = torch.empty((P, k, n), dtype=torch.int8, device="cuda")
            self.rc = torch.empty((P, m, n), dtype=torch.int8, device="cuda")
            shape = (m, n, cfg.limbs) if cfg.kind == "exact" else (m, n)
            self.out = torch.empty(shape, dtype=torch.int64, device="cuda")
            self.sbytes = lib.rns8_cuda_gemm_rns_scratch_bytes(dev, m, n, k, P)
        self.scratch = torch.empty(max(1, self.sbytes), dtype=torch.uint8, device="cuda")
        self.status = torch.zeros(4, dtype=torch.int32, device="cuda")
        gemm_launches = (1 + (1 if self.sbytes > 0 else 0)) * ((bt + 31) // 32 if cfg.kind == "finite" else 1)
        self.launches_per_step = 2 + gemm_launches + (0 if cfg.kind == "wrap" else 1)
        footprint = sum(t.numel() * t.element_size() for t in (self.A, self.B, self.ra, self.rb, self.rc, self.out))
        self.fits_l2 = footprint < (512 << 20)  # L2 is 126 MB: below this, flush it between steps

    @property
    def sptr(self):
        """The current stream (a graph capture's stream while capturing)."""
        return C.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    @staticmethod
    def _check(st, what):
        if st != 0:
            raise RuntimeError(f"{what} failed with status {st}")

    def pack(self):
        cfg, lib, d, s = self.cfg, self.lib, self.dev, self.sptr
        m, n, k, bt = cfg.m, cfg.n, cfg.k, cfg.batch
        if cfg.kind == "finite":
            self._check(lib.rns8_cuda_pack_finite_u8_device(d, self.A.data_ptr(), bt * m, k, k, cfg.modulus,
                                                            self.ra.data_ptr(), s), "pack A")
            self._check(lib.rns8_cuda_pack_finite_u8_device(d, self.B.data_ptr(), bt * k, n, n, cfg.modulus,
                                                            self.rb.data_ptr(), s), "pack B")
            return
        if cfg.kind == "wrap":
            self._check(lib.rns8_cuda_pack_wrap_u64_device(d, self.A.data_ptr(), m, k, k, self.ra.data_ptr(), s),
                        "pack A")
            self._check(lib.rns8_cuda_pack_wrap_u64_device(d, self.B.data_ptr(), k, n, n, self.rb.data_ptr(), s),
                        "pack B")
            return
        fn = lib.rns8_cuda_pack_u64_device if cfg.kind == "u64" else lib.rns8_cuda_pack_i64_device
        self._check(fn(d, self.A.data_ptr(), m, k, k, cfg.prefix, self.ra.data_ptr(), s), "pack A")
        self._check(fn(d, self.B.data_ptr(), k, n, n, cfg.prefix, self.rb.data_ptr(), s), "pack B")

    def gemm(self):
        cfg, lib, d, s = self.cfg, self.lib, self.dev, self.sptr
        if cfg.kind == "wrap":  # C = A x B mod 2^64, left in HBM as uint64
            self._check(lib.rns8_cuda_gemm_wrap_u64_device(d, self.ra.data_ptr(), self.rb.data_ptr(),
                                                           self.out.data_ptr(), cfg.m, cfg.n, cfg.k, 0,
                                                           self.status.data_ptr(), s), "wrap gemm")
            return
        if cfg.kind == "finite":
            self._check(lib.rns8_cuda_gemm_finite_u8_grouped_device(
                d, self.pa, self.pb, self.pc, cfg.batch, cfg.m, cfg.n, cfg.k, cfg.modulus, 0,
                self.scratch.data_ptr(), self.sbytes, self.status.data_ptr(), s), "grouped gemm")
            return
        self._check(lib.rns8_cuda_gemm_rns_device(d, self.ra.data_ptr(), self.rb.data_ptr(), self.rc.data_ptr(),
                                                  cfg.m, cfg.n, cfg.k, cfg.prefix, 0, self.scratch.data_ptr(),
                                                  self.sbytes, self.status.data_ptr(), s), "gemm")

    def export(self):
        cfg, lib, d, s = self.cfg, self.lib, self.dev, self.sptr
        m, n = cfg.m, cfg.n
        if cfg.kind == "wrap":
            return  # the GEMM already wrote uint64 C
        if cfg.kind == "finite":
            st = lib.rns8_cuda_export_finite_u8_device(d, self.rc.data_ptr(), cfg.batch * m, n, cfg.modulus,
                                                       self.out.data_ptr(), n, s)
        elif cfg.kind == "exact":
            st = lib.rns8_cuda_export_limbs_device(d, self.rc.data_ptr(), m, n, cfg.prefix, 1, cfg.limbs,
                                                   self.out.data_ptr(), n, self.status.data_ptr(), s)
        else:
            fn = lib.rns8_cuda_export_u64_device if cfg.kind == "u64" else lib.rns8_cuda_export_i64_device
            st = fn(d, self.rc.data_ptr(), m, n, cfg.prefix, cfg.bound, self.out.data_ptr(), n,
                    self.status.data_ptr(), s)
        self._check(st, "export")

    def step(self, events=None):
        stream = self.torch.cuda.current_stream()
        for i, stage in enumerate((self.pack, self.gemm, self.export)):
            if events:
                events[i].record(stream)
            stage()
        if events:
            events[3].record(stream)

    def device_status(self) -> int:
        return int(self.status[0].item())

    # Algorithmic work of each stage (ops for the GEMM, HBM bytes for pack and export).
    def stage_work(self) -> dict:
        cfg = self.cfg
        m, n, k, P, bt = cfg.m, cfg.n, cfg.k, cfg.prefix, cfg.batch
        elem_in = 1 if cfg.kind == "finite" else 8
        out_bytes = {"finite": 1, "exact": 8 * cfg.limbs}.get(cfg.kind, 8)
        if cfg.kind == "wrap":  # 36 u8 x u8 products per cell and k; no export stage
            return {"pack": ("hbm", 16 * (m * k + k * n)), "plane_gemm": ("tensor", 36 * 2.0 * m * n * k),
                    "export": ("hbm", 0)}
        return {
            "pack": ("hbm", bt * (elem_in + P) * (m * k + k * n)),
            "plane_gemm": ("tensor", bt * P * 2.0 * m * n * k),
            "export": ("hbm", bt * (P + out_bytes) * m * n),
        }


class EndToEnd:
    """The same work through the public C ABI from pinned host buffers."""

    def __init__(self, torch, r8, lib, cfg: Config, dev: int, pipe: DevicePipeline, hostA, hostB):
        self.cfg, self.lib, self.r8 = cfg, lib, r8
        self.ctx = r8.Context(dev)
        m, n, k = cfg.m, cfg.n, cfg.k
        as_t = (lambda a: torch.from_numpy(a.view("int64")) if a.dtype.itemsize == 8 else torch.from_numpy(a))
        self.hA = as_t(hostA).pin_memory()
        self.hB = as_t(hostB).pin_memory()
        self.hC = torch.empty(tuple(pipe.out.shape), dtype=pipe.out.dtype).pin_memory()
        S = r8.Semantics
        if cfg.kind == "wrap":
            self.desc = r8.gemm_desc(S.WRAP_U64_MOD_2_64, r8.BoundKind.NONE, m, n, k)
            self.oneshot = lib.rns8_gemm_wrap_u64_oneshot
            self.api = "rns8_gemm_wrap_u64_oneshot (pinned host buffers)"
        elif cfg.kind in ("i64", "u64"):
            signed = cfg.kind == "i64"
            self.desc = r8.gemm_desc(S.BOUNDED_I64 if signed else S.BOUNDED_U64,
                                     r8.BoundKind.GLOBAL_MAX_ABS if signed else r8.BoundKind.GLOBAL_MAX_UNSIGNED,
                                     m, n, k, bound=cfg.bound, max_prefix=cfg.prefix if cfg.forced else 0,
                                     flags=r8.PLAN_FORCE_FIXED_PREFIX if cfg.forced else 0)
            self.oneshot = lib.rns8_gemm_i64_oneshot if signed else lib.rns8_gemm_u64_oneshot
            self.api = ("rns8_gemm_i64_oneshot" if signed else "rns8_gemm_u64_oneshot") + " (pinned host buffers)"
        elif cfg.kind == "finite":
            desc = r8.gemm_desc(S.FINITE_FIELD_U8, r8.BoundKind.NONE, m, n, k, finite_modulus=cfg.modulus)
            self.plan = r8.Plan(self.ctx, desc)
            self.tasks = []
            for _ in range(cfg.batch):
                a, b, c = (r8.Matrix.for_plan(self.ctx, self.plan, r) for r in "abc")
                self.tasks.append((a, b, c, r8.Workspace(self.ctx, self.plan)))
            self.nA, self.nB, self.nC = self.hA.numpy(), self.hB.numpy(), self.hC.numpy()
            self.api = ("rns8_pack_finite_u8 x 128, rns8_gemm_finite_u8_grouped (64 tasks), rns8_export_finite_u8 x 64 "
                        "(pinned host buffers)")
        else:
            desc = r8.gemm_desc(S.EXACT_WIDE_SIGNED, r8.BoundKind.NONE, m, n, k, max_prefix=cfg.prefix,
                                flags=r8.PLAN_FORCE_FIXED_PREFIX)
            self.plan = r8.Plan(self.ctx, desc)
            assert self.plan.prefix == cfg.prefix
            self.a, self.b, self.c = (r8.Matrix.for_plan(self.ctx, self.plan, r) for r in "abc")
            self.ws = r8.Workspace(self.ctx, self.plan)
            self.nA, self.nB = self.hA.numpy(), self.hB.numpy()
            self.nC = self.hC.numpy().view("uint64")
            self.api = ("rns8_pack_i64 x 2, rns8_gemm_rns, rns8_export_exact_wide_signed_limbs "
                        "(pinned host buffers; includes the exact-range admission proofs, computed on the device)")
        elem_in = 1 if cfg.kind == "finite" else 8
        self.h2d = cfg.batch * elem_in * (m * k + k * n)
        self.d2h = self.hC.numel() * self.hC.element_size()

    def run(self):
        cfg, r8, lib = self.cfg, self.r8, self.lib
        if cfg.kind in ("i64", "u64", "wrap"):
            st = self.oneshot(self.ctx.handle, C.byref(self.desc), self.hA.data_ptr(), cfg.k, self.hB.data_ptr(),
                              cfg.n, self.hC.data_ptr(), cfg.n)
            DevicePipeline._check(st, self.api)
        elif cfg.kind == "finite":
            for t, (a, b, _, _) in enumerate(self.tasks):
                a.pack_finite_u8(cfg.modulus, self.nA[t])
                b.pack_finite_u8(cfg.modulus, self.nB[t])
            r8.gemm_finite_u8_grouped(self.ctx, self.plan, cfg.modulus, self.tasks)
            for t, (_, _, c, _) in enumerate(self.tasks):
                r8.export_finite_u8(self.ctx, self.plan, cfg.modulus, c, out=self.nC[t])
        else:
            self.a.pack_i64(self.nA)
            self.b.pack_i64(self.nB)
            r8.gemm_rns(self.ctx, self.plan, self.a, self.b, self.c, self.ws)
            r8.export_exact_wide_limbs(self.ctx, self.plan, self.c, cfg.limbs, signed=True, out=self.nC)

    def close(self):
        for obj in getattr(self, "tasks", []):
            for h in obj:
                h.close()
        for name in ("a", "b", "c", "ws", "plan"):
            h = getattr(self, name, None)
            if h is not None:
                h.close()
        self.ctx.close()


class ShardedProduct:
    """The config's single product split across ranks (strong scaling).

    rows:   rank r packs its row slab of A and all of B into every plane,
            multiplies and exports its slab (no exchange).
    grid:   the output split into row_groups x col_groups blocks
            (rns8_b200.shard.output_tile): rank (i, j) packs row slab i of A
            and column slab j of B, so B's pack is divided too; no exchange.
    planes: rank r packs all of A and B into its planes {p : p mod world == r},
            multiplies them for all of C with the row-slab scatter epilogue
            (each output row stored into its owner's receive buffer, over
            NVLink for peers), one NCCL barrier, then exports its own slab from
            all planes. Receive buffers alternate between steps so that the
            next step's scatter never overwrites a slab still being exported."""

    def __init__(self, torch, dist, lib, cfg: Config, dev: int, rank: int, world: int, mode: str, exchange: str,
                 sptr):
        from rns8_b200 import shard

        self.torch, self.dist, self.lib, self.cfg, self.dev, self.sptr = torch, dist, lib, cfg, dev, sptr
        self.mode, self.world, self.rank = mode, world, rank
        m, n, k, P = cfg.m, cfg.n, cfg.k, cfg.prefix
        # One product: every rank draws the same seeded A and B.
        self.hA, self.hB = seeded_inputs(cfg, 0)
        self.A = torch.from_numpy(self.hA.view("int64")).to("cuda")
        self.B = torch.from_numpy(self.hB.view("int64")).to("cuda")
        self.signed = cfg.kind != "u64"
        self.col0, self.cols = 0, n
        if mode == "planes":
            self.row0, self.rows = shard.slab_of_rank(rank, m, world)
        elif mode == "grid":
            self.row0, self.rows, self.col0, self.cols = shard.output_tile(rank, world, m, n)
        else:
            self.row0, self.rows = shard.row_slab(rank, world, m)
        self.status = torch.zeros(4, dtype=torch.int32, device="cuda")
        r, c = max(self.rows, 1), max(self.cols, 1)
        self.out = torch.empty((r, c, cfg.limbs) if cfg.kind == "exact" else (r, c), dtype=torch.int64, device="cuda")
        self.launches_per_step = 0
        if mode == "planes":
            self.mine = shard.planes_of_rank(rank, world, P)
            self.idx = (C.c_uint32 * max(1, len(self.mine)))(*self.mine)
            self.ra = torch.empty((max(1, len(self.mine)), m, k), dtype=torch.int8, device="cuda")
            self.rb = torch.empty((max(1, len(self.mine)), k, n), dtype=torch.int8, device="cuda")
            self.ex = shard.PlaneExchange(shard.LibraryIpc(lib, dev), rank, world, m, n, P, buffers=2)
            self.tables = [(C.c_void_p * self.ex.slab_count)(*self.ex.slab_table(b)) for b in range(2)]
            self.copy = exchange == "copy"
            self.sbytes = lib.rns8_cuda_gemm_rns_slabs_scratch_bytes(dev, m, n, k, max(1, len(self.mine)),
                                                                     1 if self.copy else 0) if self.mine else 0
            self.flag = torch.ones(1, device="cuda")
            self.fused = C.c_uint32(0)
            self.step_index = 0
        else:
            self.ex = None
            self.ra = torch.empty((P, r, k), dtype=torch.int8, device="cuda")
            self.rb = torch.empty((P, k, c), dtype=torch.int8, device="cuda")
            self.rc = torch.empty((P, r, c), dtype=torch.int8, device="cuda")
            self.sbytes = lib.rns8_cuda_gemm_rns_scratch_bytes(dev, r, c, k, P)
        self.scratch = torch.empty(max(1, self.sbytes), dtype=torch.uint8, device="cuda")

    def step(self, events=None):
        """One step; with `events` (four CUDA events) the pack, GEMM and export
        boundaries are recorded (row and grid modes)."""
        cfg, lib, d, s = self.cfg, self.lib, self.dev, self.sptr
        m, n, k, P = cfg.m, cfg.n, cfg.k, cfg.prefix
        chk = DevicePipeline._check
        stream = self.torch.cuda.current_stream()
        mark = (lambda i: events[i].record(stream)) if events else (lambda i: None)
        launches = 0
        if self.mode == "planes":
            b = self.step_index % 2
            self.step_index += 1
            if self.mine:
                pk = lib.rns8_cuda_pack_i64_planes_device if self.signed else lib.rns8_cuda_pack_u64_planes_device
                chk(pk(d, self.A.data_ptr(), m, k, k, self.idx, len(self.mine), self.ra.data_ptr(), s), "pack A")
                chk(pk(d, self.B.data_ptr(), k, n, n, self.idx, len(self.mine), self.rb.data_ptr(), s), "pack B")
                chk(lib.rns8_cuda_gemm_rns_slabs_device(d, self.ra.data_ptr(), self.rb.data_ptr(), m, n, k, self.idx,
                                                        len(self.mine), self.tables[b], self.ex.slab_count,
                                                        self.ex.slab_rows, 1 if self.copy else 0,
                                                        self.scratch.data_ptr(), self.sbytes, self.status.data_ptr(),
                                                        C.byref(self.fused), s), "gemm slabs")
                launches += 3
            if self.world > 1:
                self.dist.all_reduce(self.flag)  # every rank's scatter into this rank's buffer has completed
            planes = self.ex.receive_buffer(b)
            ld_out = n
        else:
            if self.rows and self.cols:
                pk = lib.rns8_cuda_pack_i64_device if self.signed else lib.rns8_cuda_pack_u64_device
                mark(0)
                chk(pk(d, self.A.data_ptr() + self.row0 * k * 8, self.rows, k, k, P, self.ra.data_ptr(), s), "pack A")
                chk(pk(d, self.B.data_ptr() + self.col0 * 8, k, self.cols, n, P, self.rb.data_ptr(), s), "pack B")
                mark(1)
                chk(lib.rns8_cuda_gemm_rns_device(d, self.ra.data_ptr(), self.rb.data_ptr(), self.rc.data_ptr(),
                                                  self.rows, self.cols, k, P, 0, self.scratch.data_ptr(), self.sbytes,
                                                  self.status.data_ptr(), s), "gemm")
                mark(2)
                launches += 3
            planes = self.rc.data_ptr()
            ld_out = self.cols
        if self.rows and self.cols:
            cols = self.cols if self.mode != "planes" else n
            if cfg.kind == "exact":
                st = lib.rns8_cuda_export_limbs_device(d, planes, self.rows, cols, P, 1, cfg.limbs,
                                                       self.out.data_ptr(), ld_out, self.status.data_ptr(), s)
            else:
                fn = lib.rns8_cuda_export_i64_device if self.signed else lib.rns8_cuda_export_u64_device
                st = fn(d, planes, self.rows, cols, P, cfg.bound, self.out.data_ptr(), ld_out,
                        self.status.data_ptr(), s)
            chk(st, "export")
            launches += 1
            if self.mode != "planes":
                mark(3)
        self.launches_per_step = launches

    def check_against_unsharded(self):
        """This rank's block against the unsharded pipeline on this GPU, and
        its first rows against the CPU oracle."""
        import numpy as np

        cfg = self.cfg
        if not self.rows or not self.cols:
            return True
        sub = dataclasses.replace(cfg, m=self.rows, n=self.cols)
        hb = np.ascontiguousarray(self.hB[:, self.col0:self.col0 + self.cols])
        pipe = DevicePipeline(self.torch, self.lib, sub, self.dev, self.hA[self.row0:self.row0 + self.rows], hb)
        pipe.step()
        self.torch.cuda.synchronize()
        same = bool(self.torch.equal(pipe.out, self.out[: self.rows, : self.cols])) and pipe.device_status() == 0
        _, want = cpu_sample(sub, self.hA[self.row0:self.row0 + self.rows], hb, min(8, self.rows))
        got = self.out[:8].cpu().numpy().view("uint64" if cfg.kind in ("u64", "exact") else "int64")
        return same and bool((got[: want.shape[0]] == want.view(got.dtype)).all())

    def close(self):
        if self.ex is not None:
            self.ex.close()


def measure_sharded(args, cfg: Config, torch, dist, lib, rank: int, world: int, local: int, mode: str,
                    exchange: str) -> dict:
    """One strong-scaling measurement: max-over-ranks device time of K steps
    of the sharded product, per-stage times (rank 0's, row and grid modes),
    and the AND over ranks of every block's check."""
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)
    job = ShardedProduct(torch, dist, lib, cfg, local, rank, world, mode, exchange, sptr)
    for _ in range(max(3, args.warmup)):
        job.step()
    torch.cuda.synchronize()
    ok = job.check_against_unsharded()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        job.step()
    stop.record(stream)
    torch.cuda.synchronize()
    stages = None
    if mode != "planes":
        recs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        job.step()  # lead-in work
        for i in range(args.steps):
            job.step(recs[i])
        torch.cuda.synchronize()
        stages = {name: statistics.median(r[i].elapsed_time(r[i + 1]) for r in recs)
                  for i, name in enumerate(("pack", "plane_gemm", "export"))}
    status = int(job.status[0].item())
    t = torch.tensor([start.elapsed_time(stop), 0.0 if (ok and status == 0) else 1.0], dtype=torch.float64,
                     device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if float(t[1].item()) != 0.0:
        raise RuntimeError("sharded result differs from the unsharded pipeline or the oracle (or a device status was set)")
    ms_per_step = float(t[0].item()) / args.steps
    from rns8_b200.shard import grid_shape

    groups = (world, 1) if mode != "grid" else grid_shape(world)
    res = {"mode": mode, "n_gpus": world, "ms_per_step": ms_per_step, "value": cfg.ops / (ms_per_step * 1e-3) / 1e9,
           "unit": "GOPS", "scaling": "strong", "block": {"rows": job.rows, "cols": job.cols},
           "grid": list(groups) if mode != "planes" else None, "stages_ms_rank0": stages,
           "exchange": (("fused epilogue scatter" if job.fused.value else "local planes + copies")
                        if mode == "planes" else "none"),
           "checked": "every rank's block equals the unsharded pipeline's and its first rows the oracle's",
           "gpu_launches": job.launches_per_step * args.steps}
    job.close()
    return res


def run_sharded(args, cfg: Config) -> None:
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    import rns8_b200 as r8

    lib = r8.lib()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    h0 = time.time()
    res = measure_sharded(args, cfg, torch, dist, lib, rank, world, local, args.shard, args.exchange)
    clocks.mark(h0, time.time())
    clock_info = clocks.stop()
    if rank == 0:
        line = {
            "metric": METRIC, "value": res["value"], "unit": "GOPS", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": cfg.workload, "name": cfg.name, "m": cfg.m, "n": cfg.n, "k": cfg.k,
                       "prefix": cfg.prefix, "parallelism": f"{args.shard} x{world}", "exchange": res["exchange"],
                       "grid": res["grid"], "block": res["block"], "seed": SEED, "l2": "inputs larger than L2"},
            "stages_ms_rank0": res["stages_ms_rank0"],
            "e2e": None, "note": "strong-scaling variant (device-resident); the benchmark line is --shard weak-rows",
            "checked": res["checked"], "clocks": clock_info, "gpu_launches": res["gpu_launches"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args, cfg = parse()
    if args.impl == "reference":
        reference_arm(args, cfg)
        return
    if args.shard != "weak-rows":
        run_sharded(args, cfg)
        return
    rank, world, local = dist_env()
    if world > 1:  # ranks share the host's cores for the oracle check (torchrun's default is one thread)
        os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 1) // world))
    hostA, hostB = seeded_inputs(cfg, rank)
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    import rns8_b200 as r8

    lib = r8.lib()
    stream = torch.cuda.current_stream()
    pipe = DevicePipeline(torch, lib, cfg, local, hostA, hostB)

    for _ in range(max(3, args.warmup)):
        pipe.step()
    torch.cuda.synchronize()
    if pipe.device_status() != 0:
        raise RuntimeError(f"device status {pipe.device_status():#x} after warm-up")

    peaks = measured_peaks()
    peak_int8, peak_note = int8_peak_tops(torch, peaks)
    torch.cuda.synchronize()

    # One step's launches captured once as a CUDA graph and replayed: the
    # kernels and their arguments are the same every step, and the replay
    # removes the host's per-launch cost, which dominates the small configs.
    graph, launch_mode = None, "host launches"
    if not args.no_graph:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                pipe.step()
            g.replay()
            torch.cuda.synchronize()
            graph, launch_mode = g, "CUDA graph replay (one capture of the step's launches)"
        except Exception as exc:  # capture unsupported: host launches
            launch_mode = f"host launches (graph capture failed: {type(exc).__name__})"
    if pipe.device_status() != 0:
        raise RuntimeError(f"device status {pipe.device_status():#x} after graph warm-up")

    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    # Small footprints are timed step by step with a 256 MiB write between
    # steps (outside the step's events) so that no step starts with a warm L2.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if pipe.fits_l2 else None
    step_events = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.time()
    start.record(stream)
    for i in range(args.steps):
        if flush is not None:
            flush.zero_()
        step_events[i][0].record(stream)
        if graph is not None:
            graph.replay()
        else:
            pipe.step()
        step_events[i][1].record(stream)
    stop.record(stream)
    torch.cuda.synchronize()
    clocks.mark(h0, time.time())
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    if flush is None:
        total_ms = start.elapsed_time(stop)
    else:
        total_ms = sum(e0.elapsed_time(e1) for e0, e1 in step_events)
    if pipe.device_status() != 0:
        raise RuntimeError(f"device status {pipe.device_status():#x} in the timed region")
    # Per-stage split (for the roofline): after the timed region, the same
    # steps with events between the stages. Each stage is replayed from its
    # own captured graph (host launches with --no-graph), one step's work is
    # queued ahead so the GPU is busy when the first event is recorded, and
    # the median over steps is kept, so that no stage time includes the
    # host's launch latency.
    stages = (pipe.pack, pipe.gemm, pipe.export)
    stage_graphs = None
    if graph is not None:
        try:
            stage_graphs = []
            for fn in stages:
                sg = torch.cuda.CUDAGraph()
                with torch.cuda.graph(sg):
                    fn()
                stage_graphs.append(sg)
        except Exception:
            stage_graphs = None
    records = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    if graph is not None:
        graph.replay()  # lead-in work
    for i in range(args.steps):
        if flush is not None:
            flush.zero_()
        for j in range(3):
            records[i][j].record(stream)
            if stage_graphs is not None:
                stage_graphs[j].replay()
            else:
                stages[j]()
        records[i][3].record(stream)
    torch.cuda.synchronize()
    stage_ms = {name: statistics.median(r[i].elapsed_time(r[i + 1]) for r in records)
                for i, name in enumerate(("pack", "plane_gemm", "export"))}
    # Each stage alone (the burst figure): after 5 ms with the GPU idle and a
    # 256 MiB write that evicts L2, the stage graph replayed once; median over
    # the steps. In a step the stages run back to back under the power drawn
    # by the GEMM and the HBM traffic of their neighbours.
    stage_alone_ms = None
    if stage_graphs is not None:
        evict = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        names = ("pack", "plane_gemm", "export")
        alone = {name: [] for name in names}
        for i in range(args.steps):
            for j, name in enumerate(names):
                torch.cuda.synchronize()
                time.sleep(0.005)
                evict.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                stage_graphs[j].replay()
                e1.record(stream)
                torch.cuda.synchronize()
                alone[name].append(e0.elapsed_time(e1))
        stage_alone_ms = {name: statistics.median(v) for name, v in alone.items()}
        del evict
    if pipe.device_status() != 0:
        raise RuntimeError(f"device status {pipe.device_status():#x} in the stage timing")

    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    value = world * cfg.ops / (ms_per_step * 1e-3) / 1e9

    # ---- e2e through the public C ABI from pinned host buffers -------------------
    e2e = None
    if not args.no_e2e:
        ee = EndToEnd(torch, r8, lib, cfg, local, pipe, hostA, hostB)
        for _ in range(max(3, args.warmup)):
            ee.run()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ee.run()  # synchronous: every call ends with a device sync, the result in host memory
        el = torch.tensor([(time.perf_counter() - t0) * 1e3], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(el, op=dist.ReduceOp.MAX)
        e2e_ms = float(el.item()) / args.steps
        assert torch.equal(ee.hC, pipe.out.cpu()), "e2e result differs from the device-resident result"
        e2e = {"value": world * cfg.ops / (e2e_ms * 1e-3) / 1e9, "unit": "GOPS", "h2d_bytes_per_step": ee.h2d,
               "d2h_bytes_per_step": ee.d2h, "ms_per_step": e2e_ms, "api": ee.api}
        ee.close()

    # ---- parity: the GPU's output against the CPU oracle on the same inputs --------
    # Rank 0 of a one-GPU run checks the config's sample (the CPU baseline is
    # that run's timing); with several ranks each checks 16 rows (one task) of
    # its own product on its share of the host's cores. The FNV checksum of
    # the whole GPU output is reported beside it.
    cpu, parity = None, None
    if not args.no_parity:
        sample = cfg.sample if world == 1 else min(cfg.sample, 1 if cfg.kind == "finite" else 16)
        info, want = cpu_sample(cfg, hostA, hostB, sample)
        out = pipe.out.cpu().numpy()
        if cfg.kind in ("u64", "wrap"):
            out = out.view("uint64")
        elif cfg.kind == "exact":
            out = out.view("uint64")
        got = out[:sample]
        match = bool(got.shape == want.shape and (got == want.view(got.dtype)).all())
        flag = torch.tensor([0.0 if match else 1.0], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        parity = {"oracle": "CPU restatement of the reference's src/cpu path, same seeded inputs",
                  "seed": SEED, "generator": "std::mt19937_64 + std::uniform_int_distribution (libstdc++)",
                  ("tasks_checked" if cfg.kind == "finite" else "rows_checked"): sample,
                  "cells_checked": int(want.size if cfg.kind != "exact" else want.size // cfg.limbs),
                  "match": bool(float(flag.item()) == 0.0),
                  "checksum_sample_gpu": fnv_checksum(got), "checksum_sample_oracle": fnv_checksum(want),
                  "checksum_gpu_full": fnv_checksum(out)}
        if world > 1:
            parity["note"] = "every rank checked its own first rows; match is the AND over ranks"
        if rank == 0 and world == 1:
            cpu = info

    # ---- strong scaling beside the weak line: the config's one product split
    # into 2-D output blocks over the ranks (no exchange) --------------------------
    strong = None
    if world > 1 and not args.no_strong and cfg.kind in ("i64", "u64", "exact"):
        strong = measure_sharded(args, cfg, torch, dist, lib, rank, world, local, "grid", "fused")

    # Roofline of the dominant stage (one kernel launch per stage, except that
    # the grouped finite GEMM launches once per 32 tasks).
    work = pipe.stage_work()
    dominant = max(stage_ms, key=stage_ms.get)
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    hbm_note = "MEASURED_PEAKS.json hbm_gbs (STREAM copy)" if not peaks.get("fallback") else "fallback 6650 GB/s"
    kernel_names = {"pack": "pack_kernel", "plane_gemm": "tc_wrap64_kernel" if cfg.kind == "wrap" else
                    "tc_plane_gemm_kernel", "export": "export kernel"}
    def frac_of(times):
        out = {}
        for name, (bound, amount) in work.items():
            sec = max(times[name], 1e-6) * 1e-3
            out[name] = (amount / sec / 1e12 / peak_int8) if bound == "tensor" else (amount / sec / 1e9 / hbm)
        return out

    stage_frac = frac_of(stage_ms)
    stage_frac_alone = frac_of(stage_alone_ms) if stage_alone_ms else None
    bound, amount = work[dominant]
    sec = stage_ms[dominant] * 1e-3
    if bound == "tensor":
        roof = {"kernel": kernel_names[dominant], "bound": "tensor", "achieved": amount / sec / 1e12,
                "peak": peak_int8, "unit": "TOPS (int8)", "peak_source": peak_note,
                "algorithmic_ops_per_step": amount}
    else:
        roof = {"kernel": kernel_names[dominant], "bound": "hbm", "achieved": amount / sec / 1e9, "peak": hbm,
                "unit": "GB/s", "peak_source": hbm_note, "algorithmic_bytes_per_step": amount}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = profile_traffic(cfg, kernel_names[dominant])
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GOPS", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": {"finite": "uint8", "wrap": "uint64"}.get(cfg.kind, "int64"),
            "data": "synthetic",
            "config": {"workload": cfg.workload, "name": cfg.name, "m_per_rank": cfg.m, "n": cfg.n, "k": cfg.k,
                       "batch": cfg.batch, "prefix": cfg.prefix, "parallelism": f"row-slab x{world}",
                       "launch": launch_mode,
                       "l2": "L2 flushed between steps (256 MiB write outside the step's events)"
                             if pipe.fits_l2 else "inputs larger than L2"},
            "roofline": roof,
            "stages_ms": stage_ms,
            "stages_timing": ("median over the steps of events between per-stage graph replays"
                              if stage_graphs is not None else "median over the steps of events between host launches"),
            "stage_frac_of_peak": stage_frac,
            "stages_alone_ms": stage_alone_ms,
            "stage_frac_of_peak_alone": stage_frac_alone,
            "e2e": e2e, "cpu_baseline": cpu, "parity": parity, "strong_scaling": strong, "clocks": clock_info,
            "gpu_launches": pipe.launches_per_step * args.steps,
        }
        line["config"]["seed"] = SEED
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if parity is not None and not parity["match"]:
        raise SystemExit("parity FAILED: the GPU output differs from the CPU oracle on the sample")


if __name__ == "__main__":
    main()
