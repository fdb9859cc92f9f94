"""bench.py's reference arm on CPU: one JSON line with the contract's keys,
timing the CPU restatement of the reference path on a bounded sample."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "C1", "--steps",
                          "1", "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GOPS"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1


def test_bench_checksum_and_sample_helpers():
    """The FNV output checksum (rns8_bench_support.cpp:96-99) gives the same
    value for bytes as for the same values widened to uint64, and the CPU
    sample of C1 (the whole product) equals the oracle's one-shot."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    import bench
    from oracle import bridge

    rng = np.random.default_rng(5)
    u8 = rng.integers(0, 251, (3, 40, 37), dtype=np.uint8)
    assert bench.fnv_checksum(u8) == bridge.checksum(u8.astype(np.uint64).reshape(3, -1))
    big = rng.integers(0, 256, (5 << 20) + 3, dtype=np.uint8)  # more than one chunk
    assert bench.fnv_checksum(big.reshape(1, -1)) == bridge.checksum(big.astype(np.uint64).reshape(1, -1))
    cfg = bench.CONFIGS["C1"]
    A, B = bench.seeded_inputs(cfg, 0)
    info, out = bench.cpu_sample(cfg, A, B, cfg.m)
    st, want, _ = bridge.gemm_bounded_oneshot(A, B, cfg.bound)
    assert st == 0 and np.array_equal(out, want)
    assert info["kind"] == "port" and info["value"] > 0
    # Rank 1 shares rank 0's B and draws its own A.
    A1, B1 = bench.seeded_inputs(cfg, 1)
    assert np.array_equal(B1, B) and not np.array_equal(A1, A)
