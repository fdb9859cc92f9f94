"""Build librns8.so (the rns8 C ABI on sm_100a kernels) in-tree.

Every translation unit under rns8_b200/csrc is compiled by nvcc for
sm_100a only (-gencode arch=compute_100a,code=sm_100a) and linked into
rns8_b200/_build/librns8.so, which is what the Python bindings, the tests and
bench.py load. Object files are rebuilt when a source or header is newer.

    python -m rns8_b200.build [--force] [--ptxas-verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = BUILD / "librns8.so"
INCLUDE = ROOT / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-std=c++17",
    "-O3",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DRNS8_BUILDING_LIBRARY",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build librns8.so")


def host_compiler() -> list[str]:
    # The system g++ is the toolchain nvcc 12.9 is validated against here.
    return ["-ccbin", "/usr/bin/g++"] if Path("/usr/bin/g++").exists() else []


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def headers() -> list[Path]:
    return [*CSRC.glob("*.hpp"), *CSRC.glob("*.cuh"), *INCLUDE.glob("rns8/*.h")]


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), *host_compiler(), *COMMON, *ARCH_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return src, res.stdout + res.stderr


def build(force: bool = False, ptxas_verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr_time = max((h.stat().st_mtime for h in headers()), default=0.0)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    todo = []
    objs = []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            todo.append((src, obj))
    logs = []
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as pool:
            for src, log in pool.map(lambda t: _compile(t[0], t[1], extra), todo):
                if log.strip():
                    logs.append(f"--- {src.name}\n{log}")
    if todo or not LIB.exists():
        cmd = [nvcc(), *host_compiler(), *ARCH_FLAGS, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if ptxas_verbose:
        print("\n".join(logs))
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    lib = build(force=args.force, ptxas_verbose=args.ptxas_verbose)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
