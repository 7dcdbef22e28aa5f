"""Builds libsixi_smp.so (the C-ABI library of the B200 logits-to-token path) for sm_100a.

The row-engine kernel template is instantiated once per (mode, dtype) pair in its own
translation unit (csrc/smp_inst.cu compiled with -DSIXI_INST_MODE/-DSIXI_INST_DT) so the eight
instance families compile in parallel. Objects are cached under _build/ by source timestamps.
Usage: python sixi-asi_b200/build_lib.py [-j N] [--force]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = REPO / "_build" / "sixi_smp"
LIB = PKG / "lib" / "libsixi_smp.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr"]
MODES = {"sample": 0, "candidates": 1, "greedy": 2, "verify": 3}
DTYPES = {"f32": 0, "bf16": 1}


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def _stale(obj: Path, srcs: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(s.stat().st_mtime > t for s in srcs)


def _compile(src: Path, obj: Path, defines: list[str], force: bool) -> str:
    deps = [src] + _headers()
    if not force and not _stale(obj, deps):
        return f"up to date {obj.name}"
    obj.parent.mkdir(parents=True, exist_ok=True)
    cmd = [NVCC, *ARCH, *FLAGS, *defines, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name} {defines}:\n{r.stdout}\n{r.stderr}")
    return f"built {obj.name}"


def build(jobs: int | None = None, force: bool = False, verbose: bool = True) -> Path:
    jobs = jobs or max(1, os.cpu_count() or 1)
    units: list[tuple[Path, Path, list[str]]] = []
    for mname, m in MODES.items():
        for dname, d in DTYPES.items():
            units.append((CSRC / "smp_inst.cu", BUILD / f"inst_{mname}_{dname}.o",
                          [f"-DSIXI_INST_MODE={m}", f"-DSIXI_INST_DT={d}"]))
    for name in ("smp_launch", "smp_abi", "smp_shard", "smp_dist", "smp_json", "smp_numeric", "smp_suffix", "smp_schema"):
        units.append((CSRC / f"{name}.cu", BUILD / f"{name}.o", []))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_compile, s, o, d, force) for s, o, d in units]
        for f in cf.as_completed(futs):
            msg = f.result()
            if verbose:
                print(msg, flush=True)
    objs = [o for _, o, _ in units]
    if force or _stale(LIB, objs):
        LIB.parent.mkdir(parents=True, exist_ok=True)
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lrt", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"linked {LIB}", flush=True)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(args.j, args.force)
    return 0


if __name__ == "__main__":
    sys.exit(main())
