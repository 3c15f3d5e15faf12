"""Build libpyrite_b200.so in-tree for sm_100a.

    python -m pyrite_b200.build          # compile (incremental)
    python -m pyrite_b200.build --force  # rebuild everything

The library is plain CUDA C++ with a C ABI (include/pyrite_b200.h); it links
the CUDA runtime statically, so it needs only the driver at run time.
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
OBJ = PKG / "_native" / "obj"
LIB = PKG / "_native" / "libpyrite_b200.so"
SOURCES = ["capi.cu", "mv_generic.cu", "mv_tile.cu", "mm_tc.cu", "noalloc.cu", "decode.cu", "moe.cu", "allreduce.cu", "quantize.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# host code: no FMA contraction, so the quantizers round exactly like the
# Python encoders they restate
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off", "--expt-relaxed-constexpr",
              "-I", str(ROOT / "include")]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libpyrite_b200.so")
    return found


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    for name in SOURCES:
        src, obj = CSRC / name, OBJ / (Path(name).stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
            list(pool.map(lambda j: _compile(*j, verbose), jobs))
    objs = [OBJ / (Path(n).stem + ".o") for n in SOURCES]
    if force or jobs or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
