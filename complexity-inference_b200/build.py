"""Build libmuk.so (the sm_100a kernels behind mu_b200) in-tree.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` (relocatable
device code, so the device error word is shared across files) and linked
into ``mu_b200/libmuk.so``.  Objects go to ``_build/`` next to this file; a
source is recompiled only when it or a header is newer than its object.

Usage: ``python build.py [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
OUT = HERE / "mu_b200" / "libmuk.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-Wall",
    f"-I{INCLUDE}",
]


def _nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmuk.so")
    return path


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(nvcc: str, src: Path, force: bool, hdr_mtime: float) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists():
        if obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
            return obj
    cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}\n{res.stdout}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile every kernel and link ``mu_b200/libmuk.so``; returns its path."""
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr = _headers_mtime()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, force, hdr), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(OUT)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of libmuk.so failed:\n{res.stderr}\n{res.stdout}")
        if verbose:
            print(f"linked {OUT}")
    return OUT


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    out = build(force=args.force, jobs=args.jobs, verbose=True)
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
