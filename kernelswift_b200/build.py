"""Builds libmoe_b200.so (the C-ABI library of the fused-MoE operator) in-tree.

Every CUDA source under csrc/ is compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`) and linked into
kernelswift_b200/lib/libmoe_b200.so with the CUDA runtime linked statically,
so the library needs nothing but the NVIDIA driver at run time.

    python -m kernelswift_b200.build [--force] [--verbose-ptxas]
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
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
BUILD_DIR = PKG / "_build"
LIB_PATH = LIB_DIR / "libmoe_b200.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXX_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
             "-Xcompiler", "-Wall", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH_FLAGS, *CXX_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return obj, res.stdout + res.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    """Compiles stale objects and relinks the library; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    hdrs = headers()
    jobs = []
    objs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_verbose or _stale(obj, [src, *hdrs]):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile, s, o, ptxas_verbose) for s, o in jobs]
            for f in futs:
                _, log = f.result()
                if log.strip() and not quiet:
                    print(log, file=sys.stderr)
    if force or jobs or _stale(LIB_PATH, objs):
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIB_PATH), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, ptxas_verbose=args.verbose_ptxas, quiet=False)
    print(path)


if __name__ == "__main__":
    main()
