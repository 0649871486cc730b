"""Builds libchoreo_b200.so in-tree with nvcc for sm_100a.

Each .cu under csrc/ is compiled to an object under _build/ (in parallel,
skipped when up to date), then linked into choreo-ir_b200/libchoreo_b200.so
with the CUDA runtime linked statically so the library does not depend on
which libcudart another component of the process loaded first.

Usage: python choreo-ir_b200/build.py [-v] [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libchoreo_b200.so"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-Xcompiler", "-Wall", "-diag-suppress", "177",
    f"-I{ROOT / 'include'}",
]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found")
    return exe


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "choreo_b200.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = OBJ / (src.stem + ".o")
    if not _stale(obj, _deps(src)):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout, r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    if force:
        for o in OBJ.glob("*.o"):
            o.unlink()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra), srcs))
    if _stale(OUT, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcuda" if False else "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="--force" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(OUT)
