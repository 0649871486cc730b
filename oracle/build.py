"""Builds the CPU oracle (test infrastructure, never part of the product).

  oracle/liboracle.so          gcc -O2 -fopenmp -ffp-contract=off ref_cpu.c
  oracle/_ref/libchoreo_ref.so the reference's own headers, compiled
                               unmodified from REFERENCE_ROOT/include with
                               oracle/ref_shim.h force-included (nvcc, host
                               code only). Built only where the reference
                               checkout exists; elsewhere the prebuilt file
                               is used if it was shipped, else the pin tests
                               skip and the restatement stands alone.

REFERENCE_ROOT is the reference checkout: `--reference PATH`, else the
CHOREO_REFERENCE_ROOT environment variable, else a checkout named `reference`
beside this repository's root directory.

Usage: python oracle/build.py [-v] [--reference PATH]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REFERENCE_ROOT = Path(os.environ.get("CHOREO_REFERENCE_ROOT", str(HERE.parent.parent / "reference")))
LIB = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_LIB = REF_DIR / "libchoreo_ref.so"


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_oracle(verbose: bool = False) -> Path:
    src = HERE / "ref_cpu.c"
    if _stale(LIB, [src, Path(__file__)]):
        _run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-std=c11", "-Wall",
              str(src), "-o", str(LIB), "-lm"], verbose)
    return LIB


def build_reference(verbose: bool = False, reference_root: Path | None = None) -> Path | None:
    inc = Path(reference_root or REFERENCE_ROOT) / "include"
    if not (inc / "choreo-ir" / "choreo-ir.hpp").exists():
        return REF_LIB if REF_LIB.exists() else None
    srcs = [HERE / "ref_entry.cu", HERE / "ref_shim.h"]
    if _stale(REF_LIB, srcs + [Path(__file__)]):
        REF_DIR.mkdir(exist_ok=True)
        nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        objs = []
        for t in (1, 2, 3):
            obj = REF_DIR / f"ref_entry_{t}.o"
            _run([nvcc, "-std=c++17", "-O3", "-Xcompiler", "-fPIC", "-c",
                  "-gencode", "arch=compute_100a,code=sm_100a", "-diag-suppress", "20012",
                  f"-DCHOREO_REF_TYPE={t}", f"-I{inc}", "-include", str(HERE / "ref_shim.h"),
                  str(HERE / "ref_entry.cu"), "-o", str(obj)], verbose)
            objs.append(str(obj))
        _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", str(REF_LIB)],
             verbose)
        for o in objs:
            Path(o).unlink()
    return REF_LIB


def build(verbose: bool = False, reference_root: Path | None = None) -> None:
    build_oracle(verbose)
    build_reference(verbose, reference_root)


if __name__ == "__main__":
    ref = None
    if "--reference" in sys.argv:
        ref = Path(sys.argv[sys.argv.index("--reference") + 1])
    build(verbose="-v" in sys.argv, reference_root=ref)
    print(LIB, REF_LIB if REF_LIB.exists() else "(reference not built)")
