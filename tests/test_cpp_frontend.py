"""Builds tests/cpp/test_frontend.cu against the C++ API (include/choreo-ir/)
and libchoreo_b200.so, and runs its CPU cases here and its GPU cases on a
B200. The cases mirror the reference's own C++ unit and end-to-end tests."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "cpp" / "test_frontend.cu"
OUT = ROOT / "tests" / "cpp" / "_build" / "test_frontend"
LIB = ROOT / "choreo-ir_b200" / "libchoreo_b200.so"


def build() -> Path:
    deps = [SRC, ROOT / "tests" / "cpp" / "mini_test.hpp", LIB, ROOT / "include" / "choreo_b200.h",
            *sorted((ROOT / "include" / "choreo-ir").rglob("*.hpp"))]
    if OUT.exists() and all(d.stat().st_mtime <= OUT.stat().st_mtime for d in deps):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
           f"-I{ROOT / 'include'}", f"-I{ROOT / 'tests' / 'cpp'}", str(SRC), "-o", str(OUT),
           f"-L{LIB.parent}", "-lchoreo_b200", f"-Xlinker", f"-rpath={LIB.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return OUT


def run(group: str) -> str:
    exe = build()
    r = subprocess.run([str(exe), group], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    return r.stdout


def test_cpp_frontend_cpu_cases():
    out = run("cpu")
    assert " 0 failures" in out


@pytest.mark.gpu
def test_cpp_frontend_gpu_cases():
    out = run("gpu")
    assert " 0 failures" in out
