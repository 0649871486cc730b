"""Shared pytest setup.

Markers: `gpu` — needs a CUDA device (run with -m gpu on a B200); everything
else runs on a CPU-only host. The oracle (oracle/) is the checker only; the
code under test is libchoreo_b200.so, reached through its C ABI.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _ensure_built() -> None:
    oracle_lib = ROOT / "oracle" / "liboracle.so"
    if not oracle_lib.exists():
        spec = importlib.util.spec_from_file_location("oracle_build", ROOT / "oracle" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    if not (ROOT / "choreo-ir_b200" / "libchoreo_b200.so").exists():
        spec = importlib.util.spec_from_file_location("choreo_build", ROOT / "choreo-ir_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()


_ensure_built()


def load_choreo():
    """The ctypes binding of libchoreo_b200.so (package dir has a hyphen)."""
    if "choreo_b200" in sys.modules:
        return sys.modules["choreo_b200"]
    spec = importlib.util.spec_from_file_location("choreo_b200", ROOT / "choreo-ir_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["choreo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def cb():
    return load_choreo()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected on a host without CUDA")
    return torch
