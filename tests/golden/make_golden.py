"""Generates the golden fixtures in tests/golden/ from the reference itself.

Inputs are drawn the way the reference's own tests draw them (std::mt19937
with std::uniform_real_distribution<float>, glibc rand(); via
gen_std_random.cpp compiled with g++), or from seeded numpy generators; the
expected outputs come from the reference's host code compiled from its
sources (oracle/_ref/libchoreo_ref.so, built by oracle/build.py from the
reference checkout). Run where the reference checkout exists:

    python oracle/build.py && python tests/golden/make_golden.py

The fixtures are committed; the tests only read them.
"""
from __future__ import annotations

import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
from oracle import oracle as orc  # noqa: E402

F16, F32, BF16 = orc.F16, orc.F32, orc.BF16


def std_random(gen: Path, *args) -> np.ndarray:
    out = subprocess.run([str(gen), *map(str, args)], capture_output=True, text=True, check=True).stdout.split()
    return np.array([int(h, 16) for h in out], dtype=np.uint32).view(np.float32)


def ref_matmul(a, b, dt):
    """The reference's compiled operator* (host branch)."""
    return orc.ref_matmul(a, b, dt, use_reference_lib=True)


def main() -> None:
    if orc.ref is None:
        raise SystemExit("oracle/_ref/libchoreo_ref.so is missing: run python oracle/build.py where the reference exists")
    manifest = {}
    with tempfile.TemporaryDirectory() as td:
        gen = Path(td) / "gen_std_random"
        subprocess.run(["g++", "-O2", "-std=c++17", str(HERE / "gen_std_random.cpp"), "-o", str(gen)], check=True)

        # 1. A = [[1,2],[3,4]], B = I  (tests/test_debug_cpu.cpp:23-29, test_baselines.cpp:38-66)
        a = np.array([[1, 2], [3, 4]], np.float32)
        b = np.eye(2, dtype=np.float32)
        np.savez(HERE / "kat_identity_2x2.npz", a_f32=a, b_f32=b, c_f32=ref_matmul(a, b, F32),
                 a_f16=orc.to_bits(a, F16), b_f16=orc.to_bits(b, F16),
                 c_f16=ref_matmul(orc.to_bits(a, F16), orc.to_bits(b, F16), F16))
        manifest["kat_identity_2x2.npz"] = "[[1,2],[3,4]] * I through the reference operator* (f32, f16); tests/test_debug_cpu.cpp:23-29"

        # 2. single 16^3 tile, mt19937(42) U[-2,2] fp16, A then B (tests/compute/test_wmma.cu:33-39);
        #    expected = the test's host fp32 loop (:48-52) = the reference f32 operator* on the fp16 values
        v = std_random(gen, "mt19937", 42, 16 * 16 * 2, -2.0, 2.0)
        a16 = orc.to_bits(v[:256].reshape(16, 16), F16)
        b16 = orc.to_bits(v[256:].reshape(16, 16), F16)
        c32 = ref_matmul(orc.bits_to_f32(a16, F16), orc.bits_to_f32(b16, F16), F32)
        np.savez(HERE / "wmma_tile_16.npz", a_f16=a16, b_f16=b16, c_f32=c32, tol=np.float32(1e-2))
        manifest["wmma_tile_16.npz"] = "16x16x16 fp16, mt19937(42) U[-2,2], expected = host fp32 loop, tol 1e-2; tests/compute/test_wmma.cu:33-60"

        # 3. ReLU exactness on mt19937(42) U[-2,2] 64x32 floats (tests/test_end2end.cpp:211-234)
        x = std_random(gen, "mt19937", 42, 64 * 32, -2.0, 2.0).reshape(64, 32)
        y = np.empty_like(x)
        assert orc.ref.choreo_ref_relu_f32(x.ctypes.data, y.ctypes.data, x.size) == 0
        x16 = orc.to_bits(x, F16)
        y16 = np.empty_like(x16)
        assert orc.ref.choreo_ref_relu_f16(x16.ctypes.data, y16.ctypes.data, x16.size) == 0
        np.savez(HERE / "end2end_relu_64x32.npz", x_f32=x, y_f32=y, x_f16=x16, y_f16=y16)
        manifest["end2end_relu_64x32.npz"] = "relu through the reference (f32, f16), mt19937(42) U[-2,2]; tests/test_end2end.cpp:211-234"

        # 4. 64^3 f32 with glibc rand()/RAND_MAX, A then B (tests/test_baselines.cpp:236-305), tol 1e-4
        v = std_random(gen, "rand", 64 * 64 * 2)
        a = v[: 64 * 64].reshape(64, 64)
        b = v[64 * 64:].reshape(64, 64)
        np.savez(HERE / "baselines_64_f32.npz", a=a, b=b, c=ref_matmul(a, b, F32), tol=np.float32(1e-4))
        manifest["baselines_64_f32.npz"] = "64^3 f32, rand()/RAND_MAX inputs, expected = reference f32 operator*, tol 1e-4; tests/test_baselines.cpp:236-305"

        # 5. DifferentDataTypes: 64x48 * 48x32 with create_random_matrix (fresh mt19937(42) U[0,1) per matrix)
        #    for f32 and f16 (tests/test_end2end.cpp:293-309, generator :31-53)
        va = std_random(gen, "mt19937", 42, 64 * 48, 0.0, 1.0).reshape(64, 48)
        vb = std_random(gen, "mt19937", 42, 48 * 32, 0.0, 1.0).reshape(48, 32)
        np.savez(HERE / "end2end_types_64x32x48.npz", a_f32=va, b_f32=vb, c_f32=ref_matmul(va, vb, F32),
                 a_f16=orc.to_bits(va, F16), b_f16=orc.to_bits(vb, F16),
                 c_f16=ref_matmul(orc.to_bits(va, F16), orc.to_bits(vb, F16), F16))
        manifest["end2end_types_64x32x48.npz"] = "A(64x48)*B(48x32), mt19937(42) U[0,1) per matrix, reference operator* f32/f16; tests/test_end2end.cpp:293-309"

        # 6. seeded numpy inputs through the reference operator* in each type
        for name, (M, N, K), dt, seed in (("ref_matmul_f16_64x48x80.npz", (64, 48, 80), F16, 7),
                                          ("ref_matmul_bf16_32x24x40.npz", (32, 24, 40), BF16, 8),
                                          ("ref_matmul_f32_24x16x40.npz", (24, 16, 40), F32, 9)):
            a = orc.uniform((M, K), -1, 1, seed)
            b = orc.uniform((K, N), -1, 1, seed + 100)
            if dt != F32:
                a, b = orc.to_bits(a, dt), orc.to_bits(b, dt)
            np.savez(HERE / name, a=a, b=b, c=ref_matmul(a, b, dt), dtype=np.int32(dt))
            manifest[name] = f"numpy default_rng({seed}/{seed + 100}) U[-1,1], reference operator* (choreo-ir.hpp:71-101)"

    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print("wrote", len(manifest), "fixtures")


if __name__ == "__main__":
    main()
