"""ctypes/numpy front end of the CPU oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker. The product never imports it.

Two libraries:
  liboracle.so           this repository's C restatement (oracle/ref_cpu.c)
  _ref/libchoreo_ref.so  the reference's own headers compiled from source
                         (oracle/build.py), present only where it was built.
16-bit values travel as numpy uint16 bit patterns (bf16 has no numpy dtype).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
F16, F32, BF16 = 8, 9, 11

_i64 = C.c_int64
_vp = C.c_void_p


def _load_oracle() -> C.CDLL:
    path = HERE / "liboracle.so"
    if not path.exists():
        raise RuntimeError(f"{path} is missing: run `python oracle/build.py`")
    lib = C.CDLL(str(path))
    lib.oracle_max_threads.restype = C.c_int
    lib.oracle_ref_matmul_f16.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, C.c_int]
    lib.oracle_ref_matmul_bf16.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, C.c_int]
    lib.oracle_ref_matmul_f32.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, C.c_int]
    lib.oracle_ref_relu_f16.argtypes = [_vp, _vp, _i64]
    lib.oracle_ref_relu_f32.argtypes = [_vp, _vp, _i64]
    lib.oracle_ref_add_f16.argtypes = [_vp, _vp, _vp, _i64]
    lib.oracle_ref_add_f32.argtypes = [_vp, _vp, _vp, _i64]
    lib.oracle_ref_conv2d_f16.argtypes = [_vp, _vp, _vp] + [_i64] * 7 + [C.c_int] * 4 + [_i64, _i64, C.c_int]
    lib.oracle_gemm_f64.argtypes = [C.c_int, _vp, _i64, C.c_int, _vp, _i64, C.c_int, _i64, _i64, _i64,
                                    C.c_double, C.c_double, C.c_int, _vp, _i64, C.c_int, _vp, C.c_int,
                                    _vp, _i64, _vp, C.c_int]
    lib.oracle_conv2d_f64.argtypes = [C.c_int, _vp, _vp] + [_i64] * 7 + [C.c_int] * 6 + \
        [C.c_double, C.c_int, _vp, C.c_int, _vp, _i64, _vp, C.c_int]
    lib.oracle_f32_to_f16.argtypes = [_vp, _vp, _i64]
    lib.oracle_f32_to_bf16.argtypes = [_vp, _vp, _i64]
    lib.oracle_f16_to_f32.argtypes = [_vp, _vp, _i64]
    lib.oracle_bf16_to_f32.argtypes = [_vp, _vp, _i64]
    return lib


lib = _load_oracle()


def _load_ref() -> C.CDLL | None:
    path = HERE / "_ref" / "libchoreo_ref.so"
    if not path.exists():
        return None
    r = C.CDLL(str(path))
    for n in ("choreo_ref_matmul_f16", "choreo_ref_matmul_bf16", "choreo_ref_matmul_f32"):
        getattr(r, n).argtypes = [_vp, _vp, _vp, _i64, _i64, _i64]
    for n in ("choreo_ref_matmul_f16_rows", "choreo_ref_matmul_bf16_rows"):
        getattr(r, n).argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, C.c_int]
    r.choreo_ref_relu_f16.argtypes = [_vp, _vp, _i64]
    r.choreo_ref_relu_f32.argtypes = [_vp, _vp, _i64]
    r.choreo_ref_add_mismatch_f32.argtypes = [_i64, _i64]
    r.choreo_ref_matmul_mismatch_f32.argtypes = [_i64, _i64, _i64, _i64]
    return r


ref = _load_ref()


def threads() -> int:
    return int(lib.oracle_max_threads())


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


# ----------------------------------------------------------------- conversion
def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib.oracle_f32_to_f16(_p(x), _p(out), x.size)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib.oracle_f32_to_bf16(_p(x), _p(out), x.size)
    return out


def bits_to_f32(bits: np.ndarray, dtype: int) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, np.float32)
    (lib.oracle_bf16_to_f32 if dtype == BF16 else lib.oracle_f16_to_f32)(_p(bits), _p(out), bits.size)
    return out


def to_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    """fp32 values rounded (RNE) to the 16-bit type, as uint16 bit patterns."""
    return f32_to_bf16_bits(x) if dtype == BF16 else f32_to_f16_bits(x)


# ----------------------------------------------------------------- generators
def uniform(shape, lo: float, hi: float, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).uniform(lo, hi, size=shape).astype(np.float32)


def normal(shape, mean: float, std: float, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).normal(mean, std, size=shape).astype(np.float32)


# ----------------------------------------------------------------- reference restatement
def ref_matmul(a: np.ndarray, b: np.ndarray, dtype: int, rows: tuple[int, int] | None = None,
               nthreads: int = 1, use_reference_lib: bool = False) -> np.ndarray:
    """The reference host operator* (choreo-ir.hpp:71-101) on contiguous
    row-major A (M x K) and B (K x N). 16-bit inputs as uint16 bits, f32 as
    float32. Returns rows [r0, r1) of C (all rows by default)."""
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    r0, r1 = rows if rows else (0, M)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    c = np.zeros((r1 - r0, N), np.float32 if dtype == F32 else np.uint16)
    # The C routines index C by absolute row; hand them a base pointer r0 rows
    # before the slab so only the slab is allocated.
    cbase = _p(c) - r0 * N * c.itemsize
    if use_reference_lib:
        if ref is None:
            raise RuntimeError("reference library oracle/_ref was not built")
        if dtype == F16:
            rc = ref.choreo_ref_matmul_f16_rows(_p(a), _p(b), cbase, M, N, K, r0, r1, nthreads)
        elif dtype == BF16:
            rc = ref.choreo_ref_matmul_bf16_rows(_p(a), _p(b), cbase, M, N, K, r0, r1, nthreads)
        else:
            sub = np.ascontiguousarray(a[r0:r1])
            rc = ref.choreo_ref_matmul_f32(_p(sub), _p(b), _p(c), r1 - r0, N, K)
        if rc != 0:
            raise RuntimeError(f"reference operator* failed ({rc})")
    else:
        fn = {F16: lib.oracle_ref_matmul_f16, BF16: lib.oracle_ref_matmul_bf16, F32: lib.oracle_ref_matmul_f32}[dtype]
        fn(_p(a), _p(b), cbase, M, N, K, r0, r1, nthreads)
    return c


def ref_relu(x: np.ndarray, dtype: int) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    (lib.oracle_ref_relu_f32 if dtype == F32 else lib.oracle_ref_relu_f16)(_p(x), _p(out), x.size)
    return out


def ref_add(a: np.ndarray, b: np.ndarray, dtype: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    out = np.empty_like(a)
    (lib.oracle_ref_add_f32 if dtype == F32 else lib.oracle_ref_add_f16)(_p(a), _p(b), _p(out), a.size)
    return out


def ref_conv2d_f16(x: np.ndarray, w: np.ndarray, stride: int, pad: int, pix: tuple[int, int] | None = None,
                   nthreads: int = 1) -> np.ndarray:
    """conv2d_kernel's fp16-accumulating loop (gemm_example.cu:230-247) over
    NHWC x (uint16 bits) and KRSC w; returns [npix, K] for output pixels
    [p0, p1) in NHW order."""
    N, H, W, Cc = x.shape
    K, R, S, _ = w.shape
    P = (H + 2 * pad - R) // stride + 1
    Q = (W + 2 * pad - S) // stride + 1
    p0, p1 = pix if pix else (0, N * P * Q)
    out = np.zeros((N * P * Q, K), np.uint16)
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w)
    lib.oracle_ref_conv2d_f16(_p(x), _p(w), _p(out), N, H, W, Cc, K, R, S, stride, stride, pad, pad, p0, p1,
                              nthreads)
    return out[p0:p1]


# ----------------------------------------------------------------- fp64 checkers
def gemm_f64(a: np.ndarray, b: np.ndarray, dtype: int, *, trans_a=False, trans_b=False, m=None, n=None, k=None,
             lda=None, ldb=None, alpha=1.0, beta=0.0, c0: np.ndarray | None = None, dtype_c0: int = F32,
             bias: np.ndarray | None = None, dtype_bias: int = F32, relu=False, rows=None,
             nthreads: int | None = None) -> np.ndarray:
    """fp64 op(A) op(B) epilogue over the given rows (all by default).
    a, b: 2-D arrays as stored (uint16 bits or float32)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if m is None:
        m = a.shape[1] if trans_a else a.shape[0]
    if k is None:
        k = a.shape[0] if trans_a else a.shape[1]
    if n is None:
        n = b.shape[0] if trans_b else b.shape[1]
    lda = lda if lda is not None else a.shape[1]
    ldb = ldb if ldb is not None else b.shape[1]
    rows = np.arange(m, dtype=np.int64) if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((rows.size, n), np.float64)
    c0p = None
    ldc0 = 0
    if c0 is not None:
        c0 = np.ascontiguousarray(c0)
        c0p, ldc0 = _p(c0), c0.shape[1]
    bp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias)
        bp = _p(bias)
    lib.oracle_gemm_f64(dtype, _p(a), lda, int(trans_a), _p(b), ldb, int(trans_b), m, n, k, alpha, beta,
                        dtype_c0, c0p, ldc0, dtype_bias, bp, int(relu), _p(rows), rows.size, _p(out),
                        nthreads or threads())
    return out


def conv2d_f64(x: np.ndarray, w: np.ndarray, dtype: int, *, stride=1, pad=1, dil=1, alpha=1.0,
               bias: np.ndarray | None = None, dtype_bias: int = F32, relu=False, pixels=None,
               nthreads: int | None = None) -> np.ndarray:
    N, H, W, Cc = x.shape
    K, R, S, _ = w.shape
    P = (H + 2 * pad - dil * (R - 1) - 1) // stride + 1
    Q = (W + 2 * pad - dil * (S - 1) - 1) // stride + 1
    pixels = np.arange(N * P * Q, dtype=np.int64) if pixels is None else np.ascontiguousarray(pixels, dtype=np.int64)
    out = np.empty((pixels.size, K), np.float64)
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w)
    bp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias)
        bp = _p(bias)
    lib.oracle_conv2d_f64(dtype, _p(x), _p(w), N, H, W, Cc, K, R, S, stride, stride, pad, pad, dil, dil,
                          alpha, dtype_bias, bp, int(relu), _p(pixels), pixels.size, _p(out),
                          nthreads or threads())
    return out


# ----------------------------------------------------------------- tolerance
def rel_err(y: np.ndarray, r: np.ndarray, k: int | None = None) -> float:
    """max_i |y - r| / max(|r|, tau): per-element relative error with a floor
    so outputs that cancel to ~0 do not divide by ~0. tau = 1e-3 * rms(r),
    widened by sqrt(K / 1024) for reductions longer than 1024 terms, because
    the absolute error of an fp32 accumulation grows like sqrt(K) * rms."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    grow = np.sqrt(max(1.0, (k or 1024) / 1024.0))
    tau = 1e-3 * grow * float(np.sqrt(np.mean(r * r))) + 1e-300
    return float(np.max(np.abs(y - r) / np.maximum(np.abs(r), tau)))


def normwise_err(y: np.ndarray, r: np.ndarray) -> float:
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.max(np.abs(y - r)) / max(float(np.max(np.abs(r))), 1e-300))
