/*
 * oracle/ref_cpu.c — CPU oracle for the dense-contraction path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (libchoreo_b200.so, the
 * C++ headers in include/) uses this file. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg load it, as the checker and the timed
 * reference CPU path.
 *
 * Two kinds of routines:
 *  1. Restatements of the reference's own CPU arithmetic, element for element:
 *     - oracle_ref_matmul_{f16,bf16,f32}: the host branch of operator*
 *       (include/choreo-ir/choreo-ir.hpp:71-101): C zero-filled, i-j-k loop
 *       over contiguous row-major A[i*K+k], B[k*N+j]; fp16 converts to float,
 *       computes c + a*b in float and rounds C back to fp16 after every k
 *       (:82-94); float and bf16 do C += A*B in T (:96), where bf16's host
 *       operators round the product and the sum to bf16.
 *     - oracle_ref_relu_* / oracle_ref_add_*: relu (:196-222), operator+
 *       (:150-191).
 *     - oracle_ref_conv2d_f16: the loop of the reference's only convolution,
 *       conv2d_kernel (benchmark/kernels/gemm_example.cu:208-253: for c, r, s,
 *       sum += in * w in T with zero padding), restated over NHWC / KRSC
 *       storage; for T = half each product and each sum is rounded to fp16.
 *     These are pinned bit-for-bit against the reference headers compiled
 *     from source (oracle/_ref, see oracle/build.py) and the fixtures in
 *     tests/golden/.
 *  2. fp64 checkers over the same rounded inputs: oracle_gemm_f64 and
 *     oracle_conv2d_f64, the per-element reference for the tolerance tests
 *     (fp32-accumulating kernels are compared against these, since the
 *     reference's fp16-accumulating path is itself off by up to ~1e-2
 *     relative).
 *
 * Build: gcc -O2 -fopenmp -ffp-contract=off (no FMA contraction, so float
 * expressions round exactly as the reference's host code does).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* IEEE-754 binary16 / bfloat16 conversions, round-to-nearest-even.          */

static inline uint32_t f32_bits(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  return x;
}
static inline float bits_f32(uint32_t x) {
  float f;
  memcpy(&f, &x, 4);
  return f;
}

float oracle_h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    /* zero or subnormal: man * 2^-24, exact in float */
    const float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return bits_f32(sign | 0x7f800000u | (man << 13));
  return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_f2h(float f) {
  const uint32_t x = f32_bits(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t a = x & 0x7fffffffu;
  if (a >= 0x7f800000u) /* inf / nan */
    return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? (0x200u | ((a >> 13) & 0x3ffu)) : 0u));
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (a >= 0x38800000u) {                                  /* normal half */
    uint32_t t = a - (112u << 23);
    t += 0x0fffu + ((t >> 13) & 1u);
    return (uint16_t)(sign | (t >> 13));
  }
  /* subnormal half (or zero): value / 2^-24 rounded to an integer, ties to even */
  const uint32_t e = a >> 23;
  if (e < 102) return sign; /* below 2^-25 */
  const uint32_t m = (a & 0x7fffffu) | 0x800000u;
  const uint32_t s = 126u - e; /* 14..24 */
  uint32_t q = m >> s;
  const uint32_t rem = m & ((1u << s) - 1u);
  const uint32_t half = 1u << (s - 1u);
  if (rem > half || (rem == half && (q & 1u))) ++q;
  return (uint16_t)(sign | q);
}

float oracle_bf2f(uint16_t b) { return bits_f32((uint32_t)b << 16); }

uint16_t oracle_f2bf(float f) {
  const uint32_t x = f32_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u); /* quiet nan */
  const uint32_t t = x + 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(t >> 16);
}

void oracle_f32_to_f16(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f2h(src[i]);
}
void oracle_f32_to_bf16(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f2bf(src[i]);
}
void oracle_f16_to_f32(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_h2f(src[i]);
}
void oracle_bf16_to_f32(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_bf2f(src[i]);
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* 1. Restatements of the reference's host arithmetic.                       */
/* Rows [row0, row1) of C are computed; nthreads > 1 splits rows across host  */
/* threads (each element's arithmetic and order are unchanged).               */

void oracle_ref_matmul_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N,
                           int64_t K, int64_t row0, int64_t row1, int nthreads) {
  (void)M;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t i = row0; i < row1; ++i) {
    for (int64_t j = 0; j < N; ++j) {
      uint16_t c = 0; /* std::fill with __float2half(0.0f) */
      for (int64_t k = 0; k < K; ++k) {
        const float a = oracle_h2f(A[i * K + k]);
        const float b = oracle_h2f(B[k * N + j]);
        const float cf = oracle_h2f(c);
        const float r = cf + a * b;
        c = oracle_f2h(r);
      }
      C[i * N + j] = c;
    }
  }
}

void oracle_ref_matmul_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N,
                            int64_t K, int64_t row0, int64_t row1, int nthreads) {
  (void)M;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t i = row0; i < row1; ++i) {
    for (int64_t j = 0; j < N; ++j) {
      uint16_t c = 0;
      for (int64_t k = 0; k < K; ++k) {
        /* T(a) * T(b) rounds to bf16, then C += rounds the sum to bf16 */
        const uint16_t p = oracle_f2bf(oracle_bf2f(A[i * K + k]) * oracle_bf2f(B[k * N + j]));
        c = oracle_f2bf(oracle_bf2f(c) + oracle_bf2f(p));
      }
      C[i * N + j] = c;
    }
  }
}

void oracle_ref_matmul_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                           int64_t row0, int64_t row1, int nthreads) {
  (void)M;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t i = row0; i < row1; ++i) {
    for (int64_t j = 0; j < N; ++j) {
      float c = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        const float p = A[i * K + k] * B[k * N + j];
        c = c + p;
      }
      C[i * N + j] = c;
    }
  }
}

/* relu: max(x, 0) through float for half (choreo-ir.hpp:209-217). */
void oracle_ref_relu_f16(const uint16_t* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float x = oracle_h2f(in[i]);
    out[i] = oracle_f2h(x < 0.0f ? 0.0f : x); /* std::max(x, 0.0f) */
  }
}
void oracle_ref_relu_f32(const float* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = in[i] < 0.0f ? 0.0f : in[i];
}
/* operator+: through float for half (choreo-ir.hpp:179-187). */
void oracle_ref_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f2h(oracle_h2f(a[i]) + oracle_h2f(b[i]));
}
void oracle_ref_add_f32(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* conv2d_kernel's loop (gemm_example.cu:230-247) with T = half: for each
 * output element, sum over c, then r, then s of in*w, product and running sum
 * each rounded to fp16; zero padding skips out-of-image taps. Storage here is
 * NHWC input, KRSC weight, NHWC output. Output pixels [pix0, pix1). */
void oracle_ref_conv2d_f16(const uint16_t* x, const uint16_t* w, uint16_t* out, int64_t N, int64_t H,
                           int64_t W, int64_t C, int64_t K, int64_t R, int64_t S, int stride_h,
                           int stride_w, int pad_h, int pad_w, int64_t pix0, int64_t pix1, int nthreads) {
  const int64_t P = (H + 2 * pad_h - R) / stride_h + 1;
  const int64_t Q = (W + 2 * pad_w - S) / stride_w + 1;
  (void)N;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t pix = pix0; pix < pix1; ++pix) {
    const int64_t n = pix / (P * Q);
    const int64_t p = (pix / Q) % P;
    const int64_t q = pix % Q;
    for (int64_t k = 0; k < K; ++k) {
      uint16_t sum = 0;
      for (int64_t c = 0; c < C; ++c)
        for (int64_t r = 0; r < R; ++r)
          for (int64_t s = 0; s < S; ++s) {
            const int64_t hi = p * stride_h - pad_h + r;
            const int64_t wi = q * stride_w - pad_w + s;
            if (hi >= 0 && hi < H && wi >= 0 && wi < W) {
              const uint16_t prod =
                  oracle_f2h(oracle_h2f(x[((n * H + hi) * W + wi) * C + c]) * oracle_h2f(w[((k * R + r) * S + s) * C + c]));
              sum = oracle_f2h(oracle_h2f(sum) + oracle_h2f(prod));
            }
          }
      out[pix * K + k] = sum;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* 2. fp64 checkers.                                                          */

enum { DT_F16 = 8, DT_F32 = 9, DT_BF16 = 11 };

static inline double load_elem(int dt, const void* p, int64_t i) {
  if (dt == DT_F32) return (double)((const float*)p)[i];
  if (dt == DT_BF16) return (double)oracle_bf2f(((const uint16_t*)p)[i]);
  return (double)oracle_h2f(((const uint16_t*)p)[i]);
}

/* out[r][j] = act(alpha * sum_k op(A)[rows[r], k] * op(B)[k, j]
 *                 + beta * C0[rows[r] * ldc0 + j] + bias[j])
 * for the listed rows, all N columns. op(A) = A (M x K, ld lda) or, with
 * trans_a, A stored K x M; op(B) = B (K x N) or, with trans_b, B stored N x K.
 * C0 (may be NULL) and bias (may be NULL) in their own dtypes. */
void oracle_gemm_f64(int dt_ab, const void* A, int64_t lda, int trans_a, const void* B, int64_t ldb,
                     int trans_b, int64_t M, int64_t N, int64_t K, double alpha, double beta, int dt_c0,
                     const void* C0, int64_t ldc0, int dt_bias, const void* bias, int relu,
                     const int64_t* rows, int64_t nrows, double* out, int nthreads) {
  (void)M;
  /* B as float, N x K (k contiguous): exact for f16/bf16/f32 values. */
  float* Bt = (float*)malloc(sizeof(float) * (size_t)N * (size_t)K);
  if (!Bt) return;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t j = 0; j < N; ++j)
    for (int64_t k = 0; k < K; ++k)
      Bt[j * K + k] = (float)load_elem(dt_ab, B, trans_b ? j * ldb + k : k * ldb + j);
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    double* arow = (double*)malloc(sizeof(double) * (size_t)K);
#pragma omp for schedule(dynamic, 1)
    for (int64_t r = 0; r < nrows; ++r) {
      const int64_t i = rows[r];
      for (int64_t k = 0; k < K; ++k) arow[k] = load_elem(dt_ab, A, trans_a ? k * lda + i : i * lda + k);
      for (int64_t j = 0; j < N; ++j) {
        const float* bj = Bt + j * K;
        double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        int64_t k = 0;
        for (; k + 4 <= K; k += 4) {
          s0 += arow[k] * bj[k];
          s1 += arow[k + 1] * bj[k + 1];
          s2 += arow[k + 2] * bj[k + 2];
          s3 += arow[k + 3] * bj[k + 3];
        }
        for (; k < K; ++k) s0 += arow[k] * bj[k];
        double v = alpha * ((s0 + s1) + (s2 + s3));
        if (C0) v += beta * load_elem(dt_c0, C0, i * ldc0 + j);
        if (bias) v += load_elem(dt_bias, bias, j);
        if (relu && v < 0) v = 0;
        out[r * N + j] = v;
      }
    }
    free(arow);
  }
  free(Bt);
}

/* out[r][k] for the listed output pixels (n*P*Q + p*Q + q), all K channels:
 * act(alpha * sum_{r,s,c} x[n, p*sh - ph + r*dh, q*sw - pw + s*dw, c]
 *                         * w[k, r, s, c] + bias[k]), zero outside the image. */
void oracle_conv2d_f64(int dt, const void* x, const void* w, int64_t N, int64_t H, int64_t W,
                       int64_t C, int64_t K, int64_t R, int64_t S, int stride_h, int stride_w,
                       int pad_h, int pad_w, int dil_h, int dil_w, double alpha, int dt_bias,
                       const void* bias, int relu, const int64_t* pixels, int64_t npix, double* out,
                       int nthreads) {
  const int64_t P = (H + 2 * pad_h - dil_h * (R - 1) - 1) / stride_h + 1;
  const int64_t Q = (W + 2 * pad_w - dil_w * (S - 1) - 1) / stride_w + 1;
  (void)N;
  float* wf = (float*)malloc(sizeof(float) * (size_t)(K * R * S * C));
  if (!wf) return;
  for (int64_t i = 0; i < K * R * S * C; ++i) wf[i] = (float)load_elem(dt, w, i);
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    double* patch = (double*)malloc(sizeof(double) * (size_t)(R * S * C));
#pragma omp for schedule(dynamic, 1)
    for (int64_t t = 0; t < npix; ++t) {
      const int64_t pix = pixels[t];
      const int64_t n = pix / (P * Q);
      const int64_t p = (pix / Q) % P;
      const int64_t q = pix % Q;
      for (int64_t r = 0; r < R; ++r)
        for (int64_t s = 0; s < S; ++s) {
          const int64_t hi = p * stride_h - pad_h + r * dil_h;
          const int64_t wi = q * stride_w - pad_w + s * dil_w;
          const int inside = hi >= 0 && hi < H && wi >= 0 && wi < W;
          for (int64_t c = 0; c < C; ++c)
            patch[(r * S + s) * C + c] = inside ? load_elem(dt, x, ((n * H + hi) * W + wi) * C + c) : 0.0;
        }
      for (int64_t k = 0; k < K; ++k) {
        const float* wk = wf + k * R * S * C;
        double acc = 0;
        for (int64_t i = 0; i < R * S * C; ++i) acc += patch[i] * wk[i];
        double v = alpha * acc;
        if (bias) v += load_elem(dt_bias, bias, k);
        if (relu && v < 0) v = 0;
        out[t * K + k] = v;
      }
    }
    free(patch);
  }
  free(wf);
}
