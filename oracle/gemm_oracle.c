/*
 * gemm_oracle.c — CPU restatement of the reference's BF16 GEMM arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline use it, as the checker.
 *
 * What it restates (typr7/CUDA-Kernels, bf16_matmul/):
 *   - operands: A [M,K] bf16 row-major, B [N,K] bf16 row-major ("column-major
 *     B", bf16_matmul/README.md:7; the kernels step B rows by K,
 *     bf16_matmul/matmul_v1.cu:64), plus the [K,N] row-major B of the
 *     BASELINE configuration;
 *   - accumulation: fp32 accumulators start at zero
 *     (bf16_matmul/matmul_v8_tuned.cu:78) and receive one K=16 partial sum per
 *     mma.sync.m16n8k16 (common.hpp:55-68), K-blocks taken in increasing order
 *     (matmul_v8_tuned.cu:98-143).  Here each 16-wide partial sum is formed in
 *     fp32 in increasing k and then added to the accumulator.  Products of
 *     two bf16 values are exact in fp32, so only the summation order can
 *     differ from the hardware's;
 *   - output: fp32 -> bf16 round-to-nearest-even (__float22bfloat162_rn,
 *     matmul_v8_tuned.cu:161-164).
 *
 * The fp32 -> bf16 rounding below is the standard bias-and-truncate
 * round-half-to-even on the IEEE-754 bit pattern.
 *
 * Pinning: tests/golden/ holds outputs of the reference's own matmul_v8_tuned
 * (compiled from its sources for sm_100a by oracle/Makefile and run on a
 * B200 by tests/golden/make_golden.py); tests/test_oracle.py checks this
 * restatement against them.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_MB 8   /* rows of A per task */
#define OR_NB 64  /* columns of C per task */
#define OR_KC 16  /* K per partial sum (the mma.sync K) */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)0x7fffu; /* NaN -> canonical quiet NaN */
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

void oracle_bf16_to_f32(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = bf16_to_f32(x[i]);
}

void oracle_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f32_to_bf16_rne(x[i]);
}

/* B (either layout) -> fp32 panel Bt[K][Np], Np = N rounded up to OR_NB, zero padded. */
static float* make_bt(const uint16_t* B, int64_t N, int64_t K, int64_t ldb, int b_layout, int64_t Np, int threads) {
  float* bt = (float*)calloc((size_t)K * (size_t)Np, sizeof(float));
  if (!bt) return NULL;
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t k = 0; k < K; ++k) {
    float* row = bt + k * Np;
    if (b_layout == 0) {
      for (int64_t n = 0; n < N; ++n) row[n] = bf16_to_f32(B[n * ldb + k]);
    } else {
      for (int64_t n = 0; n < N; ++n) row[n] = bf16_to_f32(B[k * ldb + n]);
    }
  }
  return bt;
}

static void block_f32acc(const uint16_t* A, const float* bt, float* C, int64_t m0, int64_t mrows, int64_t n0,
                         int64_t ncols, int64_t K, int64_t lda, int64_t ldc, int64_t Np) {
  float acc[OR_MB][OR_NB];
  memset(acc, 0, sizeof(acc));
  for (int64_t kc = 0; kc < K; kc += OR_KC) {
    const int64_t kn = (K - kc) < OR_KC ? (K - kc) : OR_KC;
    for (int64_t i = 0; i < mrows; ++i) {
      const uint16_t* arow = A + (m0 + i) * lda + kc;
      float part[OR_NB];
      for (int j = 0; j < OR_NB; ++j) part[j] = 0.0f;
      for (int64_t kk = 0; kk < kn; ++kk) {
        const float av = bf16_to_f32(arow[kk]);
        const float* brow = bt + (kc + kk) * Np + n0;
        for (int j = 0; j < OR_NB; ++j) part[j] += av * brow[j];
      }
      for (int j = 0; j < OR_NB; ++j) acc[i][j] += part[j];
    }
  }
  for (int64_t i = 0; i < mrows; ++i)
    for (int64_t j = 0; j < ncols; ++j) C[(m0 + i) * ldc + n0 + j] = acc[i][j];
}

/*
 * C32[M,N] (fp32, pitch ldc) = A[M,K] * op(B) with fp32 accumulation in K=16
 * partial sums.  b_layout 0: B is [N,K] (pitch ldb); 1: B is [K,N] (pitch ldb).
 * threads <= 0 uses every available thread.  Returns 0, or -1 on bad input /
 * allocation failure.
 */
int oracle_gemm_bf16_f32acc(const uint16_t* A, const uint16_t* B, float* C, int64_t M, int64_t N, int64_t K,
                            int64_t lda, int64_t ldb, int64_t ldc, int b_layout, int threads) {
  if (M < 0 || N < 0 || K < 0 || (b_layout != 0 && b_layout != 1)) return -1;
  if (M == 0 || N == 0) return 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#else
  threads = 1;
#endif
  if (K == 0) {
    for (int64_t m = 0; m < M; ++m)
      for (int64_t n = 0; n < N; ++n) C[m * ldc + n] = 0.0f;
    return 0;
  }
  const int64_t Np = (N + OR_NB - 1) / OR_NB * OR_NB;
  float* bt = make_bt(B, N, K, ldb, b_layout, Np, threads);
  if (!bt) return -1;
  const int64_t mblocks = (M + OR_MB - 1) / OR_MB;
  const int64_t nblocks = Np / OR_NB;
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads)
  for (int64_t t = 0; t < mblocks * nblocks; ++t) {
    const int64_t mb = t / nblocks, nb = t % nblocks;
    const int64_t m0 = mb * OR_MB, n0 = nb * OR_NB;
    const int64_t mrows = (M - m0) < OR_MB ? (M - m0) : OR_MB;
    const int64_t ncols = (N - n0) < OR_NB ? (N - n0) : OR_NB;
    block_f32acc(A, bt, C, m0, mrows, n0, ncols, K, lda, ldc, Np);
  }
  free(bt);
  return 0;
}

/* Same product rounded to bf16 (round-to-nearest-even), C pitch ldc. */
int oracle_gemm_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                     int64_t ldb, int64_t ldc, int b_layout, int threads) {
  if (M <= 0 || N <= 0) return (M < 0 || N < 0) ? -1 : 0;
  float* c32 = (float*)malloc((size_t)M * (size_t)N * sizeof(float));
  if (!c32) return -1;
  int rc = oracle_gemm_bf16_f32acc(A, B, c32, M, N, K, lda, ldb, N, b_layout, threads);
  if (rc == 0) {
    for (int64_t m = 0; m < M; ++m)
      for (int64_t n = 0; n < N; ++n) C[m * ldc + n] = f32_to_bf16_rne(c32[m * N + n]);
  }
  free(c32);
  return rc;
}

/*
 * Near-exact product in fp64 (every bf16 product is exact in fp64; only the
 * fp64 summation rounds).  Used by the tests as the "true" value when
 * measuring ulp errors.  Also writes sum_k |a*b| to `absC` (may be NULL),
 * the scale of the worst-case accumulation error.
 */
int oracle_gemm_bf16_f64(const uint16_t* A, const uint16_t* B, double* C, double* absC, int64_t M, int64_t N,
                         int64_t K, int64_t lda, int64_t ldb, int b_layout, int threads) {
  if (M < 0 || N < 0 || K < 0 || (b_layout != 0 && b_layout != 1)) return -1;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#else
  threads = 1;
#endif
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double s = 0.0, sa = 0.0;
      for (int64_t k = 0; k < K; ++k) {
        const double a = (double)bf16_to_f32(A[m * lda + k]);
        const double b = (double)bf16_to_f32(b_layout == 0 ? B[n * ldb + k] : B[k * ldb + n]);
        s += a * b;
        sa += fabs(a * b);
      }
      C[m * N + n] = s;
      if (absC) absC[m * N + n] = sa;
    }
  }
  return 0;
}

/*
 * FP32 GEMM of the reference's fp32_matmul/ operator: A [M,K] fp32 row-major
 * times B fp32, row-major [K,N] (fp32_matmul/README.md:8, b_layout 1) or
 * [N,K] (b_layout 0), C fp32.  Restates the reference's plain kernel
 * (fp32_matmul/matmul.cu:18-36): one fp32 accumulator per output starting at
 * zero, k in increasing order, acc += a * b — which nvcc contracts to a fused
 * multiply-add, restated here with fmaf.
 */
int oracle_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                    int64_t ldb, int b_layout, int threads) {
  if (M < 0 || N < 0 || K < 0 || (b_layout != 0 && b_layout != 1)) return -1;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#else
  threads = 1;
#endif
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        acc = fmaf(A[m * lda + k], b_layout == 0 ? B[n * ldb + k] : B[k * ldb + n], acc);
      }
      C[m * N + n] = acc;
    }
  }
  return 0;
}

/* Near-exact fp64 product of fp32 operands (and sum_k |a*b|), for error bounds. */
int oracle_gemm_f32_f64(const float* A, const float* B, double* C, double* absC, int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb, int b_layout, int threads) {
  if (M < 0 || N < 0 || K < 0 || (b_layout != 0 && b_layout != 1)) return -1;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#else
  threads = 1;
#endif
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double s = 0.0, sa = 0.0;
      for (int64_t k = 0; k < K; ++k) {
        const double p = (double)A[m * lda + k] * (double)(b_layout == 0 ? B[n * ldb + k] : B[k * ldb + n]);
        s += p;
        sa += fabs(p);
      }
      C[m * N + n] = s;
      if (absC) absC[m * N + n] = sa;
    }
  }
  return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
