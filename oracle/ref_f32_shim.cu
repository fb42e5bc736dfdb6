// ref_f32_shim.cu — C entry points onto the reference's fp32 kernels.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified fp32_matmul/matmul.cu (read in place from the
// reference checkout, never copied) into oracle/_ref/libref_f32.so for
// sm_100a.  tests/golden/make_golden_f32.py and tests/ call it to pin the fp32
// CPU restatement (oracle_gemm_f32) to the reference itself.
#include <cuda_runtime.h>

// The reference's host signature (fp32_matmul/matmul.cpp:3-8).
using MatmulFn = void(const float* A, const float* B, float* C, int M, int N, int K);
MatmulFn matmul_v1;
MatmulFn matmul_v5;

// v1, one thread per output with a bounds check (fp32_matmul/matmul.cu:18-36,
// host launcher :342-355): any shape.  Returns 0 on success, 2 when the
// launch failed.  Runs on the legacy default stream, as the reference does.
extern "C" int ref_matmul_f32_v1(const void* A, const void* B, void* C, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 1;
  matmul_v1(static_cast<const float*>(A), static_cast<const float*>(B), static_cast<float*>(C), M, N, K);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// v5, the reference's best fp32 kernel (fp32_matmul/matmul.cu:231-325,
// launcher :405-431); its tiles (128 x 128 x 32) have no edge handling, so
// only whole-tile shapes are accepted (1 otherwise).
extern "C" int ref_matmul_f32_v5(const void* A, const void* B, void* C, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 != 0 || N % 128 != 0 || K % 32 != 0) return 1;
  matmul_v5(static_cast<const float*>(A), static_cast<const float*>(B), static_cast<float*>(C), M, N, K);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
