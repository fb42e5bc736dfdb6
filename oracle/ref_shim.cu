// ref_shim.cu — C entry point onto the reference's own best kernel.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified bf16_matmul/matmul_v8_tuned.cu (read in place
// from the reference checkout, never copied) into oracle/_ref/libref_v8_tuned.so
// for sm_100a.  Tests and tests/golden/make_golden.py call it to compare the
// new kernel and the CPU restatement with the reference itself.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

// The reference's host signature (bf16_matmul/matmul.cpp:5-10).
using MatmulFn = void(const nv_bfloat16* A, const nv_bfloat16* B, nv_bfloat16* C, int M, int N, int K);
MatmulFn matmul_v8_tuned;

// Returns 0 on success, 1 for shapes the reference rejects with a host assert
// (M % 128, N % 64, K % 64 must all be 0: bf16_matmul/matmul_v8_tuned.cu:238),
// 2 when the launch failed.  Runs on the legacy default stream, as the
// reference does (matmul_v8_tuned.cu:256).
extern "C" int ref_matmul_v8_tuned(const void* A, const void* B, void* C, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 != 0 || N % 64 != 0 || K % 64 != 0) return 1;
  matmul_v8_tuned(static_cast<const nv_bfloat16*>(A), static_cast<const nv_bfloat16*>(B),
                  static_cast<nv_bfloat16*>(C), M, N, K);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
