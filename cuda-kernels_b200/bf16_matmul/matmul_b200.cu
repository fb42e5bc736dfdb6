// matmul_b200.cu — the B200 GEMM as a reference-style MatmulFn launcher.
//
// The reference's profiling flow builds `<name>.cu` together with its
// profile_entry.cpp and calls the C++ function named after the file's
// basename (scripts/profile.sh:95-123, bf16_matmul/profile_entry.cpp:16-20),
// with the signature
//     void(const nv_bfloat16* A, const nv_bfloat16* B, nv_bfloat16* C, int M, int N, int K)
// (bf16_matmul/profile_entry.cpp:9-14, bf16_matmul/matmul.cpp:5-10).
//
// This file compiles the library sources into the same translation unit, so
// with this file placed beside the reference's profile_entry.cpp,
//   CUDA_ARCH=sm_100a EXTRA_NVCC_FLAGS="-I<repo>/include -I<repo>/cuda-kernels_b200/csrc" \
//   EXTRA_NCU_ARGS="--clock-control none" scripts/profile.sh bf16_matmul/matmul_b200.cu
// builds and links it; the tensor-map encoder is fetched through the runtime,
// so no -lcuda is needed.
//
// Semantics match the reference launchers: A [M,K] row-major, B [N,K] row-major
// (C = A * B^T), C [M,N] row-major, legacy default stream, asynchronous.  Where
// the reference would host-assert (matmul_v8_tuned.cu:238) this accepts any
// shape; on an argument error it prints the reason to stderr.  The MatmulFn
// signature returns nothing, so a device-side wait that gave up (the library's
// status word) is reported on stderr when the process exits.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include <cuda_bf16.h>

#include "b200_gemm.cu"  // cuda-kernels_b200/csrc/ (pass -I to it and to include/)

namespace {
void report_device_status() {
  uint32_t bits = 0;
  const int rc = b200_gemm_status(nullptr, &bits);
  if (rc != B200_OK) std::fprintf(stderr, "matmul_b200: device status %s (bits 0x%x)\n", b200_gemm_strerror(rc), bits);
}
std::once_flag g_atexit_once;
}  // namespace

void matmul_b200(const nv_bfloat16* A, const nv_bfloat16* B, nv_bfloat16* C, int M, int N, int K) {
  // Registered after the CUDA runtime has initialised, so it runs before the
  // runtime's own teardown at exit.
  std::call_once(g_atexit_once, [] { std::atexit(report_device_status); });
  const int rc = b200_gemm_bf16(A, B, C, M, N, K, K, K, N, B200_B_NK, nullptr);
  if (rc != B200_OK) std::fprintf(stderr, "matmul_b200: %s\n", b200_gemm_strerror(rc));
}
