// Torch-extension binding of the B200 GEMM, shaped like the reference's
// bf16_matmul/matmul.cpp (the `matmul<fn>(A, B)` template, matmul.cpp:24-42,
// registered per kernel in PYBIND11_MODULE, matmul.cpp:44-56).
//
// Differences from the reference binding, all deliberate:
//   * N comes from B.size(0) for the reference's [N,K] B (the reference reads
//     B.size(1), matmul.cpp:29, which is K; only square shapes worked);
//   * dtype, device, rank and row-major layout are checked instead of assumed;
//   * the kernel runs on torch's current CUDA stream, not the legacy stream;
//   * launch errors raise instead of being ignored.
// The product is computed by the C ABI entry point b200_gemm_bf16
// (include/b200_gemm.h); this file only adapts torch tensors to it.
//
// Errors are raised as standard C++ exceptions, which pybind11 turns into
// Python ValueError (std::invalid_argument) and RuntimeError
// (std::runtime_error).  TORCH_CHECK is not used: with the torch 2.11 build in
// this image, a TORCH_CHECK whose message contains an integer crashes the
// process inside an extension module instead of raising.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>

#include "b200_gemm.h"

namespace {

[[noreturn]] void bad_arg(const std::string& msg) { throw std::invalid_argument(msg); }

void check_operand(const torch::Tensor& t, const char* name) {
  if (t.scalar_type() != torch::kBFloat16) bad_arg(std::string(name) + " must be bfloat16");
  if (!t.is_cuda()) bad_arg(std::string(name) + " must be a CUDA tensor");
  if (t.dim() != 2) bad_arg(std::string(name) + " must be 2-D");
  if (t.numel() != 0 && t.stride(1) != 1) bad_arg(std::string(name) + " must be row-major");
}

torch::Tensor run(const torch::Tensor& A, const torch::Tensor& B, int b_layout) {
  check_operand(A, "A");
  check_operand(B, "B");
  if (A.device() != B.device()) bad_arg("A and B must be on the same device");
  const int64_t M = A.size(0);
  const int64_t K = A.size(1);
  const int64_t N = (b_layout == B200_B_NK) ? B.size(0) : B.size(1);
  const int64_t Kb = (b_layout == B200_B_NK) ? B.size(1) : B.size(0);
  if (Kb != K)
    bad_arg("inner dimensions differ: A is [" + std::to_string(M) + "," + std::to_string(K) + "], B gives K=" +
            std::to_string(Kb));
  const c10::cuda::CUDAGuard guard(A.device());
  auto C = torch::empty({M, N}, A.options());
  // Sequential-K product (no split-K tail), so results match the reference
  // kernels' and cuBLAS's summation order, as the reference's own check
  // (assert_close against torch.matmul, bf16_matmul/main.py:44-54) expects.
  const int rc = b200_gemm_bf16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, std::max<int64_t>(A.stride(0), 1),
                                std::max<int64_t>(B.stride(0), 1), std::max<int64_t>(C.stride(0), 1), b_layout,
                                at::cuda::getCurrentCUDAStream(A.device().index()).stream());
  if (rc != B200_OK) throw std::runtime_error(std::string("b200_gemm_bf16 failed: ") + b200_gemm_strerror(rc));
  return C;
}

// Reference semantics: B is [N,K] ("column-major B"), C = A @ B^T.
torch::Tensor matmul_b200(torch::Tensor A, torch::Tensor B) { return run(A, B, B200_B_NK); }

// B stored [K,N] row-major, C = A @ B.
torch::Tensor matmul_b200_kn(torch::Tensor A, torch::Tensor B) { return run(A, B, B200_B_KN); }

// The reference's fp32 operator (fp32_matmul/matmul.cpp:20-33): A [M,K] and
// B [K,N] fp32 row-major, C = A @ B fp32 (N from B.size(1), as there).
torch::Tensor matmul_b200_f32(torch::Tensor A, torch::Tensor B) {
  for (const auto* t : {&A, &B}) {
    if (t->scalar_type() != torch::kFloat32) bad_arg("A and B must be float32");
    if (!t->is_cuda()) bad_arg("A and B must be CUDA tensors");
    if (t->dim() != 2) bad_arg("A and B must be 2-D");
    if (t->numel() != 0 && t->stride(1) != 1) bad_arg("A and B must be row-major");
  }
  if (A.device() != B.device()) bad_arg("A and B must be on the same device");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(1);
  if (B.size(0) != K) bad_arg("inner dimensions differ");
  const c10::cuda::CUDAGuard guard(A.device());
  // C is written by TMA, whose row pitch must be a multiple of 4 floats.
  const int64_t ldc = (N + 3) / 4 * 4;
  auto Cbuf = torch::empty({M, ldc}, A.options());
  auto C = Cbuf.narrow(1, 0, N);
  size_t ws_bytes = 0;
  int rc = b200_gemm_f32_workspace_bytes(M, N, K, B200_B_KN, &ws_bytes);
  if (rc != B200_OK) throw std::runtime_error(std::string("b200_gemm_f32 failed: ") + b200_gemm_strerror(rc));
  auto ws = torch::empty({(int64_t)ws_bytes + 256}, A.options().dtype(torch::kUInt8));
  void* ws_ptr = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~uintptr_t(255));
  rc = b200_gemm_f32(A.data_ptr<float>(), B.data_ptr<float>(), C.data_ptr<float>(), M, N, K,
                     std::max<int64_t>(A.stride(0), 1), std::max<int64_t>(B.stride(0), 1),
                     ldc, B200_B_KN, ws_ptr, ws_bytes, at::cuda::getCurrentCUDAStream(A.device().index()).stream());
  if (rc != B200_OK) throw std::runtime_error(std::string("b200_gemm_f32 failed: ") + b200_gemm_strerror(rc));
  return ldc == N ? C : C.contiguous();
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("matmul_b200", &matmul_b200, "B200 tcgen05 BF16 matmul, B given [N,K] (C = A @ B^T)");
  m.def("matmul_b200_kn", &matmul_b200_kn, "B200 tcgen05 BF16 matmul, B given [K,N] (C = A @ B)");
  m.def("matmul_b200_f32", &matmul_b200_f32, "B200 FP32 matmul on the bf16 tensor cores (3-way split), C = A @ B");
}
