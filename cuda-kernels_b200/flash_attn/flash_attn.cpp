// Torch-extension binding of the B200 flash attention forward, shaped like the
// reference's flash_attn/flash_attn.cpp: `flash_attn<fn>(Q, K, V)` allocates O
// like Q and runs the kernel (flash_attn.cpp:16-26), registered as
// `fa2_tma_lazy_rescale` (flash_attn.cpp:28-30).
//
// Q is [batch, seq, heads, 128] bf16, K and V [batch, seq, kv_heads, 128] with
// heads a multiple of kv_heads (grouped-query attention).  The reference's
// operator is always causal; `flash_attn_b200` takes `causal` as an argument
// (default true) and `fa2_tma_lazy_rescale` is the causal form under the
// reference's name.  Differences from the reference binding, all deliberate:
//   * inputs whose last dimension is contiguous but whose other strides are
//     not those of a packed tensor are packed first (the reference's 4-D
//     tensor maps take the strides; the C ABI takes packed tensors);
//   * dtype, device, rank and shapes are checked, errors raise.
// The attention is computed by the C ABI entry point b200_flash_attn_bf16
// (include/b200_gemm.h).  Errors are standard C++ exceptions (pybind11 turns
// them into ValueError / RuntimeError); TORCH_CHECK is not used, as in the
// GEMM binding.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>

#include "b200_gemm.h"

namespace {

[[noreturn]] void bad_arg(const std::string& msg) { throw std::invalid_argument(msg); }

torch::Tensor attention(torch::Tensor Q, torch::Tensor K, torch::Tensor V, bool causal) {
  for (const auto* t : {&Q, &K, &V}) {
    if (t->dim() != 4) bad_arg("Q, K and V must be 4-D [batch, seq_len, heads, head_dim]");
    if (t->scalar_type() != torch::kBFloat16) bad_arg("Q, K and V must be bfloat16");
    if (!t->is_cuda()) bad_arg("Q, K and V must be CUDA tensors");
  }
  if (K.device() != Q.device() || V.device() != Q.device()) bad_arg("Q, K and V must be on the same device");
  const int64_t batch = Q.size(0), seq_len = Q.size(1), heads = Q.size(2), head_dim = Q.size(3);
  const int64_t kv_heads = K.size(2);
  if (K.size(0) != batch || K.size(1) != seq_len || K.size(3) != head_dim || !K.sizes().equals(V.sizes()))
    bad_arg("K and V must be [batch, seq_len, kv_heads, head_dim] with Q's batch, seq_len and head_dim");
  if (head_dim != 128) bad_arg("head_dim must be 128, got " + std::to_string(head_dim));
  if ((kv_heads == 0 && heads != 0) || (kv_heads != 0 && heads % kv_heads != 0))
    bad_arg("heads (" + std::to_string(heads) + ") must be a multiple of kv_heads (" + std::to_string(kv_heads) +
            ")");
  const c10::cuda::CUDAGuard guard(Q.device());
  const auto q = Q.contiguous(), k = K.contiguous(), v = V.contiguous();
  auto O = torch::empty({batch, seq_len, heads, head_dim}, Q.options());
  const int rc = b200_flash_attn_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), O.data_ptr(), batch, seq_len, heads,
                                      kv_heads, head_dim, causal ? 1 : 0,
                                      at::cuda::getCurrentCUDAStream(Q.device().index()).stream());
  if (rc != B200_OK) throw std::runtime_error(std::string("b200_flash_attn_bf16 failed: ") + b200_gemm_strerror(rc));
  return O;
}

torch::Tensor fa2_tma_lazy_rescale(torch::Tensor Q, torch::Tensor K, torch::Tensor V) {
  return attention(Q, K, V, true);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("flash_attn_b200", &attention, "B200 tcgen05 flash attention forward, O = softmax(Q K^T / sqrt(D)) V",
        pybind11::arg("Q"), pybind11::arg("K"), pybind11::arg("V"), pybind11::arg("causal") = true);
  m.def("fa2_tma_lazy_rescale", &fa2_tma_lazy_rescale,
        "Causal flash attention forward under the reference operator's name (B200 tcgen05 kernel)");
}
