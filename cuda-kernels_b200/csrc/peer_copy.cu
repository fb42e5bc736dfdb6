// Copy engines and stream-ordered flags between GPUs (C ABI in
// include/b200_gemm.h): the primitives the multi-GPU driver uses to move B
// from rank to rank over NVLink while the GEMM of the previous step holds
// every SM.
//
// A collective kernel (NCCL) needs SMs, and a persistent GEMM occupies all of
// them, so a broadcast queued beside the GEMM only runs between GEMMs.  Here
// the data moves with cudaMemcpyAsync between this GPU's memory and a peer's
// buffer mapped through CUDA IPC (the copy engines, no SMs), and readiness is
// signalled with stream memory operations: a 32-bit flag written into the
// reader's memory after the copy in the writer's stream, and a stream that
// waits for the flag before the kernel that reads the data.  Neither runs on
// an SM.  The driver entry points are fetched through the runtime, so
// nothing links against libcuda.
//
// The reference has no multi-GPU code; these have no counterpart there.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "b200_gemm.h"

namespace {

std::once_flag g_memop_once;
PFN_cuStreamWriteValue32_v11070 g_write32 = nullptr;
PFN_cuStreamWaitValue32_v11070 g_wait32 = nullptr;

void load_memops() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion("cuStreamWriteValue32", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_write32 = reinterpret_cast<PFN_cuStreamWriteValue32_v11070>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuStreamWaitValue32", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_wait32 = reinterpret_cast<PFN_cuStreamWaitValue32_v11070>(fn);
}

bool memops_ready() {
  std::call_once(g_memop_once, load_memops);
  return g_write32 != nullptr && g_wait32 != nullptr;
}

inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

extern "C" B200_API int b200_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return B200_OK;
  if (dst == nullptr || src == nullptr) return B200_ERR_INVALID_ARG;
  if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_CUDA;
  }
  return B200_OK;
}

extern "C" B200_API int b200_signal_u32(void* flag, uint32_t value, void* stream) {
  if (flag == nullptr || !aligned4(flag)) return B200_ERR_INVALID_ARG;
  if (!memops_ready()) return B200_ERR_CUDA;
  // Default flags: the write is ordered after (and made visible after) all
  // earlier work in the stream, including copies into the flag owner's memory.
  const CUresult r = g_write32(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value,
                               CU_STREAM_WRITE_VALUE_DEFAULT);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_CUDA;
}

extern "C" B200_API int b200_wait_u32(const void* flag, uint32_t value, void* stream) {
  if (flag == nullptr || !aligned4(flag)) return B200_ERR_INVALID_ARG;
  if (!memops_ready()) return B200_ERR_CUDA;
  // Later work in the stream starts once (int32_t)(*flag - value) >= 0.
  const CUresult r = g_wait32(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(const_cast<void*>(flag)),
                              value, CU_STREAM_WAIT_VALUE_GEQ);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_CUDA;
}
