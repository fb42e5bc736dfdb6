/*
 * b200_gemm.h — C ABI of the B200 (sm_100a) BF16 GEMM.
 *
 * Drop-in boundary for the reference's `bf16_matmul` operator.  The reference
 * exposes one C++ host signature per kernel,
 *
 *     using MatmulFn = void(const nv_bfloat16* A, const nv_bfloat16* B,
 *                           nv_bfloat16* C, int M, int N, int K);
 *
 * (bf16_matmul/matmul.cpp:5-10, bf16_matmul/profile_entry.cpp:9-14,
 * bf16_matmul/common.hpp:169-174), implemented by e.g. `matmul_v8_tuned`
 * (bf16_matmul/matmul_v8_tuned.cu:215-257), and bound to Python by the
 * template `matmul<fn>` (bf16_matmul/matmul.cpp:24-42).  Those launchers take
 * raw device pointers, run on the legacy default stream, return nothing and
 * assert on unsupported shapes.
 *
 * This header replaces that surface with a plain C ABI: raw pointers, 64-bit
 * sizes, an explicit stream, and an integer status instead of a host assert.
 * No GEMM entry point allocates device memory (scratch comes from the
 * caller's workspace or, for b200_gemm_bf16_noalloc, a static buffer); only
 * b200_ipc_alloc, whose job it is, does.  No call throws or exits the process.
 *
 * All functions are thread-safe.  Device memory passed in must belong to the
 * device that is current on the calling thread.
 */
#ifndef B200_GEMM_H_
#define B200_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define B200_OK 0
#define B200_ERR_INVALID_ARG 1       /* null pointer, negative size, bad layout, ld too small */
#define B200_ERR_ALIGNMENT 2         /* pointer not 16-byte aligned or row pitch not a multiple of 8 elements */
#define B200_ERR_UNSUPPORTED_DEVICE 3 /* current device is not compute capability 10.0 (sm_100a) */
#define B200_ERR_CUDA 4              /* a CUDA runtime call (launch, attribute, entry point) failed */
#define B200_ERR_TENSOR_MAP 5        /* cuTensorMapEncodeTiled rejected a descriptor */
#define B200_ERR_DEVICE_TIMEOUT 6    /* a kernel wait hit its time limit (see b200_gemm_status) */
#define B200_ERR_TOO_LARGE 7         /* a dimension exceeds 2^31-1 */
#define B200_ERR_SCRATCH_LIMIT 8     /* b200_gemm_bf16_noalloc: split-K scratch beyond its 16 MiB static buffer */

/* Layout of the B operand. */
#define B200_B_NK 0 /* B stored [N,K] row-major (K contiguous): C = A * B^T.  The reference's layout. */
#define B200_B_KN 1 /* B stored [K,N] row-major (N contiguous): C = A * B. */

/*
 * C[M,N] = A[M,K] * op(B), bf16 inputs, fp32 accumulation, bf16 output
 * rounded to nearest-even.
 *
 *   A       device pointer, bf16, row-major [M, lda >= K]
 *   B       device pointer, bf16, [N, ldb >= K] if b_layout == B200_B_NK,
 *                                 [K, ldb >= N] if b_layout == B200_B_KN
 *   C       device pointer, bf16, row-major [M, ldc >= N]; fully overwritten
 *   M,N,K   any values >= 0 (M==0 or N==0: no-op; K==0: C is zero-filled)
 *   lda/ldb/ldc  row pitches in elements, multiples of 8 (TMA needs 16-byte pitches)
 *   stream  cudaStream_t to run on (NULL = legacy default stream)
 *
 * Asynchronous: returns after the launch.  Launch-time problems are returned
 * directly; a device-side wait that times out is reported by
 * b200_gemm_status().
 *
 * Replaces: matmul_v8_tuned (bf16_matmul/matmul_v8_tuned.cu:215-257) called
 * through MatmulFn (bf16_matmul/matmul.cpp:5-10); with b_layout = B200_B_NK,
 * lda = ldb = K, ldc = N and the default stream it computes the same product.
 */
B200_API int b200_gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                   int64_t ldb, int64_t ldc, int b_layout, void* stream);

/*
 * Same product as b200_gemm_bf16, with a caller-provided device workspace.
 * When the tiles of a problem do not fill the last wave of the GPU's CTA
 * pairs, the tiles of that wave are split along K across several pairs; the
 * partial sums meet in `workspace` (fp32 partial tiles plus hand-off flags).
 * Needs workspace_bytes >= b200_gemm_workspace_bytes(...) and a 256-byte
 * aligned pointer; with less (or NULL, 0) it runs without the split, exactly
 * like b200_gemm_bf16.  The workspace needs no initialisation; calls that may
 * run at the same time on the GPU must not share a workspace.  Results are
 * deterministic (partials are added in a fixed order) and within the bf16
 * tolerance of the exact product, but split tiles sum K in a different order
 * than b200_gemm_bf16, cuBLAS or the reference kernels, so near-zero outputs
 * (cancellation) can differ from theirs in the last bits.  b200_gemm_bf16 is
 * the sequential-K default.
 * No reference counterpart: the reference launches one CTA per tile
 * (bf16_matmul/matmul_v8_tuned.cu:255-256) and has no tail handling.
 */
B200_API int b200_gemm_bf16_ws(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                               int64_t ldb, int64_t ldc, int b_layout, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Row-sharded GEMM with the C all-gather fused in.  This rank computes rows
 * [row0, row0 + M_local) of C = A op(B) (A_local holds exactly those rows)
 * and its epilogue stores every C tile into each of the num_outputs
 * gathered-C buffers: outputs[r] is rank r's [M_total, ldc] bf16 C, mapped in
 * this process (this rank's own buffer, and the peers' opened with
 * b200_ipc_open).  Tiles leave over NVLink while later tiles are computed,
 * so no separate all-gather pass over C is needed.  When every rank's
 * kernel has completed (e.g. after a collective on the same stream), every
 * buffer holds all M_total rows.  num_outputs <= 8, K >= 1; no fused
 * epilogue, sequential K.  No reference counterpart: the reference has no
 * multi-GPU path; this replaces GEMM + NCCL all-gather of C in the sharded
 * driver.
 */
B200_API int b200_gemm_bf16_allgather(const void* A_local, const void* B, void* const* outputs, int num_outputs,
                                      int64_t M_local, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                                      int64_t row0, int64_t M_total, int b_layout, void* stream);

/*
 * CUDA IPC helpers for the gathering GEMM's buffers (one process per GPU).
 * b200_ipc_alloc: cudaMalloc `bytes` on the current device and write its
 * B200_IPC_HANDLE_BYTES-byte handle; b200_ipc_open: map a peer's buffer from
 * its handle into this process (peer access enabled); b200_ipc_close /
 * b200_ipc_free undo them.  No reference counterpart.
 */
#define B200_IPC_HANDLE_BYTES 64
B200_API int b200_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
B200_API int b200_ipc_free(void* dev_ptr);
B200_API int b200_ipc_open(const void* handle, void** dev_ptr);
B200_API int b200_ipc_close(void* dev_ptr);

/*
 * Copy engines and stream-ordered flags between GPUs, for moving data from
 * rank to rank over NVLink while a GEMM occupies every SM (a collective
 * kernel would wait for SMs; these use none).  Peer buffers are mapped with
 * b200_ipc_open; all calls are asynchronous on `stream`.
 *   b200_copy_async  cudaMemcpyAsync of `bytes` device to device (either side
 *                    may be a peer's mapped buffer): the copy engines.
 *   b200_signal_u32  once all earlier work of `stream` is complete and
 *                    visible, write `value` to the 4-byte-aligned `flag`
 *                    (local or a peer's mapped memory).
 *   b200_wait_u32    later work of `stream` starts once
 *                    (int32_t)(*flag - value) >= 0 (wrap-aware "flag has
 *                    reached value"; flags count up by step).
 * A wait is a stream operation, not a kernel: if its flag is never written
 * (a peer that stopped), the stream stays blocked until the process exits.
 * No reference counterpart: the reference has no multi-GPU code.
 */
B200_API int b200_copy_async(void* dst, const void* src, size_t bytes, void* stream);
B200_API int b200_signal_u32(void* flag, uint32_t value, void* stream);
B200_API int b200_wait_u32(const void* flag, uint32_t value, void* stream);

/*
 * Per-step broadcast of one buffer from rank 0 to every rank, built on the
 * three calls above (the multi-GPU driver's B exchange; one process per GPU,
 * world <= 8).  Every rank owns B200_BCAST_SLOTS receive slots of `nbytes`
 * (step s uses slot s % B200_BCAST_SLOTS, so up to two steps can be in flight
 * ahead of the one being read) and a flag array of
 * b200_bcast_flag_bytes(world) bytes, zeroed
 * before first use; all of them are mapped in every process (b200_ipc_*).
 * Rank 0 sends piece q-1 (b200_bcast_piece: world-1 pieces, 256-byte
 * aligned) to rank q, and rank q forwards its piece to the other receiving
 * ranks once it has landed, so every byte leaves rank 0 once.
 *   b200_bcast_create   slots[r * B200_BCAST_SLOTS + k] = rank r's slot k and flags[r] =
 *                       rank r's flags, as mapped in this process.
 *   b200_bcast_issue    queue step `step`'s copies on `stream` (rank 0 from
 *                       `src`; the others forward); every rank calls it.
 *   b200_bcast_wait     `stream` waits until this rank's slot of `step` is
 *                       complete (no-op on rank 0, which reads src).
 *   b200_bcast_release  after the work on `stream` that reads the slot of
 *                       `step`: its writers may overwrite it B200_BCAST_SLOTS
 *                       steps on.
 * Steps count up from 0 on every rank, each call made by every rank in the
 * same order.  No SMs are used.  A rank that stops calling leaves the
 * others' streams waiting (no time limit, see b200_wait_u32).
 * No reference counterpart: the reference has no multi-GPU code.
 */
#define B200_BCAST_SLOTS 3
typedef struct b200_bcast b200_bcast;
B200_API int b200_bcast_piece(int world, size_t nbytes, int index, size_t* offset, size_t* length);
B200_API size_t b200_bcast_flag_bytes(int world);
B200_API int b200_bcast_create(int rank, int world, size_t nbytes, void* const* slots, void* const* flags,
                               b200_bcast** out);
B200_API int b200_bcast_issue(b200_bcast* b, int64_t step, const void* src, void* stream);
/* The same for bytes [offset, offset + length) of the buffer only (offset a
   multiple of 256): they land at the same offsets of the step's slot. */
B200_API int b200_bcast_issue_range(b200_bcast* b, int64_t step, const void* src, size_t offset, size_t length,
                                    void* stream);
B200_API int b200_bcast_wait(b200_bcast* b, int64_t step, void* stream);
B200_API int b200_bcast_release(b200_bcast* b, int64_t step, void* stream);
B200_API void b200_bcast_destroy(b200_bcast* b);

/*
 * The GEMM of exchange step `step` on this rank: C = A * op(B) with B at
 * byte `b_offset` of this rank's receive slot of that step (rank 0: B0, its
 * own source buffer), in the layout rank 0 sent (ldb as for b200_gemm_bf16).  In place of
 * b200_bcast_wait before and b200_bcast_release after: on the CTA-pair
 * kernel the producer waits for the step's flags itself (bounded: a flag
 * that does not arrive within the wait limit is reported by
 * b200_gemm_status) and the last CTA pair to finish loading B releases the
 * slot, so nothing stands between consecutive launches on `stream` and they
 * keep their programmatic overlap; the other kernels get the stream
 * operations around their launch.  Calls on one rank go on one stream.
 * No reference counterpart.
 */
B200_API int b200_bcast_gemm(b200_bcast* b, int64_t step, size_t b_offset, const void* A, const void* B0, void* C,
                             int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int b_layout,
                             void* stream);

/*
 * FP32 GEMM, the reference's fp32_matmul operator (fp32_matmul/matmul.cpp:3-9,
 * MatmulFn over float; B stored [K,N] row-major there, B200_B_KN here; [N,K]
 * also accepted): C[M,N] fp32 = A[M,K] fp32 x op(B) fp32, computed on the bf16
 * tensor cores.  Each operand is split exactly into three bf16 parts and the
 * six products above fp32 rounding are summed by one bf16 GEMM with K' = 6K
 * and fp32 accumulation, written as fp32 (accuracy of an fp32 GEMM; see
 * csrc/split_f32.cuh).  The split operands live in a caller workspace of
 * b200_gemm_f32_workspace_bytes() bytes, 256-byte aligned.  C: 16-byte
 * aligned, ldc a multiple of 4; A and B: 4-byte aligned, any pitch.
 * Replaces the SIMT kernels matmul_v1..v5 (fp32_matmul/matmul.cu:18-325,
 * launchers :342-431).
 */
B200_API int b200_gemm_f32_workspace_bytes(int64_t M, int64_t N, int64_t K, int b_layout, size_t* bytes);
B200_API int b200_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                           int64_t ldb, int64_t ldc, int b_layout, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Flash attention forward, the reference's flash_attn operator
 * (flash_attn/flash_attn.cpp:5-30 and :16-25, launch_fa2_tma_lazy_rescale in
 * fa2_tma_lazy_rescale.cu:369-451): O = softmax(Q K^T / sqrt(head_dim)) V,
 * causal or not, bf16 Q and O of shape [batch, seq_len, heads, head_dim] and
 * K, V of shape [batch, seq_len, kv_heads, head_dim] (all contiguous, 16-byte
 * aligned); heads must be a multiple of kv_heads, and query head h attends
 * with key/value head h / (heads / kv_heads) (grouped-query attention, as
 * fa2_tma_lazy_rescale.cu:113-114).  head_dim = 128 (as the reference
 * requires); fp32 softmax statistics and accumulation on the tcgen05 tensor
 * cores.  No allocation; asynchronous on `stream`.
 */
B200_API int b200_flash_attn_bf16(const void* Q, const void* K, const void* V, void* O, int64_t batch,
                                  int64_t seq_len, int64_t heads, int64_t kv_heads, int64_t head_dim, int causal,
                                  void* stream);

/*
 * Attention kernel selection for later b200_flash_attn_bf16 calls in this
 * process (all devices):
 *   B200_ATTN_KERNEL_AUTO   (0) default: the faster kernel, on B200 SINGLE
 *   B200_ATTN_KERNEL_SINGLE (1) one CTA per two 128-row query tiles
 *   B200_ATTN_KERNEL_PAIR   (2) a CTA pair per four query tiles (cta_group::2
 *                               products, each SM holding half of every K and
 *                               V tile; slower on B200)
 * For testing and tuning; every choice computes the same attention.  No
 * reference counterpart (the reference has one attention kernel).
 */
#define B200_ATTN_KERNEL_AUTO 0
#define B200_ATTN_KERNEL_SINGLE 1
#define B200_ATTN_KERNEL_PAIR 2
B200_API int b200_flash_attn_set_kernel(int which);

/* Element type of D for b200_gemm_bf16_ex. */
#define B200_DTYPE_BF16 0
#define B200_DTYPE_F32 1

/*
 * Fused epilogue: D[m, n] = alpha * (A op(B))[m, n] + bias[n] + beta * c_in[m, n],
 * computed in fp32 from the fp32 accumulator, one operation at a time in that
 * order (no fused multiply-add), then stored as d_dtype.
 */
typedef struct b200_epilogue {
  float alpha;       /* scale of the product (1 for none) */
  float beta;        /* scale of c_in; 0 = c_in is not read */
  const void* c_in;  /* bf16 [M, N] row-major, leading dimension ldc_in (>= N, multiple of 8), 16-byte aligned;
                        may be D itself (in-place accumulate) when D is bf16 with ldd == ldc_in */
  int64_t ldc_in;
  const void* bias;  /* bf16 [N], 16-byte aligned, added to every row; NULL for none */
  int d_dtype;       /* B200_DTYPE_BF16 or B200_DTYPE_F32 */
} b200_epilogue;

/*
 * b200_gemm_bf16 with a fused epilogue (bias, residual / beta * C, alpha,
 * fp32 output) applied to the fp32 accumulator before D is written once.
 * D is [M, N] of d_dtype with leading dimension ldd elements (bf16: multiple
 * of 8; fp32: multiple of 4), 16-byte aligned.  epi == NULL is exactly
 * b200_gemm_bf16.  K must be >= 1 when an epilogue is given
 * (B200_ERR_INVALID_ARG otherwise).  Always sequential K order (no split-K).
 * No reference counterpart: the reference's kernels write only
 * C = bf16(A * B^T) (bf16_matmul/matmul_v8_tuned.cu:152-178); this is the
 * epilogue fusion its callers would otherwise do with extra passes over C.
 */
B200_API int b200_gemm_bf16_ex(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K, int64_t lda,
                               int64_t ldb, int64_t ldd, int b_layout, const b200_epilogue* epi, void* stream);

/*
 * Workspace b200_gemm_bf16_ws wants for this shape on the current device
 * (0 when it would not split; on a 148-SM B200 at most 15.75 MiB of fp32
 * partial tiles plus 1 KiB of hand-off flags).  Depends on the device's SM
 * count and on b200_gemm_set_kernel.
 */
B200_API int b200_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int b_layout, size_t* bytes);

/*
 * Same product as b200_gemm_bf16_ws, for callers that cannot allocate device
 * memory when they multiply (a serving engine that reserves all of HBM at
 * start-up and keeps cudaMalloc off its request path, or a plugin whose host
 * hands it buffers but no allocator).  It allocates nothing: its split-K
 * scratch is a 16 MiB static array inside this library, held by every GPU
 * that loads the library until the process exits.  Shapes that would need
 * more scratch than that are rejected with B200_ERR_SCRATCH_LIMIT (none do
 * on a 148-SM B200).
 *
 * The first call on each device also looks up the device address of that
 * array (with that device current); make that first call before any stream
 * capture.  Every call shares the one array, and the array keeps whatever the
 * last call left in it, which is harmless (partials are fully rewritten and
 * hand-off flags carry a per-launch tag) — but calls whose kernels can overlap
 * on the GPU (other streams, other host threads) race on it: issue them on
 * one stream, or use b200_gemm_bf16_ws with separate workspaces.
 * No counterpart in the reference, which allocates nothing of its own.
 */
B200_API int b200_gemm_bf16_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                    int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* stream);

/*
 * Waits for `stream`, then reads and clears the current device's status word.
 * Returns B200_OK, B200_ERR_DEVICE_TIMEOUT (a kernel gave up on a wait; the
 * raw bits are stored to *device_bits if non-NULL), or B200_ERR_CUDA.
 * The reference has no error reporting at all (host assert only,
 * bf16_matmul/matmul_v8_tuned.cu:238).
 */
B200_API int b200_gemm_status(void* stream, uint32_t* device_bits);

/*
 * Sets the time limit, in nanoseconds, that every device-side wait of later
 * launches on this device gets (default 4e9 ns).  0 restores the default.
 * No reference counterpart (its waits are unbounded, bf16_matmul/common.hpp:128-145).
 */
B200_API int b200_gemm_set_timeout_ns(uint64_t timeout_ns);

/*
 * Kernel selection for later calls in this process (all devices):
 *   B200_KERNEL_AUTO   (0) default: M <= 128 -> swap-AB split-K kernel,
 *                          otherwise the CTA-pair kernel (256-row tiles)
 *   B200_KERNEL_SINGLE (1) one CTA per 128 x 256 tile, any M
 *   B200_KERNEL_PAIR   (2) CTA pair per 256 x 256 tile, any M
 *   B200_KERNEL_SKINNY (3) swap-AB split-K, M <= 128 only (else B200_ERR_INVALID_ARG at launch)
 * For testing and tuning; every choice computes the same product.  No
 * reference counterpart (the reference picks a kernel by calling a different
 * launcher, bf16_matmul/matmul.cpp:44-56).
 */
#define B200_KERNEL_AUTO 0
#define B200_KERNEL_SINGLE 1
#define B200_KERNEL_PAIR 2
#define B200_KERNEL_SKINNY 3
B200_API int b200_gemm_set_kernel(int which);

/*
 * Failure-detection self-test: launches one CTA that waits, with the same
 * bounded wait every GEMM kernel uses, on an mbarrier that nothing arrives at
 * (timeout_ns in (0, 1e10]).  The wait gives up after timeout_ns; the next
 * b200_gemm_status() then returns B200_ERR_DEVICE_TIMEOUT, and the device
 * stays usable.  No reference counterpart (the reference's waits spin
 * forever, bf16_matmul/common.hpp:128-145).
 */
B200_API int b200_gemm_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/* Static text for a return code. */
B200_API const char* b200_gemm_strerror(int code);

/* Library version, e.g. "b200_gemm 0.1.0 sm_100a". */
B200_API const char* b200_gemm_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* B200_GEMM_H_ */
