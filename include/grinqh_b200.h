/*
 * grinqh_b200.h -- C ABI of the B200 (sm_100a) GRINQH quantized-linear hot path.
 *
 * Plain pointers, sizes and a CUDA stream; no torch types. Every pointer named
 * `*_dev` is device memory; thresholds are host memory. All entry points are
 * asynchronous on `stream` (no host synchronisation, no device->host reads), so
 * they can be recorded into CUDA graphs, and return a grinqh_status code
 * (GRINQH_OK == 0). On error, grinqh_last_error() returns a message for the
 * calling thread.
 *
 * Reference interfaces replaced (paths relative to the reference project root):
 *   grinqh_pack_words        <- grinqh/utils.py:125-146  pack_triton / _pack_kernel_uint32 (:100-122)
 *   grinqh_pack_codes        <- grinqh/grinqh.py:202-211 process_weights_after_loading
 *                               (grinqh_input_preshuffle utils.py:17-22, << (8-b), pack_triton)
 *   grinqh_unpack_checkpoint <- grinqh/grinqh.py:154-168 weight loader (unpack_from_int32 + narrow + copy)
 *   grinqh_gemv_allreduce    <- grinqh/grinqh.py:236-247 apply + vLLM's row-parallel all-reduce (M = 1)
 *   grinqh_gemm_allreduce    <- the same for one graded row or 2..64 dense rows (batched decode)
 *   grinqh_unpack            <- grinqh/utils.py:149-177  unpack_pyt, :209-223 unpack_triton
 *   grinqh_grade             <- grinqh/kernel.py:100-116 threshold masks of the graded GEMV
 *   grinqh_gemm_or_gemv      <- grinqh/kernel.py:646-710 torch.ops.grinqh.gemm_or_gemv
 *   grinqh_gemv_batch_union  <- grinqh/kernel.py:607-643 grinqh_gemv_batch_union
 *   grinqh_prefill_gemm      <- grinqh/kernel.py:561-587 grinqh_prefill_gemm_compiled
 *   grinqh_rmsnorm_grade, grinqh_silu_mul_grade, grinqh_gemv_batch_union_masked
 *                            <- the grading of kernel.py:100-116 moved into the producer of x
 *                               (vLLM's RMSNorm / SiluAndMul, which precede qkv, gate_up, down)
 *
 * Tensor layouts (row-major, contiguous unless a leading dimension is given):
 *   x              [M, K]            activations, dtype (bf16 or fp16)
 *   weight_packed  [K, (b/2)*N/16]   uint32 bit planes (grinqh/utils.py:100-122 layout)
 *   weight_scale   [K/group, N]      dtype, one scale per (K group, output column)
 *   bias           [N] or NULL       dtype
 *   y              [M, N]            dtype
 * with b = max_bits in {2,4,6,8}, N % 16 == 0, K % group_size == 0,
 * group_size % 32 == 0, and N == 4 * original_n of the reference signature.
 */
#ifndef GRINQH_B200_H
#define GRINQH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Identical to cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st *grinqh_stream_t;

typedef enum grinqh_status {
  GRINQH_OK = 0,
  GRINQH_ERR_INVALID = 1,     /* bad argument: null pointer, shape, alignment       */
  GRINQH_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. max_bits = 3)       */
  GRINQH_ERR_CUDA = 3,        /* CUDA launch / runtime error                         */
  GRINQH_ERR_WORKSPACE = 4,   /* workspace missing or smaller than required          */
  GRINQH_ERR_DEVICE = 5       /* current device is not an sm_100 (B200-class) GPU    */
} grinqh_status;

typedef enum grinqh_dtype {
  GRINQH_F16 = 0,
  GRINQH_BF16 = 1
} grinqh_dtype;

/* How rows of x pick the weight planes they read (grinqh_gemm_or_gemv):
 *   AUTO   -- the reference dispatch (kernel.py:663-705): one row -> graded GEMV,
 *             several rows -> dense x @ dtype(w*s), thresholds ignored;
 *   DENSE  -- always the dense path;
 *   GRADED -- every row graded by its own activations (the reference's one-row
 *             GEMV applied row by row; this build's opt-in graded prefill);
 *   UNION  -- rows graded by max_m |x[m,k]| (grinqh_gemv_batch_union semantics). */
typedef enum grinqh_mode {
  GRINQH_MODE_AUTO = 0,
  GRINQH_MODE_DENSE = 1,
  GRINQH_MODE_GRADED = 2,
  GRINQH_MODE_UNION = 3
} grinqh_mode;

/* OR into `mode` of grinqh_gemm_or_gemv: the caller promises that the workspace is
 * all zero bytes on entry -- freshly zeroed, or last used by a call of this library on
 * the same stream, which always leaves it zero -- so the call skips clearing its
 * tickets (one fewer operation on the stream per call). No reference counterpart. */
#define GRINQH_WORKSPACE_ZEROED 0x100

int grinqh_abi_version(void);
const char *grinqh_status_string(int status);
const char *grinqh_last_error(void);

/* Number of bounded waits in this library's kernels on the current device (pipeline
 * mbarriers, split-K fix-ups, the fused all-reduce's wait for the other ranks) that
 * gave up since the last call, then reset to 0. Non-zero means a kernel gave up
 * waiting and its output is not valid; once one wait has given up, later waits give
 * up at once until this call clears the count. Synchronous.
 * (No reference counterpart: the reference's Triton kernels have no device waits.) */
int grinqh_take_error_flags(unsigned *timeouts);

/* Bit-plane pack of already preshuffled and shifted code words.
 * words_dev [K, n_words] uint32 (4 code bytes per word, codes in the MSBs),
 * n_words % 4 == 0; out_dev [K, (b/2)*n_words/4] uint32.
 * Replaces pack_triton (grinqh/utils.py:125-146), bit-exact. */
int grinqh_pack_words(const uint32_t *words_dev, uint32_t *out_dev, int64_t K, int64_t n_words,
                      int max_bits, grinqh_stream_t stream);

/* Load-time transform fused in one pass: column preshuffle, << (8-b), pack.
 * codes_dev [K, N] int8 signed codes in [-2^(b-1), 2^(b-1)-1] (K-major, row stride ld >= N);
 * out_dev [K, (b/2)*N/16] uint32. Replaces grinqh/grinqh.py:202-211, bit-exact. */
int grinqh_pack_codes(const int8_t *codes_dev, int64_t ld, uint32_t *out_dev, int64_t K, int64_t N,
                      int max_bits, grinqh_stream_t stream);

/* Checkpoint codes -> this rank's staging codes in one pass (load time).
 * src_dev: the compressed-tensors pack-quantized weight of one shard, rows = output
 * features, src_ld int32 words per row, 32/b offset-binary fields per word LSB first
 * along K (b = 2, 4, 8); for b = 6 the int8 codes themselves, src_ld bytes per row.
 * Writes dst_dev[k * ld + n] = code(row r0 + n, column k0 + k) as int8 for n < rows,
 * k < k_local; k0 a multiple of 32/b. Replaces unpack_from_int32 + the narrowing +
 * the transposed copy of grinqh/grinqh.py:154-168 (compressed_tensors
 * compressors/pack_quantized/helpers.py unpack_from_int32), bit-exact. */
int grinqh_unpack_checkpoint(const void *src_dev, int64_t src_ld, int max_bits, int64_t r0, int64_t rows,
                             int64_t k0, int64_t k_local, int8_t *dst_dev, int64_t ld,
                             grinqh_stream_t stream);

/* Inverse of grinqh_pack_words: out_dev [K, N] uint8, byte = shifted_code >> (8-b)
 * (unsigned, preshuffled column order), exactly unpack_pyt (grinqh/utils.py:149-177). */
int grinqh_unpack(const uint32_t *packed_dev, uint8_t *out_dev, int64_t K, int64_t N, int max_bits,
                  grinqh_stream_t stream);

/* Grade activations: masks_dev [M, K] uint8 with bit z set iff fp32|x[m,k]| > fp32(t_z)
 * for z < b/2 (strict; NaN never active), grinqh/kernel.py:100-116.
 * union_dev [K] uint8 (may be NULL) = OR over rows. thresholds: 4 host floats. */
int grinqh_grade(const void *x_dev, int dtype, int64_t M, int64_t K, const float *thresholds,
                 int max_bits, uint8_t *masks_dev, uint8_t *union_dev, grinqh_stream_t stream);

/* Scratch bytes grinqh_gemm_or_gemv / grinqh_gemv_batch_union / grinqh_prefill_gemm
 * need for these sizes, group size and mode (0 is possible). Host-only. */
size_t grinqh_workspace_size(int64_t M, int64_t K, int64_t N, int max_bits, int group_size, int mode);

/* The quantized linear y = x @ W (+ bias), torch.ops.grinqh.gemm_or_gemv
 * (grinqh/kernel.py:646-710). workspace_dev: grinqh_workspace_size() bytes,
 * 256-byte aligned; its contents need no initialisation and are not preserved.
 * thresholds: 4 host floats (ignored by DENSE / AUTO with M > 1). */
int grinqh_gemm_or_gemv(const void *x_dev, int dtype, int64_t M, int64_t K,
                        const uint32_t *weight_packed_dev, const void *weight_scale_dev,
                        const void *bias_dev, int max_bits, int group_size, int64_t N,
                        const float *thresholds, int mode, void *y_dev, void *workspace_dev,
                        size_t workspace_bytes, grinqh_stream_t stream);

/* Small-batch GEMV graded by the row union (grinqh/kernel.py:607-643); same as
 * grinqh_gemm_or_gemv with mode = GRINQH_MODE_UNION. */
int grinqh_gemv_batch_union(const void *x_dev, int dtype, int64_t M, int64_t K,
                            const uint32_t *weight_packed_dev, const void *weight_scale_dev,
                            const void *bias_dev, int max_bits, int group_size, int64_t N,
                            const float *thresholds, void *y_dev, void *workspace_dev,
                            size_t workspace_bytes, grinqh_stream_t stream);

/* grinqh_gemv_batch_union with the rows' union of grades supplied (union_mask_dev [K]
 * uint8, from grinqh_rmsnorm_grade / grinqh_silu_mul_grade or grinqh_grade on the same
 * x and thresholds) instead of graded again from every row of x inside the GEMV. */
int grinqh_gemv_batch_union_masked(const void *x_dev, int dtype, int64_t M, int64_t K,
                                   const uint32_t *weight_packed_dev, const void *weight_scale_dev,
                                   const void *bias_dev, int max_bits, int group_size, int64_t N,
                                   const float *thresholds, const uint8_t *union_mask_dev, void *y_dev,
                                   void *workspace_dev, size_t workspace_bytes, grinqh_stream_t stream);

/* ---- Producers of x with the grading fused in (no counterpart in the reference,
 * which grades inside its GEMV, grinqh/kernel.py:100-116, or in a separate pass over x).
 * Each writes x for the next linear, its grade masks (masks_dev [M, K], as grinqh_grade;
 * NULL: not written) and their union over the rows (union_dev [K], cleared on the
 * stream first; NULL: not written), graded from the written (rounded) values.
 * thresholds: 4 host floats (may be NULL when neither mask is asked for). K % 8 == 0;
 * x, residual, weight and out 16-byte aligned, masks 8-byte, union 4-byte.
 *   grinqh_rmsnorm_grade: vLLM's rms_norm / fused_add_rms_norm
 *     (vllm/ir/ops/layernorm.py:10-58): s = x (+ residual; residual_dev, if not NULL,
 *     is replaced by dtype(s)); out = dtype(dtype(s * rsqrt(mean(s^2) + eps)) * weight)
 *     (weight_dev NULL: no weight). x and out [M, K]; K * 4 bytes must fit in shared
 *     memory (K <= 58112).
 *   grinqh_silu_mul_grade: vLLM's SiluAndMul on x_dev [M, 2K] = [gate | up]:
 *     out [M, K] = dtype(dtype(gate / (1 + exp(-gate))) * up). */
int grinqh_rmsnorm_grade(const void *x_dev, void *residual_dev, const void *weight_dev, int dtype, int64_t M,
                         int64_t K, float eps, const float *thresholds, int max_bits, void *out_dev,
                         uint8_t *masks_dev, uint8_t *union_dev, grinqh_stream_t stream);
int grinqh_silu_mul_grade(const void *x_dev, int dtype, int64_t M, int64_t K, const float *thresholds,
                          int max_bits, void *out_dev, uint8_t *masks_dev, uint8_t *union_dev,
                          grinqh_stream_t stream);

/* Dense path y = x @ dtype(w * s) for any M >= 1 (grinqh/kernel.py:561-587); same as
 * grinqh_gemm_or_gemv with mode = GRINQH_MODE_DENSE. */
int grinqh_prefill_gemm(const void *x_dev, int dtype, int64_t M, int64_t K,
                        const uint32_t *weight_packed_dev, const void *weight_scale_dev,
                        const void *bias_dev, int max_bits, int group_size, int64_t N,
                        void *y_dev, void *workspace_dev, size_t workspace_bytes,
                        grinqh_stream_t stream);

/* Single-row graded GEMV that allocates nothing (no counterpart in the reference,
 * whose kernels always take their scratch from the torch allocator).
 *
 * For callers that cannot allocate device memory when they run the layer: code
 * with a fixed memory budget reserved at start-up (embedded or real-time inference
 * loops, plugin hosts that forbid allocation after initialisation) or hot paths
 * that must not enter an allocator, which may synchronise the device or fail
 * under fragmentation. Same computation as grinqh_gemm_or_gemv with M = 1 and
 * mode GRINQH_MODE_AUTO (x [K], y [N]); the kernel's scratch lives in a 256 KiB
 * device array inside this library instead of a caller workspace. Every GPU that
 * loads the library holds that array until the process exits.
 *   - The first call on a device looks up the array's device address (once per
 *     device, with that device current); make that first call before any stream
 *     capture. The address is kept for the life of the process and belongs to the
 *     device's primary context: after cudaDeviceReset on a device, do not call this
 *     entry point on that device again.
 *   - A launch plan whose scratch would exceed 256 KiB returns
 *     GRINQH_ERR_WORKSPACE (the kernel's K split keeps every shape below it on a
 *     148-SM B200, so this is a guard).
 *   - All calls share the array: calls that can overlap on the GPU (different
 *     streams, or graphs replayed concurrently) race and give wrong results;
 *     serialise them, or use grinqh_gemm_or_gemv with separate workspaces. */
int grinqh_gemv_noalloc(const void *x_dev, int dtype, int64_t K, const uint32_t *weight_packed_dev,
                        const void *weight_scale_dev, const void *bias_dev, int max_bits, int group_size,
                        int64_t N, const float *thresholds, void *y_dev, grinqh_stream_t stream);

/* ---- Row-parallel linear with its all-reduce fused in (tensor parallelism).
 * Replaces the plugin's apply (grinqh/grinqh.py:236-247) followed by vLLM's
 * row-parallel all-reduce of the partial outputs (vllm/model_executor/layers/linear.py,
 * RowParallelLinear.forward) for one row (the graded GEMV) and for 2..64 rows (the
 * dense skinny GEMM, batched decode): each rank computes the product of its K slice,
 * and the kernel that does so also sums the ranks' fp32 partials over NVLink (plain
 * 64-bit peer stores of {partial, launch epoch} into every rank's buffer, bounded
 * waits on the epochs) and writes the summed y (+ bias, applied once) on every rank,
 * the same bits on every rank.
 *   - Every rank owns one peer buffer of grinqh_allreduce_buffer_bytes(world, cap)
 *     bytes from grinqh_allreduce_buffer_alloc (zeroed), cap = the largest M * N a call
 *     will use; the ranks exchange grinqh_ipc_get_handle handles (64 bytes) and open
 *     each other's with grinqh_ipc_open_handle; buffers_dev[r] is rank r's buffer as
 *     mapped in this process (buffers_dev[rank] the own one). At most 8 ranks.
 *   - Every rank must make the same sequence of calls on its buffer (launch epochs are
 *     counted on the device, so calls can be recorded in CUDA graphs). A rank that
 *     never arrives makes the others give up after GRINQH_ALLREDUCE_WAIT_MS
 *     milliseconds (environment, read on every call; default 2000):
 *     grinqh_take_error_flags then reports a non-zero count, y is not valid, and
 *     every rank should call grinqh_take_error_flags before its next launch.
 *   - grinqh_gemm_allreduce: mode as for grinqh_gemm_or_gemv (AUTO: one row graded,
 *     more rows dense; GRINQH_WORKSPACE_ZEROED honoured); shapes the fused kernels do
 *     not take (graded rows beyond one, dense rows beyond 64, unaligned views) return
 *     GRINQH_ERR_UNSUPPORTED before anything is launched -- the same answer on every
 *     rank -- and the caller takes the unfused path. The workspace is
 *     grinqh_allreduce_workspace_size bytes (it may differ from grinqh_workspace_size:
 *     the fused grid must be resident at once, which can take fewer K splits).
 *   - grinqh_gemv_allreduce: the one-row form (x [K], y [N]); mode is 0 or
 *     GRINQH_WORKSPACE_ZEROED; its workspace is grinqh_workspace_size(1, ...).
 *   - thresholds: 4 host floats (graded rows; may be NULL for dense rows). */
size_t grinqh_allreduce_buffer_bytes(int world, int64_t cap);
int grinqh_allreduce_buffer_alloc(size_t bytes, void **buf_dev);
int grinqh_allreduce_buffer_free(void *buf_dev);
int grinqh_ipc_get_handle(const void *buf_dev, unsigned char *handle64);
int grinqh_ipc_open_handle(const unsigned char *handle64, void **buf_dev);
int grinqh_ipc_close_handle(void *buf_dev);
size_t grinqh_allreduce_workspace_size(int64_t M, int64_t K, int64_t N, int max_bits, int group_size, int mode);
int grinqh_gemm_allreduce(const void *x_dev, int dtype, int64_t M, int64_t K, const uint32_t *weight_packed_dev,
                          const void *weight_scale_dev, const void *bias_dev, int max_bits, int group_size,
                          int64_t N, const float *thresholds, int mode, void *y_dev, void *workspace_dev,
                          size_t workspace_bytes, int rank, int world, void *const *buffers_dev, int64_t cap,
                          grinqh_stream_t stream);
int grinqh_gemv_allreduce(const void *x_dev, int dtype, int64_t K, const uint32_t *weight_packed_dev,
                          const void *weight_scale_dev, const void *bias_dev, int max_bits, int group_size,
                          int64_t N, const float *thresholds, void *y_dev, void *workspace_dev,
                          size_t workspace_bytes, int rank, int world, void *const *buffers_dev, int64_t cap,
                          int mode, grinqh_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GRINQH_B200_H */
