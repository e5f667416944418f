// Host-side interface of the two-pass dense GEMM (gemm_bf16.cu): dequantize the
// planes to dtype(w * s) once, then a TMA-fed tcgen05 GEMM.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace grinqh {

struct Bf16GemmArgs {
  const void* x;        // [M, K] dtype, row-major, 16-byte aligned
  const uint32_t* w;    // [K, nz*N/16] packed planes
  const void* s;        // [K/group, N] dtype
  const void* bias;     // [N] dtype or null
  void* y;              // [M, N] dtype, 16-byte aligned
  void* wbuf;           // [K, N] dtype scratch for dtype(w * s), 256-byte aligned
  float* slots;         // [splits, M, N] fp32 split-K sums (splits > 1)
  unsigned* counters;   // [tiles] tickets (splits > 1); zero before the first launch, left zero
  int M, K, N, group, splits;
  // graded prefill only (null otherwise): per (256-row tile of x, 64-deep K step) a
  // non-zero word if the step has any non-zero activation (steps without one are
  // skipped), and a device float the fp32 sums are multiplied by before the cast
  const unsigned* active;
  const float* out_scale;
};

// The opt-in per-token graded prefill (GRINQH_MODE_GRADED, many rows) on the same
// tensor-core GEMM: y = [x masked by zone 0 | ... | by zone b/2 - 1] @ [B_0; ...], one
// fp16 GEMM over K' = (b/2) K with B_z = s (D_z + Delta_z 2^shift) / 2^shift, the zone's
// weight contribution plus its mid-point bias (grinqh/kernel.py:73-158), exact in fp16.
bool graded_gemm_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* w,
                           const void* s, const void* y);
size_t graded_gemm_workspace(int64_t M, int64_t K, int64_t N, int nz, int sm_count);
int launch_graded_gemm(const Bf16GemmArgs& a, const float* thresholds, void* workspace, int dtype, int nz,
                       int sm_count, cudaStream_t st);

bool bf16_gemm_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* w, const void* s,
                         const void* y);
size_t bf16_gemm_buffer_bytes(int64_t K, int64_t N);
int bf16_gemm_splits(int64_t M, int64_t K, int64_t N, int sm_count);
size_t bf16_gemm_slot_bytes(int64_t M, int64_t N, int splits);
int launch_bf16_gemm(const Bf16GemmArgs& a, int dtype, int nz, cudaStream_t st);
unsigned take_bf16_gemm_timeouts();

}  // namespace grinqh
