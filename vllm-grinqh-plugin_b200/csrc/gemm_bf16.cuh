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
};

bool bf16_gemm_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* w, const void* s,
                         const void* y);
size_t bf16_gemm_buffer_bytes(int64_t K, int64_t N);
int bf16_gemm_splits(int64_t M, int64_t K, int64_t N, int sm_count);
size_t bf16_gemm_slot_bytes(int64_t M, int64_t N, int splits);
int launch_bf16_gemm(const Bf16GemmArgs& a, int dtype, int nz, cudaStream_t st);
unsigned take_bf16_gemm_timeouts();

}  // namespace grinqh
