// Host-side interface of the single-row graded GEMV (decode_m1.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "peer_reduce.cuh"

namespace grinqh {

struct M1Args {
  const void* x;        // [K] dtype
  const uint32_t* w;    // [K, nz*N/16] packed planes
  const void* s;        // [K/group, N] dtype
  const void* bias;     // [N] dtype or null
  void* y;              // [N] dtype
  float* slots;         // [tiles, clusters per tile, 1024] fp32 (several clusters per tile)
  unsigned* counters;   // [tiles] tickets; zero before the first launch, left zero
  int K, N, group, rows_per_warp, rows_per_cta;
  float t[4];
  PeerReduce ar;        // used by the fused all-reduce launch only (cap >= N)
};

struct M1Plan {
  int tiles, rows_per_warp, rows_per_cta, cluster, grid_splits;
  size_t slot_bytes, counter_bytes, smem_bytes;
};

// staged per-row metadata (x, bias*x, grade), 16 bytes a row
__host__ __device__ inline size_t m1_meta_bytes(int rows_per_cta) {
  return (size_t)rows_per_cta * 16;
}

bool m1_supported(int64_t M, int64_t K, int64_t N, int group);
// the kernel reads two packed words (8 bytes) and two scales (4 bytes) at a time
inline bool m1_pointers_ok(const void* w, const void* s) {
  return (reinterpret_cast<uintptr_t>(w) % 8) == 0 && (reinterpret_cast<uintptr_t>(s) % 4) == 0;
}
// few_slots: clusters of 8 CTAs wherever the split count allows, for the fewest fp32
// slots (the fixed scratch of grinqh_gemv_noalloc), at some cost in time.
M1Plan plan_m1(int64_t K, int64_t N, int group, int sm_count, bool few_slots = false);
// the plan's shared memory fits one CTA (rows_per_cta grows with K when N is so wide
// that the column slices alone fill the GPU)
inline bool m1_plan_fits(const M1Plan& p) { return p.smem_bytes <= 227u * 1024u; }
int launch_m1(const M1Args& a, const M1Plan& p, int dtype, int nz, cudaStream_t st, bool allreduce = false);
// Reads and clears the count of fused all-reduce waits that gave up (this file's copy
// of the bounded-wait counter).
unsigned take_m1_timeouts();

}  // namespace grinqh
