// Host-side interface of the skinny tcgen05 GEMM (gemm_skinny.cu): dense rows
// 2..64 with the weights as the MMA's A operand and the tokens as its N.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "peer_reduce.cuh"

namespace grinqh {

struct SkinnyArgs {
  const void* x;        // [M, K] dtype, row-major, 16-byte aligned
  const uint32_t* w;    // [K, nz*N/16] packed planes
  const void* s;        // [K/group, N] dtype
  const void* bias;     // [N] dtype or null
  void* y;              // [M, N] dtype
  float* slots;         // [tiles, clusters, Mp * 512] fp32 cluster sums (several clusters per tile)
  unsigned* counters;   // [tiles, cluster size] tickets; zero before the first launch, left zero
  int M, K, N, group;
  int tiles, splits, cluster, steps_per_split;
  PeerReduce ar;        // used by the fused all-reduce launch only (cap >= M * N)
};

struct SkinnyPlan {
  int mp;                // tokens rounded up to 16 (the MMA's N)
  int tiles, splits, cluster, steps_per_split;
  size_t slot_bytes, counter_bytes;
};

bool skinny_supported(int64_t M, int64_t K, int64_t N, int group);
bool skinny_pointers_ok(const void* x, const void* w, const void* s);
// A plan whose whole grid is resident at once (smaller clusters or fewer K splits
// where the default does not fit); false if none is, or no device can be asked. The
// fused all-reduce launch requires it: its CTAs wait on the peer ranks' CTAs, which
// must all be running.
bool plan_skinny_resident(int64_t M, int64_t K, int64_t N, int sm_count, SkinnyPlan* out);
// The launch plan: the resident plan where there is one (a grid one cluster too large
// would run that cluster as a second wave), else the default.
SkinnyPlan plan_skinny(int64_t M, int64_t K, int64_t N, int sm_count);
int launch_skinny(const SkinnyArgs& a, const SkinnyPlan& p, int dtype, int nz, cudaStream_t st,
                  bool allreduce = false);
unsigned take_skinny_timeouts();

}  // namespace grinqh
