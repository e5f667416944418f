// Host-side interface of the tensor-core single-row graded GEMV (decode_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace grinqh {

struct M1TcArgs {
  const void* x;        // [K] dtype
  const uint32_t* w;    // [K, nz*N/16] packed planes
  const void* s;        // [K/128, N] dtype
  const void* bias;     // [N] dtype or null
  void* y;              // [N] dtype
  float* slots;         // [ctas + tiles, 512] fp32 partial sums
  unsigned* counters;   // [tiles] tickets; zero before the first launch, left zero
  int K, N, tiles, units_per_cta;
  float t[4];
};

struct M1TcPlan {
  int tiles, units_per_cta, ctas;
  size_t slot_bytes, counter_bytes;
  uint32_t smem_bytes;
};

bool m1tc_supported(int64_t M, int64_t K, int64_t N, int group);
M1TcPlan plan_m1tc(int64_t K, int64_t N, int sm_count);
int launch_m1tc(const M1TcArgs& a, const M1TcPlan& p, int dtype, int nz, cudaStream_t st);
unsigned take_m1tc_timeouts();

}  // namespace grinqh
