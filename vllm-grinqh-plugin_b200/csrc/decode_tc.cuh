// Host-side interface of the tensor-core single-row graded GEMV (decode_tc.cu).
#pragma once

#include <cuda.h>
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
  int bslots;           // B slots in shared memory: min(units_per_cta, K / 64)
  int tma_min_rows;     // a unit's plane with more graded rows than this comes by TMA
  float t[4];
};

struct M1TcPlan {
  int tiles, units_per_cta, ctas;
  int plane_stages;  // plane stages in shared memory (4)
  int bslots;        // x-digit tiles kept in shared memory
  size_t slot_bytes, counter_bytes;
  uint32_t smem_bytes;
};

bool m1tc_supported(int64_t M, int64_t K, int64_t N, int group);
bool m1tc_plan_fits(const M1TcPlan& p);
bool m1tc_pointers_ok(const void* w);  // the planes are read in 16-byte chunks
M1TcPlan plan_m1tc(int64_t K, int64_t N, int nz, int sm_count);
int launch_m1tc(const M1TcArgs& a, const M1TcPlan& p, int dtype, int nz, cudaStream_t st);
unsigned take_m1tc_timeouts();

}  // namespace grinqh
