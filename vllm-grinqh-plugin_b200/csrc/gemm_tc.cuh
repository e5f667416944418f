// Host-side interface of the tcgen05 dense GEMM (gemm_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace grinqh {

struct GemmArgs {
  const void* x;        // [M, K] dtype, row-major, 16-byte aligned
  const uint32_t* w;    // [K, nz*N/16] packed planes
  const void* s;        // [K/group, N] dtype
  const void* bias;     // [N] dtype or null
  void* y;              // [M, N] dtype
  int M, K, N, group;
};

bool gemm_tc_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* y);
int launch_gemm_tc(const GemmArgs& a, int dtype, int nz, cudaStream_t st);
unsigned take_gemm_timeouts();

}  // namespace grinqh
