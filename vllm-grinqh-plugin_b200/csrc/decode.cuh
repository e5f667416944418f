// Host-side interface of the small-M kernels (decode.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace grinqh {

enum : int { kModeGraded = 0, kModeUnion = 1, kModeDense = 2 };

constexpr int kDecodeMaxRows = 512;  // K rows staged per CTA

struct DecodeArgs {
  const void* x;        // [M, K] dtype
  const uint32_t* w;    // [K, nz*N/16] packed planes
  const void* s;        // [K/group, N] dtype
  const void* bias;     // [N] dtype or null
  void* y;              // [M, N] dtype
  float* partial;       // [ksplit, M, N] fp32 (ksplit > 1)
  unsigned* counters;   // [chunks, jtiles] tickets, zero before launch
  int M, K, N, group, rows_per_cta, ksplit;
  float t[4];
  const uint8_t* umask;  // [K] union of the rows' grades (union mode), or null: graded here
};

struct DecodePlan {
  int mt, jtiles, chunks, ksplit, rows_per_cta;
  size_t partial_bytes, counter_bytes;
};

DecodePlan plan_decode(int64_t M, int64_t K, int64_t N, int mode, int sm_count);
int launch_decode(const DecodeArgs& a, const DecodePlan& p, int mode, int dtype, int nz, cudaStream_t st);

}  // namespace grinqh
