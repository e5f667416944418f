// Shared helpers for the GRINQH sm_100a kernels: status plumbing, dtype traits and
// the bit-plane merge that turns b/2 packed 2-bit planes back into code bytes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "grinqh_b200.h"

namespace grinqh {

// ------------------------------------------------------------------ status / errors
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
int check_device();  // GRINQH_ERR_DEVICE unless the current device is sm_100

#define GRINQH_REQUIRE(cond, ...)                                  \
  do {                                                             \
    if (!(cond)) return ::grinqh::set_error(GRINQH_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define GRINQH_RETURN_IF(st)          \
  do {                                \
    int _s = (st);                    \
    if (_s != GRINQH_OK) return _s;   \
  } while (0)

inline bool valid_bits(int b) { return b == 2 || b == 4 || b == 6 || b == 8; }
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------------ dtype traits
template <typename T> struct Act;
template <> struct Act<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  // round a float to the activation dtype and back (torch's w.to(dtype) * s rounding)
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct Act<__half> {
  static constexpr bool kBf16 = false;
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

// ------------------------------------------------------------------ bit-plane merge
// Packed word of plane z (grinqh/utils.py:100-122): byte lane L holds, at bits
// (7-2i, 6-2i), the zone-z bit pair of neighbour i (i = 0..3). Within each byte
// lane the four plane words form a 4x4 matrix of 2-bit fields F[z][i]; the code
// byte of neighbour i is column i: F[0][i] F[1][i] F[2][i] F[3][i] (MSB first).
// Transpose it with two block-swap stages (nibbles, then bit pairs). Byte L of the
// result q[i] is the shifted code of output column 16*j' + 4i + L of the
// preshuffled order, i.e. original column (4i + L) * N/16 + j'.
__device__ __forceinline__ void merge_planes(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t q[4]) {
  const uint32_t r0 = (a0 & 0xF0F0F0F0u) | ((a2 >> 4) & 0x0F0F0F0Fu);
  const uint32_t r2 = ((a0 << 4) & 0xF0F0F0F0u) | (a2 & 0x0F0F0F0Fu);
  const uint32_t r1 = (a1 & 0xF0F0F0F0u) | ((a3 >> 4) & 0x0F0F0F0Fu);
  const uint32_t r3 = ((a1 << 4) & 0xF0F0F0F0u) | (a3 & 0x0F0F0F0Fu);
  q[0] = (r0 & 0xCCCCCCCCu) | ((r1 >> 2) & 0x33333333u);
  q[1] = ((r0 << 2) & 0xCCCCCCCCu) | (r1 & 0x33333333u);
  q[2] = (r2 & 0xCCCCCCCCu) | ((r3 >> 2) & 0x33333333u);
  q[3] = ((r2 << 2) & 0xCCCCCCCCu) | (r3 & 0x33333333u);
}

// Flipping the top bit of every plane-0 field (0xAA pattern) turns each merged
// two's-complement byte b into the offset-binary byte u = b + 128.
constexpr uint32_t kSignFlip = 0xAAAAAAAAu;

// u (offset-binary byte L of q) -> exact float b = u - 128, via the 2^23 magic:
// float bits 0x4B0000uu == 2^23 + u.
template <int L>
__device__ __forceinline__ float byte_to_float(uint32_t q) {
  return __int_as_float(__byte_perm(q, 0x4B000000u, 0x7440u | L)) - 8388736.0f;
}

}  // namespace grinqh
