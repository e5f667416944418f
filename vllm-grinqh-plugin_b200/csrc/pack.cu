// Load-time weight codec (pack / unpack) and the activation grading kernel.
//
// Layout restated from the reference (grinqh/utils.py:100-122): for shifted code
// words a (K, N/4) -- 4 code bytes per word, codes in the MSBs -- the packed row is
// b/2 planes of N/16 words; plane z word j holds, in byte lane L at bits
// (7-2i, 6-2i), bits (7-2z, 6-2z) of byte L of word 4j+i.
#include "common.cuh"

namespace grinqh {
namespace {

// One thread per (row k, output word column j): reads the four words 4j..4j+3
// (one 16-byte load) and writes one word per plane.
template <int NZ>
__global__ void pack_words_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                  int64_t K, int64_t n_words) {
  const int64_t n_zone = n_words / 4;
  const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (j >= n_zone) return;
  for (int64_t k = blockIdx.y; k < K; k += gridDim.y) {
  const uint4 a = *reinterpret_cast<const uint4*>(in + k * n_words + 4 * j);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
  uint32_t* orow = out + k * (NZ * n_zone);
#pragma unroll
  for (int z = 0; z < NZ; ++z) {
    uint32_t acc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc |= ((w[i] >> (6 - 2 * z)) & 0x03030303u) << (6 - 2 * i);
    orow[z * n_zone + j] = acc;
  }
  }
}

// Fused preshuffle + shift + pack from signed int8 codes (grinqh/grinqh.py:202-211).
// Preshuffled column 16j + 4i + L is original column (4i + L) * (N/16) + j
// (grinqh/utils.py:17-22), so thread (k, j) gathers the 16 codes j + c*N/16.
template <int NZ>
__global__ void pack_codes_kernel(const int8_t* __restrict__ codes, int64_t ld, uint32_t* __restrict__ out,
                                  int64_t K, int64_t N) {
  constexpr int kShift = 8 - 2 * NZ;
  const int64_t n16 = N / 16;
  const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (j >= n16) return;
  for (int64_t k = blockIdx.y; k < K; k += gridDim.y) {
  const int8_t* crow = codes + k * ld;
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t word = 0;
#pragma unroll
    for (int L = 0; L < 4; ++L) {
      const uint32_t byte = ((uint32_t)(uint8_t)crow[(4 * i + L) * n16 + j] << kShift) & 0xFFu;
      word |= byte << (8 * L);
    }
    w[i] = word;
  }
  uint32_t* orow = out + k * (NZ * n16);
#pragma unroll
  for (int z = 0; z < NZ; ++z) {
    uint32_t acc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc |= ((w[i] >> (6 - 2 * z)) & 0x03030303u) << (6 - 2 * i);
    orow[z * n16 + j] = acc;
  }
  }
}

// unpack_pyt (grinqh/utils.py:149-177): word 4j+i = sum over planes z of
// ((plane_z[j] >> (6-2i)) & 0x03030303) << 2(NZ-1-z).
template <int NZ>
__global__ void unpack_kernel(const uint32_t* __restrict__ packed, uint32_t* __restrict__ out,
                              int64_t K, int64_t N) {
  const int64_t n16 = N / 16;
  const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (j >= n16) return;
  for (int64_t k = blockIdx.y; k < K; k += gridDim.y) {
  const uint32_t* prow = packed + k * (NZ * n16);
  uint32_t p[NZ];
#pragma unroll
  for (int z = 0; z < NZ; ++z) p[z] = prow[z * n16 + j];
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t acc = 0;
#pragma unroll
    for (int z = 0; z < NZ; ++z) acc |= ((p[z] >> (6 - 2 * i)) & 0x03030303u) << (2 * (NZ - 1 - z));
    w[i] = acc;
  }
  *reinterpret_cast<uint4*>(out + k * (N / 4) + 4 * j) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Grade: bit z of mask iff fp32|x| > t_z, z < nz (grinqh/kernel.py:100-116).
// One thread per column k walks the M rows so the union is a register OR.
template <typename T>
__global__ void grade_kernel(const T* __restrict__ x, int64_t M, int64_t K, float t0, float t1, float t2,
                             float t3, int nz, uint8_t* __restrict__ masks, uint8_t* __restrict__ uni) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= K) return;
  uint32_t u = 0;
  for (int64_t m = 0; m < M; ++m) {
    const float a = fabsf(Act<T>::to_f(x[m * K + k]));
    uint32_t g = (uint32_t)(a > t0) | ((uint32_t)(a > t1) << 1) | ((uint32_t)(a > t2) << 2) |
                 ((uint32_t)(a > t3) << 3);
    g &= (1u << nz) - 1u;
    u |= g;
    if (masks) masks[m * K + k] = (uint8_t)g;
  }
  if (uni) uni[k] = (uint8_t)u;
}

}  // namespace
}  // namespace grinqh

using namespace grinqh;

extern "C" int grinqh_pack_words(const uint32_t* words, uint32_t* out, int64_t K, int64_t n_words,
                                 int max_bits, grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(words && out, "null pointer");
  GRINQH_REQUIRE(K >= 0 && n_words >= 0 && n_words % 4 == 0, "n_words must be a multiple of 4 (got %lld)", (long long)n_words);
  GRINQH_REQUIRE(aligned(words, 16) && aligned(out, 4), "words must be 16-byte aligned");
  if (K == 0 || n_words == 0) return GRINQH_OK;
  const int64_t n_zone = n_words / 4;
  const dim3 block(128), grid((unsigned)((n_zone + 127) / 128), (unsigned)(K < 65535 ? K : 65535));
  switch (max_bits) {
    case 2: pack_words_kernel<1><<<grid, block, 0, stream>>>(words, out, K, n_words); break;
    case 4: pack_words_kernel<2><<<grid, block, 0, stream>>>(words, out, K, n_words); break;
    case 6: pack_words_kernel<3><<<grid, block, 0, stream>>>(words, out, K, n_words); break;
    default: pack_words_kernel<4><<<grid, block, 0, stream>>>(words, out, K, n_words); break;
  }
  return check_launch("pack_words");
}

extern "C" int grinqh_pack_codes(const int8_t* codes, int64_t ld, uint32_t* out, int64_t K, int64_t N,
                                 int max_bits, grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(codes && out, "null pointer");
  GRINQH_REQUIRE(K >= 0 && N >= 0 && N % 16 == 0, "N must be divisible by 16 for this layout (got %lld)", (long long)N);
  GRINQH_REQUIRE(ld >= N, "ld (%lld) < N (%lld)", (long long)ld, (long long)N);
  if (K == 0 || N == 0) return GRINQH_OK;
  const int64_t n16 = N / 16;
  const dim3 block(128), grid((unsigned)((n16 + 127) / 128), (unsigned)(K < 65535 ? K : 65535));
  switch (max_bits) {
    case 2: pack_codes_kernel<1><<<grid, block, 0, stream>>>(codes, ld, out, K, N); break;
    case 4: pack_codes_kernel<2><<<grid, block, 0, stream>>>(codes, ld, out, K, N); break;
    case 6: pack_codes_kernel<3><<<grid, block, 0, stream>>>(codes, ld, out, K, N); break;
    default: pack_codes_kernel<4><<<grid, block, 0, stream>>>(codes, ld, out, K, N); break;
  }
  return check_launch("pack_codes");
}

extern "C" int grinqh_unpack(const uint32_t* packed, uint8_t* out, int64_t K, int64_t N, int max_bits,
                             grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(packed && out, "null pointer");
  GRINQH_REQUIRE(K >= 0 && N >= 0 && N % 16 == 0, "N must be divisible by 16 (got %lld)", (long long)N);
  GRINQH_REQUIRE(aligned(out, 16) && aligned(packed, 4), "out must be 16-byte aligned");
  if (K == 0 || N == 0) return GRINQH_OK;
  const int64_t n16 = N / 16;
  const dim3 block(128), grid((unsigned)((n16 + 127) / 128), (unsigned)(K < 65535 ? K : 65535));
  uint32_t* o = reinterpret_cast<uint32_t*>(out);
  switch (max_bits) {
    case 2: unpack_kernel<1><<<grid, block, 0, stream>>>(packed, o, K, N); break;
    case 4: unpack_kernel<2><<<grid, block, 0, stream>>>(packed, o, K, N); break;
    case 6: unpack_kernel<3><<<grid, block, 0, stream>>>(packed, o, K, N); break;
    default: unpack_kernel<4><<<grid, block, 0, stream>>>(packed, o, K, N); break;
  }
  return check_launch("unpack");
}

extern "C" int grinqh_grade(const void* x, int dtype, int64_t M, int64_t K, const float* thresholds,
                            int max_bits, uint8_t* masks, uint8_t* uni, grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(x && thresholds && (masks || uni), "null pointer");
  GRINQH_REQUIRE(M >= 0 && K >= 0, "negative size");
  GRINQH_REQUIRE(dtype == GRINQH_BF16 || dtype == GRINQH_F16, "dtype must be GRINQH_BF16 or GRINQH_F16");
  if (K == 0) return GRINQH_OK;
  const dim3 block(256), grid((unsigned)((K + 255) / 256));
  const float* t = thresholds;
  if (dtype == GRINQH_BF16)
    grade_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), M, K, t[0], t[1],
                                                            t[2], t[3], max_bits / 2, masks, uni);
  else
    grade_kernel<__half><<<grid, block, 0, stream>>>(static_cast<const __half*>(x), M, K, t[0], t[1], t[2], t[3],
                                                     max_bits / 2, masks, uni);
  return check_launch("grade");
}
