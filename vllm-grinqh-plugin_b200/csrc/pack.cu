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


// Checkpoint -> staging codes (load time): the compressed-tensors pack-quantized
// weight (rows = output features, packed_dim 1: 32/b offset-binary fields per int32,
// LSB first along K; compressed_tensors .../pack_quantized/helpers.py unpack_from_int32)
// narrowed to rows [r0, r0 + rows) and columns [k0, k0 + k_local), transposed into
// dst[k * ld + n] as signed int8 codes. PF = fields per word; PF = 1 reads int8 codes
// directly (b = 6 checkpoints store the codes unpacked, grinqh/grinqh.py:131-132).
// A 64 x 64 tile goes through shared memory so that both the reads (along K) and the
// writes (along N) are contiguous.
constexpr int kCkTile = 64;

template <int B, int PF>
__global__ void __launch_bounds__(256) unpack_checkpoint_kernel(const void* __restrict__ src, int64_t src_ld,
                                                               int64_t r0, int64_t rows, int64_t k0,
                                                               int64_t k_local, int8_t* __restrict__ dst,
                                                               int64_t ld, bool vec_store) {
  __shared__ int8_t tile[kCkTile][kCkTile + 4];  // [k][n]
  const int64_t nb = blockIdx.x * (int64_t)kCkTile, kb = blockIdx.y * (int64_t)kCkTile;
  constexpr int kUnits = PF > 1 ? kCkTile / PF : kCkTile / 4;  // loads per tile row
  for (int t = threadIdx.x; t < kCkTile * kUnits; t += blockDim.x) {
    const int rr = t / kUnits, u = t % kUnits;
    const int64_t n = nb + rr;
    if (n >= rows) continue;
    if (PF > 1) {
      const int64_t kk0 = kb + (int64_t)u * PF;  // first column of this word within the rank slice
      if (kk0 >= k_local) continue;
      const uint32_t w =
          static_cast<const uint32_t*>(src)[(r0 + n) * src_ld + (k0 + kk0) / PF];  // k0 % PF == 0
#pragma unroll
      for (int i = 0; i < PF; ++i)
        if (kk0 + i < k_local)
          tile[u * PF + i][rr] = (int8_t)((int)((w >> (B * i)) & ((1u << B) - 1u)) - (1 << (B - 1)));
    } else {
      const int8_t* row = static_cast<const int8_t*>(src) + (r0 + n) * src_ld + k0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t kk = kb + 4 * u + i;
        if (kk < k_local) tile[4 * u + i][rr] = row[kk];
      }
    }
  }
  __syncthreads();
  // 16 threads per k row, 4 consecutive n each
  for (int t = threadIdx.x; t < kCkTile * (kCkTile / 4); t += blockDim.x) {
    const int kk = t / (kCkTile / 4), q = t % (kCkTile / 4);
    const int64_t k = kb + kk, n = nb + 4 * q;
    if (k >= k_local || n >= rows) continue;
    int8_t* o = dst + k * ld + n;
    if (vec_store && n + 4 <= rows) {
      *reinterpret_cast<char4*>(o) =
          make_char4(tile[kk][4 * q], tile[kk][4 * q + 1], tile[kk][4 * q + 2], tile[kk][4 * q + 3]);
    } else {
      for (int i = 0; i < 4 && n + i < rows; ++i) o[i] = tile[kk][4 * q + i];
    }
  }
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

extern "C" int grinqh_unpack_checkpoint(const void* src, int64_t src_ld, int max_bits, int64_t r0, int64_t rows,
                                        int64_t k0, int64_t k_local, int8_t* dst, int64_t ld,
                                        grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(src && dst, "null pointer");
  GRINQH_REQUIRE(r0 >= 0 && rows >= 0 && k0 >= 0 && k_local >= 0 && ld >= rows, "invalid slice");
  const int pf = max_bits == 6 ? 1 : 32 / max_bits;
  GRINQH_REQUIRE(k0 % (pf > 1 ? pf : 1) == 0, "k0 (%lld) must be a multiple of %d", (long long)k0, pf);
  GRINQH_REQUIRE(pf == 1 ? src_ld >= k0 + k_local : src_ld * pf >= k0 + k_local,
                 "source row of %lld elements is shorter than k0 + k_local", (long long)src_ld);
  if (rows == 0 || k_local == 0) return GRINQH_OK;
  const bool vec = aligned(dst, 4) && ld % 4 == 0;
  const dim3 grid((unsigned)((rows + kCkTile - 1) / kCkTile), (unsigned)((k_local + kCkTile - 1) / kCkTile));
  GRINQH_REQUIRE(grid.y <= 65535, "k_local too large");
  switch (max_bits) {
    case 2: unpack_checkpoint_kernel<2, 16><<<grid, 256, 0, stream>>>(src, src_ld, r0, rows, k0, k_local, dst, ld, vec); break;
    case 4: unpack_checkpoint_kernel<4, 8><<<grid, 256, 0, stream>>>(src, src_ld, r0, rows, k0, k_local, dst, ld, vec); break;
    case 6: unpack_checkpoint_kernel<8, 1><<<grid, 256, 0, stream>>>(src, src_ld, r0, rows, k0, k_local, dst, ld, vec); break;
    default: unpack_checkpoint_kernel<8, 4><<<grid, 256, 0, stream>>>(src, src_ld, r0, rows, k0, k_local, dst, ld, vec); break;
  }
  return check_launch("unpack_checkpoint");
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
