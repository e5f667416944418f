// Dense quantized GEMM for many rows in two passes, the reference's structure
// (grinqh/kernel.py:561-587: unpack, dtype(w * s), x @ w) with both passes on this
// library's kernels:
//   1. dequant_kernel turns the packed planes into W = dtype(w * s) [K, N] in the
//      original column order (HBM-bound: b/8 bytes read, 2 written per weight);
//   2. gemm_bf16_kernel computes y = x @ W on the tcgen05 tensor cores with both
//      operands loaded by TMA: warp 0 loads a 256 x 64 x tile (K-major) and four
//      64 x 64 boxes of W (128-byte swizzle, which is the MN-major operand layout)
//      per stage, warp 1 issues the MMAs from one thread (two M = 128 halves,
//      N = 256), warps 2-9 are the epilogue (tcgen05.ld, cast, bias, store).
// For many rows the dequantization is paid once per call while the fused kernel
// (gemm_tc.cu) converts every weight once per 256-row tile of x; above a few hundred
// rows the separate pass is cheaper. Both give dtype(w * s) bit for bit.
#include <cuda.h>

#include "common.cuh"
#include "gemm_bf16.cuh"
#include "ptx.cuh"

namespace grinqh {
namespace {

constexpr int BM = 256, BN = 256, BK = 64, STAGES = 3;
// Tile order: CTAs are launched in groups of kGroupM row tiles x every column tile,
// row tile fastest. A wave of one CTA per SM then reads a few row panels of x, each
// reused from L2 by all of its column tiles, instead of every row panel of x once per
// wave (qkv at M = 8192 read 3.7x its algorithmic bytes in row-tile-major order).
constexpr int kGroupM = 8;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kStageA = BM * BK * 2;  // 32 KB
constexpr uint32_t kStageB = BN * BK * 2;  // 32 KB
constexpr uint32_t kBoxB = 64 * BK * 2;    // one 64-column box of W: 8 KB
constexpr uint32_t kSmemBytes = STAGES * (kStageA + kStageB) + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kLboB = 8 * 1024;  // B: stride between 64-column MN atoms
constexpr uint32_t kSboB = 1024;      // B: stride between 8-row K groups
constexpr uint32_t kSboA = 1024;      // A: stride between 8-row M groups (128 B rows)

template <typename T> struct Fmt;
template <> struct Fmt<__nv_bfloat16> {
  static constexpr uint32_t v = 1;
  static constexpr CUtensorMapDataType tma = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <> struct Fmt<__half> {
  static constexpr uint32_t v = 0;
  static constexpr CUtensorMapDataType tma = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};

// ---------------------------------------------------------------- pass 1: dequantize
// Thread (chunk, pair): packed words 2p, 2p + 1 of kDqRows consecutive rows inside one
// scale group. The b/2 plane words of word j of row k hold the 16 codes of columns
// c * N/16 + j (c = 0..15), so the two words give, for every c, two neighbouring
// columns: one packed store per column pair, and the group's scales are loaded once
// as pairs. W[k, n] = dtype(code * s[k / group, n]).
constexpr int kDqRows = 8;

template <int NZ, typename T>
__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ w, const T* __restrict__ s,
                                                      T* __restrict__ out, int K, int N, int group) {
  constexpr int kShift = 8 - 2 * NZ;
  // byte u (offset binary, code = u - 128, shifted left by 8 - b) -> u / 2^shift plus
  // 2^(23-shift) exactly: the float with bits 0x4B000000 - (shift << 23) | u
  constexpr uint32_t kMagicBits = 0x4B000000u - ((uint32_t)kShift << 23);
  constexpr float kMagic = (float)(8388608.0 + 128.0) / float(1 << kShift);
  const int n16 = N >> 4;          // even (N % 32 == 0)
  const int pairs = n16 >> 1;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= pairs) return;
  const int j = 2 * p;
  const int k0 = blockIdx.y * kDqRows;
  if (k0 >= K) return;
  const int k1 = min(K, k0 + kDqRows);  // kDqRows divides the group: one scale group
  const size_t row_words = (size_t)NZ * n16;
  // scales of the two columns of every column group, and the exact fused-multiply-add
  // addends -(2^23 + 128) * s / 2^shift (bf16 scales have 8 significant bits)
  float2 sc[16], sn[16];
  {
    const uint32_t* sp = reinterpret_cast<const uint32_t*>(s + (size_t)(k0 / group) * N + j);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint32_t bits = __ldg(sp + (size_t)c * (n16 >> 1));
      if constexpr (Act<T>::kBf16) {
        sc[c] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bits));
      } else {
        sc[c] = __half22float2(*reinterpret_cast<const __half2*>(&bits));
      }
      sn[c] = make_float2(-kMagic * sc[c].x, -kMagic * sc[c].y);
    }
  }
  const uint32_t* wp = w + (size_t)k0 * row_words + j;
  T* op = out + (size_t)k0 * N + j;
#pragma unroll 2
  for (int k = k0; k < k1; ++k, wp += row_words, op += N) {
    uint2 P[4];
#pragma unroll
    for (int z = 0; z < 4; ++z)
      P[z] = z < NZ ? __ldcs(reinterpret_cast<const uint2*>(wp + (size_t)z * n16)) : make_uint2(0u, 0u);
    uint32_t qa[4], qb[4];
    merge_planes(P[0].x ^ kSignFlip, P[1].x, P[2].x, P[3].x, qa);
    merge_planes(P[0].y ^ kSignFlip, P[1].y, P[2].y, P[3].y, qb);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int L = 0; L < 4; ++L) {
        const int c = 4 * i + L;
        const uint32_t sel = 0x7440u | (uint32_t)L;
        const float2 f = make_float2(__int_as_float(__byte_perm(qa[i], kMagicBits, sel)),
                                     __int_as_float(__byte_perm(qb[i], kMagicBits, sel)));
        // code * s exactly in fp32, rounded once to the activation dtype (kernel.py:586)
        float2 v;
        if constexpr (Act<T>::kBf16) {
          v = __ffma2_rn(f, sc[c], sn[c]);
        } else {
          v = __fmul2_rn(__fadd2_rn(f, make_float2(-kMagic, -kMagic)), sc[c]);
        }
        uint32_t packed;
        if constexpr (Act<T>::kBf16) {
          __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
          packed = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(v.x, v.y);
          packed = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint32_t*>(op + (size_t)c * n16) = packed;
      }
  }
}

// ---------------------------------------------------------------- pass 2: x @ W
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// TI: operand type of x and W (bf16 / fp16); TO: output type (the activation dtype)
template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads, 1) gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                  const __grid_constant__ CUtensorMap tmap_w,
                                                                  const Bf16GemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + STAGES * kStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * (kStageA + kStageB));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's (row tile, column tile) in the grouped order; gridDim.x x gridDim.y tiles
  int mt, nt;
  {
    const int mtiles = (int)gridDim.x, ntiles = (int)gridDim.y;
    const int t = (int)(blockIdx.y * gridDim.x + blockIdx.x);
    const int g = t / (kGroupM * ntiles), r = t % (kGroupM * ntiles);
    const int gm = min(kGroupM, mtiles - g * kGroupM);  // row tiles in this group
    mt = g * kGroupM + r % gm;
    nt = r / gm;
  }
  const int m0 = mt * BM;
  const int n0 = nt * BN;
  // K steps of this split (blockIdx.z of a.splits; the planner leaves none empty)
  const int nk_all = a.K / BK;
  const int per = (nk_all + a.splits - 1) / a.splits;
  const int q_begin = blockIdx.z * per;
  const int nk = max(0, min(nk_all, q_begin + per) - q_begin);
  const unsigned* active = a.active;
  const size_t act_base = (size_t)mt * nk_all + q_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      prefetch_tmap(&tmap_w);
      int qa = 0;  // K steps loaded so far (steps without an active row are skipped)
      for (int q = 0; q < nk; ++q) {
        if (active && active[act_base + q] == 0u) continue;
        const int s = qa % STAGES;
        if (qa >= STAGES) mbar_wait(&empty[s], ((qa / STAGES) - 1) & 1);
        mbar_arrive_expect_tx(&full[s], kStageA + kStageB);
        tma_load_2d(sA + s * kStageA, &tmap_x, (q_begin + q) * BK, m0, &full[s]);
#pragma unroll
        for (int b = 0; b < BN / 64; ++b)
          tma_load_2d(sB + s * kStageB + b * kBoxB, &tmap_w, n0 + 64 * b, (q_begin + q) * BK, &full[s]);
        ++qa;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(1, Fmt<TI>::v, Fmt<TI>::v, 0, 1, BN, 128);
      int qa = 0;
      for (int q = 0; q < nk; ++q) {
        if (active && active[act_base + q] == 0u) continue;
        const int s = qa % STAGES;
        mbar_wait(&full[s], (qa / STAGES) & 1);
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * kStageA);
        const uint32_t b_base = smem_u32(sB + s * kStageB);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t bdesc = smem_desc(b_base + kk * 2 * kSboB, kLboB, kSboB, 2);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t adesc = smem_desc(a_base + h * 128 * 128 + kk * 32, 16, kSboA, 2);
            mma_f16_ss(tmem + h * BN, adesc, bdesc, idesc, (qa > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
        ++qa;
      }
      mma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // warp w reads TMEM lanes 32 * (w % 4) .. of accumulator half (w - 2) / 4: each
    // thread owns one output row and writes it in 64-byte runs of 32 columns
    mbar_wait(acc_full, 0);
    tc_fence_after();
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int m = m0 + half * 128 + quarter * 32 + lane;
    TO* y = static_cast<TO*>(a.y);
    const TO* bias = static_cast<const TO*>(a.bias);
    const float osc = a.out_scale ? *a.out_scale : 1.0f;
    // with skipped K steps, whether this split's accumulator was written at all
    bool any_mma = nk > 0;
    if (active) {
      bool any = false;
      for (int q = lane; q < nk; q += 32) any |= active[act_base + q] != 0u;
      any_mma = __any_sync(0xFFFFFFFFu, any);
    }
    // 8 columns (16 bytes of y) of row mm at a time: cast, bias, one 16-byte store
    auto store8 = [&](int mm, int n, const float* v) {
      uint32_t o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        TO lo = Act<TO>::from_f(v[2 * t] * osc);
        TO hi = Act<TO>::from_f(v[2 * t + 1] * osc);
        if (bias) {
          lo = Act<TO>::from_f(Act<TO>::to_f(lo) + Act<TO>::to_f(bias[n + 2 * t]));
          hi = Act<TO>::from_f(Act<TO>::to_f(hi) + Act<TO>::to_f(bias[n + 2 * t + 1]));
        }
        o[t] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
      }
      *reinterpret_cast<uint4*>(y + (size_t)mm * a.N + n) = make_uint4(o[0], o[1], o[2], o[3]);
    };
    const bool split = a.splits > 1;
#pragma unroll 1
    for (int cc = 0; cc < BN / 32; ++cc) {
      uint32_t r[32];
      if (any_mma) {
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + half * BN + cc * 32, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) r[t] = 0u;
      }
      if (m >= a.M) continue;
      const int nb = n0 + 32 * cc;
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // N is a multiple of 16, so runs of 8 are whole
        const int n = nb + 8 * e;
        if (n >= a.N) break;
        if (split) {  // this split's fp32 sums: slots[split][m][n]
          float4* dst = reinterpret_cast<float4*>(a.slots + ((size_t)blockIdx.z * a.M + m) * a.N + n);
          __stcg(dst, make_float4(__uint_as_float(r[8 * e]), __uint_as_float(r[8 * e + 1]), __uint_as_float(r[8 * e + 2]),
                                  __uint_as_float(r[8 * e + 3])));
          __stcg(dst + 1, make_float4(__uint_as_float(r[8 * e + 4]), __uint_as_float(r[8 * e + 5]),
                                      __uint_as_float(r[8 * e + 6]), __uint_as_float(r[8 * e + 7])));
        } else {
          float v[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) v[t] = __uint_as_float(r[8 * e + t]);
          store8(m, n, v);
        }
      }
    }
    if (split) {
      // Split-K fix-up, shared by the tile's splits: each one arrives on the tile's
      // ticket, waits until every split has written its sums (the grid is launched
      // cooperatively, so they are all resident; the wait is bounded), then adds
      // its share of the tile's rows over the splits in split order and stores them.
      // A second count on the same ticket lets the last one reset it.
      constexpr int kEpiThreads = 32 * kEpiWarps;
      const int et = threadIdx.x - 64;  // 0 .. kEpiThreads - 1
      unsigned* ticket = a.counters + mt * gridDim.y + nt;
      __threadfence();
      named_barrier(1, kEpiThreads);
      if (et == 0) {
        atomicAdd(ticket, 1u);
        if (ld_acquire_gpu(ticket) < (unsigned)a.splits) {
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t it = 1;; ++it) {
            __nanosleep(128);
            if (ld_acquire_gpu(ticket) >= (unsigned)a.splits) break;
            if ((it & 255u) == 0) {
              if (*reinterpret_cast<volatile unsigned*>(&g_wait_timeouts) != 0u) break;
              if (globaltimer_ns() - t0 > kWaitNs) {
                atomicAdd(&g_wait_timeouts, 1u);
                break;
              }
            }
          }
        }
      }
      named_barrier(1, kEpiThreads);
      __threadfence();
      const int rows = min(BM, a.M - m0);
      const int r0 = (int)((int64_t)rows * blockIdx.z / a.splits);
      const int r1 = (int)((int64_t)rows * (blockIdx.z + 1) / a.splits);
      const int chunks = min(BN, a.N - n0) / 8;  // 8-column runs of this tile
      for (int i = et; i < (r1 - r0) * chunks; i += kEpiThreads) {
        const int mm = m0 + r0 + i / chunks;
        const int n = n0 + 8 * (i % chunks);
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int z = 0; z < a.splits; ++z) {
          const float4* src = reinterpret_cast<const float4*>(a.slots + ((size_t)z * a.M + mm) * a.N + n);
          const float4 p0 = __ldcg(src), p1 = __ldcg(src + 1);
          v[0] += p0.x; v[1] += p0.y; v[2] += p0.z; v[3] += p0.w;
          v[4] += p1.x; v[5] += p1.y; v[6] += p1.z; v[7] += p1.w;
        }
        store8(mm, n, v);
      }
      named_barrier(1, kEpiThreads);
      if (et == 0 && atomicAdd(ticket, 1u) == 2u * a.splits - 1u) *ticket = 0u;  // ready for the next launch
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// y = x @ W on the tensor cores: x [M, a.K] and W = a.wbuf [a.K, N] of operand type TI,
// y of type TO (a.splits K splits, a.active / a.out_scale as set).
template <typename TI, typename TO>
int launch_gemm_pass(const Bf16GemmArgs& a, cudaStream_t st) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint32_t estride[2] = {1, 1};
  CUtensorMap tmap_x, tmap_w;
  {
    const cuuint64_t gdim[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
    const cuuint64_t gstride[1] = {(cuuint64_t)a.K * 2};
    const cuuint32_t box[2] = {BK, BM};
    const CUresult r = enc(&tmap_x, Fmt<TI>::tma, 2, const_cast<void*>(a.x), gdim, gstride, box, estride,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled(x) failed (%d)", (int)r);
  }
  {
    // W [K, N]: boxes of 64 columns (128 bytes) x 64 rows with the 128-byte swizzle,
    // which is the MN-major operand layout (8-row K groups of 1 KB, 64-column atoms)
    const cuuint64_t gdim[2] = {(cuuint64_t)a.N, (cuuint64_t)a.K};
    const cuuint64_t gstride[1] = {(cuuint64_t)a.N * 2};
    const cuuint32_t box[2] = {64, BK};
    const CUresult r = enc(&tmap_w, Fmt<TI>::tma, 2, a.wbuf, gdim, gstride, box, estride,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled(w) failed (%d)", (int)r);
  }
  auto kern = gemm_bf16_kernel<TI, TO>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const dim3 grid((unsigned)((a.M + BM - 1) / BM), (unsigned)((a.N + BN - 1) / BN), (unsigned)a.splits);
  if (a.splits <= 1) {
    kern<<<grid, kThreads, kSmemBytes, st>>>(tmap_x, tmap_w, a);
    return check_launch("gemm_bf16");
  }
  // The splits of a tile wait for one another in the fix-up, so every CTA of the grid
  // must be resident at once. A cooperative launch guarantees that (the planner keeps
  // the grid within one CTA per SM), also when kernels of other streams hold SMs; a
  // grid that could not be co-resident fails to launch instead of waiting.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e2 = cudaLaunchKernelEx(&cfg, kern, tmap_x, tmap_w, a);
  if (e2 != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "gemm_bf16 (split-K) launch: %s", cudaGetErrorString(e2));
  return check_launch("gemm_bf16");
}

template <int NZ, typename T>
int launch_t(const Bf16GemmArgs& a, cudaStream_t st) {
  // pass 1
  {
    const int pairs = a.N / 32;
    const dim3 grid((unsigned)((pairs + 127) / 128), (unsigned)((a.K + kDqRows - 1) / kDqRows));
    dequant_kernel<NZ, T><<<grid, 128, 0, st>>>(a.w, static_cast<const T*>(a.s), static_cast<T*>(a.wbuf), a.K, a.N,
                                                a.group);
    GRINQH_RETURN_IF(check_launch("dequant"));
  }
  // pass 2
  return launch_gemm_pass<T, T>(a, st);
}

}  // namespace

unsigned take_bf16_gemm_timeouts() {
  unsigned v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof(z));
  return v;
}

bool bf16_gemm_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* w, const void* s,
                         const void* y) {
  // TMA needs 16-byte aligned bases and row pitches (K, N multiples of 8), whole 64-deep
  // K steps; the epilogue stores 16-byte runs (N a multiple of 16, y 16-byte aligned)
  // the dequantization pass takes pairs of words (N % 32) and 32-row chunks of one
  // scale group (group % 32, checked by the caller's validation)
  (void)group;
  return M >= 1 && K % BK == 0 && N % 32 == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(w) % 8) == 0 && (reinterpret_cast<uintptr_t>(s) % 4) == 0 &&
         (reinterpret_cast<uintptr_t>(y) % 16) == 0 && K < (1LL << 31) && N < (1LL << 31);
}

size_t bf16_gemm_buffer_bytes(int64_t K, int64_t N) { return (size_t)K * (size_t)N * 2; }

int bf16_gemm_splits(int64_t M, int64_t K, int64_t N, int sm_count) {
  // one CTA per SM (about 197 KB of shared memory): split K when the output tiles
  // leave most SMs idle, keeping at least 4 K steps per split, no split empty and the
  // whole grid within one wave (the splits of a tile wait for each other)
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int64_t nk = K / BK;
  const int64_t sms = sm_count > 0 ? sm_count : 148;
  // the fix-up writes and re-reads splits x M x N fp32 sums: with a quarter of the SMs
  // busy already and short K (under 128 steps) that costs more than it saves (B200:
  // 4096 x 6144 at M = 512, 4096 x 4096 at M = 1024)
  if (tiles > sms / 4 && nk < 128) return 1;
  int64_t splits = sms / (tiles > 0 ? tiles : 1);
  if (splits > nk / 4) splits = nk / 4;
  if (splits < 1) splits = 1;
  const int64_t per = (nk + splits - 1) / splits;
  splits = (nk + per - 1) / per;
  return (int)splits;
}

size_t bf16_gemm_slot_bytes(int64_t M, int64_t N, int splits) {
  return splits > 1 ? (size_t)splits * (size_t)M * (size_t)N * sizeof(float) : 0;
}

int launch_bf16_gemm(const Bf16GemmArgs& a, int dtype, int nz, cudaStream_t st) {
  if (dtype == GRINQH_BF16) {
    switch (nz) {
      case 1: return launch_t<1, __nv_bfloat16>(a, st);
      case 2: return launch_t<2, __nv_bfloat16>(a, st);
      case 3: return launch_t<3, __nv_bfloat16>(a, st);
      default: return launch_t<4, __nv_bfloat16>(a, st);
    }
  }
  switch (nz) {
    case 1: return launch_t<1, __half>(a, st);
    case 2: return launch_t<2, __half>(a, st);
    case 3: return launch_t<3, __half>(a, st);
    default: return launch_t<4, __half>(a, st);
  }
}


// ---------------------------------------------------------------- graded prefill
// Every row graded by its own activations (the reference's one-row GEMV applied row by
// row, grinqh/kernel.py:100-158), for many rows, on the tensor cores. For element
// (m, k) with active zones Z, the reference adds s * x * (w_Z + bias(Z)) with
// w_Z = int8(byte & zone bits) >> shift and bias(Z) = sum_{z in Z} Delta_z. Both are
// sums over the active zones: w_Z = sum_{z in Z} D_z / 2^shift with D_0 the signed top
// bit pair * 64 and D_z = (bit pair z) * 4^(3-z), so
//   y[m, n] = sum_z sum_k A_z[m, k] B_z[k, n],
//   A_z[m, k] = x[m, k] if |x[m, k]| > t_z else 0,
//   B_z[k, n] = s[k / g, n] * (D_z + Delta_z 2^shift) / 2^shift,
// one GEMM over K' = (b/2) K. (D_z + Delta_z 2^shift) is 2^p times an odd number below 4
// (or 0), so B_z has at most 10 significant bits: exact in fp16 (not in bf16). Both
// operands are scaled by powers of two into fp16's range (x's largest |x| near 2^14, the
// largest |B| below 2^15) and the sums scaled back in the GEMM's epilogue.
namespace {

constexpr size_t kGradedHead = 16 << 10;  // split-K tickets; then 3 words of scaling; then the step flags

__device__ __forceinline__ void atomic_max_pos(unsigned* p, float v) {
  // non-negative floats order like their bit patterns
  atomicMax(p, __float_as_uint(v));
}

// scal[0] = bits of max |x| (finite), scal[1] = bits of max |s| (finite)
template <typename T>
__global__ void __launch_bounds__(256) graded_max_kernel(const T* __restrict__ x, size_t nx, const T* __restrict__ s,
                                                         size_t ns, unsigned* scal) {
  float mx = 0.f, ms = 0.f;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nx; i += stride) {
    const float v = fabsf(Act<T>::to_f(x[i]));
    if (v < INFINITY) mx = fmaxf(mx, v);
  }
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < ns; i += stride) {
    const float v = fabsf(Act<T>::to_f(s[i]));
    if (v < INFINITY) ms = fmaxf(ms, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    ms = fmaxf(ms, __shfl_xor_sync(0xFFFFFFFFu, ms, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomic_max_pos(scal, mx);
    atomic_max_pos(scal + 1, ms);
  }
}

__device__ __forceinline__ int exp_for(unsigned bits, int top) {  // 2^e puts the max below 2^top
  const float m = __uint_as_float(bits);
  if (!(m > 0.f) || !(m < INFINITY)) return 0;
  return max(-60, min(60, ilogbf(m) - (top - 1)));
}

// A_z = fp16(x * 2^-eA) where |x| > t_z, else 0, for the zones z < NZ: row m of A' holds
// [A_0 | A_1 | ...] (NZ K columns). flags[(m / 256) * nk' + k' / 64] = 1 where a 64-deep
// step of a 256-row tile has a non-zero value. Thread: 8 consecutive k of one row.
template <int NZ, typename T>
__global__ void __launch_bounds__(256) graded_a_kernel(const T* __restrict__ x, int M, int K, float t0, float t1,
                                                       float t2, float t3, unsigned* scal, __half* __restrict__ A,
                                                       unsigned* flags) {
  const int per_row = K / 8;
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int eA = exp_for(scal[0], 14);
  if (idx == 0) {  // the GEMM's output scale 2^(eA + eB)
    const int eB = exp_for(scal[1], 8);  // |B| <= 128 max|s| < 2^15
    reinterpret_cast<float*>(scal)[2] = ldexpf(1.0f, eA + eB);
  }
  if (idx >= (size_t)M * per_row) return;
  const int m = (int)(idx / per_row), k = (int)(idx % per_row) * 8;
  const float down = ldexpf(1.0f, -eA);
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * K + k));
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
  float xf[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint16_t bits = (uint16_t)(wv[e >> 1] >> (16 * (e & 1)));
    xf[e] = Act<T>::to_f(*reinterpret_cast<const T*>(&bits));
  }
  const float th[4] = {t0, t1, t2, t3};
  const int nk = NZ * K / 64;
#pragma unroll
  for (int z = 0; z < NZ; ++z) {
    uint32_t o[4];
    bool any = false;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      // fp32 |x| > t_z, strict; NaN is never active (kernel.py:100-116)
      const float a0 = fabsf(xf[e]) > th[z] ? xf[e] * down : 0.f;
      const float a1 = fabsf(xf[e + 1]) > th[z] ? xf[e + 1] * down : 0.f;
      any |= (a0 != 0.f) | (a1 != 0.f);
      __half2 h = __floats2half2_rn(a0, a1);
      o[e / 2] = *reinterpret_cast<uint32_t*>(&h);
    }
    const size_t col = (size_t)z * K + k;
    *reinterpret_cast<uint4*>(A + (size_t)m * NZ * K + col) = make_uint4(o[0], o[1], o[2], o[3]);
    if (any) flags[(size_t)(m / 256) * nk + col / 64] = 1u;
  }
}

// B_z[k, n] = fp16(s[k / g, n] * (D_z + Delta_z 2^shift) / 2^shift * 2^-eB) for z < NZ,
// rows z K + k of B' [NZ K, N] in the original column order. Thread: the packed words
// 2p, 2p + 1 of kDqRows consecutive rows of one scale group (as dequant_kernel).
template <int NZ, typename T>
__global__ void __launch_bounds__(128) graded_b_kernel(const uint32_t* __restrict__ w, const T* __restrict__ s,
                                                       const unsigned* scal, __half* __restrict__ B, int K, int N,
                                                       int group) {
  constexpr int kShift = 8 - 2 * NZ;
  const int n16 = N >> 4;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= (n16 >> 1)) return;
  const int j = 2 * p;
  const int k0 = blockIdx.y * kDqRows;
  if (k0 >= K) return;
  const int k1 = min(K, k0 + kDqRows);
  const size_t row_words = (size_t)NZ * n16;
  // per zone: (D_z + Delta_z 2^shift) = coef_z(field) * 2^p_z, taken from the byte below;
  // Delta_z = B_z - B_{z-1}, B_z = 2^(b-1) >> (2z + 2) (kernel.py:73-82)
  int delta[4];
  {
    const int base = 1 << (2 * NZ - 1);
    int prev = 0;
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const int bz = base >> (2 * z + 2);
      delta[z] = bz - prev;
      prev = bz;
    }
  }
  const float post = ldexpf(1.0f, -kShift - exp_for(scal[1], 8));  // 2^-shift * 2^-eB
  float2 sc[16];
  {
    const uint32_t* sp = reinterpret_cast<const uint32_t*>(s + (size_t)(k0 / group) * N + j);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint32_t bits = __ldg(sp + (size_t)c * (n16 >> 1));
      if constexpr (Act<T>::kBf16) {
        sc[c] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bits));
      } else {
        sc[c] = __half22float2(*reinterpret_cast<const __half2*>(&bits));
      }
      sc[c].x *= post;  // exact: a power of two
      sc[c].y *= post;
    }
  }
  const uint32_t* wp = w + (size_t)k0 * row_words + j;
  for (int k = k0; k < k1; ++k, wp += row_words) {
    uint2 P[4];
#pragma unroll
    for (int z = 0; z < 4; ++z)
      P[z] = z < NZ ? __ldcs(reinterpret_cast<const uint2*>(wp + (size_t)z * n16)) : make_uint2(0u, 0u);
    uint32_t qa[4], qb[4];
    // plain merge (no sign flip): the bytes are the shifted two's-complement codes
    merge_planes(P[0].x, P[1].x, P[2].x, P[3].x, qa);
    merge_planes(P[0].y, P[1].y, P[2].y, P[3].y, qb);
#pragma unroll
    for (int z = 0; z < NZ; ++z) {
      __half* op = B + ((size_t)z * K + k) * N + j;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int L = 0; L < 4; ++L) {
          const int c = 4 * i + L;
          const int ba = (int)((qa[i] >> (8 * L)) & 0xFFu), bb = (int)((qb[i] >> (8 * L)) & 0xFFu);
          // D_z: the signed top bit pair * 64 for z = 0, bit pair z * 4^(3-z) otherwise
          const int da = z == 0 ? ((int)(int8_t)ba >> 6) * 64 : ((ba >> (6 - 2 * z)) & 3) << (6 - 2 * z);
          const int db = z == 0 ? ((int)(int8_t)bb >> 6) * 64 : ((bb >> (6 - 2 * z)) & 3) << (6 - 2 * z);
          const int ea = da + (delta[z] << kShift), eb = db + (delta[z] << kShift);
          __half2 h = __floats2half2_rn((float)ea * sc[c].x, (float)eb * sc[c].y);
          *reinterpret_cast<__half2*>(op + (size_t)c * n16) = h;
        }
    }
  }
}

template <int NZ, typename T>
int launch_graded_t(const Bf16GemmArgs& a, const float* th, void* ws, int sms, cudaStream_t st) {
  char* base = static_cast<char*>(ws);
  const int nkp = NZ * a.K / BK;  // 64-deep steps of K'
  const int mtiles = (a.M + BM - 1) / BM;
  unsigned* counters = reinterpret_cast<unsigned*>(base);
  unsigned* scal = reinterpret_cast<unsigned*>(base + kGradedHead);
  unsigned* flags = scal + 4;
  const size_t head = kGradedHead + 16 + (size_t)mtiles * nkp * 4;
  __half* A = reinterpret_cast<__half*>(base + (head + 255) / 256 * 256);
  const size_t a_bytes = (size_t)a.M * NZ * a.K * 2;
  __half* Bw = reinterpret_cast<__half*>(reinterpret_cast<char*>(A) + (a_bytes + 255) / 256 * 256);
  const size_t b_bytes = (size_t)NZ * a.K * a.N * 2;
  float* slots = reinterpret_cast<float*>(reinterpret_cast<char*>(Bw) + (b_bytes + 255) / 256 * 256);
  cudaError_t e = cudaMemsetAsync(base, 0, head, st);  // tickets, scaling, flags
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  graded_max_kernel<T><<<sms * 4, 256, 0, st>>>(static_cast<const T*>(a.x), (size_t)a.M * a.K,
                                                  static_cast<const T*>(a.s), (size_t)(a.K / a.group) * a.N, scal);
  GRINQH_RETURN_IF(check_launch("graded max"));
  {
    const size_t threads = (size_t)a.M * (a.K / 8);
    graded_a_kernel<NZ, T><<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        static_cast<const T*>(a.x), a.M, a.K, th[0], th[1], th[2], th[3], scal, A, flags);
    GRINQH_RETURN_IF(check_launch("graded A"));
  }
  {
    const int pairs = a.N / 32;
    const dim3 grid((unsigned)((pairs + 127) / 128), (unsigned)((a.K + kDqRows - 1) / kDqRows));
    graded_b_kernel<NZ, T><<<grid, 128, 0, st>>>(a.w, static_cast<const T*>(a.s), scal, Bw, a.K, a.N, a.group);
    GRINQH_RETURN_IF(check_launch("graded B"));
  }
  Bf16GemmArgs g = a;
  g.x = A;
  g.K = NZ * a.K;
  g.wbuf = Bw;
  g.splits = bf16_gemm_splits(a.M, g.K, a.N, sms);
  g.counters = counters;
  g.slots = slots;
  g.active = flags;
  g.out_scale = reinterpret_cast<const float*>(scal) + 2;
  return launch_gemm_pass<__half, T>(g, st);
}

}  // namespace

bool graded_gemm_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* w, const void* s,
                           const void* y) {
  return bf16_gemm_supported(M, K, N, group, x, w, s, y) && K % 8 == 0 && group % kDqRows == 0;
}

size_t graded_gemm_workspace(int64_t M, int64_t K, int64_t N, int nz, int sm_count) {
  const int64_t nkp = nz * K / BK, mtiles = (M + BM - 1) / BM;
  const size_t head = kGradedHead + 16 + (size_t)mtiles * nkp * 4;
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  const int splits = bf16_gemm_splits(M, nz * K, N, sm_count);
  return up(head) + up((size_t)M * nz * K * 2) + up((size_t)nz * K * N * 2) +
         up(bf16_gemm_slot_bytes(M, N, splits));
}

int launch_graded_gemm(const Bf16GemmArgs& a, const float* th, void* ws, int dtype, int nz, int sms,
                       cudaStream_t st) {
  if (dtype == GRINQH_BF16) {
    switch (nz) {
      case 1: return launch_graded_t<1, __nv_bfloat16>(a, th, ws, sms, st);
      case 2: return launch_graded_t<2, __nv_bfloat16>(a, th, ws, sms, st);
      case 3: return launch_graded_t<3, __nv_bfloat16>(a, th, ws, sms, st);
      default: return launch_graded_t<4, __nv_bfloat16>(a, th, ws, sms, st);
    }
  }
  switch (nz) {
    case 1: return launch_graded_t<1, __half>(a, th, ws, sms, st);
    case 2: return launch_graded_t<2, __half>(a, th, ws, sms, st);
    case 3: return launch_graded_t<3, __half>(a, th, ws, sms, st);
    default: return launch_graded_t<4, __half>(a, th, ws, sms, st);
  }
}

}  // namespace grinqh
