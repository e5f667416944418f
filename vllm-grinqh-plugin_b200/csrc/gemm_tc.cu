// Dense quantized GEMM on the 5th-generation tensor cores (tcgen05 / TMEM / TMA):
// y = x @ dtype(w * s) for many rows, the reference's M > 1 path
// (grinqh/kernel.py:561-587) without a materialised weight.
//
// One CTA computes a 256 x 256 tile of y (rows = tokens, columns = 16 packed words
// of 16 output columns each) over K in steps of 64:
//   warp 0      TMA producer: the 256 x 64 activation tile, 128-byte swizzled,
//               K-major (operand A);
//   warp 1      allocates 512 TMEM columns and issues the MMAs from one thread:
//               per 16-deep K slice two tcgen05.mma kind::f16 (M = 128 halves of the
//               tile, N = 256) into two fp32 accumulators, then tcgen05.commit
//               frees the stage;
//   warps 2-9   converters: load the planes of 64 rows x 16 words, merge them into
//               codes, multiply by the group scale and round to the activation dtype
//               -- bit for bit the reference's dtype(w * s) -- and store the 256 x 64
//               weight tile MN-major, 128-byte swizzled (operand B): a lane's 16
//               columns of one row are 32 contiguous bytes, so no transpose is needed.
//               After the K loop they are the epilogue: tcgen05.ld of the
//               accumulators, cast, bias, store.
// Three stages of A + B (64 KB each) are in flight; every mbarrier wait is bounded.
#include "common.cuh"
#include "gemm_tc.cuh"
#include "ptx.cuh"

#include <cuda.h>

namespace grinqh {
namespace {

constexpr int BM = 256, BN = 256, BK = 64, STAGES = 3;
constexpr int kTileWords = BN / 16;                 // packed words per tile
constexpr int kConvWarps = 8;
constexpr int kThreads = 32 * (2 + kConvWarps);
constexpr uint32_t kStageA = BM * BK * 2;           // 32 KB
constexpr uint32_t kStageB = BN * BK * 2;           // 32 KB
constexpr uint32_t kSmemBytes = STAGES * (kStageA + kStageB) + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kLboB = 8 * 1024;   // B: stride between 64-column MN atoms (8 K atoms of 1 KB)
constexpr uint32_t kSboB = 1024;       // B: stride between 8-row K atoms
constexpr uint32_t kSboA = 1024;       // A: stride between 8-row M groups (128 B rows)

template <typename T> struct Fmt;
template <> struct Fmt<__nv_bfloat16> {
  static constexpr uint32_t v = 1;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Fmt<__half> {
  static constexpr uint32_t v = 0;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// byte offset of element (n', k) inside a B stage (MN-major, 128-byte swizzle)
__device__ __forceinline__ uint32_t b_off(int chunk16, int k) {
  // chunk16 = n' / 8 (16-byte chunk along N), k = row within the 64-deep stage
  const int atom_mn = chunk16 >> 3, c = chunk16 & 7;
  const int atom_k = k >> 3, r = k & 7;
  return (uint32_t)(atom_mn * kLboB + atom_k * kSboB + r * 128 + ((c ^ r) << 4));
}

template <int NZ, typename T>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                const GemmArgs a) {
  constexpr int kShift = 8 - 2 * NZ;
  constexpr float kInvShift = 1.0f / float(1 << kShift);
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + STAGES * kStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * (kStageA + kStageB));
  uint64_t* a_full = bars;
  uint64_t* b_full = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* acc_full = bars + 3 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int jt0 = blockIdx.y * kTileWords;  // first packed word of the tile
  const int n16 = a.N >> 4;
  const int nk = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&b_full[s], kConvWarps);
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
      for (int q = 0; q < nk; ++q) {
        const int s = q % STAGES;
        if (q >= STAGES) mbar_wait(&empty[s], ((q / STAGES) - 1) & 1);
        mbar_arrive_expect_tx(&a_full[s], kStageA);
        tma_load_2d(sA + s * kStageA, &tmap_x, q * BK, m0, &a_full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(1, Fmt<T>::v, Fmt<T>::v, 0, 1, BN, 128);
      for (int q = 0; q < nk; ++q) {
        const int s = q % STAGES;
        const uint32_t ph = (q / STAGES) & 1;
        mbar_wait(&a_full[s], ph);
        mbar_wait(&b_full[s], ph);
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * kStageA);
        const uint32_t b_base = smem_u32(sB + s * kStageB);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t bdesc = smem_desc(b_base + kk * 2 * kSboB, kLboB, kSboB, 2);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t adesc = smem_desc(a_base + h * 128 * 128 + kk * 32, 16, kSboA, 2);
            mma_f16_ss(tmem + h * BN, adesc, bdesc, idesc, (q > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
      }
      mma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ converters
    const int ct = threadIdx.x - 64;          // 0..255
    const int jj = ct & 15;                   // word of the tile this thread converts
    const int r0 = ct >> 4;                   // rows r0 + 16 i, i = 0..3
    const int jw = jt0 + jj;
    const bool jvalid = jw < n16;
    const size_t row_words = (size_t)NZ * n16;
    const uint32_t* wcol = a.w + (jvalid ? jw : 0);
    const T* sc = static_cast<const T*>(a.s);
    float sreg[16], snext[16];
    auto load_scales = [&](float (&dst)[16], int g) {
#pragma unroll
      for (int c = 0; c < 16; ++c)
        dst[c] = jvalid ? Act<T>::to_f(sc[(size_t)g * a.N + (size_t)c * n16 + jw]) * kInvShift : 0.f;
    };
    // plane words of K steps q+1 and q+2 are in flight while step q is converted
    uint32_t P1[4][4], P2[4][4];
    auto load_planes = [&](uint32_t (&P)[4][4], int q) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t* wr = wcol + (size_t)(q * BK + r0 + 16 * i) * row_words;
#pragma unroll
        for (int z = 0; z < 4; ++z) P[i][z] = (z < NZ && jvalid && q < nk) ? __ldcs(wr + (size_t)z * n16) : 0u;
      }
    };
    const int steps_per_group = a.group / BK;
    load_scales(sreg, 0);
    if (nk > steps_per_group) load_scales(snext, 1);
    auto convert_step = [&](const uint32_t (&Pc)[4][4], int q) {
      const int s = q % STAGES;
      if (q > 0 && q % steps_per_group == 0) {  // next K group: its scales were prefetched
        const int g = q / steps_per_group;
#pragma unroll
        for (int c = 0; c < 16; ++c) sreg[c] = snext[c];
        if ((g + 1) * steps_per_group < nk) load_scales(snext, g + 1);
      }
      if (q >= STAGES) mbar_wait(&empty[s], ((q / STAGES) - 1) & 1);
      unsigned char* bst = sB + s * kStageB;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t qv[4];
        merge_planes(Pc[i][0] ^ kSignFlip, Pc[i][1], Pc[i][2], Pc[i][3], qv);
        uint32_t out[8];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          // code * s exactly in fp32, rounded once to the activation dtype (kernel.py:586)
          const float f0 = byte_to_float<0>(qv[t]) * sreg[4 * t + 0];
          const float f1 = byte_to_float<1>(qv[t]) * sreg[4 * t + 1];
          const float f2 = byte_to_float<2>(qv[t]) * sreg[4 * t + 2];
          const float f3 = byte_to_float<3>(qv[t]) * sreg[4 * t + 3];
          out[2 * t] = Fmt<T>::pack(f0, f1);
          out[2 * t + 1] = Fmt<T>::pack(f2, f3);
        }
        const int k = r0 + 16 * i;
        *reinterpret_cast<uint4*>(bst + b_off(2 * jj, k)) = make_uint4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<uint4*>(bst + b_off(2 * jj + 1, k)) = make_uint4(out[4], out[5], out[6], out[7]);
      }
      fence_proxy_async_smem();  // make the generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_full[s]);
    };
    // the plane buffers rotate by name: a register copy of a pending load would wait for it
    load_planes(P1, 0);
    load_planes(P2, 1);
    for (int q = 0; q < nk; q += 2) {
      convert_step(P1, q);
      load_planes(P1, q + 2);
      if (q + 1 < nk) {
        convert_step(P2, q + 1);
        load_planes(P2, q + 3);
      }
    }

    // ------------------------------------------------------------ epilogue
    // Accumulator rows are staged through the (now idle) stage buffers so that each
    // store instruction writes one output row's 16 runs of 16 columns (32 B each).
    mbar_wait(acc_full, 0);
    tc_fence_after();
    const int quarter = warp & 3;       // TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;   // accumulator (M half)
    const int wl = warp - 2;            // 0..7
    uint32_t* stage_w = reinterpret_cast<uint32_t*>(smem) + wl * 32 * (BN / 2 + 1);  // 32 rows x 256 cols (+1 word pad)
    T* y = static_cast<T*>(a.y);
    const T* bias = static_cast<const T*>(a.bias);
#pragma unroll 1
    for (int cc = 0; cc < BN / 32; ++cc) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + half * BN + cc * 32, r);
      tmem_ld_wait();
      // tile column 32cc + 16u + c = output column c * n16 + jt0 + 2cc + u; store the row
      // as [c][jj] (16 x 16 dtype) so that (c, jj..jj+7) is 16 contiguous bytes
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int jx = jt0 + 2 * cc;
        float v0 = __uint_as_float(r[c]), v1 = __uint_as_float(r[16 + c]);
        T o0 = Act<T>::from_f(v0), o1 = Act<T>::from_f(v1);
        if (bias) {
          if (jx < n16) o0 = Act<T>::from_f(Act<T>::to_f(o0) + Act<T>::to_f(bias[c * n16 + jx]));
          if (jx + 1 < n16) o1 = Act<T>::from_f(Act<T>::to_f(o1) + Act<T>::to_f(bias[c * n16 + jx + 1]));
        }
        const uint32_t pr = (uint32_t)(*reinterpret_cast<uint16_t*>(&o0)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&o1)) << 16);
        // word (c, cc) of this lane's row; rows padded by one word against bank conflicts
        stage_w[lane * (BN / 2 + 1) + c * 8 + cc] = pr;
      }
    }
    __syncwarp();
    // each lane writes 16 B = 8 columns (c, jj0..jj0+7) of one row per instruction
    {
      const int c = lane >> 1, part = lane & 1;
      const int jx0 = jt0 + part * 8;
      for (int rr = 0; rr < 32; ++rr) {
        const int m = m0 + half * 128 + quarter * 32 + rr;
        if (m >= a.M) break;
        const uint32_t* src = stage_w + rr * (BN / 2 + 1) + c * 8 + part * 4;
        if (jx0 + 8 <= n16 && ((c * n16 + jx0) & 7) == 0) {
          *reinterpret_cast<uint4*>(y + (size_t)m * a.N + c * n16 + jx0) = make_uint4(src[0], src[1], src[2], src[3]);
        } else {
          const uint16_t* h = reinterpret_cast<const uint16_t*>(src);
          for (int e = 0; e < 8; ++e)
            if (jx0 + e < n16) reinterpret_cast<uint16_t*>(y)[(size_t)m * a.N + c * n16 + jx0 + e] = h[e];
        }
      }
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

template <int NZ, typename T>
int launch_t(const GemmArgs& a, cudaStream_t st) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap tmap;
  const cuuint64_t gdim[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.K * 2};
  const cuuint32_t box[2] = {BK, BM};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = enc(&tmap, Fmt<T>::v ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                         const_cast<void*>(a.x), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  auto kern = gemm_tc_kernel<NZ, T>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const dim3 grid((unsigned)((a.M + BM - 1) / BM), (unsigned)((a.N / 16 + kTileWords - 1) / kTileWords));
  kern<<<grid, kThreads, kSmemBytes, st>>>(tmap, a);
  return check_launch("gemm_tc");
}

}  // namespace

unsigned take_gemm_timeouts() {
  unsigned v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof(z));
  return v;
}

bool gemm_tc_supported(int64_t M, int64_t K, int64_t N, int group, const void* x, const void* y) {
  // TMA needs a 16-byte aligned base and row pitch; the K loop needs whole 64-deep
  // steps that never straddle a scale group; the epilogue stores 16-byte runs
  static_assert(8 * 32 * (BN / 2 + 1) * 4 <= STAGES * (kStageA + kStageB), "epilogue staging must fit");
  return M >= 1 && K % BK == 0 && group % BK == 0 && N % 16 == 0 && (K * 2) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(x) % 16) == 0 && (reinterpret_cast<uintptr_t>(y) % 16) == 0;
}

int launch_gemm_tc(const GemmArgs& a, int dtype, int nz, cudaStream_t st) {
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

}  // namespace grinqh
