// Dense quantized GEMM for few rows (2..64 tokens) on the 5th-generation tensor
// cores: y = x @ dtype(w * s), the reference's M > 1 path (grinqh/kernel.py:561-587),
// with the roles of the operands swapped so that no MMA work is spent on padding
// rows: the weights are operand A (M = 128 weight columns per MMA) and the tokens
// are operand B (N = the row count rounded up to 16).
//
// A CTA owns a tile of 32 packed words (512 output columns) and a range of K steps
// of 64 rows:
//   warps 0-15  converters: load the planes of 64 rows x 32 words (two steps ahead),
//               merge them into codes, multiply by the group scale, round to the
//               activation dtype -- the reference's dtype(w * s), bit for bit -- and
//               store the 512 x 64 tile MN-major with the 128-byte swizzle (a lane's
//               16 columns of one row are 32 contiguous bytes). After the K loop they
//               are the epilogue.
//   warp 16     TMA producer: the Mp x 64 activation tile (rows past M read as 0),
//               K-major, 128-byte swizzle.
//   warp 17     allocates TMEM and issues, per 16-deep K slice, four
//               tcgen05.mma kind::f16 (one per 128-column block, N = Mp) from one
//               thread; tcgen05.commit frees the stage.
// Three stages (64 KB of weights + up to 8 KB of activations each) are in flight.
//
// K is split over the CTAs of a thread-block cluster (and over several clusters for
// long K). Each CTA stages its fp32 partial tile in shared memory; rank r of the
// cluster adds the ranks' values for its share of the (row, column-group) pairs over
// distributed shared memory, in rank order. With one cluster per tile that sum is the
// result; otherwise it goes to an fp32 slot and the last cluster to finish a share
// (atomic ticket) adds the clusters' slots in order. Deterministic; every wait is
// bounded.
#include <cooperative_groups.h>
#include <cuda.h>

#include "common.cuh"
#include "gemm_skinny.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace grinqh {
namespace {

constexpr int TW = 32;         // packed words per tile
constexpr int TN = 16 * TW;    // output columns per tile
constexpr int BK = 64, STAGES = 3;
constexpr int kConvWarps = 16;
constexpr int kProdWarp = 16, kMmaWarp = 17;
constexpr int kThreads = 32 * (kConvWarps + 2);
constexpr int kMaxMp = 64;
constexpr uint32_t kStageW = TN * BK * 2;      // 64 KB
constexpr uint32_t kStageX = kMaxMp * BK * 2;  // 8 KB
constexpr uint32_t kSmemBytes = STAGES * (kStageW + kStageX) + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kLbo = 8 * 1024;  // weights: stride between 64-column MN atoms (8 K atoms of 1 KB)
constexpr uint32_t kSbo = 1024;      // stride between 8-row K groups
constexpr int kPartRow = 16 * 33;    // fp32 partial staging [m][c][word], words padded to 33

static_assert((size_t)kMaxMp * kPartRow * 4 <= (size_t)STAGES * (kStageW + kStageX), "partial tile must fit");

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

// byte offset of the 16-byte chunk `chunk16` (8 columns) of row k in a weight stage
// (MN-major, 128-byte swizzle)
__device__ __forceinline__ uint32_t w_off(int chunk16, int k) {
  const int atom_mn = chunk16 >> 3, c = chunk16 & 7;
  const int atom_k = k >> 3, r = k & 7;
  return (uint32_t)(atom_mn * kLbo + atom_k * kSbo + r * 128 + ((c ^ r) << 4));
}

template <int NZ, typename T>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmap_x, const SkinnyArgs a, const int mp) {
  constexpr int kShift = 8 - 2 * NZ;
  constexpr float kInvShift = 1.0f / float(1 << kShift);
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sW = smem;
  unsigned char* sX = smem + STAGES * kStageW;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * (kStageW + kStageX));
  uint64_t* x_full = bars;
  uint64_t* w_full = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* acc_full = bars + 3 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int jt0 = tile * TW;  // first packed word of the tile
  const int n16 = a.N >> 4;
  const int nk = a.K / BK;
  const int q0 = split * a.steps_per_split;
  const int nq = max(0, min(nk, q0 + a.steps_per_split) - q0);
  const uint32_t cstride = mp <= 32 ? 32u : 64u;  // TMEM columns per 128-column block
  const uint32_t tcols = 4 * cstride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&w_full[s], kConvWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      const uint32_t xbytes = (uint32_t)mp * BK * 2;
      for (int i = 0; i < nq; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES) mbar_wait(&empty[s], ((i / STAGES) - 1) & 1);
        mbar_arrive_expect_tx(&x_full[s], xbytes);
        tma_load_2d(sX + s * kStageX, &tmap_x, (q0 + i) * BK, 0, &x_full[s]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc(1, Fmt<T>::v, Fmt<T>::v, 1, 0, (uint32_t)mp, 128);
      for (int i = 0; i < nq; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        mbar_wait(&x_full[s], ph);
        mbar_wait(&w_full[s], ph);
        tc_fence_after();
        const uint32_t wbase = smem_u32(sW + s * kStageW);
        const uint32_t xbase = smem_u32(sX + s * kStageX);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t bdesc = smem_desc(xbase + kk * 32, 16, 1024, 2);
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint64_t adesc = smem_desc(wbase + b * 2 * kLbo + kk * 2 * kSbo, kLbo, kSbo, 2);
            mma_f16_ss(tmem + b * cstride, adesc, bdesc, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
      }
      mma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ converters
    const int ct = threadIdx.x;      // 0..511
    const int jj = ct & (TW - 1);    // word of the tile this thread converts
    const int r0 = ct / TW;          // rows r0 + 16 i, i = 0..3
    const int jw = jt0 + jj;
    const bool jvalid = jw < n16;
    const size_t row_words = (size_t)NZ * n16;
    const uint32_t* wcol = a.w + (jvalid ? jw : 0);
    const T* sc = static_cast<const T*>(a.s);
    const int spg = a.group / BK;  // K steps per scale group
    float sreg[16], snext[16];
    auto load_scales = [&](float (&dst)[16], int g) {
#pragma unroll
      for (int c = 0; c < 16; ++c)
        dst[c] = jvalid ? Act<T>::to_f(sc[(size_t)g * a.N + (size_t)c * n16 + jw]) * kInvShift : 0.f;
    };
    uint32_t P1[4][4], P2[4][4];
    auto load_planes = [&](uint32_t (&P)[4][4], int i) {
      const int q = q0 + i;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t* wr = wcol + (size_t)(q * BK + r0 + 16 * r) * row_words;
#pragma unroll
        for (int z = 0; z < 4; ++z) P[r][z] = (z < NZ && jvalid && i < nq) ? __ldcs(wr + (size_t)z * n16) : 0u;
      }
    };
    if (nq > 0) {
      const int g0 = q0 / spg;
      load_scales(sreg, g0);
      if ((g0 + 1) * spg < q0 + nq) load_scales(snext, g0 + 1);
    }
    auto convert_step = [&](const uint32_t (&Pc)[4][4], int i) {
      const int q = q0 + i, s = i % STAGES;
      if (i > 0 && q % spg == 0) {  // next scale group: its scales were prefetched
        const int g = q / spg;
#pragma unroll
        for (int c = 0; c < 16; ++c) sreg[c] = snext[c];
        if ((g + 1) * spg < q0 + nq) load_scales(snext, g + 1);
      }
      if (i >= STAGES) mbar_wait(&empty[s], ((i / STAGES) - 1) & 1);
      unsigned char* wst = sW + s * kStageW;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        uint32_t qv[4];
        merge_planes(Pc[r][0] ^ kSignFlip, Pc[r][1], Pc[r][2], Pc[r][3], qv);
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
        const int k = r0 + 16 * r;
        *reinterpret_cast<uint4*>(wst + w_off(2 * jj, k)) = make_uint4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<uint4*>(wst + w_off(2 * jj + 1, k)) = make_uint4(out[4], out[5], out[6], out[7]);
      }
      fence_proxy_async_smem();  // make the generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&w_full[s]);
    };
    // the plane buffers rotate by name: a register copy of a pending load would wait for it
    load_planes(P1, 0);
    load_planes(P2, 1);
    for (int i = 0; i < nq; i += 2) {
      convert_step(P1, i);
      load_planes(P1, i + 2);
      if (i + 1 < nq) {
        convert_step(P2, i + 1);
        load_planes(P2, i + 3);
      }
    }

    // ------------------------------------------------------------ partial tile -> smem
    // accumulator block b, TMEM lane p (this warp may read lanes 32 * (warp % 4) ..):
    // tile position P = 128 b + p, word P / 16, column group P % 16 (the converters'
    // order); TMEM column m = token m.
    mbar_wait(acc_full, 0);
    tc_fence_after();
    float* part = reinterpret_cast<float*>(smem);  // the stages are idle now
    const int quarter = warp & 3, blk = warp >> 2;
    const int pos = blk * 128 + quarter * 32 + lane;
    const int pw = pos >> 4, pc = pos & 15;
    for (int h = 0; h < (int)cstride; h += 32) {
      uint32_t r[32];
      if (nq > 0) {
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + blk * cstride + h, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) r[t] = 0u;
      }
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (h + t < mp) part[(h + t) * kPartRow + pc * 33 + pw] = __uint_as_float(r[t]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, tcols);

  // ------------------------------------------------------------ reduction and store
  T* y = static_cast<T*>(a.y);
  const T* bias = static_cast<const T*>(a.bias);
  const float* part = reinterpret_cast<const float*>(smem);
  // (row m, column group c, word jj) -> y[m, c * n16 + jt0 + jj]; one warp writes a
  // pair's 32 words (64 contiguous bytes)
  auto store_y = [&](int m, int c, int w, float v) {
    if (m >= a.M || jt0 + w >= n16) return;
    const int n = c * n16 + jt0 + w;
    T out = Act<T>::from_f(v);
    if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[n]));
    y[(size_t)m * a.N + n] = out;
  };
  const int npairs = mp * 16;
  if (a.splits == 1) {
    for (int pr = warp; pr < npairs; pr += kThreads / 32)
      store_y(pr >> 4, pr & 15, lane, part[(pr >> 4) * kPartRow + (pr & 15) * 33 + lane]);
    return;
  }
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = a.cluster;
  const int crank = (int)cluster.block_rank();
  const int nclu = a.splits / cs, clu = split / cs;
  const size_t slot_elems = (size_t)npairs * 32;
  float* myslot = a.slots + ((size_t)tile * nclu + clu) * slot_elems;
  cluster.sync();
  // this rank's pairs: crank, crank + cs, ...; summed over the ranks in rank order
  for (int k = warp; crank + cs * k < npairs; k += kThreads / 32) {
    const int pr = crank + cs * k;
    const int off = (pr >> 4) * kPartRow + (pr & 15) * 33 + lane;
    float v = 0.f;
    for (int rr = 0; rr < cs; ++rr) v += cluster.map_shared_rank(part, rr)[off];
    if (nclu == 1) store_y(pr >> 4, pr & 15, lane, v);
    else __stcg(myslot + (size_t)pr * 32 + lane, v);
  }
  cluster.sync();  // every rank keeps its shared memory until the others have read it
  if (nclu == 1) return;
  __threadfence();
  __syncthreads();
  unsigned* ticket = a.counters + (size_t)tile * cs + crank;
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1u) == (unsigned)(nclu - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int k = warp; crank + cs * k < npairs; k += kThreads / 32) {
    const int pr = crank + cs * k;
    float v = 0.f;
    for (int cl = 0; cl < nclu; ++cl)
      v += __ldcg(a.slots + ((size_t)tile * nclu + cl) * slot_elems + (size_t)pr * 32 + lane);
    store_y(pr >> 4, pr & 15, lane, v);
  }
  if (threadIdx.x == 0) *ticket = 0u;  // ready for the next launch
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
int launch_t(const SkinnyArgs& a, const SkinnyPlan& p, cudaStream_t st) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap tmap;
  const cuuint64_t gdim[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.K * 2};
  const cuuint32_t box[2] = {BK, (cuuint32_t)p.mp};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = enc(&tmap, Fmt<T>::v ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                         const_cast<void*>(a.x), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  auto kern = skinny_kernel<NZ, T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)p.tiles, (unsigned)p.splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.cluster;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tmap, a, p.mp);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "skinny GEMM launch: %s", cudaGetErrorString(e));
  return check_launch("skinny GEMM");
}

}  // namespace

unsigned take_skinny_timeouts() {
  unsigned v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof(z));
  return v;
}

bool skinny_supported(int64_t M, int64_t K, int64_t N, int group) {
  // TMA rows of 64 K-elements, K steps that never straddle a scale group, N / 16 words
  return M >= 2 && M <= kMaxMp && K % BK == 0 && group % BK == 0 && N % 16 == 0 && K < (1LL << 31);
}

bool skinny_pointers_ok(const void* x, const void* y) {
  (void)y;
  return (reinterpret_cast<uintptr_t>(x) % 16) == 0;
}

SkinnyPlan plan_skinny(int64_t M, int64_t K, int64_t N, int sm_count) {
  SkinnyPlan p{};
  p.mp = (int)((M + 15) / 16 * 16);
  const int64_t n16 = N / 16;
  p.tiles = (int)((n16 + TW - 1) / TW);
  const int64_t nk = K / BK;
  // one CTA per SM (about 218 KB of shared memory each); clusters of up to 8 pack
  // into the GPCs less densely than single CTAs, so aim a little under the SM count
  const int64_t target = (sm_count > 0 ? sm_count : 148) * 7 / 8;
  int64_t splits = target / p.tiles;
  if (splits > nk) splits = nk;
  if (splits < 1) splits = 1;
  int64_t steps = (nk + splits - 1) / splits;
  splits = (nk + steps - 1) / steps;  // no empty splits
  // cluster: the largest size <= 8 that divides the split count
  int cl = 1;
  for (int c = 8; c >= 1; --c)
    if (splits % c == 0) {
      cl = c;
      break;
    }
  p.splits = (int)splits;
  p.cluster = cl;
  p.steps_per_split = (int)steps;
  const int nclu = p.splits / p.cluster;
  p.slot_bytes = nclu > 1 ? (size_t)p.tiles * nclu * p.mp * TN * sizeof(float) : 0;
  p.counter_bytes = nclu > 1 ? (size_t)p.tiles * p.cluster * sizeof(unsigned) : 0;
  return p;
}

int launch_skinny(const SkinnyArgs& a, const SkinnyPlan& p, int dtype, int nz, cudaStream_t st) {
  if (dtype == GRINQH_BF16) {
    switch (nz) {
      case 1: return launch_t<1, __nv_bfloat16>(a, p, st);
      case 2: return launch_t<2, __nv_bfloat16>(a, p, st);
      case 3: return launch_t<3, __nv_bfloat16>(a, p, st);
      default: return launch_t<4, __nv_bfloat16>(a, p, st);
    }
  }
  switch (nz) {
    case 1: return launch_t<1, __half>(a, p, st);
    case 2: return launch_t<2, __half>(a, p, st);
    case 3: return launch_t<3, __half>(a, p, st);
    default: return launch_t<4, __half>(a, p, st);
  }
}

}  // namespace grinqh
