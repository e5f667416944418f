// Single-row graded GEMV (the reference's M == 1 path, grinqh/kernel.py:39-167)
// streamed from HBM through registers.
//
// Tile: a warp owns 32 packed-word columns (one word = 16 output columns per lane,
// 128 B per plane row) and a contiguous chunk of K rows; the 8 warps of a CTA take
// consecutive chunks of the CTA's row range for the same 32 words. Each lane keeps
// a D-deep ring of plane words in registers: while row r is merged and multiplied,
// the active planes of row r + D are already in flight (a row graded 0 issues no
// load), so a CTA keeps 8 * D * 4 * 128 B of weights in flight.
//
// Scales are applied per K group, s * (sum(code * x) + sum(bias * x)) as in
// kernel.py:148-158. The 8 warps are summed in shared memory; up to 8 CTAs that
// split the same tile along K form a thread-block cluster and rank 0 adds their
// partials over distributed shared memory; when a tile has several clusters, their
// sums go to fp32 slots and the last cluster leader (atomic ticket) adds them in
// cluster order. Every sum has a fixed order, so results are deterministic.
#include <cooperative_groups.h>

#include "common.cuh"
#include "decode_m1.cuh"

namespace cg = cooperative_groups;

namespace grinqh {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kTileJ = 32;
constexpr int kTileN = 16 * kTileJ;

struct RowMeta {
  float x, bx;
  uint32_t m, pad;
};

template <int NZ>
__device__ __forceinline__ int zone_bias(uint32_t m) {
  constexpr int base = 1 << (2 * NZ - 1);
  constexpr int b0 = base >> 2, b1 = base >> 4, b2 = base >> 6, b3 = base >> 8;
  int v = 0;
  if (NZ > 0 && (m & 1)) v += b0;
  if (NZ > 1 && (m & 2)) v += b1 - b0;
  if (NZ > 2 && (m & 4)) v += b2 - b1;
  if (NZ > 3 && (m & 8)) v += b3 - b2;
  return v;
}

// acc[p]: columns c = 2p, 2p+1 of the lane's packed word (c = 4i + L)
__device__ __forceinline__ void fma_word(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, float2 xv,
                                         float2 (&acc)[8]) {
  uint32_t q[4];
  merge_planes(a0 ^ kSignFlip, a1, a2, a3, q);
  const float2 magic = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f01 = make_float2(__int_as_float(__byte_perm(q[i], 0x4B000000u, 0x7440u)),
                             __int_as_float(__byte_perm(q[i], 0x4B000000u, 0x7441u)));
    float2 f23 = make_float2(__int_as_float(__byte_perm(q[i], 0x4B000000u, 0x7442u)),
                             __int_as_float(__byte_perm(q[i], 0x4B000000u, 0x7443u)));
    acc[2 * i] = __ffma2_rn(__fadd2_rn(f01, magic), xv, acc[2 * i]);
    acc[2 * i + 1] = __ffma2_rn(__fadd2_rn(f23, magic), xv, acc[2 * i + 1]);
  }
}

template <int NZ, int D, typename T>
__global__ void __launch_bounds__(kThreads, 2) m1_kernel(const M1Args a) {
  constexpr int kShift = 8 - 2 * NZ;
  constexpr float kInvShift = 1.0f / float(1 << kShift);
  extern __shared__ __align__(16) unsigned char smem[];
  RowMeta* rows = reinterpret_cast<RowMeta*>(smem);                       // staged rows of the CTA
  float* red = reinterpret_cast<float*>(smem);                            // aliases rows after the loop
  float* part = reinterpret_cast<float*>(smem + m1_meta_bytes(a.rows_per_cta));  // CTA partial (DSMEM)
  __shared__ int s_last;

  cg::cluster_group cluster = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n16 = a.N >> 4;
  const int jw = tile * kTileJ + lane;
  const bool jvalid = jw < n16;
  const int k0 = split * a.rows_per_cta;
  const int k1 = min(k0 + a.rows_per_cta, a.K);
  const int nrows = max(0, k1 - k0);
  const T* x = static_cast<const T*>(a.x);
  const T* sc = static_cast<const T*>(a.s);
  const size_t row_words = (size_t)NZ * n16;

  // grade the CTA's rows once (kernel.py:100-116): fp32 |x| > t_z, bias * x
  for (int i = threadIdx.x; i < nrows; i += kThreads) {
    const float xv = Act<T>::to_f(x[k0 + i]);
    const float ax = fabsf(xv);
    uint32_t g = (uint32_t)(ax > a.t[0]) | ((uint32_t)(ax > a.t[1]) << 1) | ((uint32_t)(ax > a.t[2]) << 2) |
                 ((uint32_t)(ax > a.t[3]) << 3);
    g &= (1u << NZ) - 1u;
    rows[i] = RowMeta{xv, float(zone_bias<NZ>(g)) * xv, g, 0u};
  }
  __syncthreads();

  float2 acc[8], gacc[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) acc[p] = gacc[p] = make_float2(0.f, 0.f);
  float bsum = 0.f;
  float sreg[16];

  const int rb = min(nrows, warp * a.rows_per_warp), re = min(nrows, rb + a.rows_per_warp);
  const uint32_t* wcol = a.w + jw;

  auto load_row = [&](uint32_t (&P)[4], int i) {
    const uint32_t m = jvalid ? rows[i].m : 0u;
    const uint32_t* wr = wcol + (size_t)(k0 + i) * row_words;
#pragma unroll
    for (int z = 0; z < 4; ++z) P[z] = (z < NZ && ((m >> z) & 1u)) ? __ldcs(wr + (size_t)z * n16) : 0u;
  };
  auto load_scales = [&](int g) {
#pragma unroll
    for (int c = 0; c < 16; ++c) sreg[c] = jvalid ? Act<T>::to_f(sc[(size_t)g * a.N + (size_t)c * n16 + jw]) : 0.f;
  };
  auto flush = [&]() {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      acc[p].x = fmaf(sreg[2 * p], fmaf(gacc[p].x, kInvShift, bsum), acc[p].x);
      acc[p].y = fmaf(sreg[2 * p + 1], fmaf(gacc[p].y, kInvShift, bsum), acc[p].y);
      gacc[p] = make_float2(0.f, 0.f);
    }
    bsum = 0.f;
  };

  if (rb < re) {
    int g = (k0 + rb) / a.group;
    int next_group_k = (g + 1) * a.group;
    load_scales(g);
    uint32_t P[D][4];
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (rb + d < re) load_row(P[d], rb + d);
    for (int r = rb; r < re; r += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const int i = r + d;
        if (i < re) {
          if (k0 + i == next_group_k) {  // K group boundary: apply the finished group's scales
            flush();
            next_group_k += a.group;
            load_scales(++g);
          }
          const RowMeta rm = rows[i];
          bsum += rm.bx;
          if (rm.m) fma_word(P[d][0], P[d][1], P[d][2], P[d][3], make_float2(rm.x, rm.x), gacc);
          if (i + D < re) load_row(P[d], i + D);
        }
      }
    }
    flush();
  }

  // ---- sum the 8 warps (red aliases the staged rows: wait for every warp first)
  __syncthreads();
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    red[warp * kTileN + (2 * p) * kTileJ + lane] = acc[p].x;
    red[warp * kTileN + (2 * p + 1) * kTileJ + lane] = acc[p].y;
  }
  __syncthreads();
  for (int col = threadIdx.x; col < kTileN; col += kThreads) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w * kTileN + col];
    part[col] = v;
  }

  // ---- cluster: rank 0 adds the ranks' partials in rank order over DSMEM
  cluster.sync();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  float sum2[kTileN / kThreads];
  if (crank == 0) {
#pragma unroll
    for (int h = 0; h < kTileN / kThreads; ++h) {
      const int col = threadIdx.x + h * kThreads;
      float v = 0.f;
      for (int r = 0; r < csize; ++r) v += cluster.map_shared_rank(part, r)[col];
      sum2[h] = v;
    }
  }
  cluster.sync();  // other ranks keep their shared memory alive until rank 0 has read it
  if (crank != 0) return;

  T* y = static_cast<T*>(a.y);
  const T* bias = static_cast<const T*>(a.bias);
  auto store_y = [&](int col, float v) {
    const int c = col / kTileJ, jj = col % kTileJ;
    const int jx = tile * kTileJ + jj;
    if (jx >= n16) return;
    const int n = c * n16 + jx;
    T out = Act<T>::from_f(v);
    if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[n]));
    y[n] = out;
  };
  const int nclu = gridDim.y / csize;
  if (nclu == 1) {
#pragma unroll
    for (int h = 0; h < kTileN / kThreads; ++h) store_y(threadIdx.x + h * kThreads, sum2[h]);
    return;
  }
  const int clu = split / csize;
#pragma unroll
  for (int h = 0; h < kTileN / kThreads; ++h)
    __stcg(a.slots + ((size_t)tile * nclu + clu) * kTileN + threadIdx.x + h * kThreads, sum2[h]);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.counters + tile, 1u) == (unsigned)(nclu - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
#pragma unroll
  for (int h = 0; h < kTileN / kThreads; ++h) {
    const int col = threadIdx.x + h * kThreads;
    float v = 0.f;
    for (int c0 = 0; c0 < nclu; c0 += 8) {
      float buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        buf[u] = (c0 + u < nclu) ? __ldcg(a.slots + ((size_t)tile * nclu + c0 + u) * kTileN + col) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) v += buf[u];
    }
    store_y(col, v);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;  // ready for the next launch
}

template <int NZ, typename T>
int launch_t(const M1Args& a, const M1Plan& p, cudaStream_t st) {
  constexpr int D = 8;
  auto kern = m1_kernel<NZ, D, T>;
  const size_t smem = p.smem_bytes;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)p.tiles, (unsigned)p.grid_splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.cluster;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "m1 GEMV launch: %s", cudaGetErrorString(e));
  return check_launch("m1 GEMV");
}

}  // namespace

bool m1_supported(int64_t M, int64_t K, int64_t N, int group) {
  return M == 1 && N % 16 == 0 && K % group == 0 && group % 8 == 0;
}

M1Plan plan_m1(int64_t K, int64_t N, int group, int sm_count) {
  constexpr int D = 8;
  M1Plan p{};
  const int64_t n16 = N / 16;
  p.tiles = (int)((n16 + kTileJ - 1) / kTileJ);
  const int64_t target = 2LL * (sm_count > 0 ? sm_count : 148);
  int64_t splits = (target + p.tiles / 2) / p.tiles;
  const int64_t max_splits = (K + kWarps * D - 1) / (kWarps * D);
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int64_t rpw = ((K + splits - 1) / splits + kWarps - 1) / kWarps;
  rpw = (rpw + D - 1) / D * D;
  p.rows_per_warp = (int)rpw;
  p.rows_per_cta = (int)(rpw * kWarps);
  const int64_t real = (K + p.rows_per_cta - 1) / p.rows_per_cta;
  p.cluster = (int)(real < 8 ? real : 8);
  p.grid_splits = (int)((real + p.cluster - 1) / p.cluster * p.cluster);
  const int nclu = p.grid_splits / p.cluster;
  p.slot_bytes = nclu > 1 ? (size_t)p.tiles * nclu * kTileN * sizeof(float) : 0;
  p.counter_bytes = nclu > 1 ? (size_t)p.tiles * sizeof(unsigned) : 0;
  p.smem_bytes = m1_meta_bytes(p.rows_per_cta) + kTileN * sizeof(float);
  return p;
}

int launch_m1(const M1Args& a, const M1Plan& p, int dtype, int nz, cudaStream_t st) {
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
