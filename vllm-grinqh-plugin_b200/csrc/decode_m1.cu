// Single-row graded GEMV (the reference's M == 1 path, grinqh/kernel.py:39-167)
// streamed from HBM through registers.
//
// Tile: a CTA owns a slice of 64 packed words (1024 output columns); each lane owns
// two neighbouring words and reads both with one 8-byte load per active plane, so a
// warp reads 256 contiguous bytes of every plane row it needs. The 8 warps of a CTA
// take consecutive chunks of the CTA's K range. Each warp grades its own rows into
// shared memory (no CTA-wide barrier before the first weight load) and keeps a
// kD-row ring of plane words in flight: while row r is merged and multiplied, the
// active planes of row r + kD are already loading. A row graded 0 issues no load
// and no arithmetic.
//
// Scales are applied per K group, s * (sum(code * x) + sum(bias * x)) as in
// kernel.py:148-158, at group boundaries and at the end of a chunk. The 8 warps are
// summed in shared memory; up to 8 CTAs that split the same slice along K form a
// thread-block cluster and rank 0 adds their partials over distributed shared
// memory; when a slice has several clusters, their sums go to fp32 slots and the
// last cluster leader (atomic ticket) adds them in cluster order. Every sum has a
// fixed order, so results are deterministic.
#include <cooperative_groups.h>

#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "decode_m1.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace grinqh {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kWpl = 2;                // packed words per lane
constexpr int kSliceW = 32 * kWpl;     // words per slice
constexpr int kSliceN = 16 * kSliceW;  // output columns per slice
constexpr int kD = 4;                  // rows in flight per warp

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

// acc[p]: columns c = 2p, 2p+1 of one packed word (c = 4i + L)
__device__ __forceinline__ void fma_word(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, float2 xv,
                                         float2* acc) {
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

// The active planes of one row for this lane's two words: P[z] = plane z words
// (zero when the row's grade does not include zone z).
template <int NZ>
__device__ __forceinline__ void load_row(uint2 (&P)[4], const uint32_t* wr, uint32_t m, uint32_t pstride) {
#pragma unroll
  for (int z = 0; z < 4; ++z) {
    P[z] = make_uint2(0u, 0u);
    if (z < NZ && (m & (1u << z))) P[z] = __ldcs(reinterpret_cast<const uint2*>(wr + (size_t)z * pstride));
  }
}

template <typename T>
__device__ __forceinline__ float2 scale2(uint32_t bits);
template <>
__device__ __forceinline__ float2 scale2<__nv_bfloat16>(uint32_t bits) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bits));
}
template <>
__device__ __forceinline__ float2 scale2<__half>(uint32_t bits) {
  return __half22float2(*reinterpret_cast<const __half2*>(&bits));
}

// Rows [kb, ke) of slice `tile` for this warp: grade them, stream their planes and
// add s * partial sums into this lane's 32 columns of wacc (kernel.py:100-158).
template <int NZ, typename T>
__device__ __forceinline__ void warp_chunk(const M1Args& a, int tile, int kb, int ke, RowMeta* wrows,
                                           float* wacc) {
  constexpr int kShift = 8 - 2 * NZ;
  constexpr float kInvShift = 1.0f / float(1 << kShift);
  const int lane = threadIdx.x & 31;
  const int n16 = a.N >> 4;
  const int j0 = tile * kSliceW + kWpl * lane;  // this lane's first word (n16 is even)
  const bool jvalid = j0 < n16;
  const T* x = static_cast<const T*>(a.x);
  const uint32_t pstride = (uint32_t)n16;
  const size_t row_words = (size_t)NZ * n16;
  const int n = ke - kb;  // a multiple of kD (chunk bounds, K and the group size are)

  // grade (kernel.py:100-116): fp32 |x| > t_z, bias * x
  for (int i = lane; i < n; i += 32) {
    const float xv = Act<T>::to_f(x[kb + i]);
    const float ax = fabsf(xv);
    uint32_t g = (uint32_t)(ax > a.t[0]) | ((uint32_t)(ax > a.t[1]) << 1) | ((uint32_t)(ax > a.t[2]) << 2) |
                 ((uint32_t)(ax > a.t[3]) << 3);
    g &= (1u << NZ) - 1u;
    wrows[i] = RowMeta{xv, float(zone_bias<NZ>(g)) * xv, g, 0u};
  }
  __syncwarp();
  if (n <= 0) return;

  float2 gacc[16];
#pragma unroll
  for (int p = 0; p < 16; ++p) gacc[p] = make_float2(0.f, 0.f);
  float bsum = 0.f;
  const uint32_t* wr = a.w + (size_t)kb * row_words + (jvalid ? j0 : 0);
  int g = kb / a.group;
  int next_group_k = (g + 1) * a.group;
  // scales of the current group as packed dtype pairs: s[g, c * n16 + j0 .. j0 + 1]
  uint32_t sv[16];
  auto load_scales = [&](int gi) {
    const uint32_t* sp =
        reinterpret_cast<const uint32_t*>(static_cast<const T*>(a.s) + (size_t)gi * a.N + (jvalid ? j0 : 0));
#pragma unroll
    for (int c = 0; c < 16; ++c) sv[c] = __ldg(sp + (size_t)c * (n16 >> 1));
  };
  load_scales(g);
  // wacc += s * (sum(code * x) / 2^shift + sum(bias * x)) for the finished group
  auto flush = [&]() {
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      // gacc[h * 8 + p] holds word h, columns 2p, 2p+1
      const int p = c >> 1;
      const float w0 = (c & 1) ? gacc[p].y : gacc[p].x;
      const float w1 = (c & 1) ? gacc[8 + p].y : gacc[8 + p].x;
      const float2 s2 = scale2<T>(sv[c]);
      float2* dst = reinterpret_cast<float2*>(wacc + c * kSliceW);
      float2 v = *dst;
      v.x = fmaf(s2.x, fmaf(w0, kInvShift, bsum), v.x);
      v.y = fmaf(s2.y, fmaf(w1, kInvShift, bsum), v.y);
      *dst = v;
    }
#pragma unroll
    for (int p = 0; p < 16; ++p) gacc[p] = make_float2(0.f, 0.f);
    bsum = 0.f;
  };

  // lanes past the last word load nothing (their grades read as 0)
  const uint32_t lmask = jvalid ? 0xFu : 0u;
  uint2 P0[4], P1[4], P2[4], P3[4];
  load_row<NZ>(P0, wr, wrows[0].m & lmask, pstride);
  load_row<NZ>(P1, wr + row_words, wrows[1].m & lmask, pstride);
  load_row<NZ>(P2, wr + 2 * row_words, wrows[2].m & lmask, pstride);
  load_row<NZ>(P3, wr + 3 * row_words, wrows[3].m & lmask, pstride);
  const uint32_t* wn = wr + kD * row_words;  // plane words of row i + kD

  auto step = [&](uint2 (&P)[4], int i) {
    const RowMeta rm = wrows[i];
    bsum += rm.bx;
    if (rm.m) {
      const float2 xv = make_float2(rm.x, rm.x);
      fma_word(P[0].x, P[1].x, P[2].x, P[3].x, xv, gacc);
      fma_word(P[0].y, P[1].y, P[2].y, P[3].y, xv, gacc + 8);
    }
    load_row<NZ>(P, wn, i + kD < n ? (wrows[i + kD].m & lmask) : 0u, pstride);
    wn += row_words;
  };

  // a block of kD rows never straddles a group (kb and the group size are multiples of kD)
  for (int i = 0; i < n; i += kD) {
    if (kb + i == next_group_k) {  // K group boundary: apply the finished group's scales
      flush();
      next_group_k += a.group;
      load_scales(++g);
    }
    step(P0, i);
    step(P1, i + 1);
    step(P2, i + 2);
    step(P3, i + 3);
  }
  flush();
}

// ---------------------------------------------------------------- fused all-reduce
// Runs in the CTA that finalises column slice `tile`, after it has stored the slice's
// sums into every rank's buffer: waits (bounded) until every rank's partial of each of
// this thread's columns carries this launch's epoch, adds them in rank order, adds the
// bias and writes y. The slices finalise independently; a waiting CTA waits only on the
// peer CTAs that finalise the same slice, which wait on nothing on their own GPU.
template <typename T>
__device__ void allreduce_tail(const M1Args& a, int tile, unsigned epoch) {
  constexpr int kH = kSliceN / kThreads;
  const int n16 = a.N >> 4;
  size_t nn[kH];
  bool ok[kH];
#pragma unroll
  for (int h = 0; h < kH; ++h) {  // the columns store_y published for this thread
    const int col = threadIdx.x + h * kThreads;
    const int jx = tile * kSliceW + col % kSliceW;
    ok[h] = jx < n16;
    nn[h] = (size_t)(col / kSliceW) * n16 + jx;
  }
  float v[kH];
  peer_sum<kH>(a.ar, epoch, nn, ok, v);  // on a timeout y is invalid; the host sees the count
  T* y = static_cast<T*>(a.y);
  const T* bias = static_cast<const T*>(a.bias);
#pragma unroll
  for (int h = 0; h < kH; ++h) {
    if (!ok[h]) continue;
    T out = Act<T>::from_f(v[h]);
    if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[nn[h]]));
    y[nn[h]] = out;
  }
}

template <int NZ, typename T, bool kAR>
__global__ void __launch_bounds__(kThreads, 2) m1_kernel(const M1Args a) {
  extern __shared__ __align__(16) unsigned char smem[];
  RowMeta* rows = reinterpret_cast<RowMeta*>(smem);  // staged rows of the CTA
  // per-warp scaled accumulators [warp][column], column = c * kSliceW + word; they
  // are also the buffer the 8 warps are summed from
  float* red = reinterpret_cast<float*>(smem + m1_meta_bytes(a.rows_per_cta));
  float* part = red + kWarps * kSliceN;  // CTA partial (read by the cluster over DSMEM)
  __shared__ int s_last;

  cg::cluster_group cluster = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n16 = a.N >> 4;
  const int k0 = split * a.rows_per_cta;
  const int rb = min(a.K, k0 + warp * a.rows_per_warp);
  const int re = min(a.K, rb + a.rows_per_warp);
  float* wacc = red + warp * kSliceN + kWpl * lane;  // this lane's columns: wacc[c * kSliceW + h]
#pragma unroll
  for (int c = 0; c < 16; ++c) *reinterpret_cast<float2*>(wacc + c * kSliceW) = make_float2(0.f, 0.f);
  // While an earlier kernel on the stream finishes (dependent launch), bring the planes
  // of this warp's first rows into L2: the weights are never written by other kernels.
  {
    const int n16p = a.N >> 4, j0p = tile * kSliceW + kWpl * lane;
    if (j0p < n16p && rb < re) {
      const size_t rw = (size_t)NZ * n16p;
#pragma unroll
      for (int r = 0; r < kD; ++r)
        if (rb + r < re)
#pragma unroll
          for (int z = 0; z < NZ; ++z) prefetch_l2(a.w + (size_t)(rb + r) * rw + (size_t)z * n16p + j0p);
    }
  }
  wait_prior_grid();  // x and the outputs belong to the stream order from here on
  // epoch of this launch (fused all-reduce): one more than the last completed one
  const unsigned ar_epoch = kAR ? peer_epoch(a.ar) : 0u;
  warp_chunk<NZ, T>(a, tile, rb, re, rows + (rb - k0), wacc);
  allow_dependent_grid();

  // ---- sum the 8 warps' accumulators
  __syncthreads();
  for (int col = threadIdx.x; col < kSliceN; col += kThreads) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w * kSliceN + col];
    part[col] = v;
  }

  // ---- cluster: rank 0 adds the ranks' partials in rank order over DSMEM
  cluster.sync();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  float sum2[kSliceN / kThreads];
  if (crank == 0) {
#pragma unroll
    for (int h = 0; h < kSliceN / kThreads; ++h) {
      const int col = threadIdx.x + h * kThreads;
      float v = 0.f;
      for (int r = 0; r < csize; ++r) v += cluster.map_shared_rank(part, r)[col];
      sum2[h] = v;
    }
  }
  cluster.sync();  // other ranks keep their shared memory alive until rank 0 has read it
  if (crank != 0) {
    peer_cta_done<kAR>(a.ar, ar_epoch);
    return;
  }

  T* y = static_cast<T*>(a.y);
  const T* bias = static_cast<const T*>(a.bias);
  auto store_y = [&](int col, float v) {
    const int c = col / kSliceW, jj = col % kSliceW;
    const int jx = tile * kSliceW + jj;
    if (jx >= n16) return;
    const int nn = c * n16 + jx;
    if constexpr (kAR) {  // this rank's partial, into every rank's buffer (NVLink stores)
      peer_publish(a.ar, ar_epoch, (size_t)nn, v);
      return;
    }
    T out = Act<T>::from_f(v);
    if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[nn]));
    y[nn] = out;
  };
  const int nclu = gridDim.y / csize;
  if (nclu == 1) {
#pragma unroll
    for (int h = 0; h < kSliceN / kThreads; ++h) store_y(threadIdx.x + h * kThreads, sum2[h]);
    if constexpr (kAR) allreduce_tail<T>(a, tile, ar_epoch);
    peer_cta_done<kAR>(a.ar, ar_epoch);
    return;
  }
  const int clu = split / csize;
#pragma unroll
  for (int h = 0; h < kSliceN / kThreads; ++h)
    __stcg(a.slots + ((size_t)tile * nclu + clu) * kSliceN + threadIdx.x + h * kThreads, sum2[h]);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.counters + tile, 1u) == (unsigned)(nclu - 1);
  __syncthreads();
  if (!s_last) {
    peer_cta_done<kAR>(a.ar, ar_epoch);
    return;
  }
  __threadfence();
#pragma unroll
  for (int h = 0; h < kSliceN / kThreads; ++h) {
    const int col = threadIdx.x + h * kThreads;
    float v = 0.f;
    for (int c0 = 0; c0 < nclu; c0 += 8) {
      float buf[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        buf[u] = (c0 + u < nclu) ? __ldcg(a.slots + ((size_t)tile * nclu + c0 + u) * kSliceN + col) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) v += buf[u];
    }
    store_y(col, v);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;  // ready for the next launch
  if constexpr (kAR) allreduce_tail<T>(a, tile, ar_epoch);
  peer_cta_done<kAR>(a.ar, ar_epoch);
}

template <int NZ, typename T, bool kAR>
int launch_t(const M1Args& a, const M1Plan& p, cudaStream_t st) {
  auto kern = m1_kernel<NZ, T, kAR>;
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
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.cluster;
  attr[0].val.clusterDim.z = 1;
  // may start while the previous kernel on the stream finishes (the kernel waits for
  // it before touching x, the output or the workspace)
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "m1 GEMV launch: %s", cudaGetErrorString(e));
  return check_launch("m1 GEMV");
}

}  // namespace

unsigned take_m1_timeouts() {
  unsigned v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof(z));
  return v;
}

bool m1_supported(int64_t M, int64_t K, int64_t N, int group) {
  // two words per lane: N / 16 even; kD-row blocks never straddle a group
  return M == 1 && N % 32 == 0 && K % group == 0 && group % kD == 0;
}

static M1Plan plan_for(int64_t K, int64_t N, int64_t target, bool few_slots) {
  M1Plan p{};
  const int64_t n16 = N / 16;
  p.tiles = (int)((n16 + kSliceW - 1) / kSliceW);
  int64_t splits = target / p.tiles;
  const int64_t max_splits = (K + kWarps * kD - 1) / (kWarps * kD);
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  // Cluster size: the split count is rounded down to a multiple of it, and larger
  // clusters leave fewer fp32 slots for the last CTA to add. Measured on the Llama
  // shapes (µs, clusters of 8 / 4 / 2): qkv 16.2 / 14.5 / 16.2, o 14.9 / 12.7 / 14.4,
  // gate_up 35.6 / 38.4 / 33.2, down 23.2 / 22.3 / 24.4. So clusters of 4 where they
  // keep more splits than clusters of 8, else clusters of 2 where those do, else 8.
  if (splits < 8 || few_slots) {
    p.cluster = (int)(splits < 8 ? splits : 8);
  } else if (splits / 4 * 4 > splits / 8 * 8) {
    p.cluster = 4;
  } else if (splits / 2 * 2 > splits / 8 * 8) {
    p.cluster = 2;
  } else {
    p.cluster = 8;
  }
  splits = splits / p.cluster * p.cluster;
  int64_t rpw = ((K + splits - 1) / splits + kWarps - 1) / kWarps;
  rpw = (rpw + kD - 1) / kD * kD;
  p.rows_per_warp = (int)rpw;
  p.rows_per_cta = (int)(rpw * kWarps);
  const int64_t real = (K + p.rows_per_cta - 1) / p.rows_per_cta;
  p.grid_splits = (int)((real + p.cluster - 1) / p.cluster * p.cluster);
  const int nclu = p.grid_splits / p.cluster;
  p.slot_bytes = nclu > 1 ? (size_t)p.tiles * nclu * kSliceN * sizeof(float) : 0;
  p.counter_bytes = nclu > 1 ? (size_t)p.tiles * sizeof(unsigned) : 0;
  p.smem_bytes = m1_meta_bytes(p.rows_per_cta) + (kWarps + 1) * kSliceN * sizeof(float);
  return p;
}

// Clusters of `cluster` CTAs with `smem` bytes of dynamic shared memory each that the
// current device holds at once; 0 if no device can be asked. Every instantiation of
// the kernel has the same block size and register bound, so one answers for all.
static int resident_clusters(int cluster, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(dev, cluster, smem);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kern = m1_kernel<4, __nv_bfloat16, false>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1, (unsigned)cluster, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)cluster;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cache[key] = n;
  return n;
}

M1Plan plan_m1(int64_t K, int64_t N, int group, int sm_count, bool few_slots) {
  // One wave: 2 CTAs fit per SM, and a target of 1.9 CTAs per SM measured best on a
  // 148-SM B200. Clusters live inside one GPC, so 8-CTA clusters do not tile all SMs:
  // a grid with more clusters than the device holds at once would run the rest as a
  // second wave (and the fused all-reduce launch needs every CTA running), so the split
  // count drops one cluster per tile at a time until the grid is resident. Without a
  // device to ask (host-only queries) the first plan stands.
  (void)group;
  int64_t target = (int64_t)(sm_count > 0 ? sm_count : 148) * 19 / 10;
  M1Plan p = plan_for(K, N, target, few_slots);
  for (;;) {
    const int have = resident_clusters(p.cluster, p.smem_bytes);
    if (have <= 0 || (int64_t)p.tiles * p.grid_splits <= (int64_t)have * p.cluster) return p;
    if (p.grid_splits <= p.cluster) return p;  // one cluster per tile is the least
    target = (int64_t)p.tiles * (p.grid_splits - p.cluster);
    const M1Plan q = plan_for(K, N, target, few_slots);
    if ((int64_t)q.tiles * q.grid_splits >= (int64_t)p.tiles * p.grid_splits) return p;
    p = q;
  }
}

template <bool kAR>
int launch_m1_t(const M1Args& a, const M1Plan& p, int dtype, int nz, cudaStream_t st) {
  if (dtype == GRINQH_BF16) {
    switch (nz) {
      case 1: return launch_t<1, __nv_bfloat16, kAR>(a, p, st);
      case 2: return launch_t<2, __nv_bfloat16, kAR>(a, p, st);
      case 3: return launch_t<3, __nv_bfloat16, kAR>(a, p, st);
      default: return launch_t<4, __nv_bfloat16, kAR>(a, p, st);
    }
  }
  switch (nz) {
    case 1: return launch_t<1, __half, kAR>(a, p, st);
    case 2: return launch_t<2, __half, kAR>(a, p, st);
    case 3: return launch_t<3, __half, kAR>(a, p, st);
    default: return launch_t<4, __half, kAR>(a, p, st);
  }
}

int launch_m1(const M1Args& a, const M1Plan& p, int dtype, int nz, cudaStream_t st, bool allreduce) {
  return allreduce ? launch_m1_t<true>(a, p, dtype, nz, st) : launch_m1_t<false>(a, p, dtype, nz, st);
}

}  // namespace grinqh
