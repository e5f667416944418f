// Dense quantized GEMM for few rows (2..64 tokens) on the 5th-generation tensor
// cores: y = x @ dtype(w * s), the reference's M > 1 path (grinqh/kernel.py:561-587),
// with the roles of the operands swapped so that no MMA work is spent on padding
// rows: the weights are operand A (M = 128 weight columns per MMA) and the tokens
// are operand B (N = the row count rounded up to 16).
//
// A CTA owns a tile of 32 packed words (512 output columns) and a range of K steps
// of 32 rows. Three rings of shared-memory stages:
//   planes  (5 x 16 KB)  the b/2 plane words of 32 rows x 32 words, one 2-D TMA box
//                        per plane (128-byte swizzle), loaded up to five steps ahead
//                        by the loader warp;
//   weights (4 x 32 KB)  operand A: dtype(w * s) for 512 columns x 32 rows, MN-major
//                        with the 128-byte swizzle;
//   x       (4 x 4 KB)   operand B: Mp x 32 activations, K-major with the 64-byte
//                        swizzle (rows past M read as 0), loaded by TMA.
// Warps 0-15 convert (a warp covers 8 rows x 4 word pairs, so that every
// shared-memory access is free of bank conflicts): each thread owns two neighbouring
// words of one row (same scales' rows), reads their planes from shared memory, merges
// them into codes, forms the exact code in fp32, packs it to the activation dtype
// (exact: |code| <= 128) and multiplies it by the packed scale pair with one rounding
// -- the reference's dtype(w * s), bit for bit -- and stores the weight stage. Four
// converter warps per scheduler (96 registers a thread) hide the latency of that
// chain. Warp 16 loads the planes; warp 17 issues the MMAs (per 16-deep K slice, one
// tcgen05.mma kind::f16 per 128-column block, N = Mp) from one thread into TMEM;
// tcgen05.commit frees the stage, and warp 18 then loads the x tile of the step that
// reuses it (the x loads stay off the plane loader's TMA queue and out of the
// converters' loop). The converters never wait on global memory: the
// plane ring hides its latency.
//
// K is split over the CTAs of a thread-block cluster (and over several clusters for
// long K). Each CTA stages its fp32 partial tile in shared memory; rank r of the
// cluster adds the ranks' values for its share of the (row, column-group) pairs over
// distributed shared memory, in rank order. With one cluster per tile that sum is the
// result; otherwise it goes to an fp32 slot and the last cluster to finish a share
// (atomic ticket) adds the clusters' slots in order. Deterministic; every wait is
// bounded.
//
// Fused all-reduce (kAR, tensor-parallel row-parallel layers): where a CTA would write
// an entry of y it stores its fp32 value, tagged with the launch epoch, into every
// rank's peer buffer instead (peer_reduce.cuh), then waits for every rank's value of
// the same entries, adds them in rank order and writes y. A CTA waits on peer CTAs
// only, never on another CTA of its own grid, but the peer CTAs must be running: the
// host keeps the whole grid resident at once (plan_skinny_resident).
#include <cooperative_groups.h>
#include <cuda.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "gemm_skinny.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace grinqh {
namespace {

constexpr int TW = 32;         // packed words per tile
constexpr int TN = 16 * TW;    // output columns per tile
constexpr int BK = 32;         // rows per K step
constexpr int SP = 5, SW = 4;  // plane stages; weight / activation stages
#ifndef GRINQH_SKINNY_CONV_WARPS
#define GRINQH_SKINNY_CONV_WARPS 16
#endif
constexpr int kConvWarps = GRINQH_SKINNY_CONV_WARPS;  // 8 (two rows a thread) or 16 (one row)
static_assert(kConvWarps == 8 || kConvWarps == 16, "converter warps");
constexpr int kRowsPerThread = 16 / kConvWarps;       // rows of a step per converter thread
constexpr int kLoadWarp = kConvWarps, kMmaWarp = kConvWarps + 1, kXWarp = kConvWarps + 2;
constexpr int kThreads = 32 * (kConvWarps + 3);
constexpr int kMaxMp = 64;
constexpr uint32_t kPlaneBytes = BK * TW * 4;  // one plane of a step: 4 KB
constexpr uint32_t kStageP = 4 * kPlaneBytes;  // 16 KB
constexpr uint32_t kStageW = TN * BK * 2;      // 32 KB
constexpr uint32_t kStageX = kMaxMp * BK * 2;  // 4 KB
constexpr uint32_t kOffW = SP * kStageP;
constexpr uint32_t kOffX = kOffW + SW * kStageW;
constexpr uint32_t kOffBar = kOffX + SW * kStageX;
constexpr uint32_t kSmemBytes = kOffBar + 256 /*barriers*/ + 1024 /*align*/;
constexpr uint32_t kLbo = 4 * 1024;  // weights: stride between 64-column MN atoms (4 K atoms of 1 KB)
constexpr uint32_t kSbo = 1024;      // weights: stride between 8-row K groups
constexpr uint32_t kSboX = 512;      // x: stride between 8-row groups of 64-byte rows
constexpr int kPartRow = 16 * 33;    // fp32 partial staging [m][c][word], words padded to 33

static_assert((size_t)kMaxMp * kPartRow * 4 <= kOffBar, "partial tile must fit in the stages");
static_assert(kSmemBytes <= 227 * 1024, "shared memory");

template <typename T> struct Fmt;
template <> struct Fmt<__nv_bfloat16> {
  static constexpr uint32_t v = 1;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t bits) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bits));
  }
  // a * b per half, rounded once to the dtype (the exact product of two dtype values)
  static __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};
template <> struct Fmt<__half> {
  static constexpr uint32_t v = 0;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t bits) {
    return __half22float2(*reinterpret_cast<const __half2*>(&bits));
  }
  static __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

__device__ __forceinline__ uint64_t* bar_at(unsigned char* smem, int i) {
  return reinterpret_cast<uint64_t*>(smem + kOffBar) + i;
}

template <int NZ, typename T, bool kAR>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                  const SkinnyArgs a, const int mp) {
  constexpr int kShift = 8 - 2 * NZ;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sP = smem;
  unsigned char* sW = smem + kOffW;
  unsigned char* sX = smem + kOffX;
  uint64_t* p_full = bar_at(smem, 0);
  uint64_t* p_empty = bar_at(smem, SP);
  uint64_t* x_full = bar_at(smem, 2 * SP);
  uint64_t* w_full = bar_at(smem, 2 * SP + SW);
  uint64_t* empty = bar_at(smem, 2 * SP + 2 * SW);
  uint64_t* acc_full = bar_at(smem, 2 * SP + 3 * SW);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_at(smem, 2 * SP + 3 * SW + 1));
  __shared__ int s_last;
  __shared__ unsigned s_epoch;

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
    for (int s = 0; s < SP; ++s) {
      mbar_init(&p_full[s], 1);
      mbar_init(&p_empty[s], kConvWarps);
    }
    for (int s = 0; s < SW; ++s) {
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

  // Dependent launch: only the plane loader may run ahead of the previous kernel on
  // the stream (the weights are never written by other kernels); everything that
  // reads x or writes the output or the workspace waits for it first.
  const bool loader = warp == kLoadWarp && lane == 0;
  if (!loader) wait_prior_grid();
  if (warp == kLoadWarp) {
    // ------------------------------------------------------------ plane loader
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      for (int i = 0; i < nq; ++i) {
        const int s = i % SP;
        if (i >= SP) mbar_wait(&p_empty[s], ((i / SP) - 1) & 1);
        mbar_arrive_expect_tx(&p_full[s], NZ * kPlaneBytes);
        const int row = (q0 + i) * BK;
#pragma unroll
        for (int z = 0; z < NZ; ++z)
          tma_load_2d(sP + s * kStageP + z * kPlaneBytes, &tmap_w, z * n16 + jt0, row, &p_full[s]);
      }
      wait_prior_grid();
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc(1, Fmt<T>::v, Fmt<T>::v, 1, 0, (uint32_t)mp, 128);
      for (int i = 0; i < nq; ++i) {
        const int s = i % SW;
        const uint32_t ph = (i / SW) & 1;
        mbar_wait(&x_full[s], ph);
        mbar_wait(&w_full[s], ph);
        tc_fence_after();
        const uint32_t wbase = smem_u32(sW + s * kStageW);
        const uint32_t xbase = smem_u32(sX + s * kStageX);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t bdesc = smem_desc(xbase + kk * 32, 16, kSboX, 4);
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
    __syncwarp();
  } else if (warp == kXWarp) {
    // ------------------------------------------------------------ activation loader
    // x of step i into stage i % SW as soon as the MMAs of step i - SW have released
    // it, so the load is in flight well before the MMAs need it. A warp of its own: a
    // lane of the MMA warp waiting on a barrier would hold back a lane of the same warp
    // that must act for the barrier to complete.
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      const uint32_t xbytes = (uint32_t)mp * BK * 2;
      for (int i = 0; i < nq; ++i) {
        const int s = i % SW;
        if (i >= SW) mbar_wait(&empty[s], ((i / SW) - 1) & 1);
        mbar_arrive_expect_tx(&x_full[s], xbytes);
        tma_load_2d(sX + s * kStageX, &tmap_x, (q0 + i) * BK, 0, &x_full[s]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ converters
    // a warp covers 8 rows x 4 word pairs (kRowsPerThread times): in every
    // shared-memory access the 8 lanes of a phase are 8 different rows, which the
    // 128-byte swizzle spreads over all banks
    constexpr int kWarpRowSets = 4 / kRowsPerThread;          // warps side by side along the rows
    const int rr = 8 * kRowsPerThread * (warp % kWarpRowSets) + (lane & 7);  // rows rr + 8 h
    const int jp = 4 * (warp / kWarpRowSets) + (lane >> 3);   // this thread's words: 2 jp, 2 jp + 1
    const int jw = jt0 + 2 * jp;
    const bool jvalid = jw < n16;      // n16 is even: both words are valid or neither
    const int spg = a.group / BK;      // K steps per scale group
    // byte u (offset binary, code = u - 128, shifted left by 8 - b) -> u / 2^shift plus
    // 2^(23-shift), exactly: the float with bits 0x4B000000 - (shift << 23) | u; minus
    // the magic constant that is the unshifted code, exactly
    constexpr uint32_t kMagicBits = 0x4B000000u - ((uint32_t)kShift << 23);
    constexpr float kMagic = (float)(8388608.0 + 128.0) / float(1 << kShift);
    // Scales of the current group as packed dtype pairs of neighbouring column groups:
    // sa[2t + p] = (s[4t + 2p], s[4t + 2p + 1]) of word 2 jp, sb the same of word
    // 2 jp + 1, where s[c] = s[g, c * n16 + word]. The next group's scales are
    // prefetched as they lie in memory (snext[c] = both words of column group c).
    uint32_t sa[8], sb[8], snext[16];
    auto load_scales = [&](int g) {
      const uint32_t* sp =
          reinterpret_cast<const uint32_t*>(static_cast<const T*>(a.s) + (size_t)g * a.N + (jvalid ? jw : 0));
#pragma unroll
      for (int c = 0; c < 16; ++c) snext[c] = jvalid ? __ldg(sp + (size_t)c * (n16 >> 1)) : 0u;
    };
    auto unpack_scales = [&]() {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        sa[k] = __byte_perm(snext[2 * k], snext[2 * k + 1], 0x5410u);
        sb[k] = __byte_perm(snext[2 * k], snext[2 * k + 1], 0x7632u);
      }
    };
    int g_next = 0;  // first K step of the next scale group
    if (nq > 0) {
      const int g0 = q0 / spg;
      load_scales(g0);
      unpack_scales();
      g_next = (g0 + 1) * spg;
      if (g_next < q0 + nq) load_scales(g0 + 1);
    }
    // store offsets of rows rr + 8 h in the weight stage (MN-major, 128-byte swizzle:
    // 16-byte chunk c of row k sits at (c ^ (k & 7)); every row has k & 7 = rr & 7)
    const uint32_t rsw = (uint32_t)(rr & 7);
    const uint32_t c0 = (uint32_t)(4 * jp) & 7u;  // first of the thread's four chunks (0 or 4)
    uint32_t row_base[kRowsPerThread];
#pragma unroll
    for (int h = 0; h < kRowsPerThread; ++h) {
      const int k = rr + 8 * h;
      row_base[h] = (uint32_t)(((4 * jp) >> 3) * kLbo + (k >> 3) * kSbo + (k & 7) * 128);
    }
    uint32_t chunk_off[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) chunk_off[e] = ((c0 + (uint32_t)e) ^ rsw) << 4;
    // plane words of the thread's rows (the TMA swizzles the 128-byte plane rows: 16-byte
    // chunk c of row r at chunk c ^ (r & 7)); the same offset in every stage
    const uint32_t poff =
        (uint32_t)(rr * (TW * 4)) + ((((uint32_t)jp >> 1) ^ (uint32_t)(rr & 7)) << 4) + (uint32_t)(jp & 1) * 8u;

    // code bytes of one merged word -> dtype(code * s) for its 16 columns, as 8 packed
    // pairs (columns 4t + 2p, 4t + 2p + 1): exact code in fp32, packed to the dtype
    // (|code| <= 128 is exact there), one rounded multiply by the scale pair
    auto convert = [&](const uint32_t (&q)[4], const uint32_t (&sc)[8], uint32_t (&o)[8]) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 f = make_float2(__int_as_float(__byte_perm(q[t], kMagicBits, 0x7440u | (2u * p))),
                                       __int_as_float(__byte_perm(q[t], kMagicBits, 0x7440u | (2u * p + 1u))));
          const float2 c = __fadd2_rn(f, make_float2(-kMagic, -kMagic));
          o[2 * t + p] = Fmt<T>::mul2(Fmt<T>::pack(c.x, c.y), sc[2 * t + p]);
        }
      }
    };

    for (int i = 0; i < nq; ++i) {
      const int q = q0 + i, s = i % SW, ps = i % SP;
      if (q == g_next) {  // next scale group: its scales were prefetched
        unpack_scales();
        g_next += spg;
        if (g_next < q0 + nq) load_scales(g_next / spg);
      }
      if (i >= SW) mbar_wait_inline(&empty[s], ((i / SW) - 1) & 1);
      mbar_wait_inline(&p_full[ps], (i / SP) & 1);
      uint2 P[kRowsPerThread][4];
      const unsigned char* pst = sP + ps * kStageP + poff;
#pragma unroll
      for (int h = 0; h < kRowsPerThread; ++h)
#pragma unroll
        for (int z = 0; z < 4; ++z)
          P[h][z] = z < NZ ? *reinterpret_cast<const uint2*>(pst + h * 8 * (TW * 4) + z * kPlaneBytes)
                           : make_uint2(0u, 0u);
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_empty[ps]);

      unsigned char* wst = sW + s * kStageW;
#pragma unroll
      for (int h = 0; h < kRowsPerThread; ++h) {
        uint32_t qa[4], qb[4];  // merged code bytes of word 2 jp (a) and 2 jp + 1 (b)
        merge_planes(P[h][0].x ^ kSignFlip, P[h][1].x, P[h][2].x, P[h][3].x, qa);
        merge_planes(P[h][0].y ^ kSignFlip, P[h][1].y, P[h][2].y, P[h][3].y, qb);
        uint32_t oa[8], ob[8];
        convert(qa, sa, oa);  // dtype(code * s) rounded once (kernel.py:586)
        convert(qb, sb, ob);
        unsigned char* rowp = wst + row_base[h];
        *reinterpret_cast<uint4*>(rowp + chunk_off[0]) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
        *reinterpret_cast<uint4*>(rowp + chunk_off[1]) = make_uint4(oa[4], oa[5], oa[6], oa[7]);
        *reinterpret_cast<uint4*>(rowp + chunk_off[2]) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
        *reinterpret_cast<uint4*>(rowp + chunk_off[3]) = make_uint4(ob[4], ob[5], ob[6], ob[7]);
      }
      fence_proxy_async_smem();  // make the generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&w_full[s]);
    }

    allow_dependent_grid();

    // ------------------------------------------------------------ partial tile -> smem
    // accumulator block b, TMEM lane p (this warp may read lanes 32 * (warp % 4) ..):
    // tile position P = 128 b + p, word P / 16, column group P % 16 (the converters'
    // order); TMEM column m = token m.
    mbar_wait(acc_full, 0);
    tc_fence_after();
    float* part = reinterpret_cast<float*>(smem);  // the stages are idle now
    const int quarter = warp & 3;
#pragma unroll 1
    for (int blk = warp >> 2; blk < 4; blk += kConvWarps / 4) {
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
  }
  // fused all-reduce: the epoch of this launch (thread 0 is past wait_prior_grid)
  if constexpr (kAR)
    if (threadIdx.x == 0) s_epoch = peer_epoch(a.ar);
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, tcols);

  // ------------------------------------------------------------ reduction and store
  T* y = static_cast<T*>(a.y);
  const T* bias = static_cast<const T*>(a.bias);
  const float* part = reinterpret_cast<const float*>(smem);
  const unsigned epoch = kAR ? s_epoch : 0u;
  // (row m, column group c, word w) -> y[m, c * n16 + jt0 + w]; one warp writes a
  // pair's 32 words (64 contiguous bytes)
  auto store_y = [&](int m, int c, int w, float v) {
    if (m >= a.M || jt0 + w >= n16) return;
    const int n = c * n16 + jt0 + w;
    T out = Act<T>::from_f(v);
    if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[n]));
    y[(size_t)m * a.N + n] = out;
  };
  // the final K sum of an entry: y, or with the fused all-reduce this rank's partial,
  // stored into every rank's buffer (a warp stores a pair's 32 words, 256 contiguous
  // bytes, into each); the ranks' sums follow in peer_gather
  auto finish = [&](int m, int c, int w, float v) {
    if constexpr (kAR) {
      if (m >= a.M || jt0 + w >= n16) return;
      peer_publish(a.ar, epoch, (size_t)m * a.N + c * n16 + jt0 + w, v);
    } else {
      store_y(m, c, w, v);
    }
  };
  // fused all-reduce, second half: for the pairs first, first + stride, ... (below
  // npairs) that this warp published, every rank's partial summed in rank order (four
  // pairs' words in flight at a time), the bias added, y written. A CTA waits only on
  // the peer CTAs that publish the same entries, which publish before they wait.
  const int npairs = mp * 16;
  auto peer_gather = [&](int first, int stride) {
    if constexpr (kAR) {
      for (int p0 = first; p0 < npairs; p0 += 4 * stride) {
        size_t e[4];
        bool ok[4];
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int pr = p0 + i * stride, m = pr >> 4;
          ok[i] = pr < npairs && m < a.M && jt0 + lane < n16;
          e[i] = (size_t)m * a.N + (pr & 15) * n16 + jt0 + lane;
        }
        peer_sum<4>(a.ar, epoch, e, ok, v);  // on a timeout y is invalid; the host sees the count
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (ok[i]) store_y((p0 + i * stride) >> 4, (p0 + i * stride) & 15, lane, v[i]);
      }
    }
  };
  if (a.splits == 1) {
    for (int pr = warp; pr < npairs; pr += kThreads / 32)
      finish(pr >> 4, pr & 15, lane, part[(pr >> 4) * kPartRow + (pr & 15) * 33 + lane]);
    peer_gather(warp, kThreads / 32);
    peer_cta_done<kAR>(a.ar, epoch);
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
    for (int r = 0; r < cs; ++r) v += cluster.map_shared_rank(part, r)[off];
    if (nclu == 1) finish(pr >> 4, pr & 15, lane, v);
    else __stcg(myslot + (size_t)pr * 32 + lane, v);
  }
  cluster.sync();  // every rank keeps its shared memory until the others have read it
  if (nclu == 1) {
    peer_gather(crank + cs * warp, cs * (kThreads / 32));
    peer_cta_done<kAR>(a.ar, epoch);
    return;
  }
  __threadfence();
  __syncthreads();
  unsigned* ticket = a.counters + (size_t)tile * cs + crank;
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1u) == (unsigned)(nclu - 1);
  __syncthreads();
  if (!s_last) {
    peer_cta_done<kAR>(a.ar, epoch);
    return;
  }
  __threadfence();
  for (int k = warp; crank + cs * k < npairs; k += kThreads / 32) {
    const int pr = crank + cs * k;
    float v = 0.f;
    for (int cl = 0; cl < nclu; ++cl)
      v += __ldcg(a.slots + ((size_t)tile * nclu + cl) * slot_elems + (size_t)pr * 32 + lane);
    finish(pr >> 4, pr & 15, lane, v);
  }
  if (threadIdx.x == 0) *ticket = 0u;  // ready for the next launch
  peer_gather(crank + cs * warp, cs * (kThreads / 32));
  peer_cta_done<kAR>(a.ar, epoch);
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

template <int NZ, typename T, bool kAR>
int launch_t(const SkinnyArgs& a, const SkinnyPlan& p, cudaStream_t st) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint32_t estride[2] = {1, 1};
  // activations [M, K]: boxes of 32 K-elements (64 bytes) x Mp rows, 64-byte swizzle
  CUtensorMap tmap_x;
  {
    const cuuint64_t gdim[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
    const cuuint64_t gstride[1] = {(cuuint64_t)a.K * 2};
    const cuuint32_t box[2] = {BK, (cuuint32_t)p.mp};
    const CUresult r = enc(&tmap_x, Fmt<T>::v ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           2, const_cast<void*>(a.x), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled(x) failed (%d)", (int)r);
  }
  // packed planes [K, nz * N/16] uint32: boxes of 32 words (128 bytes) x 32 rows,
  // 128-byte swizzle (conflict-free reads by the converters)
  CUtensorMap tmap_w;
  {
    const cuuint64_t gdim[2] = {(cuuint64_t)NZ * (a.N / 16), (cuuint64_t)a.K};
    const cuuint64_t gstride[1] = {(cuuint64_t)NZ * (a.N / 16) * 4};
    const cuuint32_t box[2] = {TW, BK};
    const CUresult r = enc(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(a.w), gdim, gstride,
                           box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled(w) failed (%d)", (int)r);
  }
  auto kern = skinny_kernel<NZ, T, kAR>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)p.tiles, (unsigned)p.splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.cluster;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see wait_prior_grid()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, tmap_x, tmap_w, a, p.mp);
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
  // K steps of 32 rows that never straddle a scale group; plane boxes start on 16-byte
  // boundaries (N / 16 words per plane a multiple of 4, so N % 64 == 0); a thread's two
  // words and their two scales are one 8-byte and one 4-byte load
  return M >= 2 && M <= kMaxMp && K % BK == 0 && group % BK == 0 && N % 64 == 0 && K < (1LL << 31);
}

bool skinny_pointers_ok(const void* x, const void* w, const void* s) {
  return (reinterpret_cast<uintptr_t>(x) % 16) == 0 && (reinterpret_cast<uintptr_t>(w) % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(s) % 4) == 0;
}

static SkinnyPlan plan_for(int64_t M, int64_t K, int64_t N, int64_t target, int max_cluster = 8) {
  SkinnyPlan p{};
  p.mp = (int)((M + 15) / 16 * 16);
  const int64_t n16 = N / 16;
  p.tiles = (int)((n16 + TW - 1) / TW);
  const int64_t nk = K / BK;
  int64_t splits = target / p.tiles;
  if (splits > nk) splits = nk;
  if (splits < 1) splits = 1;
  int64_t steps = (nk + splits - 1) / splits;
  splits = (nk + steps - 1) / steps;  // no empty splits
  // cluster: the largest size <= max_cluster (8) that divides the split count
  int cl = 1;
  for (int c = max_cluster; c >= 1; --c)
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


// Clusters of `cluster` CTAs that the current device holds at once. Every
// instantiation of the kernel has the same block size, shared memory and register
// bound (one CTA per SM), so one of them answers for all.
static int resident_clusters(int cluster) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(dev, cluster);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kern = skinny_kernel<4, __nv_bfloat16, true>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1, (unsigned)cluster, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
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

bool plan_skinny_resident(int64_t M, int64_t K, int64_t N, int sm_count, SkinnyPlan* out) {
  int64_t target = (int64_t)(sm_count > 0 ? sm_count : 148) * 7 / 8;
  for (;;) {
    // the split count of plan_skinny with the largest cluster whose grid is resident
    // (clusters live inside one GPC, so smaller ones pack the SMs more densely)
    SkinnyPlan p{};
    for (int cmax = 8; cmax >= 1; cmax = p.cluster - 1) {
      p = plan_for(M, K, N, target, cmax);
      const int have = resident_clusters(p.cluster);
      if (have > 0 && (int64_t)p.tiles * p.splits <= (int64_t)have * p.cluster) {
        *out = p;
        return true;
      }
      if (have <= 0) return false;
    }
    if (p.splits == 1) return false;           // even one CTA per tile does not fit
    target = (int64_t)p.tiles * p.splits - 1;  // fewer splits
  }
}

template <bool kAR>
static int launch_ar(const SkinnyArgs& a, const SkinnyPlan& p, int dtype, int nz, cudaStream_t st) {
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

SkinnyPlan plan_skinny(int64_t M, int64_t K, int64_t N, int sm_count) {
  // One CTA per SM (about 225 KB of shared memory each), aiming a little under the SM
  // count. Clusters live inside one GPC, so 8-CTA clusters do not tile all SMs (a
  // 148-SM B200 holds 15 of them, 120 CTAs): a grid one cluster too large would run
  // that cluster as a second wave, doubling the time. The resident plan avoids that;
  // without a device to ask (host-only queries) the plain plan is used.
  SkinnyPlan p{};
  if (plan_skinny_resident(M, K, N, sm_count, &p)) return p;
  return plan_for(M, K, N, (int64_t)(sm_count > 0 ? sm_count : 148) * 7 / 8);
}

int launch_skinny(const SkinnyArgs& a, const SkinnyPlan& p, int dtype, int nz, cudaStream_t st, bool allreduce) {
  return allreduce ? launch_ar<true>(a, p, dtype, nz, st) : launch_ar<false>(a, p, dtype, nz, st);
}

}  // namespace grinqh
