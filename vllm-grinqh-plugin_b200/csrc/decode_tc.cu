// Single-row graded GEMV (the reference's M == 1 path, grinqh/kernel.py:39-167) on
// the tensor cores as an exact integer dot-product engine.
//
// Per unit -- 64 rows (half a K group) of a column tile of 32 packed words = 512
// output columns, four MMA blocks of M = 128:
//   A  [512 columns x 64 rows] int8 -- the merged planes of every graded row are
//      exactly the shifted codes int8(code << (8-b)) with inactive zones cleared
//      (kernel.py:120-146), written MN-major with a 128-byte swizzle: a lane's 16
//      columns of one row are one 16-byte store;
//   B  [16 x 64 rows] int8 -- three digits of x in 21-bit fixed point at the
//      unit's power-of-two scale 2^e: x ~= 2^(e-21) (d0 2^14 + d1 2^7 + d2); rows
//      graded 0 get zero digits, so their weight rows are never loaded or merged;
//   D  = A * B with tcgen05.mma kind::i8 into int32 TMEM columns (exact).
// The epilogue (four output columns per thread) adds, per unit of group g,
//   s[g, n] * (2^(e-21-shift) (D0 2^14 + D1 2^7 + D2) + sum_k bias_k x_k)
// i.e. s * (sum(code * x) + sum(bias * x)) of kernel.py:148-158.
//
// A warp reads 128 contiguous bytes per plane row, so every DRAM line is fetched
// once. Warps: 0-7 convert (plane loads two units ahead in registers, merge, store A),
// 8 builds B and issues the MMAs from one thread, 9-12 are the epilogue (TMEM lane
// quarters 1, 2, 3, 0). Units (tile, group) are walked tile-major and split into
// one contiguous range per CTA; CTAs that share a tile write partial slots and the
// last one (atomic ticket) adds them in CTA order, so results are deterministic.
#include "common.cuh"
#include "decode_tc.cuh"
#include "ptx.cuh"

namespace grinqh {
namespace {

constexpr int kConvWarps = 8;
constexpr int kThreads = 32 * (kConvWarps + 1 + 4);
constexpr int kGroup = 128;                 // K group of the scales
constexpr int kRowsU = 64;                  // rows per unit (half a group)
constexpr int kTileW = 32;                  // packed words per column tile (128 B per plane row)
constexpr int kTileCols = 16 * kTileW;      // 512 output columns = 4 MMA blocks of M = 128
constexpr int kMBlocks = kTileCols / 128;
constexpr int kStages = 4;
constexpr uint32_t kAtomLbo = (kRowsU / 8) * 1024;  // A: stride between 128-column MN atoms
constexpr uint32_t kStageA = kTileCols * kRowsU;    // 32 KB int8
constexpr uint32_t kStageB = 16 * 128;              // 2 KB int8 (rows of 128 B, first 64 used)
constexpr int kAccCols = 16;                        // TMEM columns per MMA block and unit
constexpr int kAccBlocks = 8;                       // MMAs may run this many units ahead of the epilogue
constexpr uint32_t kTmemCols = kAccCols * kMBlocks * kAccBlocks;  // 512
constexpr int kFix = 21;                           // fixed-point bits of the x digits

struct Smem {
  static constexpr uint32_t a = 0;
  static constexpr uint32_t b = a + kStages * kStageA;
  static constexpr uint32_t masks = b + kStages * kStageB;
};

// per-unit fp32 pairs (2^(e-21-shift), sum bias*x) follow the K grade bytes, then
// the barriers
__host__ __device__ inline uint32_t ex_offset(int K) { return Smem::masks + ((uint32_t)K + 15) / 16 * 16; }
__host__ __device__ inline uint32_t bars_offset(int K, int upc) { return ex_offset(K) + (uint32_t)upc * 8; }
__host__ __device__ inline uint32_t smem_bytes_tc(int K, int upc) { return 1024 + bars_offset(K, upc) + 512; }

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

template <int NZ>
__device__ __forceinline__ uint32_t grade_of(float xv, const M1TcArgs& a) {
  const float ax = fabsf(xv);
  uint32_t g = (uint32_t)(ax > a.t[0]) | ((uint32_t)(ax > a.t[1]) << 1) | ((uint32_t)(ax > a.t[2]) << 2) |
               ((uint32_t)(ax > a.t[3]) << 3);
  return g & ((1u << NZ) - 1u);
}

template <int NZ, typename T>
__global__ void __launch_bounds__(kThreads, 1) m1tc_kernel(const M1TcArgs a) {
  constexpr int kShift = 8 - 2 * NZ;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem + Smem::a;
  unsigned char* sB = smem + Smem::b;
  uint8_t* masks = smem + Smem::masks;                                    // grade of every row of K
  float* sEx = reinterpret_cast<float*>(smem + ex_offset(a.K));           // [unit][2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bars_offset(a.K, a.units_per_cta));
  uint64_t* full = bars;                   // converters (8) + B builder (1)
  uint64_t* empty = bars + kStages;        // MMA commit
  uint64_t* acc_full = bars + 2 * kStages;     // [kAccBlocks] MMA commit
  uint64_t* acc_empty = acc_full + kAccBlocks; // [kAccBlocks] epilogue warps (4)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kAccBlocks);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n16 = a.N >> 4;
  const int ngroups = a.K / kRowsU;  // units per tile
  const int64_t total = (int64_t)a.tiles * ngroups;
  const int64_t u_begin = (int64_t)blockIdx.x * a.units_per_cta;
  const int64_t u_end = min(total, u_begin + a.units_per_cta);
  const int nunits = (int)(u_end - u_begin);
  const T* x = static_cast<const T*>(a.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], kConvWarps + 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBlocks; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_mbar_init();
  }
  for (int k = threadIdx.x; k < a.K; k += kThreads) masks[k] = (uint8_t)grade_of<NZ>(Act<T>::to_f(x[k]), a);
  if (warp == kConvWarps) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kConvWarps) {
    // ------------------------------------------------------------ converters
    const int jj = lane;               // word of the tile
    const int rw = warp;               // rows rw + 8 i of the unit
    const size_t row_words = (size_t)NZ * n16;
    uint32_t P1[8][4], P2[8][4];
    // row k's plane z word of this lane: a.w + k * row_words + z * n16 + jw; the unit's
    // rows are rw + 8 i, so successive rows of a lane are 8 * row_words apart
    const uint32_t row8 = (uint32_t)(8 * row_words);
    auto load_unit = [&](uint32_t (&P)[8][4], int ui) {
      const int64_t u = u_begin + ui;
      const int tile = (int)(u / ngroups), g = (int)(u - (int64_t)tile * ngroups);
      const int jw = tile * kTileW + jj;
      const bool ok = ui < nunits && jw < n16;
      const int kb = g * kRowsU + rw;
      const uint32_t* wb = a.w + (size_t)kb * row_words + jw;
      // grades of the lane's 8 rows, one byte each (masks is 16-byte aligned, rows rw + 8 i)
      uint32_t mrow[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mrow[i] = ok ? (uint32_t)masks[kb + 8 * i] : 0u;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t* wr = wb + (size_t)i * row8;
#pragma unroll
        for (int z = 0; z < 4; ++z) P[i][z] = z < NZ ? ld_cs_if(wr + (size_t)z * n16, mrow[i], 1u << z) : 0u;
      }
    };
    const uint32_t col_off = (uint32_t)(jj >> 3) * kAtomLbo;  // MN atom of this word
    const int chunk = jj & 7;
    auto store_unit = [&](const uint32_t (&P)[8][4], int ui) {
      const int s = ui % kStages;
      if (ui >= kStages) mbar_wait(&empty[s], ((ui / kStages) - 1) & 1);
      unsigned char* ast = sA + s * kStageA + col_off;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t q[4];
        merge_planes(P[i][0], P[i][1], P[i][2], P[i][3], q);  // int8 codes << shift, inactive zones 0
        const int k = rw + 8 * i;
        // MN-major, 128-byte swizzle: 8-row K atoms of 1 KB, 16-byte chunk of row k
        *reinterpret_cast<uint4*>(ast + (k >> 3) * 1024 + (k & 7) * 128 + ((chunk ^ (k & 7)) << 4)) =
            make_uint4(q[0], q[1], q[2], q[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    };
    // the buffers rotate by name: a register copy of a pending load would wait for it
    load_unit(P1, 0);
    load_unit(P2, 1);
    for (int ui = 0; ui < nunits; ui += 2) {
      store_unit(P1, ui);
      load_unit(P1, ui + 2);
      if (ui + 1 < nunits) {
        store_unit(P2, ui + 1);
        load_unit(P2, ui + 3);
      }
    }
  } else if (warp == kConvWarps) {
    // ------------------------------------------------------------ B builder + MMA issuer
    constexpr uint32_t idesc = instr_desc(2 /*s32*/, 1 /*s8*/, 1 /*s8*/, 1 /*A MN-major*/, 0 /*B K-major*/, 16, 128);
    // x of the next unit's group is loaded while the current one is built
    T xa[2], xb[2];
    auto load_x = [&](T (&dst)[2], int ui) {
      const int g = (int)((u_begin + ui) % ngroups);
#pragma unroll
      for (int i = 0; i < 2; ++i) dst[i] = ui < nunits ? x[g * kRowsU + lane * 2 + i] : Act<T>::from_f(0.f);
    };
    load_x(xa, 0);
    load_x(xb, 1);
    for (int ui = 0; ui < nunits; ++ui) {
      const int s = ui % kStages;
      const int64_t u = u_begin + ui;
      const int g = (int)(u % ngroups);
      const int acc_b = ui % kAccBlocks;
      float xcur[2];
      if (ui & 1) {
#pragma unroll
        for (int i = 0; i < 2; ++i) xcur[i] = Act<T>::to_f(xb[i]);
        load_x(xb, ui + 2);
      } else {
#pragma unroll
        for (int i = 0; i < 2; ++i) xcur[i] = Act<T>::to_f(xa[i]);
        load_x(xa, ui + 2);
      }
      if (ui >= kStages) mbar_wait(&empty[s], ((ui / kStages) - 1) & 1);
      // digits of x for the unit's 64 rows (2 per lane); graded-0 rows get zeros
      float xv[2];
      uint32_t mk[2];
      float amax = 0.f, bsum = 0.f;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int k = g * kRowsU + lane * 2 + i;
        xv[i] = xcur[i];
        mk[i] = masks[k];
        if (mk[i]) amax = fmaxf(amax, fabsf(xv[i]));
        bsum += float(zone_bias<NZ>(mk[i])) * xv[i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
      }
      // 2^e > amax; q = rint(x * 2^(21-e)) fits 22 bits signed
      int e = 0;
      if (amax > 0.f) frexpf(amax, &e);
      const float to_fix = ldexpf(1.0f, kFix - e);
      uint32_t d0 = 0, d1 = 0, d2 = 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int qv = mk[i] ? max(-(1 << kFix) + 1, min((1 << kFix) - 1, __float2int_rn(xv[i] * to_fix))) : 0;
        d0 |= (uint32_t)((qv >> 14) & 0xFF) << (8 * i);
        d1 |= (uint32_t)((qv >> 7) & 0x7F) << (8 * i);
        d2 |= (uint32_t)(qv & 0x7F) << (8 * i);
      }
      // B: K-major, 128-byte swizzle, row t = digit column (rows 3..15 stay zero);
      // k = 2 lane + i is byte (2 lane + i) of the row: chunk lane/8, 2-byte slot
      unsigned char* bst = sB + s * kStageB;
      const int chunk = lane >> 3, within = (lane & 7) * 2;
      const uint32_t dig[3] = {d0, d1, d2};
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const uint32_t v = t < 3 ? dig[t] : 0u;
        const int r = t & 7, atom = t >> 3;
        *reinterpret_cast<uint16_t*>(bst + atom * 1024 + r * 128 + ((chunk ^ r) << 4) + within) = (uint16_t)v;
      }
      if (lane == 0) {
        sEx[ui * 2 + 0] = ldexpf(1.0f, e - kFix - kShift);
        sEx[ui * 2 + 1] = bsum;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[s]);
        mbar_wait(&full[s], (ui / kStages) & 1);
        if (ui >= kAccBlocks) mbar_wait(&acc_empty[acc_b], ((ui / kAccBlocks) - 1) & 1);
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * kStageA);
        const uint32_t b_base = smem_u32(sB + s * kStageB);
#pragma unroll
        for (int kk = 0; kk < kRowsU / 32; ++kk) {
          // A: +32 rows = 4 K atoms; B: +32 bytes inside the 128-byte rows
          const uint64_t bdesc = smem_desc(b_base + kk * 32, 16, 1024, 2);
#pragma unroll
          for (int mb = 0; mb < kMBlocks; ++mb) {
            const uint64_t adesc = smem_desc(a_base + mb * kAtomLbo + kk * 4096, kAtomLbo, 1024, 2);
            mma_i8_ss(tmem + (acc_b * kMBlocks + mb) * kAccCols, adesc, bdesc, idesc, kk > 0 ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
        mma_commit(&acc_full[acc_b]);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int ml = quarter * 32 + lane;  // row of each 128-column MMA block
    const int c = ml & 15;
    const T* sc = static_cast<const T*>(a.s);
    T* y = static_cast<T*>(a.y);
    const T* bias = static_cast<const T*>(a.bias);
    float acc[kMBlocks];
#pragma unroll
    for (int mb = 0; mb < kMBlocks; ++mb) acc[mb] = 0.f;
    int cur_tile = -1;
    auto emit = [&](int tile) {
      const int first = (int)(((int64_t)tile * ngroups) / a.units_per_cta);
      const int last = (int)min((int64_t)gridDim.x - 1, ((int64_t)(tile + 1) * ngroups - 1) / a.units_per_cta);
#pragma unroll
      for (int mb = 0; mb < kMBlocks; ++mb) {
        __stcg(a.slots + (size_t)(blockIdx.x + tile) * kTileCols + mb * 128 + ml, acc[mb]);
        acc[mb] = 0.f;
      }
      __threadfence();
      named_barrier(1, 128);
      if (threadIdx.x == 32 * (kConvWarps + 1)) *s_last = atomicAdd(a.counters + tile, 1u) == (unsigned)(last - first);
      named_barrier(1, 128);
      if (!*s_last) return;
      __threadfence();
#pragma unroll 1
      for (int mb = 0; mb < kMBlocks; ++mb) {
        const int col = mb * 128 + ml;
        float v = 0.f;
        for (int sl = first; sl <= last; sl += 8) {
          float buf[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            buf[q] = (sl + q <= last) ? __ldcg(a.slots + (size_t)(sl + q + tile) * kTileCols + col) : 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) v += buf[q];
        }
        const int jw = tile * kTileW + col / 16;
        if (jw < n16) {
          const int n = c * n16 + jw;
          T o = Act<T>::from_f(v);
          if (bias) o = Act<T>::from_f(Act<T>::to_f(o) + Act<T>::to_f(bias[n]));
          y[n] = o;
        }
      }
      named_barrier(1, 128);
      if (threadIdx.x == 32 * (kConvWarps + 1)) a.counters[tile] = 0u;  // ready for the next launch
    };
    // scales of units ui+1..ui+3 are in flight while unit ui is finished
    auto load_sv = [&](float (&dst)[kMBlocks], int ui) {
      const int64_t u = u_begin + ui;
      const int tile = (int)(u / ngroups), g = (int)(u - (int64_t)tile * ngroups);
      const int grp = (g * kRowsU) / kGroup;
#pragma unroll
      for (int mb = 0; mb < kMBlocks; ++mb) {
        const int jw = tile * kTileW + (mb * 128 + ml) / 16;
        dst[mb] = (ui < nunits && jw < n16) ? Act<T>::to_f(sc[(size_t)grp * a.N + (size_t)c * n16 + jw]) : 0.f;
      }
    };
    float sva[kMBlocks], svb[kMBlocks], svc[kMBlocks];
    load_sv(sva, 0);
    load_sv(svb, 1);
    load_sv(svc, 2);
    for (int ui = 0; ui < nunits; ++ui) {
      const int64_t u = u_begin + ui;
      const int tile = (int)(u / ngroups);
      if (tile != cur_tile) {
        if (cur_tile >= 0) emit(cur_tile);
        cur_tile = tile;
      }
      float sv[kMBlocks];
      const int rot = ui % 3;
      if (rot == 0) {
#pragma unroll
        for (int mb = 0; mb < kMBlocks; ++mb) sv[mb] = sva[mb];
        load_sv(sva, ui + 3);
      } else if (rot == 1) {
#pragma unroll
        for (int mb = 0; mb < kMBlocks; ++mb) sv[mb] = svb[mb];
        load_sv(svb, ui + 3);
      } else {
#pragma unroll
        for (int mb = 0; mb < kMBlocks; ++mb) sv[mb] = svc[mb];
        load_sv(svc, ui + 3);
      }
      const int acc_b = ui % kAccBlocks;
      mbar_wait(&acc_full[acc_b], (ui / kAccBlocks) & 1);
      tc_fence_after();
      uint32_t r[kMBlocks][4];
#pragma unroll
      for (int mb = 0; mb < kMBlocks; ++mb)
        tmem_ld4(tmem + ((uint32_t)(quarter * 32) << 16) + (acc_b * kMBlocks + mb) * kAccCols, r[mb]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc_b]);
      const float scale_fix = sEx[ui * 2 + 0], bsum = sEx[ui * 2 + 1];
#pragma unroll
      for (int mb = 0; mb < kMBlocks; ++mb) {
        const float dot = fmaf((float)(int)r[mb][0], 16384.0f, fmaf((float)(int)r[mb][1], 128.0f, (float)(int)r[mb][2]));
        acc[mb] = fmaf(sv[mb], fmaf(dot, scale_fix, bsum), acc[mb]);
      }
    }
    if (cur_tile >= 0) emit(cur_tile);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kConvWarps) tmem_dealloc(tmem, kTmemCols);
}

template <int NZ, typename T>
int launch_t(const M1TcArgs& a, const M1TcPlan& p, cudaStream_t st) {
  auto kern = m1tc_kernel<NZ, T>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  kern<<<p.ctas, kThreads, p.smem_bytes, st>>>(a);
  return check_launch("m1tc GEMV");
}

}  // namespace

unsigned take_m1tc_timeouts() {
  unsigned v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof(z));
  return v;
}

bool m1tc_supported(int64_t M, int64_t K, int64_t N, int group) {
  return M == 1 && group == kGroup && K % kGroup == 0 && N % 16 == 0 && K <= 65536;
}

M1TcPlan plan_m1tc(int64_t K, int64_t N, int sm_count) {
  M1TcPlan p{};
  p.tiles = (int)((N / 16 + kTileW - 1) / kTileW);
  const int64_t total = (int64_t)p.tiles * (K / kRowsU);
  int64_t ctas = sm_count > 0 ? sm_count : 148;
  if (ctas > total) ctas = total;
  const int64_t upc = (total + ctas - 1) / ctas;
  p.units_per_cta = (int)upc;
  p.ctas = (int)((total + upc - 1) / upc);
  p.slot_bytes = (size_t)(p.ctas + p.tiles) * kTileCols * sizeof(float);
  p.counter_bytes = (size_t)p.tiles * sizeof(unsigned);
  p.smem_bytes = smem_bytes_tc((int)K, p.units_per_cta);
  return p;
}

int launch_m1tc(const M1TcArgs& a, const M1TcPlan& p, int dtype, int nz, cudaStream_t st) {
  if (p.smem_bytes > 227 * 1024) return set_error(GRINQH_ERR_UNSUPPORTED, "m1tc: shared memory plan too large");
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
