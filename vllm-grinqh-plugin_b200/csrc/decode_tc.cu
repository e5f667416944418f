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
// Plane words reach shared memory by cp.async: each converter warp owns rows
// rw + 8 i of every unit and fetches the active planes of its rows (16 bytes per lane,
// 128 contiguous bytes per plane row) kSp - 1 units ahead of the unit it converts, so
// a row graded 0 costs no load and inactive zones no bytes, and enough bytes stay in
// flight without holding them in registers. Warps: 0-7 convert (merge the staged
// planes of their rows into A; rows graded 0 are skipped, their x digits are zero),
// 8 builds B and issues the MMAs from one thread, 9-12 are the epilogue (TMEM lane
// quarters 1, 2, 3, 0). Units (tile, group) are walked tile-major and split into one
// contiguous range per CTA; CTAs that share a tile write partial slots and the last
// one (atomic ticket) adds them in CTA order, so results are deterministic.
#include "common.cuh"
#include "decode_tc.cuh"
#include "ptx.cuh"

namespace grinqh {
namespace {

#ifndef GRINQH_TC_GROUPS
#define GRINQH_TC_GROUPS 1
#endif
constexpr int kGroups = GRINQH_TC_GROUPS;     // converter groups of 8 warps, taking units in turn
constexpr int kGroupWarps = 8;
constexpr int kConvWarps = kGroups * kGroupWarps;
constexpr int kMmaWarp = kConvWarps;          // then 4 epilogue warps
constexpr int kProdWarp = kConvWarps + 5;     // TMA issuer of the plane stages
constexpr int kThreads = 32 * (kConvWarps + 1 + 4 + 1);
constexpr int kGroup = 128;                 // K group of the scales
constexpr int kRowsU = 64;                  // rows per unit (half a group)
constexpr int kTileW = 32;                  // packed words per column tile (128 B per plane row)
constexpr int kTileCols = 16 * kTileW;      // 512 output columns = 4 MMA blocks of M = 128
constexpr int kMBlocks = kTileCols / 128;
constexpr int kStagesA = 2;                 // A / B stages between converters and MMA
constexpr uint32_t kAtomLbo = (kRowsU / 8) * 1024;  // A: stride between 128-column MN atoms
constexpr uint32_t kStageA = kTileCols * kRowsU;    // 32 KB int8
// B of one 64-row group: K-major without swizzle, core matrix c (16 K bytes x 8 rows,
// 16 bytes per row) at c * 128; digit t of x is row t. Rows 3..7, and the rows 8..15
// the MMA reads one slot further on (SBO), only feed D columns the epilogue never reads.
constexpr uint32_t kBSlot = 4 * 128;
constexpr int kAccCols = 16;                        // TMEM columns per MMA block and unit
constexpr int kAccBlocks = 8;                       // MMAs may run this many units ahead of the epilogue
constexpr uint32_t kTmemCols = kAccCols * kMBlocks * kAccBlocks;  // 512
constexpr int kFix = 21;                           // fixed-point bits of the x digits
constexpr uint32_t kSmemLimit = 227 * 1024;

// Shared memory: A stages (1 KB aligned for the swizzle atoms), the B slots of the
// CTA's groups (+ one slot read past the last through SBO), the plane stages
// [kSp][NZ planes][64 rows][128 B], the zone masks of the slots' rows, the per-slot
// fp32 pairs (2^(e-21-shift), sum bias*x), the per-slot TMA plane masks, then the
// barriers.
struct TcLayout {
  uint32_t a, b, p, masks, ex, tma, bars, total;
};
__host__ __device__ inline TcLayout tc_layout(int nz, int sp, int bslots) {
  TcLayout L;
  L.a = 0;
  L.b = L.a + kStagesA * kStageA;
  L.p = L.b + (uint32_t)(bslots + 1) * kBSlot;
  L.masks = L.p + (uint32_t)sp * kRowsU * nz * 128;
  L.ex = L.masks + (uint32_t)bslots * kRowsU * 4;
  L.tma = L.ex + (uint32_t)bslots * 8;
  L.bars = (L.tma + (uint32_t)bslots + 7) / 8 * 8;
  L.total = 1024 + L.bars + 512;
  return L;
}

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

template <int NZ, typename T, int kSp>
__global__ void __launch_bounds__(kThreads, 1)
    m1tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const M1TcArgs a) {
  constexpr int kShift = 8 - 2 * NZ;
  constexpr uint32_t kPlaneBox = kRowsU * 128;  // one plane of a unit: 64 rows x 32 words
  constexpr uint32_t kStageP = NZ * kPlaneBox;
  constexpr uint32_t kAllPlanes = (1u << NZ) - 1u;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TcLayout L = tc_layout(NZ, kSp, a.bslots);
  unsigned char* sA = smem + L.a;
  unsigned char* sB = smem + L.b;
  unsigned char* sP = smem + L.p;
  // [slot][64] zone masks, warp-major: row r of a group at 8 (r % 8) + r / 8; byte mask of
  // the active zones' bits (zone z: bits 7-2z, 6-2z) replicated to the 4 bytes
  uint32_t* zmasks = reinterpret_cast<uint32_t*>(smem + L.masks);
  float* sEx = reinterpret_cast<float*>(smem + L.ex);               // [slot][2]
  uint8_t* slot_tma = smem + L.tma;                                 // [slot] planes loaded by TMA
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* full = bars;                        // converter group (8 warps)
  uint64_t* empty = bars + kStagesA;            // MMA commit
  uint64_t* acc_full = bars + 2 * kStagesA;     // [kAccBlocks] MMA commit
  uint64_t* acc_empty = acc_full + kAccBlocks;  // [kAccBlocks] epilogue warps (4)
  uint64_t* p_full = acc_empty + kAccBlocks;    // [kSp] TMA bytes of a plane stage
  uint64_t* p_empty = p_full + kSp;             // [kSp] converter group (8) done with a plane stage
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_empty + kSp);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n16 = a.N >> 4;
  const int ngroups = a.K / kRowsU;  // units per tile
  const int64_t total = (int64_t)a.tiles * ngroups;
  const int64_t u_begin = (int64_t)blockIdx.x * a.units_per_cta;
  const int64_t u_end = min(total, u_begin + a.units_per_cta);
  const int nunits = (int)(u_end - u_begin);
  const T* x = static_cast<const T*>(a.x);

  // A CTA's units are consecutive, so while they stay within one tile their groups are
  // consecutive too (slot = unit); a range that covers a whole tile uses slot = group.
  const bool by_unit = nunits <= ngroups;
  const int nslots = by_unit ? nunits : ngroups;
  auto slot_of = [&](int ui) { return by_unit ? ui : (int)((u_begin + ui) % ngroups); };
  // Planes of unit ui that the producer loads by TMA (all rows of the unit): every plane
  // of the first kSp units (issued before the grades are known), then the planes that
  // more than a.tma_min_rows of the unit's 64 rows need. The converters fetch the
  // other planes of their own graded rows.
  auto tma_planes = [&](int ui) { return ui < kSp ? kAllPlanes : (uint32_t)slot_tma[slot_of(ui)]; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesA; ++s) {
      mbar_init(&full[s], kGroupWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBlocks; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    for (int s = 0; s < kSp; ++s) {
      mbar_init(&p_full[s], 1);
      mbar_init(&p_empty[s], kGroupWarps);
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, kTmemCols);
  __syncthreads();

  // TMA of unit ui's planes in `planes` (producer lane only)
  auto tma_unit = [&](int ui, uint32_t planes) {
    const int64_t u = u_begin + ui;
    const int tile = (int)(u / ngroups), g = (int)(u - (int64_t)tile * ngroups);
    const int sp = ui % kSp;
    mbar_arrive_expect_tx(&p_full[sp], (uint32_t)__popc(planes) * kPlaneBox);
#pragma unroll
    for (int z = 0; z < NZ; ++z)
      if ((planes >> z) & 1u)
        tma_load_2d(sP + sp * kStageP + z * kPlaneBox, &tmap_w, z * n16 + tile * kTileW, g * kRowsU, &p_full[sp]);
  };
  // The weights are never written by other kernels: the first units' planes load
  // while the previous kernel on the stream finishes.
  if (warp == kProdWarp && lane == 0) {
    prefetch_tmap(&tmap_w);
    for (int ui = 0; ui < kSp && ui < nunits; ++ui) tma_unit(ui, kAllPlanes);
  }
  wait_prior_grid();  // x, the outputs and the workspace belong to the stream order from here on

  // ---- grades, TMA plane masks and x digits of the CTA's groups, all warps, one group
  // per warp at a time (the next group's x loads while one is finished)
  {
    constexpr int kAllWarps = kThreads / 32;
    auto load_x = [&](int sl, float (&d)[2]) {
      d[0] = d[1] = 0.f;
      if (sl < nslots) {
        const int g = by_unit ? (int)((u_begin + sl) % ngroups) : sl;
#pragma unroll
        for (int i = 0; i < 2; ++i) d[i] = Act<T>::to_f(x[g * kRowsU + 2 * lane + i]);
      }
    };
    float xc[2];
    load_x(warp, xc);
    for (int sl = warp; sl < nslots; sl += kAllWarps) {
      float xn[2];
      load_x(sl + kAllWarps, xn);
      uint32_t mk[2], abits = 0u;
      float bsum = 0.f;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int r = 2 * lane + i;
        mk[i] = grade_of<NZ>(xc[i], a);
        uint32_t zm = 0u;
#pragma unroll
        for (int z = 0; z < NZ; ++z)
          if ((mk[i] >> z) & 1u) zm |= 0xC0u >> (2 * z);
        zmasks[sl * kRowsU + (r & 7) * 8 + (r >> 3)] = zm * 0x01010101u;
        if (mk[i]) abits = max(abits, __float_as_uint(fabsf(xc[i])));
        bsum += float(zone_bias<NZ>(mk[i])) * xc[i];
      }
      uint32_t tplanes = 0u;
#pragma unroll
      for (int z = 0; z < NZ; ++z) {
        const int cnt = __popc(__ballot_sync(0xffffffffu, (mk[0] >> z) & 1u)) +
                        __popc(__ballot_sync(0xffffffffu, (mk[1] >> z) & 1u));
        if (cnt > a.tma_min_rows) tplanes |= 1u << z;
      }
      abits = __reduce_max_sync(0xffffffffu, abits);  // |x| bit patterns order like the values
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
      const float amax = __uint_as_float(abits);
      // 2^e > amax; q = rint(x * 2^(21-e)) fits 22 bits signed
      int e = 0;
      if (amax > 0.f) frexpf(amax, &e);
      const float to_fix = ldexpf(1.0f, kFix - e);
      uint32_t d0 = 0, d1 = 0, d2 = 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int qv =
            mk[i] ? max(-(1 << kFix) + 1, min((1 << kFix) - 1, __float2int_rn(xc[i] * to_fix))) : 0;
        d0 |= (uint32_t)((qv >> 14) & 0xFF) << (8 * i);
        d1 |= (uint32_t)((qv >> 7) & 0x7F) << (8 * i);
        d2 |= (uint32_t)(qv & 0x7F) << (8 * i);
      }
      // rows k = 2 lane, 2 lane + 1: core matrix lane / 8, bytes 2 (lane % 8) of digit row t
      unsigned char* bs = sB + sl * kBSlot + (lane >> 3) * 128 + 2 * (lane & 7);
      *reinterpret_cast<uint16_t*>(bs + 0) = (uint16_t)d0;
      *reinterpret_cast<uint16_t*>(bs + 16) = (uint16_t)d1;
      *reinterpret_cast<uint16_t*>(bs + 32) = (uint16_t)d2;
      if (lane == 0) {
        sEx[sl * 2 + 0] = ldexpf(1.0f, e - kFix - kShift);
        sEx[sl * 2 + 1] = bsum;
        slot_tma[sl] = (uint8_t)tplanes;
      }
      xc[0] = xn[0];
      xc[1] = xn[1];
    }
  }
  fence_proxy_async_smem();  // B is read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kConvWarps) {
    // ------------------------------------------------------------ converters
    // group cg = warp / 8 takes units cg, cg + kGroups, ...; each group cycles through
    // kSp / kGroups plane stages and fetches its own units kLook ahead
    const int cg = warp / kGroupWarps;
    const int rw = warp % kGroupWarps;  // rows rw + 8 i of its units
    const size_t row_words = (size_t)NZ * n16;
    // cp.async of this warp's rows of unit ui for the planes not loaded by TMA:
    // slot q = (row i, plane z), 8 lanes x 16 bytes per slot
    auto fetch = [&](int ui) {
      const int sub = lane & 7, qs = lane >> 3;
      if (ui >= kSp && ui < nunits) {
        const int64_t u = u_begin + ui;
        const int tile = (int)(u / ngroups), g = (int)(u - (int64_t)tile * ngroups);
        const int kb = g * kRowsU + rw;
        const int w0 = tile * kTileW + 4 * sub;  // n16 % 4 == 0: a chunk is all in range or all out
        const uint32_t own = ~tma_planes(ui) & kAllPlanes;
        unsigned char* ps = sP + (ui % kSp) * kStageP + rw * 128 + sub * 16;
        const uint32_t* zr = zmasks + slot_of(ui) * kRowsU + rw * 8;
        if (w0 < n16 && own) {
#pragma unroll
          for (int it = 0; it < 2 * NZ; ++it) {
            const int q = 4 * it + qs;
            const int i = q / NZ, z = q - (q / NZ) * NZ;
            if (((own >> z) & 1u) && ((zr[i] >> (6 - 2 * z)) & 1u))
              cp_async_16(ps + z * kPlaneBox + 8 * i * 128, a.w + (size_t)(kb + 8 * i) * row_words + (size_t)z * n16 + w0,
                          16);
          }
        }
      }
      cp_async_commit();  // one group per unit, empty or not
    };
    constexpr int kLook = kSp / kGroups - 1;
#pragma unroll
    for (int i = 0; i < kLook; ++i) cp_async_commit();  // units below kSp come by TMA only
    const int jj = lane;                                      // word of the tile
    const uint32_t col_off = (uint32_t)(jj >> 3) * kAtomLbo;  // MN atom of this word
    const int chunk = jj & 7;
    for (int ui = cg; ui < nunits; ui += kGroups) {
      fetch(ui + kLook * kGroups);  // this group's unit kLook ahead
      const int sp = ui % kSp;
      cp_async_wait<kLook>();                  // this lane's copies of unit ui have landed
      mbar_wait(&p_full[sp], (ui / kSp) & 1);  // the TMA planes of unit ui
      __syncwarp();                            // ... and every lane's copies
      const uint32_t* ps = reinterpret_cast<const uint32_t*>(sP + sp * kStageP + rw * 128) + jj;
      const uint4* zr = reinterpret_cast<const uint4*>(zmasks + slot_of(ui) * kRowsU + rw * 8);
      const uint4 zlo = zr[0], zhi = zr[1];
      const uint32_t zm[8] = {zlo.x, zlo.y, zlo.z, zlo.w, zhi.x, zhi.y, zhi.z, zhi.w};
      // the active plane words of the 8 rows (zone z of row i is active when bit 6 - 2z
      // of its zone mask is set); inactive zones read as zero, so a row graded 0
      // merges to zero bytes (its x digits are zero as well)
      uint32_t p[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int z = 0; z < 4; ++z)
          p[i][z] = (z < NZ && ((zm[i] >> (6 - 2 * z)) & 1u)) ? ps[(z * kPlaneBox + 8 * i * 128) / 4] : 0u;
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_empty[sp]);  // this warp is done with the plane stage
      const int s = ui % kStagesA;
      if (ui >= kStagesA) mbar_wait(&empty[s], ((ui / kStagesA) - 1) & 1);
      unsigned char* ast = sA + s * kStageA + col_off;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t q[4];
        merge_planes(p[i][0], p[i][1], p[i][2], p[i][3], q);  // int8 codes << shift, inactive zones 0
        const int k = rw + 8 * i;
        // MN-major, 128-byte swizzle: 8-row K atoms of 1 KB, 16-byte chunk of row k
        *reinterpret_cast<uint4*>(ast + (k >> 3) * 1024 + (k & 7) * 128 + ((chunk ^ (k & 7)) << 4)) =
            make_uint4(q[0], q[1], q[2], q[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
    cp_async_wait<0>();
  } else if (warp == kProdWarp) {
    // ------------------------------------------------------------ plane TMA producer
    if (lane == 0) {
      for (int ui = kSp; ui < nunits; ++ui) {
        const int sp = ui % kSp;
        mbar_wait(&p_empty[sp], ((ui / kSp) - 1) & 1);  // every converter is done with unit ui - kSp
        tma_unit(ui, tma_planes(ui));
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = instr_desc(2 /*s32*/, 1 /*s8*/, 1 /*s8*/, 1 /*A MN-major*/, 0 /*B K-major*/, 16, 128);
    if (lane == 0) {
      for (int ui = 0; ui < nunits; ++ui) {
        const int s = ui % kStagesA;
        const int acc_b = ui % kAccBlocks;
        const int sl = slot_of(ui);
        mbar_wait(&full[s], (ui / kStagesA) & 1);
        if (ui >= kAccBlocks) mbar_wait(&acc_empty[acc_b], ((ui / kAccBlocks) - 1) & 1);
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * kStageA);
        const uint32_t b_base = smem_u32(sB + sl * kBSlot);
#pragma unroll
        for (int kk = 0; kk < kRowsU / 32; ++kk) {
          // A: +32 rows = 4 K atoms; B: +2 core matrices
          const uint64_t bdesc = smem_desc(b_base + kk * 256, 128, kBSlot, 0);
#pragma unroll
          for (int mb = 0; mb < kMBlocks; ++mb) {
            const uint64_t adesc = smem_desc(a_base + mb * kAtomLbo + kk * 4096, kAtomLbo, 1024, 2);
            mma_i8_ss(tmem + (acc_b * kMBlocks + mb) * kAccCols, adesc, bdesc, idesc, kk > 0 ? 1u : 0u);
          }
        }
        mma_commit(&empty[s]);
        mma_commit(&acc_full[acc_b]);
      }
    }
    __syncwarp();
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
      const int sl = slot_of(ui);
      const float scale_fix = sEx[sl * 2 + 0], bsum = sEx[sl * 2 + 1];
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc_b]);
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

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tc_encode_fn() {
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

template <int NZ, typename T, int kSp>
int launch_t(const M1TcArgs& a, const M1TcPlan& p, cudaStream_t st) {
  EncodeTiledFn enc = tc_encode_fn();
  if (!enc) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  // packed planes [K, nz * N/16] uint32: boxes of one plane's 32 words (128 bytes) x 64
  // rows, no swizzle; x = z * N/16 + 32 tile is a multiple of 4 words (N % 64 == 0)
  CUtensorMap tmap_w;
  {
    const cuuint64_t gdim[2] = {(cuuint64_t)NZ * (a.N / 16), (cuuint64_t)a.K};
    const cuuint64_t gstride[1] = {(cuuint64_t)NZ * (a.N / 16) * 4};
    const cuuint32_t box[2] = {kTileW, kRowsU};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = enc(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(a.w), gdim, gstride,
                           box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(GRINQH_ERR_CUDA, "cuTensorMapEncodeTiled(w) failed (%d)", (int)r);
  }
  auto kern = m1tc_kernel<NZ, T, kSp>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)p.ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = st;
  // may start while the previous kernel on the stream finishes (the kernel waits for
  // it before reading x or touching the output and the workspace)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, tmap_w, a);
  if (le != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "m1tc GEMV launch: %s", cudaGetErrorString(le));
  return check_launch("m1tc GEMV");
}

template <int NZ, typename T>
int launch_sp(const M1TcArgs& a, const M1TcPlan& p, cudaStream_t st) {
  (void)p.plane_stages;  // always 4: each converter group cycles through two stages
  return launch_t<NZ, T, 4>(a, p, st);
}

}  // namespace

unsigned take_m1tc_timeouts() {
  unsigned v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return 0;
  cudaMemcpyToSymbol(g_wait_timeouts, &z, sizeof(z));
  return v;
}

bool m1tc_supported(int64_t M, int64_t K, int64_t N, int group) {
  // 16-byte plane chunks: N / 16 a multiple of 4; the grades of K and three plane
  // stages must fit in shared memory
  // (the plan's B slots are checked at launch; the dispatcher asks m1tc_plan_fits)
  return M == 1 && group == kGroup && K % kGroup == 0 && N % 64 == 0 && tc_layout(4, 4, 1).total <= kSmemLimit;
}

bool m1tc_plan_fits(const M1TcPlan& p) { return p.smem_bytes <= kSmemLimit; }

bool m1tc_pointers_ok(const void* w) { return (reinterpret_cast<uintptr_t>(w) & 15u) == 0; }

M1TcPlan plan_m1tc(int64_t K, int64_t N, int nz, int sm_count) {
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
  const int64_t ngroups = K / kRowsU;
  p.bslots = (int)(upc < ngroups ? upc : ngroups);
  p.plane_stages = 4;
  p.smem_bytes = tc_layout(nz, p.plane_stages, p.bslots).total;
  return p;
}

int launch_m1tc(const M1TcArgs& a, const M1TcPlan& p, int dtype, int nz, cudaStream_t st) {
  if (p.smem_bytes > kSmemLimit) return set_error(GRINQH_ERR_UNSUPPORTED, "m1tc: shared memory plan too large");
  if (dtype == GRINQH_BF16) {
    switch (nz) {
      case 1: return launch_sp<1, __nv_bfloat16>(a, p, st);
      case 2: return launch_sp<2, __nv_bfloat16>(a, p, st);
      case 3: return launch_sp<3, __nv_bfloat16>(a, p, st);
      default: return launch_sp<4, __nv_bfloat16>(a, p, st);
    }
  }
  switch (nz) {
    case 1: return launch_sp<1, __half>(a, p, st);
    case 2: return launch_sp<2, __half>(a, p, st);
    case 3: return launch_sp<3, __half>(a, p, st);
    default: return launch_sp<4, __half>(a, p, st);
  }
}

}  // namespace grinqh
