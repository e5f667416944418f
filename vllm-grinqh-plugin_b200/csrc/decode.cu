// Small-M quantized linear on CUDA cores: the graded GEMV of the reference
// (grinqh/kernel.py:39-167), its batch-union variant (kernel.py:170-360) and the
// dense x @ dtype(w*s) product (kernel.py:561-587) for few rows.
//
// Work decomposition: a CTA (4 warps) owns 32 packed-word columns j (512 output
// columns: j + c*N/16, c = 0..15) and a contiguous range of K rows; each warp takes
// a quarter of the rows. Per row only the planes some graded row needs are read
// (warp-uniform predicate), merged into code bytes in registers and multiplied by
// the activation in fp32. Partial sums of the K split go to an fp32 workspace; the
// last CTA of each column tile (atomic ticket) adds them in split order, which keeps
// the result deterministic, then casts and adds the bias.
#include "common.cuh"
#include "decode.cuh"

namespace grinqh {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;

// Mid-point bias of an active-zone mask (grinqh/kernel.py:73-82,108-114).
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
__device__ __forceinline__ uint32_t grade_bits(float v, const DecodeArgs& a) {
  const float x = fabsf(v);
  uint32_t g = (uint32_t)(x > a.t[0]) | ((uint32_t)(x > a.t[1]) << 1) | ((uint32_t)(x > a.t[2]) << 2) |
               ((uint32_t)(x > a.t[3]) << 3);
  return g & ((1u << NZ) - 1u);
}

template <int NZ, int MT, int MODE, typename T>
__global__ void __launch_bounds__(kThreads) decode_kernel(const DecodeArgs a) {
  constexpr int kShift = 8 - 2 * NZ;
  constexpr float kInvShift = 1.0f / float(1 << kShift);
  __shared__ float xs[kDecodeMaxRows][MT];
  __shared__ float bxs[kDecodeMaxRows][MT];
  __shared__ uint8_t rmask[kDecodeMaxRows];
  __shared__ uint8_t tmask[kDecodeMaxRows][MT];
  __shared__ float red[kWarps - 1][MT][16][32];
  __shared__ int s_last;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jt = blockIdx.x, ks = blockIdx.y, chunk = blockIdx.z;
  const int n16 = a.N >> 4;
  const int j = jt * 32 + lane;
  const bool jvalid = j < n16;
  const int m0 = chunk * MT;
  const int k0 = ks * a.rows_per_cta;
  const int k1 = min(k0 + a.rows_per_cta, a.K);
  const int R = k1 - k0;
  const T* x = static_cast<const T*>(a.x);
  const T* sc = static_cast<const T*>(a.s);

  // ---- stage activations, grades and per-row bias*x of this CTA's rows
  for (int r = threadIdx.x; r < R; r += kThreads) {
    const int k = k0 + r;
    uint32_t um = (MODE == kModeDense) ? ((1u << NZ) - 1u) : 0u;
    if (MODE == kModeUnion) {
      if (a.umask)  // graded by the producer of x (produce.cu)
        um = a.umask[k] & ((1u << NZ) - 1u);
      else
        for (int m = 0; m < a.M; ++m) um |= grade_bits<NZ>(Act<T>::to_f(x[(size_t)m * a.K + k]), a);
    }
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      const int m = m0 + mm;
      const float xv = m < a.M ? Act<T>::to_f(x[(size_t)m * a.K + k]) : 0.0f;
      const uint32_t tm = (MODE == kModeGraded && m < a.M) ? grade_bits<NZ>(xv, a) : 0u;
      if (MODE == kModeGraded) um |= tm;
      xs[r][mm] = xv;
      tmask[r][mm] = (uint8_t)tm;
      bxs[r][mm] = (MODE == kModeGraded) ? float(zone_bias<NZ>(tm)) * xv
                   : (MODE == kModeUnion) ? 0.0f : 0.0f;
    }
    rmask[r] = (uint8_t)um;
    if (MODE == kModeUnion) {
      const float bu = float(zone_bias<NZ>(um));
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) bxs[r][mm] = bu * xs[r][mm];
    }
  }
  __syncthreads();

  // ---- main loop over this warp's rows
  float acc_y[MT][16];
  float acc_g[MT][16];
  float bsum[MT];
  float scl[16];
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) {
    bsum[mm] = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) acc_y[mm][c] = acc_g[mm][c] = 0.f;
  }
#pragma unroll
  for (int c = 0; c < 16; ++c) scl[c] = 0.f;

  const int rpw = (R + kWarps - 1) / kWarps;
  const int r_begin = warp * rpw, r_end = min(R, r_begin + rpw);
  const size_t row_words = (size_t)NZ * n16;
  const uint32_t* wcol = a.w + j;
  int g_cur = -1;

  auto flush = [&](int g) {
    if constexpr (MODE != kModeDense) {
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float s = jvalid ? Act<T>::to_f(sc[(size_t)g * a.N + c * n16 + j]) : 0.f;
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) {
          acc_y[mm][c] = fmaf(s, fmaf(acc_g[mm][c], kInvShift, bsum[mm]), acc_y[mm][c]);
          acc_g[mm][c] = 0.f;
        }
      }
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) bsum[mm] = 0.f;
    }
  };

  for (int r = r_begin; r < r_end; ++r) {
    const int k = k0 + r;
    const int g = k / a.group;
    if (g != g_cur) {
      if (g_cur >= 0) flush(g_cur);
      g_cur = g;
      if (MODE == kModeDense) {
#pragma unroll
        for (int c = 0; c < 16; ++c)
          scl[c] = jvalid ? Act<T>::to_f(sc[(size_t)g * a.N + c * n16 + j]) * kInvShift : 0.f;
      }
    }
    const uint32_t um = rmask[r];
    if (um == 0) continue;
    const uint32_t* wr = wcol + (size_t)k * row_words;
    uint32_t p[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int z = 0; z < NZ; ++z) p[z] = (jvalid && ((um >> z) & 1u)) ? __ldcs(wr + (size_t)z * n16) : 0u;

#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      uint32_t q[4];
      uint32_t pz[4];
      const uint32_t tm = (MODE == kModeGraded && MT > 1) ? (uint32_t)tmask[r][mm] : um;
#pragma unroll
      for (int z = 0; z < 4; ++z) pz[z] = (z < NZ && ((tm >> z) & 1u)) ? p[z] : 0u;
      merge_planes(pz[0] ^ kSignFlip, pz[1], pz[2], pz[3], q);
      const float xv = xs[r][mm];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float f[4];
        f[0] = byte_to_float<0>(q[i]);
        f[1] = byte_to_float<1>(q[i]);
        f[2] = byte_to_float<2>(q[i]);
        f[3] = byte_to_float<3>(q[i]);
#pragma unroll
        for (int L = 0; L < 4; ++L) {
          const int c = 4 * i + L;
          if (MODE == kModeDense) {
            acc_y[mm][c] = fmaf(xv, Act<T>::round(f[L] * scl[c]), acc_y[mm][c]);
          } else {
            acc_g[mm][c] = fmaf(xv, f[L], acc_g[mm][c]);
          }
        }
      }
      if (MODE != kModeDense) bsum[mm] += bxs[r][mm];
    }
  }
  if (g_cur >= 0) flush(g_cur);

  // ---- reduce the 4 warps' row partials in shared memory (warp 0 keeps the sum)
  if (warp > 0) {
#pragma unroll
    for (int mm = 0; mm < MT; ++mm)
#pragma unroll
      for (int c = 0; c < 16; ++c) red[warp - 1][mm][c][lane] = acc_y[mm][c];
  }
  __syncthreads();

  T* y = static_cast<T*>(a.y);
  const T* bias = static_cast<const T*>(a.bias);
  if (a.ksplit == 1) {
    if (warp == 0 && jvalid) {
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) {
        const int m = m0 + mm;
        if (m >= a.M) break;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float v = acc_y[mm][c];
#pragma unroll
          for (int w = 0; w < kWarps - 1; ++w) v += red[w][mm][c][lane];
          const int n = c * n16 + j;
          T out = Act<T>::from_f(v);
          if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[n]));
          y[(size_t)m * a.N + n] = out;
        }
      }
    }
    return;
  }

  if (warp == 0 && jvalid) {
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      const int m = m0 + mm;
      if (m >= a.M) break;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float v = acc_y[mm][c];
#pragma unroll
        for (int w = 0; w < kWarps - 1; ++w) v += red[w][mm][c][lane];
        __stcg(a.partial + ((size_t)ks * a.M + m) * a.N + c * n16 + j, v);
      }
    }
  }
  // ---- ticket: the last CTA of this (column tile, row chunk) reduces the splits
  __threadfence();
  __syncthreads();
  unsigned* ctr = a.counters + (size_t)chunk * gridDim.x + jt;
  if (threadIdx.x == 0) s_last = (atomicAdd(ctr, 1u) == (unsigned)(a.ksplit - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < MT * 16 * 32; idx += kThreads) {
    const int mm = idx / 512, c = (idx / 32) % 16, jj = idx % 32;
    const int m = m0 + mm, jx = jt * 32 + jj;
    if (m >= a.M || jx >= n16) continue;
    const int n = c * n16 + jx;
    float v = 0.f;
    for (int s = 0; s < a.ksplit; ++s) v += __ldcg(a.partial + ((size_t)s * a.M + m) * a.N + n);
    T out = Act<T>::from_f(v);
    if (bias) out = Act<T>::from_f(Act<T>::to_f(out) + Act<T>::to_f(bias[n]));
    y[(size_t)m * a.N + n] = out;
  }
  if (threadIdx.x == 0) *ctr = 0u;  // leave the ticket ready for the next launch
}

template <int NZ, int MT, int MODE, typename T>
void launch_t(const DecodeArgs& a, dim3 grid, cudaStream_t st) {
  decode_kernel<NZ, MT, MODE, T><<<grid, kThreads, 0, st>>>(a);
}

template <int MT, int MODE, typename T>
void launch_nz(const DecodeArgs& a, int nz, dim3 grid, cudaStream_t st) {
  switch (nz) {
    case 1: launch_t<1, MT, MODE, T>(a, grid, st); break;
    case 2: launch_t<2, MT, MODE, T>(a, grid, st); break;
    case 3: launch_t<3, MT, MODE, T>(a, grid, st); break;
    default: launch_t<4, MT, MODE, T>(a, grid, st); break;
  }
}

template <int MODE, typename T>
void launch_mt(const DecodeArgs& a, int mt, int nz, dim3 grid, cudaStream_t st) {
  if (mt == 1) launch_nz<1, MODE, T>(a, nz, grid, st);
  else launch_nz<4, MODE, T>(a, nz, grid, st);
}

}  // namespace

DecodePlan plan_decode(int64_t M, int64_t K, int64_t N, int mode, int sm_count) {
  DecodePlan p{};
  p.mt = (M == 1) ? 1 : 4;
  p.jtiles = (int)((N / 16 + 31) / 32);
  p.chunks = (int)((M + p.mt - 1) / p.mt);
  const int64_t ctas_xy = (int64_t)p.jtiles * p.chunks;
  const int64_t target = 4LL * (sm_count > 0 ? sm_count : 148);
  int64_t ks = (target + ctas_xy - 1) / ctas_xy;
  const int64_t ks_max = (K + 31) / 32;
  const int64_t ks_min = (K + kDecodeMaxRows - 1) / kDecodeMaxRows;
  if (ks > ks_max) ks = ks_max;
  if (ks < ks_min) ks = ks_min;
  if (ks < 1) ks = 1;
  int64_t rows = (K + ks - 1) / ks;
  rows = (rows + 31) / 32 * 32;
  if (rows > kDecodeMaxRows) rows = kDecodeMaxRows;
  p.rows_per_cta = (int)rows;
  p.ksplit = (int)((K + rows - 1) / rows);
  if (p.ksplit > 1) {
    p.partial_bytes = (size_t)p.ksplit * (size_t)M * (size_t)N * sizeof(float);
    p.counter_bytes = (size_t)p.jtiles * p.chunks * sizeof(unsigned);
  }
  (void)mode;
  return p;
}

int launch_decode(const DecodeArgs& a, const DecodePlan& p, int mode, int dtype, int nz, cudaStream_t st) {
  const dim3 grid((unsigned)p.jtiles, (unsigned)p.ksplit, (unsigned)p.chunks);
  if (p.chunks > 65535 || p.ksplit > 65535)
    return set_error(GRINQH_ERR_UNSUPPORTED, "too many rows for the small-M kernel (M=%d)", a.M);
  if (dtype == GRINQH_BF16) {
    if (mode == kModeGraded) launch_mt<kModeGraded, __nv_bfloat16>(a, p.mt, nz, grid, st);
    else if (mode == kModeUnion) launch_mt<kModeUnion, __nv_bfloat16>(a, p.mt, nz, grid, st);
    else launch_mt<kModeDense, __nv_bfloat16>(a, p.mt, nz, grid, st);
  } else {
    if (mode == kModeGraded) launch_mt<kModeGraded, __half>(a, p.mt, nz, grid, st);
    else if (mode == kModeUnion) launch_mt<kModeUnion, __half>(a, p.mt, nz, grid, st);
    else launch_mt<kModeDense, __half>(a, p.mt, nz, grid, st);
  }
  return check_launch("decode");
}

}  // namespace grinqh
