// Producers of a linear's activations with the grading fused in: the threshold masks
// of the graded GEMV (grinqh/kernel.py:100-116; zone z of element k is active iff
// fp32 |x_k| > t_z) and their union over the rows (the batch-union GEMV,
// kernel.py:170-360) are computed where x is written, instead of by a separate pass
// over x (grinqh_grade) or by every CTA of the union GEMV re-reading all rows.
//
//   RMSNorm (before qkv and gate_up), with or without the residual add, as vLLM's
//   rms_norm / fused_add_rms_norm (vllm/ir/ops/layernorm.py:10-58):
//     s   = float(x) [+ float(residual)]          (residual <- dtype(s), in place)
//     out = dtype(dtype(s * rsqrt(mean(s^2) + eps)) * weight)
//   SiLU(gate) * up (before down), as vLLM's SiluAndMul on x = [gate | up]
//   (vllm/model_executor/layers/activation.py, forward_native):
//     out = dtype(dtype(gate / (1 + exp(-gate))) * up)
//
// The masks are graded from the produced, rounded out -- the values the linear reads --
// so a GEMV fed with them grades exactly as one that grades its x itself. The union
// is one byte per k, ORed over the rows with 32-bit atomics (4 bytes a word); it is
// cleared on the stream first.
#include "common.cuh"

namespace grinqh {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ uint32_t grade_of(float v, float t0, float t1, float t2, float t3, uint32_t zmask) {
  const float a = fabsf(v);
  return ((uint32_t)(a > t0) | ((uint32_t)(a > t1) << 1) | ((uint32_t)(a > t2) << 2) | ((uint32_t)(a > t3) << 3)) &
         zmask;
}

struct GradeOut {
  uint8_t* masks;  // [M, K] or null
  uint8_t* uni;    // [K] or null (cleared before the launch)
  float t0, t1, t2, t3;
  uint32_t zmask;
};

// Grades 8 produced values of row m at columns k..k+7 (k % 8 == 0): 8 mask bytes, and
// their OR into the union (two 32-bit words).
__device__ __forceinline__ void emit_grades(const GradeOut& g, int64_t m, int64_t K, int64_t k, const float (&v)[8]) {
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo |= grade_of(v[i], g.t0, g.t1, g.t2, g.t3, g.zmask) << (8 * i);
    hi |= grade_of(v[4 + i], g.t0, g.t1, g.t2, g.t3, g.zmask) << (8 * i);
  }
  if (g.masks) *reinterpret_cast<uint2*>(g.masks + m * K + k) = make_uint2(lo, hi);
  if (g.uni) {
    unsigned* u = reinterpret_cast<unsigned*>(g.uni + k);
    if (lo) atomicOr(u, lo);
    if (hi) atomicOr(u + 1, hi);
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T* h = reinterpret_cast<const T*>(&w[i]);
    v[2 * i] = Act<T>::to_f(h[0]);
    v[2 * i + 1] = Act<T>::to_f(h[1]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const T (&o)[8]) {
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(o);
}

// One CTA per row. The fp32 sums s stay in shared memory between the two passes.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_grade_kernel(const T* __restrict__ x, T* residual,
                                                                     const T* __restrict__ weight, int64_t K,
                                                                     float eps, T* __restrict__ out, GradeOut g) {
  extern __shared__ float srow[];
  __shared__ float red[kRowThreads / 32];
  const int64_t m = blockIdx.x;
  const T* xr = x + m * K;
  T* rr = residual ? residual + m * K : nullptr;
  float ss = 0.f;
  for (int64_t k = 8 * (int64_t)threadIdx.x; k < K; k += 8 * kRowThreads) {
    float v[8];
    load8(xr + k, v);
    if (rr) {
      float r[8];
      load8(rr + k, r);
      T o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] += r[i];
        o[i] = Act<T>::from_f(v[i]);
      }
      store8(rr + k, o);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      srow[k + i] = v[i];
      ss = fmaf(v[i], v[i], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / (float)K + eps);
  T* orow = out + m * K;
  for (int64_t k = 8 * (int64_t)threadIdx.x; k < K; k += 8 * kRowThreads) {
    float wv[8];
    if (weight) load8(weight + k, wv);
    T o[8];
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const T n = Act<T>::from_f(srow[k + i] * inv);
      o[i] = weight ? Act<T>::from_f(Act<T>::to_f(n) * wv[i]) : n;
      v[i] = Act<T>::to_f(o[i]);
    }
    store8(orow + k, o);
    emit_grades(g, m, K, k, v);
  }
}

// Grid-stride over the M x K/8 output vectors.
template <typename T>
__global__ void silu_mul_grade_kernel(const T* __restrict__ x, int64_t M, int64_t K, T* __restrict__ out,
                                      GradeOut g) {
  const int64_t kv = K / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < M * kv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / kv, k = (i % kv) * 8;
    float gt[8], up[8];
    load8(x + m * 2 * K + k, gt);
    load8(x + m * 2 * K + K + k, up);
    T o[8];
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const T sg = Act<T>::from_f(gt[j] / (1.0f + expf(-gt[j])));
      o[j] = Act<T>::from_f(Act<T>::to_f(sg) * up[j]);
      v[j] = Act<T>::to_f(o[j]);
    }
    store8(out + m * K + k, o);
    emit_grades(g, m, K, k, v);
  }
}

int grade_out(const float* thresholds, int max_bits, uint8_t* masks, uint8_t* uni, int64_t K, cudaStream_t st,
              GradeOut* g) {
  if ((masks || uni) && !thresholds) return set_error(GRINQH_ERR_INVALID, "thresholds required for the masks");
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(!masks || aligned(masks, 8), "masks must be 8-byte aligned");
  GRINQH_REQUIRE(!uni || aligned(uni, 4), "union must be 4-byte aligned");
  *g = GradeOut{masks, uni, 0.f, 0.f, 0.f, 0.f, (1u << (max_bits / 2)) - 1u};
  if (thresholds) {
    g->t0 = thresholds[0];
    g->t1 = thresholds[1];
    g->t2 = thresholds[2];
    g->t3 = thresholds[3];
  }
  if (uni) {
    const cudaError_t e = cudaMemsetAsync(uni, 0, (size_t)K, st);
    if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaMemsetAsync(union): %s", cudaGetErrorString(e));
  }
  return GRINQH_OK;
}

}  // namespace
}  // namespace grinqh

using namespace grinqh;

extern "C" int grinqh_rmsnorm_grade(const void* x, void* residual, const void* weight, int dtype, int64_t M,
                                    int64_t K, float eps, const float* thresholds, int max_bits, void* out,
                                    uint8_t* masks, uint8_t* uni, grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  GRINQH_REQUIRE(dtype == GRINQH_BF16 || dtype == GRINQH_F16, "dtype must be GRINQH_BF16 or GRINQH_F16");
  GRINQH_REQUIRE(M >= 0 && K > 0 && K % 8 == 0, "K must be a positive multiple of 8 (got %lld)", (long long)K);
  GRINQH_REQUIRE(M == 0 || (x && out), "null pointer");
  GRINQH_REQUIRE(aligned(x, 16) && aligned(out, 16) && (!residual || aligned(residual, 16)) &&
                     (!weight || aligned(weight, 16)),
                 "x, residual, weight and out must be 16-byte aligned");
  GRINQH_REQUIRE(M < (1LL << 31), "M exceeds int32 range");
  const size_t smem = (size_t)K * sizeof(float);
  if (smem > 227u * 1024u)
    return set_error(GRINQH_ERR_UNSUPPORTED, "K=%lld: the row does not fit in shared memory", (long long)K);
  GradeOut g;
  GRINQH_RETURN_IF(grade_out(thresholds, max_bits, masks, uni, K, stream, &g));
  if (M == 0) return GRINQH_OK;
  if (dtype == GRINQH_BF16) {
    auto k = rmsnorm_grade_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)M, kRowThreads, smem, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                  static_cast<__nv_bfloat16*>(residual),
                                                  static_cast<const __nv_bfloat16*>(weight), K, eps,
                                                  static_cast<__nv_bfloat16*>(out), g);
  } else {
    auto k = rmsnorm_grade_kernel<__half>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)M, kRowThreads, smem, stream>>>(static_cast<const __half*>(x), static_cast<__half*>(residual),
                                                  static_cast<const __half*>(weight), K, eps,
                                                  static_cast<__half*>(out), g);
  }
  return check_launch("rmsnorm_grade");
}

extern "C" int grinqh_silu_mul_grade(const void* x, int dtype, int64_t M, int64_t K, const float* thresholds,
                                     int max_bits, void* out, uint8_t* masks, uint8_t* uni, grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  GRINQH_REQUIRE(dtype == GRINQH_BF16 || dtype == GRINQH_F16, "dtype must be GRINQH_BF16 or GRINQH_F16");
  GRINQH_REQUIRE(M >= 0 && K > 0 && K % 8 == 0, "K must be a positive multiple of 8 (got %lld)", (long long)K);
  GRINQH_REQUIRE(M == 0 || (x && out), "null pointer");
  GRINQH_REQUIRE(aligned(x, 16) && aligned(out, 16), "x and out must be 16-byte aligned");
  GradeOut g;
  GRINQH_RETURN_IF(grade_out(thresholds, max_bits, masks, uni, K, stream, &g));
  if (M == 0) return GRINQH_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t vecs = M * (K / 8);
  const unsigned grid = (unsigned)std::min<int64_t>((vecs + 255) / 256, (int64_t)sms * 8);
  if (dtype == GRINQH_BF16)
    silu_mul_grade_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), M, K,
                                                                   static_cast<__nv_bfloat16*>(out), g);
  else
    silu_mul_grade_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(x), M, K,
                                                            static_cast<__half*>(out), g);
  return check_launch("silu_mul_grade");
}
