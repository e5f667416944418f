// Single-row graded GEMV for callers that cannot allocate device memory.
//
// grinqh_gemm_or_gemv asks its caller for a workspace (the K-split partial sums
// and tickets of the single-row kernel). Some callers have no way to provide one:
// code that runs inside a fixed memory budget set up once at start-up (an embedded
// or real-time inference loop, a plugin host that forbids allocations after
// initialisation), or code that must not call into an allocator on the hot path
// because that may synchronise the device or fail under fragmentation. For them
// this file keeps the scratch in a fixed device array that is part of the loaded
// library, so grinqh_gemv_noalloc itself never allocates.
#include "common.cuh"
#include "decode_m1.cuh"

#include <mutex>

namespace grinqh {
namespace {

// Fixed scratch shared by every call on a device: tickets first, then the fp32
// partial sums of the K split. The single-row kernel writes one 4 KiB slot per
// cluster of up to 8 CTAs (about 1.7 CTAs per SM in one wave), so its scratch stays
// near (1.7 * SMs / 8) slots, about 128 KiB on a 148-SM B200; 256 KiB holds that
// for every shape. A plan that would need more is rejected rather than overrun.
constexpr size_t kNoAllocScratchBytes = size_t(256) << 10;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDev = 64;
void* g_scratch_addr[kMaxDev];
std::mutex g_scratch_mu;

size_t round256(size_t v) { return (v + 255) / 256 * 256; }

// Device address of the scratch array on the current device. The array's name in
// host code is only a host-side handle, so the address must be looked up once per
// device with that device current; the lookup happens on the first call there. The
// address belongs to the device's primary context: it is not valid after that context
// is destroyed (cudaDeviceReset), so a process that resets a device must not call
// grinqh_gemv_noalloc on it again.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDev) return set_error(GRINQH_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(GRINQH_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return GRINQH_OK;
}

}  // namespace
}  // namespace grinqh

using namespace grinqh;

extern "C" int grinqh_gemv_noalloc(const void* x, int dtype, int64_t K, const uint32_t* w, const void* s,
                                   const void* bias, int max_bits, int group, int64_t N, const float* thresholds,
                                   void* y, grinqh_stream_t stream) {
  GRINQH_RETURN_IF(check_device());
  if (!valid_bits(max_bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", max_bits);
  GRINQH_REQUIRE(dtype == GRINQH_BF16 || dtype == GRINQH_F16, "dtype must be GRINQH_BF16 or GRINQH_F16");
  GRINQH_REQUIRE(x && w && s && y && thresholds, "null pointer");
  GRINQH_REQUIRE(K > 0 && N > 0 && N % 16 == 0, "N must be a positive multiple of 16 (got %lld)", (long long)N);
  GRINQH_REQUIRE(group > 0 && group % 32 == 0 && K % group == 0,
                 "group_size must be a multiple of 32 dividing K (K=%lld, group=%d)", (long long)K, group);
  GRINQH_REQUIRE(K < (1LL << 31) && N < (1LL << 31), "size exceeds int32 range");
  if (!m1_supported(1, K, N, group))
    return set_error(GRINQH_ERR_UNSUPPORTED, "shape K=%lld N=%lld group=%d not supported", (long long)K, (long long)N, group);
  if (!m1_pointers_ok(w, s))
    return set_error(GRINQH_ERR_UNSUPPORTED, "weight_packed must be 8-byte and weight_scale 4-byte aligned");

  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
  const M1Plan plan = plan_m1(K, N, group, sms, /*few_slots=*/true);
  if (!m1_plan_fits(plan))
    return set_error(GRINQH_ERR_UNSUPPORTED, "K=%lld N=%lld: the GEMV's shared memory does not fit one CTA (use "
                     "grinqh_gemm_or_gemv)", (long long)K, (long long)N);
  const size_t counters = round256(plan.counter_bytes);
  const size_t need = counters + round256(plan.slot_bytes);
  if (need > kNoAllocScratchBytes)
    return set_error(GRINQH_ERR_WORKSPACE,
                     "K=%lld N=%lld needs %zu bytes of scratch; grinqh_gemv_noalloc has %zu (use grinqh_gemm_or_gemv "
                     "with a workspace)",
                     (long long)K, (long long)N, need, kNoAllocScratchBytes);

  void* base = nullptr;
  GRINQH_RETURN_IF(scratch_address(&base));
  M1Args a{};
  a.x = x;
  a.w = w;
  a.s = s;
  a.bias = bias;
  a.y = y;
  a.K = (int)K;
  a.N = (int)N;
  a.group = group;
  a.rows_per_warp = plan.rows_per_warp;
  a.rows_per_cta = plan.rows_per_cta;
  for (int z = 0; z < 4; ++z) a.t[z] = thresholds[z];
  if (plan.counter_bytes) {
    a.counters = static_cast<unsigned*>(base);
    a.slots = reinterpret_cast<float*>(static_cast<char*>(base) + counters);
    // the tickets must start at zero; the array keeps whatever the last call left
    const cudaError_t e = cudaMemsetAsync(a.counters, 0, plan.counter_bytes, stream);
    if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  return launch_m1(a, plan, dtype, max_bits / 2, stream);
}
