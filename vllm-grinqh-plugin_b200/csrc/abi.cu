// C ABI entry points of the quantized linear and shared status plumbing.
#include <mutex>

#include <cstring>

#include "common.cuh"

#include <stdlib.h>
#include "decode.cuh"
#include "decode_m1.cuh"
#include "gemm_tc.cuh"
#include "decode_tc.cuh"
#include "gemm_skinny.cuh"
#include "gemm_bf16.cuh"

namespace grinqh {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
int g_cc_major[kMaxDevices];  // 0 = unknown
int g_sm_count[kMaxDevices];
std::mutex g_dev_mu;

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

int set_error(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return GRINQH_OK;
}

static int device_info(int* dev_out, int* sm_count) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(GRINQH_ERR_DEVICE, "device ordinal %d out of range", dev);
  if (g_cc_major[dev] == 0) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    int major = 0, sms = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    g_sm_count[dev] = sms;
    g_cc_major[dev] = major;
  }
  if (g_cc_major[dev] != 10)
    return set_error(GRINQH_ERR_DEVICE, "device %d has compute capability %d.x; this library is built for sm_100a",
                     dev, g_cc_major[dev]);
  if (dev_out) *dev_out = dev;
  if (sm_count) *sm_count = g_sm_count[dev];
  return GRINQH_OK;
}

int check_device() { return device_info(nullptr, nullptr); }

struct LinearShape {
  int64_t M, K, N;
  int bits, group, mode;
};

// Map the public mode to a kernel mode (grinqh/kernel.py:663-705 dispatch for AUTO).
static int resolve_mode(int mode, int64_t M) {
  switch (mode) {
    case GRINQH_MODE_AUTO: return M == 1 ? kModeGraded : kModeDense;
    case GRINQH_MODE_DENSE: return kModeDense;
    case GRINQH_MODE_GRADED: return kModeGraded;
    case GRINQH_MODE_UNION: return kModeUnion;
    default: return -1;
  }
}

// Workspace layout of every split-K kernel: the tickets first, in a region of at
// least kTicketBytes, then the fp32 partial sums. The kernels return every ticket to
// zero and nothing else is ever written into the ticket region, so a workspace reused
// by calls of any shape keeps that region zero (GRINQH_WORKSPACE_ZEROED).
constexpr size_t kTicketBytes = 16 << 10;

static size_t ticket_region(size_t counter_bytes) {
  return counter_bytes > kTicketBytes ? align_up(counter_bytes, 256) : kTicketBytes;
}

static size_t split_workspace(size_t partial_bytes, size_t counter_bytes) {
  if (counter_bytes == 0) return 0;
  return ticket_region(counter_bytes) + align_up(partial_bytes, 256);
}

// Points tickets and partial sums into the workspace; clears the tickets unless the
// caller says they are zero (and they fit the region that is kept zero).
static int bind_workspace(void* workspace, size_t partial_bytes, size_t counter_bytes, bool zeroed,
                          cudaStream_t stream, float** partial, unsigned** counters) {
  char* base = static_cast<char*>(workspace);
  *counters = reinterpret_cast<unsigned*>(base);
  *partial = reinterpret_cast<float*>(base + ticket_region(counter_bytes));
  if (!zeroed || counter_bytes > kTicketBytes) {
    const cudaError_t e = cudaMemsetAsync(*counters, 0, counter_bytes, stream);
    if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  return GRINQH_OK;
}

static size_t workspace_for(const DecodePlan& p) {
  if (p.ksplit <= 1) return 0;
  return split_workspace(p.partial_bytes, p.counter_bytes);
}

static size_t workspace_for(const M1Plan& p) { return split_workspace(p.slot_bytes, p.counter_bytes); }

static size_t workspace_for(const M1TcPlan& p) { return split_workspace(p.slot_bytes, p.counter_bytes); }

// The int8 tensor-core single-row kernel (decode_tc.cu) is selected only when
// GRINQH_M1_TENSOR_CORES=1: it is exact but slower than the register-streaming
// kernel on the Llama-3-8B shapes (gate_up 44 us vs 36 us at b = 8, graded; both
// are bound by the integer work of merging the 2-bit planes), so it is not the
// default. The variable is read on every call (a getenv, no allocation).
//
// A unit's plane comes by TMA for all 64 rows when more than GRINQH_TC_TMA_ROWS
// (default 0: always) of the rows need it, else by per-row cp.async of the graded
// rows only; all-TMA measured fastest (gate_up 42 us vs 47-50 us for 16-48).
static int tc_tma_min_rows() {
  const char* e = getenv("GRINQH_TC_TMA_ROWS");
  return e ? atoi(e) : 0;
}

static bool use_m1tc(int kmode, int64_t M, int64_t K, int64_t N, int group) {
  const char* e = getenv("GRINQH_M1_TENSOR_CORES");
  if (!e || e[0] != '1') return false;
  return (kmode == kModeGraded || kmode == kModeUnion) && m1tc_supported(M, K, N, group);
}


// Dense rows up to this count run the skinny tcgen05 GEMM (weights as operand A).
constexpr int64_t kSkinnyMaxRows = 64;
// Above the skinny range the weights are dequantized once per call to dtype(w * s) and
// multiplied by the TMA-fed tcgen05 GEMM (gemm_bf16.cu); the fused tcgen05 GEMM
// (gemm_tc.cu, planes converted in its converter warps) takes the shapes that path
// cannot (N / 16 odd, unaligned views).
constexpr int64_t kBf16MinRows = kSkinnyMaxRows + 1;

// Kernel choice: graded / union rows of one token use the register-streaming
// single-row kernel; dense rows 2..kSkinnyMaxRows the skinny tcgen05 GEMM; dense
// rows above that the tcgen05 GEMM; everything else the generic small-M kernel.
static bool use_m1(int kmode, int64_t M, int64_t K, int64_t N, int group) {
  return (kmode == kModeGraded || kmode == kModeUnion) && m1_supported(M, K, N, group);
}

// The dequantization pass costs about as much as streaming the weights three times, so
// it pays off with many rows, or when the fused GEMM's 256 x 256 tiles would leave more
// than half of the SMs idle.
static bool use_bf16_gemm(int kmode, int64_t M, int64_t K, int64_t N, int sms) {
  if (kmode != kModeDense || M < kBf16MinRows || K % 64 != 0 || N % 32 != 0) return false;
  const int64_t fused_ctas = ((M + 255) / 256) * ((N / 16 + 15) / 16);
  return M >= 512 || fused_ctas < sms / 2;
}

// Rows graded one by one (GRINQH_MODE_GRADED) take the tensor-core graded prefill from
// this many rows on (its per-call preparation of the zone operands costs about one pass
// over the weights); fewer rows run the generic kernel.
constexpr int64_t kGradedTcMinRows = 128;

static bool use_graded_gemm(int kmode, int64_t M) { return kmode == kModeGraded && M >= kGradedTcMinRows; }

static bool use_skinny(int kmode, int64_t M, int64_t K, int64_t N, int group) {
  return kmode == kModeDense && M >= 2 && M <= kSkinnyMaxRows && skinny_supported(M, K, N, group);
}

static size_t workspace_for(const SkinnyPlan& p) { return split_workspace(p.slot_bytes, p.counter_bytes); }

static int validate(const void* x, int dtype, int64_t M, int64_t K, const void* w, const void* s, int bits,
                    int group, int64_t N, const void* y) {
  if (!valid_bits(bits)) return set_error(GRINQH_ERR_UNSUPPORTED, "max_bits must be 2, 4, 6 or 8 (got %d)", bits);
  GRINQH_REQUIRE(dtype == GRINQH_BF16 || dtype == GRINQH_F16, "dtype must be GRINQH_BF16 or GRINQH_F16");
  GRINQH_REQUIRE(M >= 0, "M must be >= 0");
  GRINQH_REQUIRE(K > 0, "K must be > 0");
  GRINQH_REQUIRE(N > 0 && N % 16 == 0, "N must be a positive multiple of 16 (got %lld)", (long long)N);
  GRINQH_REQUIRE(group > 0 && group % 32 == 0, "group_size must be a positive multiple of 32 (got %d)", group);
  GRINQH_REQUIRE(K % group == 0, "K (%lld) must be a multiple of group_size (%d)", (long long)K, group);
  GRINQH_REQUIRE(K < (1LL << 31) && N < (1LL << 31) && M < (1LL << 31), "size exceeds int32 range");
  GRINQH_REQUIRE(M == 0 || (x && w && s && y), "null pointer");
  return GRINQH_OK;
}

}  // namespace grinqh

using namespace grinqh;

extern "C" int grinqh_abi_version(void) { return 1; }

extern "C" const char* grinqh_status_string(int status) {
  switch (status) {
    case GRINQH_OK: return "ok";
    case GRINQH_ERR_INVALID: return "invalid argument";
    case GRINQH_ERR_UNSUPPORTED: return "unsupported";
    case GRINQH_ERR_CUDA: return "CUDA error";
    case GRINQH_ERR_WORKSPACE: return "workspace too small";
    case GRINQH_ERR_DEVICE: return "unsupported device";
    default: return "unknown status";
  }
}

extern "C" const char* grinqh_last_error(void) { return g_last_error.c_str(); }

extern "C" size_t grinqh_workspace_size(int64_t M, int64_t K, int64_t N, int max_bits, int group_size, int mode) {
  if (group_size <= 0 || !valid_bits(max_bits)) return 0;
  mode &= ~GRINQH_WORKSPACE_ZEROED;
  const int km = resolve_mode(mode, M);
  if (km < 0 || M <= 0 || K <= 0 || N <= 0) return 0;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices && g_sm_count[dev] > 0) sms = g_sm_count[dev];
  if (use_m1tc(km, M, K, N, group_size)) {
    // a weight view that is not 16-byte aligned runs the streaming kernel: cover both
    const size_t a = workspace_for(plan_m1tc(K, N, max_bits / 2, sms));
    const size_t b = use_m1(km, M, K, N, group_size) ? workspace_for(plan_m1(K, N, group_size, sms))
                                                     : workspace_for(plan_decode(M, K, N, km, sms));
    const size_t c = workspace_for(plan_decode(M, K, N, km, sms));
    return a > b ? (a > c ? a : c) : (b > c ? b : c);
  }
  if (use_m1(km, M, K, N, group_size)) {
    // a weight or scale view that is not 8 / 4-byte aligned runs the generic kernel,
    // and this query does not see the pointers: cover both plans
    const size_t a = workspace_for(plan_m1(K, N, group_size, sms));
    const size_t b = workspace_for(plan_decode(M, K, N, km, sms));
    return a > b ? a : b;
  }
  // an activation or output view that the tensor-core kernels cannot take (alignment)
  // runs the generic kernel, and this query does not see the pointers: cover both
  const size_t generic = workspace_for(plan_decode(M, K, N, km, sms));
  if (use_graded_gemm(km, M) && K % 64 == 0 && N % 32 == 0) {
    const size_t a = graded_gemm_workspace(M, K, N, max_bits / 2, sms);
    return a > generic ? a : generic;
  }
  if (use_bf16_gemm(km, M, K, N, sms)) {
    // the dtype(w * s) buffer sits after the ticket region, then the split-K sums
    const int splits = bf16_gemm_splits(M, K, N, sms);
    const size_t a = kTicketBytes + align_up(bf16_gemm_buffer_bytes(K, N), 256) +
                     align_up(bf16_gemm_slot_bytes(M, N, splits), 256);
    return a > generic ? a : generic;
  }
  if (use_skinny(km, M, K, N, group_size)) {
    const size_t a = workspace_for(plan_skinny(M, K, N, sms));
    return a > generic ? a : generic;
  }
  return generic;
}

// umask: the rows' union of grades per k, from a producer that graded x as it wrote it
// (union mode with several rows; null: the kernel grades x itself).
static int gemm_or_gemv_impl(const void* x, int dtype, int64_t M, int64_t K, const uint32_t* w, const void* s,
                             const void* bias, int max_bits, int group, int64_t N, const float* thresholds, int mode,
                             void* y, void* workspace, size_t workspace_bytes, const uint8_t* umask,
                             grinqh_stream_t stream) {
  int dev = 0, sms = 0;
  GRINQH_RETURN_IF(device_info(&dev, &sms));
  GRINQH_RETURN_IF(validate(x, dtype, M, K, w, s, max_bits, group, N, y));
  const bool zeroed = (mode & GRINQH_WORKSPACE_ZEROED) != 0;  // tickets already zero: no clearing
  mode &= ~GRINQH_WORKSPACE_ZEROED;
  const int km = resolve_mode(mode, M);
  GRINQH_REQUIRE(km >= 0, "unknown mode %d", mode);
  GRINQH_REQUIRE(km == kModeDense || thresholds, "thresholds required for graded modes");
  if (M == 0) return GRINQH_OK;

  if (use_m1tc(km, M, K, N, group) && m1tc_pointers_ok(w) && m1tc_plan_fits(plan_m1tc(K, N, max_bits / 2, sms))) {
    const M1TcPlan plan = plan_m1tc(K, N, max_bits / 2, sms);
    const size_t need = workspace_for(plan);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    GRINQH_REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    M1TcArgs g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.K = (int)K;
    g.N = (int)N;
    g.tiles = plan.tiles;
    g.units_per_cta = plan.units_per_cta;
    g.bslots = plan.bslots;
    g.tma_min_rows = tc_tma_min_rows();
    for (int z = 0; z < 4; ++z) g.t[z] = thresholds[z];
    GRINQH_RETURN_IF(bind_workspace(workspace, plan.slot_bytes, plan.counter_bytes, zeroed, stream, &g.slots,
                                    &g.counters));
    return launch_m1tc(g, plan, dtype, max_bits / 2, stream);
  }

  if (use_m1(km, M, K, N, group) && m1_pointers_ok(w, s) && m1_plan_fits(plan_m1(K, N, group, sms))) {
    const M1Plan plan = plan_m1(K, N, group, sms);
    const size_t need = workspace_for(plan);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
      return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    GRINQH_REQUIRE(need == 0 || aligned(workspace, 256), "workspace must be 256-byte aligned");
    M1Args g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.K = (int)K;
    g.N = (int)N;
    g.group = group;
    g.rows_per_warp = plan.rows_per_warp;
    g.rows_per_cta = plan.rows_per_cta;
    for (int z = 0; z < 4; ++z) g.t[z] = thresholds[z];
    if (need > 0)
      GRINQH_RETURN_IF(bind_workspace(workspace, plan.slot_bytes, plan.counter_bytes, zeroed, stream, &g.slots,
                                      &g.counters));
    return launch_m1(g, plan, dtype, max_bits / 2, stream);
  }

  if (use_graded_gemm(km, M) && graded_gemm_supported(M, K, N, group, x, w, s, y)) {
    const size_t need = graded_gemm_workspace(M, K, N, max_bits / 2, sms);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    GRINQH_REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    Bf16GemmArgs g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.M = (int)M;
    g.K = (int)K;
    g.N = (int)N;
    g.group = group;
    return launch_graded_gemm(g, thresholds, workspace, dtype, max_bits / 2, sms, stream);
  }

  if (use_skinny(km, M, K, N, group) && skinny_pointers_ok(x, w, s)) {
    const SkinnyPlan plan = plan_skinny(M, K, N, sms);
    const size_t need = workspace_for(plan);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
      return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    GRINQH_REQUIRE(need == 0 || aligned(workspace, 256), "workspace must be 256-byte aligned");
    SkinnyArgs g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.M = (int)M;
    g.K = (int)K;
    g.N = (int)N;
    g.group = group;
    g.tiles = plan.tiles;
    g.splits = plan.splits;
    g.cluster = plan.cluster;
    g.steps_per_split = plan.steps_per_split;
    if (need > 0)
      GRINQH_RETURN_IF(bind_workspace(workspace, plan.slot_bytes, plan.counter_bytes, zeroed, stream, &g.slots,
                                      &g.counters));
    return launch_skinny(g, plan, dtype, max_bits / 2, stream);
  }

  if (use_bf16_gemm(km, M, K, N, sms) && bf16_gemm_supported(M, K, N, group, x, w, s, y)) {
    const int splits = bf16_gemm_splits(M, K, N, sms);
    const size_t wbuf_bytes = align_up(bf16_gemm_buffer_bytes(K, N), 256);
    const size_t need = kTicketBytes + wbuf_bytes + align_up(bf16_gemm_slot_bytes(M, N, splits), 256);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    GRINQH_REQUIRE(aligned(workspace, 256), "workspace must be 256-byte aligned");
    Bf16GemmArgs g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.wbuf = static_cast<char*>(workspace) + kTicketBytes;
    g.M = (int)M;
    g.K = (int)K;
    g.N = (int)N;
    g.group = group;
    g.splits = splits;
    if (splits > 1) {  // one ticket per output tile at the start of the workspace
      g.counters = static_cast<unsigned*>(workspace);
      g.slots = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTicketBytes + wbuf_bytes);
      const size_t tiles = (size_t)((M + 255) / 256) * (size_t)((N + 255) / 256);
      if (!zeroed) {
        const cudaError_t e = cudaMemsetAsync(g.counters, 0, tiles * sizeof(unsigned), stream);
        if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
      }
    }
    return launch_bf16_gemm(g, dtype, max_bits / 2, stream);
  }

  if (km == kModeDense && M > kSkinnyMaxRows && gemm_tc_supported(M, K, N, group, x, y)) {
    GemmArgs g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.M = (int)M;
    g.K = (int)K;
    g.N = (int)N;
    g.group = group;
    return launch_gemm_tc(g, dtype, max_bits / 2, stream);
  }

  const DecodePlan plan = plan_decode(M, K, N, km, sms);
  const size_t need = workspace_for(plan);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  GRINQH_REQUIRE(need == 0 || aligned(workspace, 256), "workspace must be 256-byte aligned");

  DecodeArgs a{};
  a.x = x;
  a.w = w;
  a.s = s;
  a.bias = bias;
  a.y = y;
  a.M = (int)M;
  a.K = (int)K;
  a.N = (int)N;
  a.group = group;
  a.rows_per_cta = plan.rows_per_cta;
  a.ksplit = plan.ksplit;
  for (int z = 0; z < 4; ++z) a.t[z] = thresholds ? thresholds[z] : 0.0f;
  a.umask = km == kModeUnion ? umask : nullptr;
  if (plan.ksplit > 1)
    GRINQH_RETURN_IF(bind_workspace(workspace, plan.partial_bytes, plan.counter_bytes, zeroed, stream, &a.partial,
                                    &a.counters));
  return launch_decode(a, plan, km, dtype, max_bits / 2, stream);
}

extern "C" int grinqh_gemm_or_gemv(const void* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                                   const void* s, const void* bias, int max_bits, int group, int64_t N,
                                   const float* thresholds, int mode, void* y, void* workspace,
                                   size_t workspace_bytes, grinqh_stream_t stream) {
  return gemm_or_gemv_impl(x, dtype, M, K, w, s, bias, max_bits, group, N, thresholds, mode, y, workspace,
                           workspace_bytes, nullptr, stream);
}

extern "C" int grinqh_gemv_batch_union_masked(const void* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                                              const void* s, const void* bias, int max_bits, int group, int64_t N,
                                              const float* thresholds, const uint8_t* union_mask, void* y,
                                              void* workspace, size_t workspace_bytes, grinqh_stream_t stream) {
  GRINQH_REQUIRE(union_mask, "union_mask required");
  return gemm_or_gemv_impl(x, dtype, M, K, w, s, bias, max_bits, group, N, thresholds, GRINQH_MODE_UNION, y,
                           workspace, workspace_bytes, union_mask, stream);
}

// ---------------------------------------------------------------- fused all-reduce
// How long a fused launch waits for the other ranks' partials before it gives up and
// counts a timeout: GRINQH_ALLREDUCE_WAIT_MS milliseconds (read on every call, default
// 2000, at least 1).
static unsigned long long allreduce_wait_ns() {
  const char* e = getenv("GRINQH_ALLREDUCE_WAIT_MS");
  long ms = e ? atol(e) : 2000;
  if (ms < 1) ms = 1;
  return (unsigned long long)ms * 1000000ull;
}

extern "C" size_t grinqh_allreduce_buffer_bytes(int world, int64_t cap) {
  if (world < 1 || world > kArMaxRanks || cap <= 0) return 0;
  return peer_reduce_buffer_bytes(world, cap);
}

// Which kernel a fused launch of M rows runs: one row graded (or union) by the
// single-row kernel, 2..kSkinnyMaxRows dense rows by the skinny GEMM; 0 if neither.
enum { kArNone = 0, kArM1 = 1, kArSkinny = 2 };
static int allreduce_kernel(int km, int64_t M, int64_t K, int64_t N, int group) {
  if (M == 1 && use_m1(km, M, K, N, group)) return kArM1;
  if (use_skinny(km, M, K, N, group)) return kArSkinny;
  return kArNone;
}

extern "C" size_t grinqh_allreduce_workspace_size(int64_t M, int64_t K, int64_t N, int max_bits, int group_size,
                                                  int mode) {
  if (group_size <= 0 || !valid_bits(max_bits) || M <= 0 || K <= 0 || N <= 0) return 0;
  const int km = resolve_mode(mode & ~GRINQH_WORKSPACE_ZEROED, M);
  if (km < 0) return 0;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices && g_sm_count[dev] > 0) sms = g_sm_count[dev];
  switch (allreduce_kernel(km, M, K, N, group_size)) {
    case kArM1: return workspace_for(plan_m1(K, N, group_size, sms));
    case kArSkinny: {
      SkinnyPlan plan{};
      return plan_skinny_resident(M, K, N, sms, &plan) ? workspace_for(plan) : 0;
    }
    default: return 0;
  }
}

extern "C" int grinqh_allreduce_buffer_alloc(size_t bytes, void** buf) {
  GRINQH_RETURN_IF(check_device());
  GRINQH_REQUIRE(buf && bytes >= kArParts, "null pointer or buffer too small");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);  // epoch, ticket and flags start at 0
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(GRINQH_ERR_CUDA, "clearing the peer buffer: %s", cudaGetErrorString(e));
  }
  *buf = p;
  return GRINQH_OK;
}

extern "C" int grinqh_allreduce_buffer_free(void* buf) {
  if (!buf) return GRINQH_OK;
  const cudaError_t e = cudaFree(buf);
  return e == cudaSuccess ? GRINQH_OK : set_error(GRINQH_ERR_CUDA, "cudaFree: %s", cudaGetErrorString(e));
}

extern "C" int grinqh_ipc_get_handle(const void* buf, unsigned char* handle64) {
  GRINQH_REQUIRE(buf && handle64, "null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buf));
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  return GRINQH_OK;
}

extern "C" int grinqh_ipc_open_handle(const unsigned char* handle64, void** buf) {
  GRINQH_REQUIRE(handle64 && buf, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  const cudaError_t e = cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(GRINQH_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return GRINQH_OK;
}

extern "C" int grinqh_ipc_close_handle(void* buf) {
  if (!buf) return GRINQH_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(buf);
  return e == cudaSuccess ? GRINQH_OK : set_error(GRINQH_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
}

extern "C" int grinqh_gemm_allreduce(const void* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                                     const void* s, const void* bias, int max_bits, int group, int64_t N,
                                     const float* thresholds, int mode, void* y, void* workspace,
                                     size_t workspace_bytes, int rank, int world, void* const* buffers, int64_t cap,
                                     grinqh_stream_t stream) {
  int dev = 0, sms = 0;
  GRINQH_RETURN_IF(device_info(&dev, &sms));
  GRINQH_RETURN_IF(validate(x, dtype, M, K, w, s, max_bits, group, N, y));
  const bool zeroed = (mode & GRINQH_WORKSPACE_ZEROED) != 0;
  const int km = resolve_mode(mode & ~GRINQH_WORKSPACE_ZEROED, M);
  GRINQH_REQUIRE(km >= 0, "unknown mode %d", mode & ~GRINQH_WORKSPACE_ZEROED);
  GRINQH_REQUIRE(km == kModeDense || thresholds, "thresholds required for graded modes");
  GRINQH_REQUIRE(world >= 1 && world <= kArMaxRanks && rank >= 0 && rank < world, "rank %d of %d (at most %d ranks)",
                 rank, world, kArMaxRanks);
  GRINQH_REQUIRE(buffers && M * N <= cap, "peer buffers hold %lld values, M * N is %lld", (long long)cap,
                 (long long)(M * N));
  for (int r = 0; r < world; ++r) GRINQH_REQUIRE(buffers[r] && aligned(buffers[r], 256), "peer buffer %d", r);
  PeerReduce ar{};
  ar.rank = rank;
  ar.world = world;
  ar.cap = cap;
  ar.wait_ns = allreduce_wait_ns();
  for (int r = 0; r < world; ++r) ar.buf[r] = static_cast<unsigned char*>(buffers[r]);
  if (M == 0) return GRINQH_OK;  // every rank skips alike: no epoch is used
  const int which = allreduce_kernel(km, M, K, N, group);

  if (which == kArM1) {
    if (!m1_pointers_ok(w, s) || !m1_plan_fits(plan_m1(K, N, group, sms)))
      return set_error(GRINQH_ERR_UNSUPPORTED, "fused all-reduce not supported: shape or alignment of the "
                       "single-row GEMV");
    const M1Plan plan = plan_m1(K, N, group, sms);
    const size_t need = workspace_for(plan);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
      return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    GRINQH_REQUIRE(need == 0 || aligned(workspace, 256), "workspace must be 256-byte aligned");
    M1Args g{};
    g.x = x;
    g.w = w;
    g.s = s;
    g.bias = bias;
    g.y = y;
    g.K = (int)K;
    g.N = (int)N;
    g.group = group;
    g.rows_per_warp = plan.rows_per_warp;
    g.rows_per_cta = plan.rows_per_cta;
    for (int z = 0; z < 4; ++z) g.t[z] = thresholds[z];
    g.ar = ar;
    if (need > 0)
      GRINQH_RETURN_IF(bind_workspace(workspace, plan.slot_bytes, plan.counter_bytes, zeroed, stream, &g.slots,
                                      &g.counters));
    return launch_m1(g, plan, dtype, max_bits / 2, stream, true);
  }

  SkinnyPlan plan{};
  if (which != kArSkinny || !skinny_pointers_ok(x, w, s) || !plan_skinny_resident(M, K, N, sms, &plan))
    return set_error(GRINQH_ERR_UNSUPPORTED,
                     "fused all-reduce not supported: M=%lld K=%lld N=%lld mode %d (the fused kernels take one "
                     "graded row, or 2..%lld dense rows, with aligned views)",
                     (long long)M, (long long)K, (long long)N, mode & ~GRINQH_WORKSPACE_ZEROED,
                     (long long)kSkinnyMaxRows);
  const size_t need = workspace_for(plan);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(GRINQH_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  GRINQH_REQUIRE(need == 0 || aligned(workspace, 256), "workspace must be 256-byte aligned");
  SkinnyArgs g{};
  g.x = x;
  g.w = w;
  g.s = s;
  g.bias = bias;
  g.y = y;
  g.M = (int)M;
  g.K = (int)K;
  g.N = (int)N;
  g.group = group;
  g.tiles = plan.tiles;
  g.splits = plan.splits;
  g.cluster = plan.cluster;
  g.steps_per_split = plan.steps_per_split;
  g.ar = ar;
  if (need > 0)
    GRINQH_RETURN_IF(bind_workspace(workspace, plan.slot_bytes, plan.counter_bytes, zeroed, stream, &g.slots,
                                    &g.counters));
  return launch_skinny(g, plan, dtype, max_bits / 2, stream, true);
}

extern "C" int grinqh_gemv_allreduce(const void* x, int dtype, int64_t K, const uint32_t* w, const void* s,
                                     const void* bias, int max_bits, int group, int64_t N, const float* thresholds,
                                     void* y, void* workspace, size_t workspace_bytes, int rank, int world,
                                     void* const* buffers, int64_t n_cap, int mode, grinqh_stream_t stream) {
  GRINQH_REQUIRE((mode & ~GRINQH_WORKSPACE_ZEROED) == 0, "mode takes only GRINQH_WORKSPACE_ZEROED");
  GRINQH_REQUIRE(thresholds, "thresholds required");
  return grinqh_gemm_allreduce(x, dtype, 1, K, w, s, bias, max_bits, group, N, thresholds, mode | GRINQH_MODE_AUTO,
                               y, workspace, workspace_bytes, rank, world, buffers, n_cap, stream);
}

extern "C" int grinqh_take_error_flags(unsigned* timeouts) {
  GRINQH_RETURN_IF(check_device());
  const unsigned v = take_gemm_timeouts() + take_m1tc_timeouts() + take_skinny_timeouts() + take_bf16_gemm_timeouts() +
                     take_m1_timeouts();
  if (timeouts) *timeouts = v;
  return GRINQH_OK;
}

extern "C" int grinqh_gemv_batch_union(const void* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                                       const void* s, const void* bias, int max_bits, int group, int64_t N,
                                       const float* thresholds, void* y, void* workspace, size_t workspace_bytes,
                                       grinqh_stream_t stream) {
  return grinqh_gemm_or_gemv(x, dtype, M, K, w, s, bias, max_bits, group, N, thresholds, GRINQH_MODE_UNION, y,
                             workspace, workspace_bytes, stream);
}

extern "C" int grinqh_prefill_gemm(const void* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                                   const void* s, const void* bias, int max_bits, int group, int64_t N, void* y,
                                   void* workspace, size_t workspace_bytes, grinqh_stream_t stream) {
  return grinqh_gemm_or_gemv(x, dtype, M, K, w, s, bias, max_bits, group, N, nullptr, GRINQH_MODE_DENSE, y,
                             workspace, workspace_bytes, stream);
}
