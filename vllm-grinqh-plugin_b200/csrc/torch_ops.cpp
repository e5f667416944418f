// torch custom ops of the GRINQH plugin. Thin shims: argument checks, output /
// workspace allocation through the caching allocator, the current CUDA stream,
// then one call into the C ABI (include/grinqh_b200.h). No CPU implementation is
// registered: a CPU tensor raises.
//
// Schemas mirror the reference's op (grinqh/kernel.py:646-657) plus the helpers
// its tests call (pack_triton utils.py:125, unpack utils.py:149/209,
// grinqh_gemv_batch_union kernel.py:607, grinqh_prefill_gemm_compiled kernel.py:561).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <optional>
#include <utility>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "grinqh_b200.h"

namespace {

// An NVTX range around each op call, so that profilers (nsys, ncu --nvtx) attribute the
// kernels to the quantized linear; without a tool attached the calls do nothing.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};

int dtype_code(const at::Tensor& t, const char* name) {
  if (t.scalar_type() == at::kBFloat16) return GRINQH_BF16;
  if (t.scalar_type() == at::kHalf) return GRINQH_F16;
  TORCH_CHECK(false, "GRINQH: ", name, " must be float16 or bfloat16, got ", t.scalar_type());
  return -1;
}

void check_ok(int st, const char* what) {
  TORCH_CHECK(st == GRINQH_OK, "GRINQH ", what, " failed (", grinqh_status_string(st), "): ", grinqh_last_error());
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "GRINQH: ", name, " must be a CUDA tensor (no CPU implementation)");
}

bool is_word32(const at::Tensor& t) {
  return t.scalar_type() == at::kInt || t.scalar_type() == at::kUInt32;
}

std::vector<float> thresholds4(at::ArrayRef<double> th) {
  // kernel.py:700 reads thresholds[0..3]; grinqh.py:113 pads with 0.0
  std::vector<float> t(4, 0.0f);
  for (size_t i = 0; i < th.size() && i < 4; ++i) t[i] = static_cast<float>(th[i]);
  return t;
}

cudaStream_t cur_stream(const at::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

// A zeroed workspace per (device, stream), grown on demand and kept for the process.
// The kernels leave their split-K tickets at zero, so a call that reuses it passes
// GRINQH_WORKSPACE_ZEROED and no clearing runs on the stream; calls on one stream are
// ordered, and other streams get their own. A workspace is only created outside
// stream capture (a capture records the zeroing instead of running it): a call
// captured before any eager call on its stream allocates per call as before.
at::Tensor stream_workspace(const at::Tensor& like, size_t bytes, cudaStream_t st, bool* zeroed) {
  static std::mutex mu;
  static std::map<std::pair<int, uintptr_t>, at::Tensor> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(static_cast<int>(like.device().index()), reinterpret_cast<uintptr_t>(st));
  auto it = cache.find(key);
  if (it != cache.end() && static_cast<size_t>(it->second.numel()) >= bytes) {
    *zeroed = true;
    return it->second;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    *zeroed = false;
    return at::empty({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
  }
  const size_t size = std::max<size_t>(bytes, size_t(1) << 20);
  at::Tensor t = at::zeros({static_cast<int64_t>(size)}, like.options().dtype(at::kByte));
  cache[key] = t;
  *zeroed = true;
  return t;
}

int env_mode_for_rows() {
  // Opt-in per-token grading for rows > 1 (this build's graded prefill).
  static const int m = [] {
    const char* v = std::getenv("GRINQH_GRADED_PREFILL");
    return (v && v[0] == '1') ? GRINQH_MODE_GRADED : GRINQH_MODE_AUTO;
  }();
  return m;
}

at::Tensor run_linear(const at::Tensor& x, const at::Tensor& weight_packed, const at::Tensor& weight_scale,
                      const std::optional<at::Tensor>& bias, int64_t max_bits, int64_t group_size,
                      int64_t original_n, at::ArrayRef<double> thresholds, int mode,
                      const at::Tensor* union_mask = nullptr) {
  const NvtxRange range("grinqh::linear");
  check_cuda(x, "x");
  check_cuda(weight_packed, "weight_packed");
  check_cuda(weight_scale, "weight_scale");
  const int dt = dtype_code(x, "x");
  TORCH_CHECK(weight_scale.scalar_type() == x.scalar_type(), "GRINQH: weight_scale dtype ", weight_scale.scalar_type(),
              " != x dtype ", x.scalar_type());
  TORCH_CHECK(is_word32(weight_packed), "GRINQH: weight_packed must be int32/uint32, got ", weight_packed.scalar_type());
  TORCH_CHECK(x.dim() >= 1, "GRINQH: x must have at least one dimension");
  TORCH_CHECK(weight_packed.dim() == 2 && weight_scale.dim() == 2, "GRINQH: weight_packed and weight_scale must be 2-D");
  const int64_t K = weight_packed.size(0);
  const int64_t N = original_n * 4;
  TORCH_CHECK(max_bits == 2 || max_bits == 4 || max_bits == 6 || max_bits == 8,
              "GRINQH: max_bits must be 2, 4, 6 or 8, got ", max_bits);
  TORCH_CHECK(x.size(-1) == K, "GRINQH: x.shape[-1] (", x.size(-1), ") != K (", K, ")");
  TORCH_CHECK(weight_packed.size(1) == (max_bits / 2) * (N / 16), "GRINQH: weight_packed has ", weight_packed.size(1),
              " columns, expected ", (max_bits / 2) * (N / 16), " for N=", N, " and max_bits=", max_bits);
  TORCH_CHECK(group_size > 0 && K % group_size == 0, "GRINQH: K must be a multiple of group_size");
  TORCH_CHECK(weight_scale.size(0) == K / group_size && weight_scale.size(1) == N, "GRINQH: weight_scale shape ",
              weight_scale.sizes(), " != [", K / group_size, ", ", N, "]");
  if (bias) {
    check_cuda(*bias, "bias");
    TORCH_CHECK(bias->scalar_type() == x.scalar_type() && bias->numel() == N, "GRINQH: bias must be [N] of x's dtype");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor xf = x.reshape({-1, K}).contiguous();
  const at::Tensor wp = weight_packed.contiguous();
  const at::Tensor sc = weight_scale.contiguous();
  const at::Tensor bc = bias ? bias->contiguous() : at::Tensor();
  const int64_t M = xf.size(0);
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = N;
  at::Tensor y = at::empty({M, N}, x.options());
  if (M == 0) return y.view(out_shape);
  const auto th = thresholds4(thresholds);
  const size_t ws_bytes = grinqh_workspace_size(M, K, N, (int)max_bits, (int)group_size, mode);
  const cudaStream_t stream = cur_stream(x);
  at::Tensor ws;
  bool zeroed = false;
  if (ws_bytes) ws = stream_workspace(x, ws_bytes, stream, &zeroed);
  const int call_mode = zeroed ? (mode | GRINQH_WORKSPACE_ZEROED) : mode;
  if (union_mask) {  // the rows' union of grades from the producer of x
    check_cuda(*union_mask, "union_mask");
    TORCH_CHECK(union_mask->scalar_type() == at::kByte && union_mask->numel() == K && union_mask->is_contiguous(),
                "GRINQH: union_mask must be a contiguous uint8 tensor of K values");
    check_ok(grinqh_gemv_batch_union_masked(
                 xf.data_ptr(), dt, M, K, reinterpret_cast<const uint32_t*>(wp.data_ptr()), sc.data_ptr(),
                 bias ? bc.data_ptr() : nullptr, (int)max_bits, (int)group_size, N, th.data(),
                 union_mask->data_ptr<uint8_t>(), y.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr,
                 ws_bytes ? static_cast<size_t>(ws.numel()) : 0, stream),
             "gemv_batch_union_masked");
    return y.view(out_shape);
  }
  const int st = grinqh_gemm_or_gemv(xf.data_ptr(), dt, M, K, reinterpret_cast<const uint32_t*>(wp.data_ptr()),
                                     sc.data_ptr(), bias ? bc.data_ptr() : nullptr, (int)max_bits, (int)group_size, N,
                                     th.data(), call_mode, y.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr,
                                     ws_bytes ? static_cast<size_t>(ws.numel()) : 0, stream);
  check_ok(st, "gemm_or_gemv");
  return y.view(out_shape);
}

// Row-parallel linear of one row with the tensor-parallel sum fused in (the C ABI's
// grinqh_gemv_allreduce): buffers are every rank's peer buffer address as mapped in
// this process, from grinqh.allreduce.PeerBuffers.
at::Tensor gemv_allreduce(const at::Tensor& x, const at::Tensor& weight_packed, const at::Tensor& weight_scale,
                          const std::optional<at::Tensor>& bias, int64_t max_bits, int64_t group_size,
                          int64_t original_n, at::ArrayRef<double> thresholds, int64_t rank, int64_t world,
                          at::ArrayRef<int64_t> buffers, int64_t n_cap) {
  const NvtxRange range("grinqh::gemv_allreduce");
  check_cuda(x, "x");
  check_cuda(weight_packed, "weight_packed");
  check_cuda(weight_scale, "weight_scale");
  const int dt = dtype_code(x, "x");
  TORCH_CHECK(weight_scale.scalar_type() == x.scalar_type(), "GRINQH: weight_scale dtype != x dtype");
  TORCH_CHECK(is_word32(weight_packed) && weight_packed.dim() == 2 && weight_scale.dim() == 2,
              "GRINQH: weight_packed must be 2-D int32/uint32 and weight_scale 2-D");
  const int64_t K = weight_packed.size(0), N = original_n * 4;
  TORCH_CHECK(x.numel() == K, "GRINQH gemv_allreduce: x must hold exactly one row of K = ", K, " values");
  TORCH_CHECK((int64_t)buffers.size() == world, "GRINQH gemv_allreduce: one buffer per rank");
  if (bias) {
    check_cuda(*bias, "bias");
    TORCH_CHECK(bias->scalar_type() == x.scalar_type() && bias->numel() == N, "GRINQH: bias must be [N] of x's dtype");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor xf = x.reshape({1, K}).contiguous();
  const at::Tensor wp = weight_packed.contiguous();
  const at::Tensor sc = weight_scale.contiguous();
  const at::Tensor bc = bias ? bias->contiguous() : at::Tensor();
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = N;
  at::Tensor y = at::empty({1, N}, x.options());
  const auto th = thresholds4(thresholds);
  const size_t ws_bytes = grinqh_workspace_size(1, K, N, (int)max_bits, (int)group_size, GRINQH_MODE_AUTO);
  const cudaStream_t stream = cur_stream(x);
  at::Tensor ws;
  bool zeroed = false;
  if (ws_bytes) ws = stream_workspace(x, ws_bytes, stream, &zeroed);
  std::vector<void*> bufs(buffers.size());
  for (size_t r = 0; r < buffers.size(); ++r) bufs[r] = reinterpret_cast<void*>(buffers[r]);
  check_ok(grinqh_gemv_allreduce(xf.data_ptr(), dt, K, reinterpret_cast<const uint32_t*>(wp.data_ptr()), sc.data_ptr(),
                                 bias ? bc.data_ptr() : nullptr, (int)max_bits, (int)group_size, N, th.data(),
                                 y.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr,
                                 ws_bytes ? static_cast<size_t>(ws.numel()) : 0, (int)rank, (int)world, bufs.data(),
                                 n_cap, zeroed ? GRINQH_WORKSPACE_ZEROED : 0, stream),
           "gemv_allreduce");
  return y.view(out_shape);
}

// Row-parallel linear of M rows with the tensor-parallel sum fused in (the C ABI's
// grinqh_gemm_allreduce): one graded row or 2..64 dense rows; any other shape raises
// "fused all-reduce not supported" before anything is launched (on every rank alike).
at::Tensor linear_allreduce(const at::Tensor& x, const at::Tensor& weight_packed, const at::Tensor& weight_scale,
                            const std::optional<at::Tensor>& bias, int64_t max_bits, int64_t group_size,
                            int64_t original_n, at::ArrayRef<double> thresholds, int64_t mode, int64_t rank,
                            int64_t world, at::ArrayRef<int64_t> buffers, int64_t cap) {
  const NvtxRange range("grinqh::linear_allreduce");
  check_cuda(x, "x");
  check_cuda(weight_packed, "weight_packed");
  check_cuda(weight_scale, "weight_scale");
  const int dt = dtype_code(x, "x");
  TORCH_CHECK(weight_scale.scalar_type() == x.scalar_type(), "GRINQH: weight_scale dtype != x dtype");
  TORCH_CHECK(is_word32(weight_packed) && weight_packed.dim() == 2 && weight_scale.dim() == 2,
              "GRINQH: weight_packed must be 2-D int32/uint32 and weight_scale 2-D");
  const int64_t K = weight_packed.size(0), N = original_n * 4;
  TORCH_CHECK(x.dim() >= 1 && x.size(-1) == K, "GRINQH linear_allreduce: x must be [..., K] with K = ", K);
  TORCH_CHECK(max_bits == 2 || max_bits == 4 || max_bits == 6 || max_bits == 8,
              "GRINQH: max_bits must be 2, 4, 6 or 8, got ", max_bits);
  TORCH_CHECK(weight_packed.size(1) == (max_bits / 2) * (N / 16), "GRINQH: weight_packed has ", weight_packed.size(1),
              " columns, expected ", (max_bits / 2) * (N / 16), " for N=", N, " and max_bits=", max_bits);
  TORCH_CHECK(group_size > 0 && K % group_size == 0 && weight_scale.size(0) == K / group_size &&
                  weight_scale.size(1) == N,
              "GRINQH: weight_scale shape ", weight_scale.sizes(), " does not match K=", K, ", N=", N);
  TORCH_CHECK((int64_t)buffers.size() == world, "GRINQH linear_allreduce: one buffer per rank");
  if (bias) {
    check_cuda(*bias, "bias");
    TORCH_CHECK(bias->scalar_type() == x.scalar_type() && bias->numel() == N, "GRINQH: bias must be [N] of x's dtype");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor xf = x.reshape({-1, K}).contiguous();
  const int64_t M = xf.size(0);
  const at::Tensor wp = weight_packed.contiguous();
  const at::Tensor sc = weight_scale.contiguous();
  const at::Tensor bc = bias ? bias->contiguous() : at::Tensor();
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = N;
  at::Tensor y = at::empty({M, N}, x.options());
  const auto th = thresholds4(thresholds);
  const size_t ws_bytes = grinqh_allreduce_workspace_size(M, K, N, (int)max_bits, (int)group_size, (int)mode);
  const cudaStream_t stream = cur_stream(x);
  at::Tensor ws;
  bool zeroed = false;
  if (ws_bytes) ws = stream_workspace(x, ws_bytes, stream, &zeroed);
  std::vector<void*> bufs(buffers.size());
  for (size_t r = 0; r < buffers.size(); ++r) bufs[r] = reinterpret_cast<void*>(buffers[r]);
  check_ok(grinqh_gemm_allreduce(xf.data_ptr(), dt, M, K, reinterpret_cast<const uint32_t*>(wp.data_ptr()),
                                 sc.data_ptr(), bias ? bc.data_ptr() : nullptr, (int)max_bits, (int)group_size, N,
                                 th.data(), zeroed ? ((int)mode | GRINQH_WORKSPACE_ZEROED) : (int)mode, y.data_ptr(),
                                 ws_bytes ? ws.data_ptr() : nullptr, ws_bytes ? static_cast<size_t>(ws.numel()) : 0,
                                 (int)rank, (int)world, bufs.data(), cap, stream),
           "linear_allreduce");
  return y.view(out_shape);
}

// torch.ops.grinqh.gemm_or_gemv -- grinqh/kernel.py:646-710. use_marlin is accepted
// for schema compatibility and ignored (no Marlin path in this build).
at::Tensor gemm_or_gemv(const at::Tensor& x, const at::Tensor& weight_packed, const at::Tensor& weight_scale,
                        const std::optional<at::Tensor>& bias, int64_t max_bits, int64_t group_size,
                        int64_t original_n, at::ArrayRef<double> thresholds, bool use_marlin) {
  (void)use_marlin;
  return run_linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds,
                    env_mode_for_rows());
}

at::Tensor linear(const at::Tensor& x, const at::Tensor& weight_packed, const at::Tensor& weight_scale,
                  const std::optional<at::Tensor>& bias, int64_t max_bits, int64_t group_size, int64_t original_n,
                  at::ArrayRef<double> thresholds, int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 3, "GRINQH: mode must be 0..3");
  return run_linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds, (int)mode);
}

// The batch-union GEMV with the union of grades from the producer of x (rmsnorm_grade /
// silu_mul_grade), which the kernel then does not recompute from every row of x.
at::Tensor union_linear_masked(const at::Tensor& x, const at::Tensor& weight_packed, const at::Tensor& weight_scale,
                               const std::optional<at::Tensor>& bias, int64_t max_bits, int64_t group_size,
                               int64_t original_n, at::ArrayRef<double> thresholds, const at::Tensor& union_mask) {
  return run_linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds,
                    GRINQH_MODE_UNION, &union_mask);
}

// x for the next linear together with its grades (C ABI grinqh_rmsnorm_grade): returns
// (out, masks [M, K] uint8, union [K] uint8); residual, if given, is updated in place
// to dtype(x + residual) as vLLM's fused_add_rms_norm does.
std::tuple<at::Tensor, at::Tensor, at::Tensor> rmsnorm_grade(const at::Tensor& x,
                                                             const std::optional<at::Tensor>& residual,
                                                             const std::optional<at::Tensor>& weight, double eps,
                                                             at::ArrayRef<double> thresholds, int64_t max_bits) {
  const NvtxRange range("grinqh::rmsnorm_grade");
  check_cuda(x, "x");
  const int dt = dtype_code(x, "x");
  TORCH_CHECK(x.is_contiguous(), "GRINQH rmsnorm_grade: x must be contiguous");
  const int64_t K = x.size(-1), M = K ? x.numel() / K : 0;
  if (residual) {
    check_cuda(*residual, "residual");
    TORCH_CHECK(residual->scalar_type() == x.scalar_type() && residual->sizes() == x.sizes() &&
                    residual->is_contiguous(),
                "GRINQH rmsnorm_grade: residual must be a contiguous tensor like x");
  }
  at::Tensor wc;
  if (weight) {
    check_cuda(*weight, "weight");
    TORCH_CHECK(weight->scalar_type() == x.scalar_type() && weight->numel() == K,
                "GRINQH rmsnorm_grade: weight must be [K] of x's dtype");
    wc = weight->contiguous();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty_like(x);
  at::Tensor masks = at::empty({M, K}, x.options().dtype(at::kByte));
  at::Tensor uni = at::empty({K}, x.options().dtype(at::kByte));
  const auto th = thresholds4(thresholds);
  check_ok(grinqh_rmsnorm_grade(x.data_ptr(), residual ? residual->data_ptr() : nullptr,
                                weight ? wc.data_ptr() : nullptr, dt, M, K, (float)eps, th.data(), (int)max_bits,
                                out.data_ptr(), masks.data_ptr<uint8_t>(), uni.data_ptr<uint8_t>(), cur_stream(x)),
           "rmsnorm_grade");
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  return {out, masks.view(shape), uni};
}

// silu(gate) * up of x = [..., 2K] with its grades (C ABI grinqh_silu_mul_grade).
std::tuple<at::Tensor, at::Tensor, at::Tensor> silu_mul_grade(const at::Tensor& x, at::ArrayRef<double> thresholds,
                                                              int64_t max_bits) {
  const NvtxRange range("grinqh::silu_mul_grade");
  check_cuda(x, "x");
  const int dt = dtype_code(x, "x");
  TORCH_CHECK(x.size(-1) % 2 == 0, "GRINQH silu_mul_grade: the last dimension must be even");
  const at::Tensor xc = x.contiguous();
  const int64_t K = x.size(-1) / 2, M = K ? x.numel() / (2 * K) : 0;
  const c10::cuda::CUDAGuard guard(x.device());
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape.back() = K;
  at::Tensor out = at::empty(shape, x.options());
  at::Tensor masks = at::empty(shape, x.options().dtype(at::kByte));
  at::Tensor uni = at::empty({K}, x.options().dtype(at::kByte));
  const auto th = thresholds4(thresholds);
  check_ok(grinqh_silu_mul_grade(xc.data_ptr(), dt, M, K, th.data(), (int)max_bits, out.data_ptr(),
                                 masks.data_ptr<uint8_t>(), uni.data_ptr<uint8_t>(), cur_stream(x)),
           "silu_mul_grade");
  return {out, masks, uni};
}

// pack_triton (grinqh/utils.py:125-146): [K, N/4] shifted code words -> [K, (b/2)*N/16]
at::Tensor pack(const at::Tensor& words, int64_t max_bits) {
  check_cuda(words, "words");
  TORCH_CHECK(is_word32(words) && words.dim() == 2, "GRINQH pack: expects a 2-D uint32/int32 tensor");
  const at::Tensor a = words.contiguous();
  const int64_t K = a.size(0), nw = a.size(1);
  TORCH_CHECK(nw % 4 == 0, "GRINQH pack: number of words must be a multiple of 4");
  const c10::cuda::CUDAGuard guard(a.device());
  at::Tensor out = at::empty({K, (max_bits / 2) * (nw / 4)}, a.options());
  check_ok(grinqh_pack_words(reinterpret_cast<const uint32_t*>(a.data_ptr()), reinterpret_cast<uint32_t*>(out.data_ptr()),
                             K, nw, (int)max_bits, cur_stream(a)),
           "pack");
  return out;
}

// process_weights_after_loading transform (grinqh/grinqh.py:202-211) from int8 codes
at::Tensor pack_codes(const at::Tensor& codes, int64_t max_bits) {
  check_cuda(codes, "codes");
  TORCH_CHECK(codes.scalar_type() == at::kChar && codes.dim() == 2, "GRINQH pack_codes: expects 2-D int8 codes [K, N]");
  const at::Tensor c = codes.stride(1) == 1 ? codes : codes.contiguous();
  const int64_t K = c.size(0), N = c.size(1);
  TORCH_CHECK(N % 16 == 0, "GRINQH pack_codes: N must be divisible by 16 for this layout");
  const c10::cuda::CUDAGuard guard(c.device());
  at::Tensor out = at::empty({K, (max_bits / 2) * (N / 16)}, c.options().dtype(at::kUInt32));
  check_ok(grinqh_pack_codes(c.data_ptr<int8_t>(), c.stride(0), reinterpret_cast<uint32_t*>(out.data_ptr()), K, N,
                             (int)max_bits, cur_stream(c)),
           "pack_codes");
  return out;
}

// checkpoint -> staging codes (grinqh/grinqh.py:154-168): src is the shard's
// compressed-tensors int32 weight [rows_total, words] (or int8 codes for b = 6);
// writes dst[:, n_off : n_off + rows] (int8 [K_local, N_local], any row stride) with
// the codes of source rows [row0, row0 + rows) and columns [k0, k0 + dst.size(0))
void unpack_checkpoint(const at::Tensor& src, int64_t max_bits, int64_t row0, int64_t rows, int64_t k0,
                       const at::Tensor& dst, int64_t n_off) {
  check_cuda(src, "src");
  check_cuda(dst, "dst");
  TORCH_CHECK(src.dim() == 2 && dst.dim() == 2, "GRINQH unpack_checkpoint: expects 2-D tensors");
  TORCH_CHECK(max_bits == 6 ? src.scalar_type() == at::kChar : src.scalar_type() == at::kInt,
              "GRINQH unpack_checkpoint: src must be int32 (int8 for max_bits 6)");
  TORCH_CHECK(dst.scalar_type() == at::kChar && dst.stride(1) == 1, "GRINQH unpack_checkpoint: dst must be int8 with unit column stride");
  TORCH_CHECK(src.device() == dst.device(), "GRINQH unpack_checkpoint: src and dst on different devices");
  TORCH_CHECK(row0 >= 0 && rows >= 0 && row0 + rows <= src.size(0), "GRINQH unpack_checkpoint: row range out of bounds");
  TORCH_CHECK(n_off >= 0 && n_off + rows <= dst.size(1), "GRINQH unpack_checkpoint: column range out of bounds");
  const at::Tensor s = src.contiguous();
  const c10::cuda::CUDAGuard guard(s.device());
  check_ok(grinqh_unpack_checkpoint(s.data_ptr(), s.size(1), (int)max_bits, row0, rows, k0, dst.size(0),
                                    dst.data_ptr<int8_t>() + n_off, dst.stride(0), cur_stream(s)),
           "unpack_checkpoint");
}

// unpack (grinqh/utils.py:149-177): [K, (b/2)*N/16] -> [K, N] uint8 (shifted code >> (8-b))
at::Tensor unpack(const at::Tensor& packed, int64_t max_bits, int64_t original_n) {
  check_cuda(packed, "packed");
  TORCH_CHECK(is_word32(packed) && packed.dim() == 2, "GRINQH unpack: expects a 2-D uint32/int32 tensor");
  const at::Tensor p = packed.contiguous();
  const int64_t K = p.size(0), N = original_n * 4;
  TORCH_CHECK(p.size(1) >= (max_bits / 2) * (N / 16), "GRINQH unpack: packed tensor too narrow");
  TORCH_CHECK(p.size(1) == (max_bits / 2) * (N / 16), "GRINQH unpack: packed width does not match max_bits/original_n");
  const c10::cuda::CUDAGuard guard(p.device());
  at::Tensor out = at::empty({K, N}, p.options().dtype(at::kByte));
  check_ok(grinqh_unpack(reinterpret_cast<const uint32_t*>(p.data_ptr()), out.data_ptr<uint8_t>(), K, N, (int)max_bits,
                         cur_stream(p)),
           "unpack");
  return out;
}

// grade (grinqh/kernel.py:100-116): per-element zone masks and their union over rows
std::tuple<at::Tensor, at::Tensor> grade(const at::Tensor& x, at::ArrayRef<double> thresholds, int64_t max_bits) {
  check_cuda(x, "x");
  const int dt = dtype_code(x, "x");
  const at::Tensor xf = x.reshape({-1, x.size(-1)}).contiguous();
  const int64_t M = xf.size(0), K = xf.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor masks = at::empty({M, K}, x.options().dtype(at::kByte));
  at::Tensor uni = at::empty({K}, x.options().dtype(at::kByte));
  const auto th = thresholds4(thresholds);
  check_ok(grinqh_grade(xf.data_ptr(), dt, M, K, th.data(), (int)max_bits, masks.data_ptr<uint8_t>(),
                        uni.data_ptr<uint8_t>(), cur_stream(x)),
           "grade");
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  return {masks.view(shape), uni};
}

}  // namespace

TORCH_LIBRARY(grinqh, m) {
  m.def("gemm_or_gemv(Tensor x, Tensor weight_packed, Tensor weight_scale, Tensor? bias, int max_bits, "
        "int group_size, int original_n, float[] thresholds, bool use_marlin=False) -> Tensor");
  m.def("linear(Tensor x, Tensor weight_packed, Tensor weight_scale, Tensor? bias, int max_bits, "
        "int group_size, int original_n, float[] thresholds, int mode) -> Tensor");
  m.def("pack(Tensor words, int max_bits) -> Tensor");
  m.def("pack_codes(Tensor codes, int max_bits) -> Tensor");
  m.def("unpack(Tensor packed, int max_bits, int original_n) -> Tensor");
  m.def("unpack_checkpoint(Tensor src, int max_bits, int row0, int rows, int k0, Tensor(a!) dst, int n_off) -> ()");
  m.def("gemv_allreduce(Tensor x, Tensor weight_packed, Tensor weight_scale, Tensor? bias, int max_bits, "
        "int group_size, int original_n, float[] thresholds, int rank, int world, int[] buffers, int n_cap) -> Tensor");
  m.def("linear_allreduce(Tensor x, Tensor weight_packed, Tensor weight_scale, Tensor? bias, int max_bits, "
        "int group_size, int original_n, float[] thresholds, int mode, int rank, int world, int[] buffers, "
        "int cap) -> Tensor");
  m.def("grade(Tensor x, float[] thresholds, int max_bits) -> (Tensor, Tensor)");
  m.def("rmsnorm_grade(Tensor x, Tensor(a!)? residual, Tensor? weight, float eps, float[] thresholds, "
        "int max_bits) -> (Tensor, Tensor, Tensor)");
  m.def("silu_mul_grade(Tensor x, float[] thresholds, int max_bits) -> (Tensor, Tensor, Tensor)");
  m.def("union_linear_masked(Tensor x, Tensor weight_packed, Tensor weight_scale, Tensor? bias, int max_bits, "
        "int group_size, int original_n, float[] thresholds, Tensor union_mask) -> Tensor");
}

TORCH_LIBRARY_IMPL(grinqh, CUDA, m) {
  m.impl("gemm_or_gemv", &gemm_or_gemv);
  m.impl("linear", &linear);
  m.impl("pack", &pack);
  m.impl("pack_codes", &pack_codes);
  m.impl("unpack", &unpack);
  m.impl("unpack_checkpoint", &unpack_checkpoint);
  m.impl("gemv_allreduce", &gemv_allreduce);
  m.impl("linear_allreduce", &linear_allreduce);
  m.impl("grade", &grade);
  m.impl("rmsnorm_grade", &rmsnorm_grade);
  m.impl("silu_mul_grade", &silu_mul_grade);
  m.impl("union_linear_masked", &union_linear_masked);
}
