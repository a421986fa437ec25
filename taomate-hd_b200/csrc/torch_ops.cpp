// torch custom operators over the C ABI of libtaomate_w8a8.so.
//
// Registers torch.ops.taomate_w8a8.* with the argument order of the vLLM
// out-variant operators the reference calls through torch.ops._C
// (src/taomate_hd/inference/w8a8.py:22-35, :71-72).  Only a CUDA kernel is
// registered: CPU tensors raise (no CPU fallback).  Every op validates
// dtype/device/layout with TORCH_CHECK (RuntimeError in Python), launches on
// the current CUDA stream.  The only allocation is the split-K workspace of
// cutlass_scaled_mm / scaled_mm_i8_ex (cached per device and stream, from
// torch's caching allocator) for shapes that use split-K.
#include <ATen/cuda/CUDAContext.h>
#include <ATen/ops/zeros.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/taomate_w8a8.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return TM_DTYPE_BF16;
    case at::kHalf: return TM_DTYPE_FP16;
    case at::kFloat: return TM_DTYPE_FP32;
    default: return -1;
  }
}

void check_status(int status, const char* op) {
  TORCH_CHECK(status == TM_OK, "taomate_w8a8.", op, " failed: ", tm_status_string(status),
              " (status ", status, ")");
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check_cuda(const at::Tensor& t, const at::Tensor& ref, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == ref.device(), name, " must be on ", ref.device());
}

// Treat `input` as [rows, cols] with unit inner stride and a row stride.
void as_rows(const at::Tensor& input, int64_t* rows, int64_t* cols, int64_t* ld) {
  TORCH_CHECK(input.dim() >= 1, "input must have at least one dimension");
  *cols = input.size(-1);
  if (input.dim() == 2 && input.stride(1) == 1) {
    *rows = input.size(0);
    *ld = input.size(0) > 1 ? input.stride(0) : *cols;
    return;
  }
  TORCH_CHECK(input.is_contiguous(), "input must be contiguous");
  *rows = *cols == 0 ? 0 : input.numel() / *cols;
  *ld = *cols;
}

void dynamic_scaled_int8_quant(at::Tensor& out, const at::Tensor& input, at::Tensor& scales,
                               const std::optional<at::Tensor>& azp) {
  check_cuda(input, input, "input");
  check_cuda(out, input, "result");
  check_cuda(scales, input, "scale");
  TORCH_CHECK(!azp.has_value(), "asymmetric int8 quantisation (azp) is not supported");
  const int dt = dtype_code(input);
  TORCH_CHECK(dt >= 0, "input dtype must be bfloat16, float16 or float32");
  TORCH_CHECK(out.scalar_type() == at::kChar && out.is_contiguous(), "result must be contiguous int8");
  TORCH_CHECK(out.numel() == input.numel(), "result must have the shape of input");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.is_contiguous(),
              "scale must be contiguous float32");
  int64_t rows, cols, ld;
  as_rows(input, &rows, &cols, &ld);
  TORCH_CHECK(scales.numel() == rows, "scale must hold one value per token");
  const c10::cuda::CUDAGuard guard(input.device());
  check_status(tm_dynamic_scaled_int8_quant(out.data_ptr<int8_t>(), input.data_ptr(), dt,
                                            scales.data_ptr<float>(), nullptr, rows, cols, ld,
                                            stream_of(input)),
               "dynamic_scaled_int8_quant");
}

void static_scaled_int8_quant(at::Tensor& out, const at::Tensor& input, const at::Tensor& scale,
                              const std::optional<at::Tensor>& azp) {
  check_cuda(input, input, "input");
  check_cuda(out, input, "result");
  check_cuda(scale, input, "scale");
  TORCH_CHECK(!azp.has_value(), "asymmetric int8 quantisation (azp) is not supported");
  const int dt = dtype_code(input);
  TORCH_CHECK(dt >= 0, "input dtype must be bfloat16, float16 or float32");
  TORCH_CHECK(out.scalar_type() == at::kChar && out.is_contiguous(), "result must be contiguous int8");
  TORCH_CHECK(out.numel() == input.numel(), "result must have the shape of input");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() == 1,
              "static scale must be one float32 value");
  int64_t rows, cols, ld;
  as_rows(input, &rows, &cols, &ld);
  const c10::cuda::CUDAGuard guard(input.device());
  check_status(tm_static_scaled_int8_quant(out.data_ptr<int8_t>(), input.data_ptr(), dt,
                                           scale.data_ptr<float>(), nullptr, rows, cols, ld,
                                           stream_of(input)),
               "static_scaled_int8_quant");
}

// Split-K workspace per (device, stream): zeroed when allocated, grown on
// demand, reused by every call on that stream (calls on one stream never
// overlap).  The kernels leave its counters at zero after each call.
at::Tensor splitk_workspace(const at::Tensor& like, uint64_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, at::Tensor> cache;
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream(like.device().index()).stream();
  const std::pair<int, cudaStream_t> key{like.device().index(), stream};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it == cache.end() || static_cast<uint64_t>(it->second.numel()) < bytes) {
    at::Tensor ws = at::zeros({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
    cache[key] = ws;
    return ws;
  }
  return it->second;
}

void scaled_mm_common(at::Tensor& out, const at::Tensor& a, const at::Tensor& b,
                      const at::Tensor& a_scales, const at::Tensor& b_scales,
                      const std::optional<at::Tensor>& bias, int64_t epilogue,
                      const std::optional<at::Tensor>& acc_debug, int64_t tile_n,
                      const char* op) {
  check_cuda(a, a, "a");
  check_cuda(b, a, "b");
  check_cuda(out, a, "out");
  check_cuda(a_scales, a, "a_scales");
  check_cuda(b_scales, a, "b_scales");
  TORCH_CHECK(a.scalar_type() == at::kChar && b.scalar_type() == at::kChar,
              "a and b must be int8");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "a, b and out must be 2-D");
  const int64_t m = a.size(0), k = a.size(1), n = b.size(1);
  TORCH_CHECK(b.size(0) == k, "a and b inner dimensions differ: ", k, " vs ", b.size(0));
  // SwiGLU: n interleaved (gate, up) columns in, n / 2 out
  const int64_t out_n = (epilogue & TM_EPI_SWIGLU) ? n / 2 : n;
  TORCH_CHECK(out.size(0) == m && out.size(1) == out_n, "out must be [", m, ", ", out_n, "]");
  TORCH_CHECK(a.stride(1) == 1, "a must be row-major");
  TORCH_CHECK(b.stride(0) == 1, "b must be column-major (pass weight.t())");
  TORCH_CHECK(out.stride(1) == 1, "out must be row-major");
  const int out_dt = dtype_code(out);
  TORCH_CHECK(out_dt == TM_DTYPE_BF16 || out_dt == TM_DTYPE_FP16, "out must be bfloat16 or float16");
  TORCH_CHECK(a_scales.scalar_type() == at::kFloat && b_scales.scalar_type() == at::kFloat,
              "scales must be float32");
  TORCH_CHECK(a_scales.is_contiguous() && b_scales.is_contiguous(), "scales must be contiguous");
  TORCH_CHECK(a_scales.numel() == 1 || a_scales.numel() == m, "a_scales must be per-tensor or per-token");
  TORCH_CHECK(b_scales.numel() == 1 || b_scales.numel() == n, "b_scales must be per-tensor or per-channel");
  const void* bias_ptr = nullptr;
  if (bias.has_value()) {
    check_cuda(*bias, a, "bias");
    TORCH_CHECK(bias->scalar_type() == out.scalar_type(), "bias must have the output dtype");
    TORCH_CHECK(bias->numel() == n && bias->is_contiguous(), "bias must be contiguous [n]");
    bias_ptr = bias->data_ptr();
  }
  int32_t* acc_ptr = nullptr;
  if (acc_debug.has_value()) {
    check_cuda(*acc_debug, a, "acc_debug");
    TORCH_CHECK(acc_debug->scalar_type() == at::kInt && acc_debug->is_contiguous() &&
                    acc_debug->numel() == m * n,
                "acc_debug must be a contiguous int32 [m, n]");
    acc_ptr = acc_debug->data_ptr<int32_t>();
  }
  const int64_t lda = m > 1 ? a.stride(0) : k;
  const int64_t ldb = n > 1 ? b.stride(1) : k;
  const int64_t ldo = m > 1 ? out.stride(0) : out_n;
  const c10::cuda::CUDAGuard guard(a.device());
  int status;
  if (tile_n != 0) {
    status = tm_scaled_mm_i8_tile(out.data_ptr(), out_dt, a.data_ptr<int8_t>(),
                                  b.data_ptr<int8_t>(), a_scales.data_ptr<float>(),
                                  a_scales.numel(), b_scales.data_ptr<float>(), b_scales.numel(),
                                  bias_ptr, m, n, k, lda, ldb, ldo,
                                  static_cast<uint32_t>(epilogue), acc_ptr,
                                  static_cast<int>(tile_n), stream_of(a));
  } else {
    uint64_t ws_bytes = 0;
    status = m > 0 ? tm_scaled_mm_i8_workspace_size(m, n, k, &ws_bytes) : TM_OK;
    if (status == TM_OK && ws_bytes > 0) {
      at::Tensor ws = splitk_workspace(a, ws_bytes);
      status = tm_scaled_mm_i8_ws(out.data_ptr(), out_dt, a.data_ptr<int8_t>(),
                                  b.data_ptr<int8_t>(), a_scales.data_ptr<float>(),
                                  a_scales.numel(), b_scales.data_ptr<float>(), b_scales.numel(),
                                  bias_ptr, m, n, k, lda, ldb, ldo,
                                  static_cast<uint32_t>(epilogue), acc_ptr, ws.data_ptr(),
                                  static_cast<uint64_t>(ws.numel()), stream_of(a));
    } else if (status == TM_OK) {
      status = tm_scaled_mm_i8_ex(out.data_ptr(), out_dt, a.data_ptr<int8_t>(),
                                  b.data_ptr<int8_t>(), a_scales.data_ptr<float>(),
                                  a_scales.numel(), b_scales.data_ptr<float>(), b_scales.numel(),
                                  bias_ptr, m, n, k, lda, ldb, ldo,
                                  static_cast<uint32_t>(epilogue), acc_ptr, stream_of(a));
    }
  }
  check_status(status, op);
}

void cutlass_scaled_mm(at::Tensor& out, const at::Tensor& a, const at::Tensor& b,
                       const at::Tensor& a_scales, const at::Tensor& b_scales,
                       const std::optional<at::Tensor>& bias) {
  scaled_mm_common(out, a, b, a_scales, b_scales, bias, 0, std::nullopt, 0, "cutlass_scaled_mm");
}

void scaled_mm_i8_ex(at::Tensor& out, const at::Tensor& a, const at::Tensor& b,
                     const at::Tensor& a_scales, const at::Tensor& b_scales,
                     const std::optional<at::Tensor>& bias, int64_t epilogue,
                     const std::optional<at::Tensor>& acc_debug, int64_t tile_n) {
  scaled_mm_common(out, a, b, a_scales, b_scales, bias, epilogue, acc_debug, tile_n,
                   "scaled_mm_i8_ex");
}

// W8A8 GEMM with the BF16 LoRA delta added in the epilogue:
// out = epi(dequant(a b) (+bias) + lora_t lora_b^T); lora_t = x A^T [m, r],
// lora_b = scale * B [n, r], both bf16 with unit inner stride, r <= 64.
void scaled_mm_i8_lora(at::Tensor& out, const at::Tensor& a, const at::Tensor& b,
                       const at::Tensor& a_scales, const at::Tensor& b_scales,
                       const std::optional<at::Tensor>& bias, const at::Tensor& lora_t,
                       const at::Tensor& lora_b, int64_t epilogue) {
  check_cuda(a, a, "a");
  check_cuda(b, a, "b");
  check_cuda(out, a, "out");
  check_cuda(a_scales, a, "a_scales");
  check_cuda(b_scales, a, "b_scales");
  check_cuda(lora_t, a, "lora_t");
  check_cuda(lora_b, a, "lora_b");
  TORCH_CHECK(a.scalar_type() == at::kChar && b.scalar_type() == at::kChar,
              "a and b must be int8");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "a, b and out must be 2-D");
  const int64_t m = a.size(0), k = a.size(1), n = b.size(1);
  TORCH_CHECK(b.size(0) == k, "a and b inner dimensions differ: ", k, " vs ", b.size(0));
  TORCH_CHECK(out.size(0) == m && out.size(1) == n, "out must be [", m, ", ", n, "]");
  TORCH_CHECK(a.stride(1) == 1, "a must be row-major");
  TORCH_CHECK(b.stride(0) == 1, "b must be column-major (pass weight.t())");
  TORCH_CHECK(out.stride(1) == 1, "out must be row-major");
  const int out_dt = dtype_code(out);
  TORCH_CHECK(out_dt == TM_DTYPE_BF16 || out_dt == TM_DTYPE_FP16, "out must be bfloat16 or float16");
  TORCH_CHECK(a_scales.scalar_type() == at::kFloat && b_scales.scalar_type() == at::kFloat,
              "scales must be float32");
  TORCH_CHECK(a_scales.is_contiguous() && b_scales.is_contiguous(), "scales must be contiguous");
  TORCH_CHECK(a_scales.numel() == 1 || a_scales.numel() == m, "a_scales must be per-tensor or per-token");
  TORCH_CHECK(b_scales.numel() == 1 || b_scales.numel() == n, "b_scales must be per-tensor or per-channel");
  TORCH_CHECK(lora_t.scalar_type() == at::kBFloat16 && lora_b.scalar_type() == at::kBFloat16,
              "lora_t and lora_b must be bfloat16");
  TORCH_CHECK(lora_t.dim() == 2 && lora_b.dim() == 2 && lora_t.stride(1) == 1 &&
                  lora_b.stride(1) == 1,
              "lora_t and lora_b must be 2-D row-major");
  const int64_t r = lora_t.size(1);
  TORCH_CHECK(lora_t.size(0) == m && lora_b.size(0) == n && lora_b.size(1) == r,
              "lora_t must be [m, r] and lora_b [n, r]");
  const void* bias_ptr = nullptr;
  if (bias.has_value()) {
    check_cuda(*bias, a, "bias");
    TORCH_CHECK(bias->scalar_type() == out.scalar_type(), "bias must have the output dtype");
    TORCH_CHECK(bias->numel() == n && bias->is_contiguous(), "bias must be contiguous [n]");
    bias_ptr = bias->data_ptr();
  }
  const int64_t lda = m > 1 ? a.stride(0) : k;
  const int64_t ldb = n > 1 ? b.stride(1) : k;
  const int64_t ldo = m > 1 ? out.stride(0) : n;
  const int64_t ldt = m > 1 ? lora_t.stride(0) : r;
  const int64_t ldlb = n > 1 ? lora_b.stride(0) : r;
  const c10::cuda::CUDAGuard guard(a.device());
  check_status(tm_scaled_mm_i8_lora(out.data_ptr(), out_dt, a.data_ptr<int8_t>(),
                                    b.data_ptr<int8_t>(), a_scales.data_ptr<float>(),
                                    a_scales.numel(), b_scales.data_ptr<float>(),
                                    b_scales.numel(), bias_ptr, lora_t.data_ptr(), ldt,
                                    lora_b.data_ptr(), ldlb, static_cast<int>(r), m, n, k, lda,
                                    ldb, ldo, static_cast<uint32_t>(epilogue), stream_of(a)),
               "scaled_mm_i8_lora");
}

// LoRA down-projection t = x a^T (tm_lora_down_proj): x bf16 [m, k],
// a bf16 [r, k], t bf16 [m, r]; rows contiguous, any row strides.
void lora_down_proj(at::Tensor& t, const at::Tensor& x, const at::Tensor& a) {
  check_cuda(x, x, "x");
  check_cuda(a, x, "a");
  check_cuda(t, x, "t");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && a.scalar_type() == at::kBFloat16 &&
                  t.scalar_type() == at::kBFloat16,
              "x, a and t must be bfloat16");
  TORCH_CHECK(x.dim() == 2 && a.dim() == 2 && t.dim() == 2, "x, a and t must be 2-D");
  const int64_t m = x.size(0), k = x.size(1), r = a.size(0);
  TORCH_CHECK(a.size(1) == k, "x and a inner dimensions differ: ", k, " vs ", a.size(1));
  TORCH_CHECK(t.size(0) == m && t.size(1) == r, "t must be [", m, ", ", r, "]");
  TORCH_CHECK(x.stride(1) == 1 && a.stride(1) == 1 && t.stride(1) == 1,
              "x, a and t must be row-major");
  const int64_t ldx = m > 1 ? x.stride(0) : k;
  const int64_t lda = r > 1 ? a.stride(0) : k;
  const int64_t ldt = m > 1 ? t.stride(0) : r;
  const c10::cuda::CUDAGuard guard(x.device());
  check_status(tm_lora_down_proj(t.data_ptr(), ldt, x.data_ptr(), ldx, a.data_ptr(), lda,
                                 static_cast<int>(r), m, k, stream_of(x)),
               "lora_down_proj");
}

// Merged QKV projection into the Ulysses all-to-all send buffer
// send [world, 3, m, ceil(heads / world) * head_dim] (tm_scaled_mm_i8_ulysses_send;
// padded head slots are zeroed).
void scaled_mm_i8_ulysses_send(at::Tensor& send, const at::Tensor& a, const at::Tensor& b,
                               const at::Tensor& a_scales, const at::Tensor& b_scales,
                               const std::optional<at::Tensor>& bias, int64_t num_heads,
                               int64_t head_dim, int64_t world) {
  check_cuda(a, a, "a");
  check_cuda(b, a, "b");
  check_cuda(send, a, "send");
  check_cuda(a_scales, a, "a_scales");
  check_cuda(b_scales, a, "b_scales");
  TORCH_CHECK(a.scalar_type() == at::kChar && b.scalar_type() == at::kChar,
              "a and b must be int8");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "a and b must be 2-D");
  const int64_t m = a.size(0), k = a.size(1), n = b.size(1);
  TORCH_CHECK(b.size(0) == k, "a and b inner dimensions differ");
  TORCH_CHECK(world > 0 && num_heads > 0, "heads and the Ulysses degree must be positive");
  TORCH_CHECK(n == 3 * num_heads * head_dim, "b must have 3 x heads x head_dim columns");
  const int64_t local = (num_heads + world - 1) / world;
  TORCH_CHECK(send.is_contiguous() && send.numel() == world * 3 * m * local * head_dim,
              "send must be a contiguous [world, 3, m, ceil(heads / world) * head_dim] buffer");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(0) == 1, "a row-major, b column-major (weight.t())");
  const int out_dt = dtype_code(send);
  TORCH_CHECK(out_dt == TM_DTYPE_BF16 || out_dt == TM_DTYPE_FP16, "send must be bf16 or fp16");
  TORCH_CHECK(a_scales.scalar_type() == at::kFloat && b_scales.scalar_type() == at::kFloat &&
                  a_scales.is_contiguous() && b_scales.is_contiguous(),
              "scales must be contiguous float32");
  const void* bias_ptr = nullptr;
  if (bias.has_value()) {
    check_cuda(*bias, a, "bias");
    TORCH_CHECK(bias->scalar_type() == send.scalar_type() && bias->numel() == n &&
                    bias->is_contiguous(),
                "bias must be contiguous [n] in the output dtype");
    bias_ptr = bias->data_ptr();
  }
  const int64_t lda = m > 1 ? a.stride(0) : k;
  const int64_t ldb = n > 1 ? b.stride(1) : k;
  const c10::cuda::CUDAGuard guard(a.device());
  check_status(tm_scaled_mm_i8_ulysses_send(send.data_ptr(), out_dt, a.data_ptr<int8_t>(),
                                            b.data_ptr<int8_t>(), a_scales.data_ptr<float>(),
                                            a_scales.numel(), b_scales.data_ptr<float>(),
                                            b_scales.numel(), bias_ptr, m, n, k, lda, ldb,
                                            static_cast<int>(num_heads),
                                            static_cast<int>(head_dim), static_cast<int>(world),
                                            stream_of(a)),
               "scaled_mm_i8_ulysses_send");
}

void quantize_weight_int8(at::Tensor& q, at::Tensor& scales, const at::Tensor& w) {
  check_cuda(w, w, "weight");
  check_cuda(q, w, "q");
  check_cuda(scales, w, "scales");
  const int dt = dtype_code(w);
  TORCH_CHECK(dt >= 0, "weight dtype must be bfloat16, float16 or float32");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous(), "weight must be a contiguous 2-D tensor");
  TORCH_CHECK(q.scalar_type() == at::kChar && q.is_contiguous() && q.sizes() == w.sizes(),
              "q must be contiguous int8 with the weight's shape");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.is_contiguous() &&
                  scales.numel() == w.size(0),
              "scales must be contiguous float32 [n]");
  const c10::cuda::CUDAGuard guard(w.device());
  check_status(tm_quantize_weight_int8(q.data_ptr<int8_t>(), scales.data_ptr<float>(), w.data_ptr(),
                                       dt, w.size(0), w.size(1), stream_of(w)),
               "quantize_weight_int8");
}

struct ModulateArgs {
  int64_t rows, cols, table_stride;
  const int64_t* index;
  void* hidden;
};

ModulateArgs check_modulate(at::Tensor& out, at::Tensor& scales,
                            const std::optional<at::Tensor>& hidden_out, const at::Tensor& x,
                            const at::Tensor& shift, const at::Tensor& scale,
                            const std::optional<at::Tensor>& index) {
  check_cuda(x, x, "x");
  check_cuda(out, x, "out");
  check_cuda(scales, x, "scales");
  check_cuda(shift, x, "shift");
  check_cuda(scale, x, "scale");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x must be contiguous bfloat16");
  ModulateArgs r{};
  r.cols = x.size(-1);
  r.rows = r.cols == 0 ? 0 : x.numel() / r.cols;
  TORCH_CHECK(out.scalar_type() == at::kChar && out.is_contiguous() && out.numel() == x.numel(),
              "out must be contiguous int8 with x's shape");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.is_contiguous() &&
                  scales.numel() == r.rows,
              "scales must be contiguous float32 [rows]");
  TORCH_CHECK(shift.scalar_type() == at::kBFloat16 && scale.scalar_type() == at::kBFloat16,
              "shift/scale must be bfloat16");
  TORCH_CHECK(shift.dim() == 2 && scale.dim() == 2 && shift.sizes() == scale.sizes(),
              "shift/scale must be 2-D tables of equal shape");
  TORCH_CHECK(shift.stride(1) == 1 && scale.stride(1) == 1 && shift.stride(0) == scale.stride(0),
              "shift/scale must be row-major with equal row strides");
  TORCH_CHECK(shift.size(1) == r.cols, "shift/scale width must equal x's last dimension");
  r.table_stride = shift.stride(0);
  if (index.has_value()) {
    check_cuda(*index, x, "index");
    TORCH_CHECK(index->scalar_type() == at::kLong && index->is_contiguous() &&
                    index->numel() == r.rows,
                "index must be contiguous int64 [rows]");
    r.index = index->data_ptr<int64_t>();
  } else {
    TORCH_CHECK(shift.size(0) == r.rows, "without index, shift/scale need one row per token");
  }
  if (hidden_out.has_value()) {
    check_cuda(*hidden_out, x, "hidden_out");
    TORCH_CHECK(hidden_out->scalar_type() == at::kBFloat16 && hidden_out->is_contiguous() &&
                    hidden_out->numel() == x.numel(),
                "hidden_out must be contiguous bfloat16 with x's shape");
    r.hidden = hidden_out->data_ptr();
  }
  return r;
}

void modulate_int8_quant(at::Tensor& out, at::Tensor& scales,
                         const std::optional<at::Tensor>& hidden_out, const at::Tensor& x,
                         const at::Tensor& shift, const at::Tensor& scale,
                         const std::optional<at::Tensor>& index) {
  const ModulateArgs r = check_modulate(out, scales, hidden_out, x, shift, scale, index);
  const c10::cuda::CUDAGuard guard(x.device());
  check_status(tm_modulate_int8_quant(out.data_ptr<int8_t>(), scales.data_ptr<float>(), r.hidden,
                                      x.data_ptr(), shift.data_ptr(), scale.data_ptr(), r.index,
                                      r.table_stride, r.rows, r.cols, stream_of(x)),
               "modulate_int8_quant");
}

void rms_norm_modulate_int8_quant(at::Tensor& out, at::Tensor& scales,
                                  const std::optional<at::Tensor>& hidden_out,
                                  const at::Tensor& x, const at::Tensor& weight, double eps,
                                  const at::Tensor& shift, const at::Tensor& scale,
                                  const std::optional<at::Tensor>& index) {
  const ModulateArgs r = check_modulate(out, scales, hidden_out, x, shift, scale, index);
  check_cuda(weight, x, "weight");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16 && weight.is_contiguous() &&
                  weight.numel() == r.cols,
              "norm weight must be contiguous bfloat16 [cols]");
  const c10::cuda::CUDAGuard guard(x.device());
  check_status(tm_rms_norm_modulate_int8_quant(out.data_ptr<int8_t>(), scales.data_ptr<float>(),
                                               r.hidden, x.data_ptr(), weight.data_ptr(),
                                               static_cast<float>(eps), shift.data_ptr(),
                                               scale.data_ptr(), r.index, r.table_stride, r.rows,
                                               r.cols, stream_of(x)),
               "rms_norm_modulate_int8_quant");
}

void residual_gate_rms_norm_modulate_int8_quant(
    at::Tensor& out, at::Tensor& scales, at::Tensor& residual_out,
    const std::optional<at::Tensor>& hidden_out, const at::Tensor& residual,
    const at::Tensor& branch, const at::Tensor& gate, const at::Tensor& weight, double eps,
    const at::Tensor& shift, const at::Tensor& scale, const std::optional<at::Tensor>& index) {
  const ModulateArgs r = check_modulate(out, scales, hidden_out, residual, shift, scale, index);
  check_cuda(weight, residual, "weight");
  check_cuda(branch, residual, "branch");
  check_cuda(gate, residual, "gate");
  check_cuda(residual_out, residual, "residual_out");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16 && weight.is_contiguous() &&
                  weight.numel() == r.cols,
              "norm weight must be contiguous bfloat16 [cols]");
  TORCH_CHECK(branch.scalar_type() == at::kBFloat16 && branch.is_contiguous() &&
                  branch.sizes() == residual.sizes(),
              "branch must be contiguous bfloat16 with the residual's shape");
  TORCH_CHECK(residual_out.scalar_type() == at::kBFloat16 && residual_out.is_contiguous() &&
                  residual_out.numel() == residual.numel(),
              "residual_out must be contiguous bfloat16 with the residual's shape");
  TORCH_CHECK(gate.scalar_type() == at::kBFloat16 && gate.sizes() == shift.sizes() &&
                  gate.stride(1) == 1 && gate.stride(0) == shift.stride(0),
              "gate must be a bfloat16 table shaped and strided like shift/scale");
  const c10::cuda::CUDAGuard guard(residual.device());
  check_status(tm_residual_gate_rms_norm_modulate_int8_quant(
                   out.data_ptr<int8_t>(), scales.data_ptr<float>(), residual_out.data_ptr(),
                   r.hidden, residual.data_ptr(), branch.data_ptr(), gate.data_ptr(),
                   weight.data_ptr(), static_cast<float>(eps), shift.data_ptr(),
                   scale.data_ptr(), r.index, r.table_stride, r.rows, r.cols,
                   stream_of(residual)),
               "residual_gate_rms_norm_modulate_int8_quant");
}

}  // namespace

TORCH_LIBRARY(taomate_w8a8, m) {
  m.def("dynamic_scaled_int8_quant(Tensor(a!) result, Tensor input, Tensor(b!) scale, Tensor? azp) -> ()");
  m.def("static_scaled_int8_quant(Tensor(a!) result, Tensor input, Tensor scale, Tensor? azp) -> ()");
  m.def(
      "cutlass_scaled_mm(Tensor(a!) out, Tensor a, Tensor b, Tensor a_scales, Tensor b_scales, "
      "Tensor? bias) -> ()");
  m.def(
      "scaled_mm_i8_ex(Tensor(a!) out, Tensor a, Tensor b, Tensor a_scales, Tensor b_scales, "
      "Tensor? bias, int epilogue, Tensor(b!)? acc_debug, int tile_n) -> ()");
  m.def(
      "scaled_mm_i8_lora(Tensor(a!) out, Tensor a, Tensor b, Tensor a_scales, Tensor b_scales, "
      "Tensor? bias, Tensor lora_t, Tensor lora_b, int epilogue) -> ()");
  m.def(
      "scaled_mm_i8_ulysses_send(Tensor(a!) send, Tensor a, Tensor b, Tensor a_scales, "
      "Tensor b_scales, Tensor? bias, int num_heads, int head_dim, int world) -> ()");
  m.def("quantize_weight_int8(Tensor(a!) q, Tensor(b!) scales, Tensor w) -> ()");
  m.def("lora_down_proj(Tensor(a!) t, Tensor x, Tensor a) -> ()");
  m.def(
      "modulate_int8_quant(Tensor(a!) out, Tensor(b!) scales, Tensor(c!)? hidden_out, Tensor x, "
      "Tensor shift, Tensor scale, Tensor? index) -> ()");
  m.def(
      "rms_norm_modulate_int8_quant(Tensor(a!) out, Tensor(b!) scales, Tensor(c!)? hidden_out, "
      "Tensor x, Tensor weight, float eps, Tensor shift, Tensor scale, Tensor? index) -> ()");
  m.def(
      "residual_gate_rms_norm_modulate_int8_quant(Tensor(a!) out, Tensor(b!) scales, "
      "Tensor(c!) residual_out, Tensor(d!)? hidden_out, Tensor residual, Tensor branch, "
      "Tensor gate, Tensor weight, float eps, Tensor shift, Tensor scale, Tensor? index) -> ()");
}

TORCH_LIBRARY_IMPL(taomate_w8a8, CUDA, m) {
  m.impl("dynamic_scaled_int8_quant", &dynamic_scaled_int8_quant);
  m.impl("static_scaled_int8_quant", &static_scaled_int8_quant);
  m.impl("cutlass_scaled_mm", &cutlass_scaled_mm);
  m.impl("scaled_mm_i8_ex", &scaled_mm_i8_ex);
  m.impl("scaled_mm_i8_lora", &scaled_mm_i8_lora);
  m.impl("scaled_mm_i8_ulysses_send", &scaled_mm_i8_ulysses_send);
  m.impl("quantize_weight_int8", &quantize_weight_int8);
  m.impl("lora_down_proj", &lora_down_proj);
  m.impl("modulate_int8_quant", &modulate_int8_quant);
  m.impl("rms_norm_modulate_int8_quant", &rms_norm_modulate_int8_quant);
  m.impl("residual_gate_rms_norm_modulate_int8_quant",
         &residual_gate_rms_norm_modulate_int8_quant);
}
