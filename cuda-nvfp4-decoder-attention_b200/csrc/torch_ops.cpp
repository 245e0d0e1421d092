// PyTorch operator library over the C ABI (libnvfp4da.so).
//
// Registers the reference's nine schemas in its namespace
// (src/bindings.cpp:888-916) so that its Python loader, wrappers and tests bind
// to this library unchanged, plus the fused forward and the device quantizer.
// Structural checks raise RuntimeError with the reference's messages (its tests
// match on them); outputs are fresh contiguous tensors on the input's device;
// everything runs on the current CUDA stream with no host synchronisation.
#include <ATen/cuda/CUDAContext.h>
#include <ATen/ops/empty.h>
#include <ATen/ops/empty_like.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <cstdint>
#include <limits>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/nvfp4_decoder_attention.h"

namespace nvfp4da_ops {
namespace {

using at::Tensor;
constexpr int64_t kI64Max = std::numeric_limits<int64_t>::max();
constexpr int64_t kI32Max = std::numeric_limits<int32_t>::max();

void* cur_stream(const Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

void check_status(int status, const char* what) {
  TORCH_CHECK(status == NVFP4DA_OK, what, " failed: ", nvfp4da_last_error());
}

const char* dtype_name(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return "torch.bfloat16";
    case at::kByte: return "torch.uint8";
    case at::kFloat: return "torch.float32";
    default: return "?";
  }
}

// Common structural requirement: CUDA, dtype, contiguous.
void expect(const Tensor& t, const char* name, at::ScalarType dtype) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dtype, name, " must have dtype ", dtype_name(dtype));
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void expect_same_device(const Tensor& t, const char* name, const Tensor& ref, const char* ref_name) {
  TORCH_CHECK(t.device() == ref.device(), name, " must be on the same CUDA device as ", ref_name);
}

// packed_values: CUDA uint8 rank-2 contiguous, nonempty (bindings.cpp:25-56).
void expect_packed(const Tensor& packed) {
  expect(packed, "packed_values", at::kByte);
  TORCH_CHECK(packed.dim() == 2, "packed_values must have rank 2, got rank ", packed.dim());
  TORCH_CHECK(packed.size(0) > 0 && packed.size(1) > 0,
              "packed_values must have nonempty N and packed-byte dimensions");
  TORCH_CHECK(packed.size(1) <= kI64Max / 2, "packed_values byte dimension is too large to derive logical K");
  TORCH_CHECK(packed.numel() <= kI64Max / 2, "packed_values has too many bytes to allocate the unpacked output");
  TORCH_CHECK((packed.numel() - 1) / 256 + 1 <= kI32Max,
              "packed_values is too large for a one-dimensional CUDA grid");
}

// block_scales + global_decode_scale against packed_values of logical [N, K].
void expect_scales(const Tensor& packed, const Tensor& scales, const Tensor& gamma, const Tensor& device_ref,
                   const char* device_ref_name) {
  expect(scales, "block_scales", at::kByte);
  TORCH_CHECK(scales.dim() == 2, "block_scales must have rank 2, got rank ", scales.dim());
  expect(gamma, "global_decode_scale", at::kFloat);
  TORCH_CHECK(gamma.dim() == 0, "global_decode_scale must be a scalar tensor with shape []");
  expect_same_device(scales, "block_scales", device_ref, device_ref_name);
  expect_same_device(gamma, "global_decode_scale", device_ref, device_ref_name);
  const int64_t n = packed.size(0), k = packed.size(1) * 2;
  TORCH_CHECK(k >= 16, "logical K must be at least 16, got ", k);
  TORCH_CHECK(k % 16 == 0, "logical K must be divisible by 16, got ", k);
  TORCH_CHECK(scales.size(0) == n, "block_scales row count must match packed_values (", scales.size(0), " != ", n,
              ")");
  TORCH_CHECK(scales.size(1) == k / 16, "block_scales must have shape [N, K/16]; expected [", n, ", ", k / 16,
              "], got [", scales.size(0), ", ", scales.size(1), "]");
}

nvfp4da_weight as_weight(const Tensor& packed, const Tensor& scales, const Tensor& gamma) {
  nvfp4da_weight w;
  w.packed_values = packed.data_ptr<uint8_t>();
  w.block_scales = scales.data_ptr<uint8_t>();
  w.global_decode_scale = gamma.data_ptr<float>();
  w.rows = packed.size(0);
  w.cols = packed.size(1) * 2;
  return w;
}

const uint16_t* bits(const Tensor& t) { return reinterpret_cast<const uint16_t*>(t.data_ptr()); }
uint16_t* mbits(const Tensor& t) { return reinterpret_cast<uint16_t*>(t.data_ptr()); }

Tensor workspace(const Tensor& like, size_t bytes) {
  return at::empty({static_cast<int64_t>(bytes > 0 ? bytes : 1)}, like.options().dtype(at::kByte));
}

void expect_rank4(const Tensor& t, const char* name) {
  expect(t, name, at::kBFloat16);
  TORCH_CHECK(t.dim() == 4, name, " must have rank 4, got rank ", t.dim());
  TORCH_CHECK(t.size(0) > 0 && t.size(1) > 0 && t.size(2) > 0 && t.size(3) > 0, name,
              " dimensions must all be positive");
}

// ---------------------------------------------------------------- ops
Tensor unpack_e2m1_codes(const Tensor& packed) {
  expect_packed(packed);
  const c10::cuda::CUDAGuard g(packed.device());
  Tensor out = at::empty({packed.size(0), packed.size(1) * 2}, packed.options());
  check_status(nvfp4da_unpack_e2m1_codes(packed.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), packed.size(0),
                                         packed.size(1), cur_stream(packed)),
               "cuda_unpack_e2m1_codes");
  return out;
}

Tensor dequantize_nvfp4(const Tensor& packed, const Tensor& scales, const Tensor& gamma) {
  expect_packed(packed);
  expect_scales(packed, scales, gamma, packed, "packed_values");
  const c10::cuda::CUDAGuard g(packed.device());
  Tensor out = at::empty({packed.size(0), packed.size(1) * 2}, packed.options().dtype(at::kFloat));
  const nvfp4da_weight w = as_weight(packed, scales, gamma);
  check_status(nvfp4da_dequantize_nvfp4(&w, out.data_ptr<float>(), cur_stream(packed)), "cuda_dequantize_nvfp4");
  return out;
}

Tensor w4a16_linear(const Tensor& x, const Tensor& packed, const Tensor& scales, const Tensor& gamma) {
  expect(x, "x", at::kBFloat16);
  TORCH_CHECK(x.dim() >= 1 && x.dim() <= 4, "x must have rank in [1, 4], got rank ", x.dim());
  TORCH_CHECK(x.numel() > 0, "x must be nonempty");
  expect_packed(packed);
  expect_same_device(packed, "packed_values", x, "x");
  expect_scales(packed, scales, gamma, x, "x");
  const int64_t n = packed.size(0), k = packed.size(1) * 2;
  TORCH_CHECK(x.size(-1) == k, "x final dimension must match logical weight K (", x.size(-1), " != ", k, ")");
  const int64_t m = x.numel() / k;
  TORCH_CHECK(m <= kI64Max / n, "M*N overflows int64");
  TORCH_CHECK(m * n <= kI32Max, "M*N is too large for a one-dimensional CUDA grid");
  std::vector<int64_t> sizes(x.sizes().begin(), x.sizes().end());
  sizes.back() = n;
  const c10::cuda::CUDAGuard g(x.device());
  Tensor y = at::empty(sizes, x.options());
  const nvfp4da_weight w = as_weight(packed, scales, gamma);
  check_status(nvfp4da_w4a16_linear(bits(x), m, &w, mbits(y), cur_stream(x)), "cuda_w4a16_linear");
  return y;
}

Tensor rms_norm(const Tensor& x, const Tensor& weight, double eps) {
  TORCH_CHECK(x.is_cuda(), "x must be a CUDA tensor");
  TORCH_CHECK(weight.is_cuda(), "weight must be a CUDA tensor");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must have dtype torch.bfloat16");
  TORCH_CHECK(weight.scalar_type() == at::kBFloat16, "weight must have dtype torch.bfloat16");
  TORCH_CHECK(x.device() == weight.device(), "x and weight must be on the same CUDA device");
  TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
  TORCH_CHECK(weight.is_contiguous(), "weight must be contiguous");
  TORCH_CHECK(x.dim() >= 1 && x.dim() <= 4, "x must have rank in [1, 4], got rank ", x.dim());
  TORCH_CHECK(weight.dim() == 1, "weight must be rank 1");
  TORCH_CHECK(x.numel() > 0, "x must be nonempty");
  TORCH_CHECK(weight.numel() > 0, "weight must be nonempty");
  TORCH_CHECK(weight.numel() == x.size(-1), "weight length must match x final dimension (", weight.numel(), " != ",
              x.size(-1), ")");
  TORCH_CHECK(std::isfinite(eps) && eps > 0.0, "eps must be finite and positive");
  const float eps32 = static_cast<float>(eps);
  TORCH_CHECK(std::isfinite(eps32) && eps32 > 0.0f, "eps must be representable as a finite positive FP32 value");
  const int64_t rows = x.numel() / x.size(-1);
  TORCH_CHECK(rows <= kI32Max, "x has too many logical rows for a one-dimensional CUDA grid");
  const c10::cuda::CUDAGuard g(x.device());
  Tensor out = at::empty_like(x);
  check_status(nvfp4da_rms_norm(bits(x), bits(weight), mbits(out), rows, x.size(-1), eps32, cur_stream(x)),
               "cuda_rms_norm");
  return out;
}

Tensor apply_rope(const Tensor& x, int64_t past_length, double theta) {
  expect(x, "x", at::kBFloat16);
  TORCH_CHECK(x.dim() == 4, "x must have rank 4, got rank ", x.dim());
  TORCH_CHECK(x.size(0) > 0 && x.size(1) > 0 && x.size(2) > 0 && x.size(3) > 0, "x dimensions must all be nonempty");
  const int64_t tokens = x.size(1), d = x.size(3);
  TORCH_CHECK(d >= 2, "x head dimension must be at least 2");
  TORCH_CHECK(d % 2 == 0, "x head dimension must be even for adjacent-pair RoPE");
  TORCH_CHECK(past_length >= 0, "past_length must be nonnegative");
  TORCH_CHECK(past_length <= kI64Max - (tokens - 1), "past_length plus token index must fit in int64");
  TORCH_CHECK(std::isfinite(theta) && theta > 0.0, "rope_theta must be finite and positive");
  const float theta32 = static_cast<float>(theta);
  TORCH_CHECK(std::isfinite(theta32) && theta32 > 0.0f,
              "rope_theta must be representable as a finite positive FP32 value");
  TORCH_CHECK((x.numel() / 2 - 1) / 256 + 1 <= kI32Max,
              "x has too many logical adjacent pairs for a one-dimensional CUDA grid");
  const c10::cuda::CUDAGuard g(x.device());
  Tensor out = at::empty_like(x);
  check_status(nvfp4da_apply_rope(bits(x), mbits(out), x.size(0), tokens, x.size(2), d, past_length, theta32,
                                  cur_stream(x)),
               "cuda_apply_rope");
  return out;
}

// Shared by the compact and the capacity-backed attention (bindings.cpp:534-782).
Tensor gqa_common(const Tensor& q, const Tensor& kc, const Tensor& vc, int64_t past_length, bool compact,
                  const char* kname, const char* vname) {
  expect_rank4(q, "q");
  expect_rank4(kc, kname);
  expect_rank4(vc, vname);
  TORCH_CHECK(vc.sizes() == kc.sizes(), vname, " must have the same shape as ", kname, "; got ", vc.sizes(), " and ",
              kc.sizes());
  TORCH_CHECK(kc.device() == q.device(), kname, " must be on the same CUDA device as q");
  TORCH_CHECK(vc.device() == q.device(), vname, " must be on the same CUDA device as q");
  const int64_t b = q.size(0), t = q.size(1), hq = q.size(2), d = q.size(3);
  const int64_t hkv = kc.size(1), c = kc.size(2);
  TORCH_CHECK(b == kc.size(0), "q and cache batch sizes must match (", b, " != ", kc.size(0), ")");
  TORCH_CHECK(d == kc.size(3), "q and cache head dimensions must match (", d, " != ", kc.size(3), ")");
  TORCH_CHECK(hq % hkv == 0, "number of query heads must be divisible by number of KV heads (", hq, " % ", hkv,
              " != 0)");
  TORCH_CHECK(past_length >= 0, "past_length must be nonnegative");
  TORCH_CHECK(past_length <= kI64Max - t, "past_length + current token count overflows int64");
  if (compact) {
    TORCH_CHECK(c == past_length + t, "cache context length must equal past_length + current token count (", c,
                " != ", past_length, " + ", t, ")");
  } else {
    TORCH_CHECK(past_length + t <= c, "past_length + current token count exceeds cache capacity (", past_length + t,
                " > ", c, ")");
  }
  TORCH_CHECK(d <= 256, "head dimension must be at most 256 (", d, ")");
  const c10::cuda::CUDAGuard g(q.device());
  Tensor ctx = at::empty({b, t, hq, d}, q.options());
  const size_t wsb = nvfp4da_gqa_attention_workspace_size(b, t, hq, hkv, d, past_length);
  Tensor ws = workspace(q, wsb);
  check_status(nvfp4da_gqa_attention_cached(bits(q), bits(kc), bits(vc), mbits(ctx), b, t, hq, hkv, c, d,
                                            past_length, nullptr, past_length, ws.data_ptr(), wsb, cur_stream(q)),
               "cuda_gqa_attention_cached");
  return ctx;
}

Tensor gqa_attention(const Tensor& q, const Tensor& k, const Tensor& v, int64_t past_length) {
  return gqa_common(q, k, v, past_length, true, "present_k", "present_v");
}

Tensor gqa_attention_cached(const Tensor& q, const Tensor& k, const Tensor& v, int64_t past_length) {
  return gqa_common(q, k, v, past_length, false, "k_cache", "v_cache");
}

void kv_cache_append_(Tensor& kc, Tensor& vc, const Tensor& nk, const Tensor& nv, int64_t past_length) {
  expect_rank4(kc, "k_cache");
  expect_rank4(vc, "v_cache");
  expect_rank4(nk, "new_k");
  expect_rank4(nv, "new_v");
  TORCH_CHECK(vc.sizes() == kc.sizes(), "v_cache must have the same shape as k_cache; got ", vc.sizes(), " and ",
              kc.sizes());
  TORCH_CHECK(nv.sizes() == nk.sizes(), "new_v must have the same shape as new_k; got ", nv.sizes(), " and ",
              nk.sizes());
  TORCH_CHECK(vc.device() == kc.device(), "v_cache must be on the same CUDA device as k_cache");
  TORCH_CHECK(nk.device() == kc.device(), "new_k must be on the same CUDA device as k_cache");
  TORCH_CHECK(nv.device() == kc.device(), "new_v must be on the same CUDA device as k_cache");
  const int64_t b = kc.size(0), hkv = kc.size(1), c = kc.size(2), d = kc.size(3), t = nk.size(1);
  TORCH_CHECK(nk.size(0) == b, "new K/V batch size must match cache batch size (", nk.size(0), " != ", b, ")");
  TORCH_CHECK(nk.size(2) == hkv, "new K/V head count must match cache KV head count (", nk.size(2), " != ", hkv,
              ")");
  TORCH_CHECK(nk.size(3) == d, "new K/V head dimension must match cache head dimension (", nk.size(3), " != ", d,
              ")");
  TORCH_CHECK(past_length >= 0, "past_length must be nonnegative");
  TORCH_CHECK(past_length <= kI64Max - t, "past_length + current token count overflows int64");
  TORCH_CHECK(past_length + t <= c, "past_length + current token count exceeds cache capacity (", past_length + t,
              " > ", c, ")");
  const c10::cuda::CUDAGuard g(kc.device());
  check_status(nvfp4da_kv_cache_append(mbits(kc), mbits(vc), bits(nk), bits(nv), b, hkv, c, d, t, past_length,
                                       nullptr, cur_stream(kc)),
               "cuda_kv_cache_append_");
}

// ---------------------------------------------------------------- fused forward
struct ForwardTensors {
  Tensor x, g_in, qp, qs, qg, kp, ks, kg, vp, vs, vg, g_q, g_k, op, os, og, kc, vc;
};

nvfp4da_forward_args forward_args(const ForwardTensors& f, Tensor& out, int64_t past_length,
                                  const Tensor* past_lengths, int64_t max_past, double eps, double theta) {
  nvfp4da_forward_args a{};
  a.x = bits(f.x);
  a.input_norm_weight = bits(f.g_in);
  a.q_weight = as_weight(f.qp, f.qs, f.qg);
  a.k_weight = as_weight(f.kp, f.ks, f.kg);
  a.v_weight = as_weight(f.vp, f.vs, f.vg);
  a.out_weight = as_weight(f.op, f.os, f.og);
  a.q_norm_weight = bits(f.g_q);
  a.k_norm_weight = bits(f.g_k);
  a.k_cache = mbits(f.kc);
  a.v_cache = mbits(f.vc);
  a.output = mbits(out);
  a.batch = f.x.size(0);
  a.tokens = f.x.size(1);
  a.hidden = f.x.size(2);
  a.kv_heads = f.kc.size(1);
  a.head_dim = f.kc.size(3);
  a.capacity = f.kc.size(2);
  a.past_length = past_length;
  a.past_lengths = past_lengths ? past_lengths->data_ptr<int64_t>() : nullptr;
  a.max_past_length = max_past;
  a.rms_eps = static_cast<float>(eps);
  a.rope_theta = static_cast<float>(theta);
  return a;
}

void expect_forward(const ForwardTensors& f) {
  expect(f.x, "x", at::kBFloat16);
  TORCH_CHECK(f.x.dim() == 3, "x must have rank 3, got rank ", f.x.dim());
  expect_rank4(f.kc, "k_cache");
  expect_rank4(f.vc, "v_cache");
  TORCH_CHECK(f.vc.sizes() == f.kc.sizes(), "v_cache must have the same shape as k_cache");
  for (const Tensor* t : {&f.g_in, &f.g_q, &f.g_k}) expect(*t, "norm weight", at::kBFloat16);
  TORCH_CHECK(f.g_in.dim() == 1 && f.g_in.size(0) == f.x.size(2), "input_norm_weight must have shape [H]");
  TORCH_CHECK(f.g_q.dim() == 1 && f.g_q.size(0) == f.kc.size(3), "q_norm_weight must have shape [D]");
  TORCH_CHECK(f.g_k.dim() == 1 && f.g_k.size(0) == f.kc.size(3), "k_norm_weight must have shape [D]");
  const Tensor* w[4][3] = {{&f.qp, &f.qs, &f.qg}, {&f.kp, &f.ks, &f.kg}, {&f.vp, &f.vs, &f.vg}, {&f.op, &f.os, &f.og}};
  for (auto& t : w) {
    expect_packed(*t[0]);
    expect_scales(*t[0], *t[1], *t[2], f.x, "x");
    expect_same_device(*t[0], "packed_values", f.x, "x");
  }
  for (const Tensor* t : {&f.g_in, &f.g_q, &f.g_k, &f.kc, &f.vc})
    TORCH_CHECK(t->device() == f.x.device(), "all forward tensors must be on the same CUDA device as x");
}

Tensor run_forward(const ForwardTensors& f, int64_t past_length, const Tensor* past_lengths, int64_t max_past,
                   double eps, double theta) {
  expect_forward(f);
  const c10::cuda::CUDAGuard g(f.x.device());
  Tensor out = at::empty(f.x.sizes(), f.x.options());
  nvfp4da_forward_args a = forward_args(f, out, past_length, past_lengths, max_past, eps, theta);
  const size_t wsb = nvfp4da_forward_workspace_size(&a);
  TORCH_CHECK(wsb > 0, "cuda_decoder_attention_forward_ rejected its arguments: ", nvfp4da_last_error());
  Tensor ws = workspace(f.x, wsb);
  check_status(nvfp4da_decoder_attention_forward(&a, ws.data_ptr(), wsb, cur_stream(f.x)),
               "cuda_decoder_attention_forward_");
  return out;
}

Tensor forward_(const Tensor& x, const Tensor& g_in, const Tensor& qp, const Tensor& qs, const Tensor& qg,
                const Tensor& kp, const Tensor& ks, const Tensor& kg, const Tensor& vp, const Tensor& vs,
                const Tensor& vg, const Tensor& g_q, const Tensor& g_k, const Tensor& op, const Tensor& os,
                const Tensor& og, Tensor& kc, Tensor& vc, int64_t past_length, double eps, double theta) {
  ForwardTensors f{x, g_in, qp, qs, qg, kp, ks, kg, vp, vs, vg, g_q, g_k, op, os, og, kc, vc};
  return run_forward(f, past_length, nullptr, past_length, eps, theta);
}

Tensor forward_varlen_(const Tensor& x, const Tensor& g_in, const Tensor& qp, const Tensor& qs, const Tensor& qg,
                       const Tensor& kp, const Tensor& ks, const Tensor& kg, const Tensor& vp, const Tensor& vs,
                       const Tensor& vg, const Tensor& g_q, const Tensor& g_k, const Tensor& op, const Tensor& os,
                       const Tensor& og, Tensor& kc, Tensor& vc, const Tensor& past_lengths, int64_t max_past_length,
                       double eps, double theta) {
  expect(past_lengths, "past_lengths", at::kLong);
  TORCH_CHECK(past_lengths.dim() == 1 && past_lengths.size(0) == x.size(0),
              "past_lengths must have shape [B] matching x");
  TORCH_CHECK(past_lengths.device() == x.device(), "past_lengths must be on the same CUDA device as x");
  ForwardTensors f{x, g_in, qp, qs, qg, kp, ks, kg, vp, vs, vg, g_q, g_k, op, os, og, kc, vc};
  return run_forward(f, 0, &past_lengths, max_past_length, eps, theta);
}

std::tuple<Tensor, Tensor, Tensor> quantize_nvfp4(const Tensor& source) {
  TORCH_CHECK(source.is_cuda(), "source must be a CUDA tensor");
  TORCH_CHECK(source.scalar_type() == at::kFloat || source.scalar_type() == at::kBFloat16,
              "source must have dtype torch.float32 or torch.bfloat16");
  TORCH_CHECK(source.dim() == 2, "source must be rank 2, got rank ", source.dim());
  TORCH_CHECK(source.is_contiguous(), "source must be contiguous");
  const int64_t n = source.size(0), k = source.size(1);
  TORCH_CHECK(n >= 1, "source must have at least one row, got ", n);
  TORCH_CHECK(k >= 16 && k % 16 == 0, "source K dimension must be a positive multiple of 16, got ", k);
  const c10::cuda::CUDAGuard g(source.device());
  Tensor packed = at::empty({n, k / 2}, source.options().dtype(at::kByte));
  Tensor scales = at::empty({n, k / 16}, source.options().dtype(at::kByte));
  Tensor gamma = at::empty({}, source.options().dtype(at::kFloat));
  const size_t wsb = nvfp4da_quantize_workspace_size(n, k);
  Tensor ws = workspace(source, wsb);
  check_status(nvfp4da_quantize_nvfp4(source.data_ptr(), source.scalar_type() == at::kBFloat16 ? 1 : 0, n, k,
                                      packed.data_ptr<uint8_t>(), scales.data_ptr<uint8_t>(), gamma.data_ptr<float>(),
                                      ws.data_ptr(), wsb, cur_stream(source)),
               "cuda_quantize_nvfp4");
  return {packed, scales, gamma};
}

}  // namespace
}  // namespace nvfp4da_ops

TORCH_LIBRARY(cuda_nvfp4_decoder_attention, m) {
  using namespace nvfp4da_ops;
  // The reference's nine schemas (src/bindings.cpp:888-916), unchanged.
  m.def("cuda_unpack_e2m1_codes(Tensor packed_values) -> Tensor", TORCH_FN(unpack_e2m1_codes));
  m.def("cuda_dequantize_nvfp4(Tensor packed_values, Tensor block_scales, Tensor global_decode_scale) -> Tensor",
        TORCH_FN(dequantize_nvfp4));
  m.def("cuda_rms_norm(Tensor x, Tensor weight, float eps) -> Tensor", TORCH_FN(rms_norm));
  m.def("cuda_apply_rope(Tensor x, int past_length, float rope_theta=10000.0) -> Tensor", TORCH_FN(apply_rope));
  m.def("cuda_w4a16_linear(Tensor x, Tensor packed_values, Tensor block_scales, Tensor global_decode_scale) -> Tensor",
        TORCH_FN(w4a16_linear));
  m.def(
      "cuda_w4a16_linear_grouped_decode(Tensor x, Tensor packed_values, Tensor block_scales, Tensor "
      "global_decode_scale) -> Tensor",
      TORCH_FN(w4a16_linear));
  m.def("cuda_gqa_attention(Tensor q, Tensor present_k, Tensor present_v, int past_length) -> Tensor",
        TORCH_FN(gqa_attention));
  m.def("cuda_gqa_attention_cached(Tensor q, Tensor k_cache, Tensor v_cache, int past_length) -> Tensor",
        TORCH_FN(gqa_attention_cached));
  m.def(
      "cuda_kv_cache_append_(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor new_k, Tensor new_v, int past_length) -> "
      "()",
      TORCH_FN(kv_cache_append_));
  // Additions: the fused forward (scalar and per-sequence past lengths) and the
  // device quantizer.
  m.def(
      "cuda_decoder_attention_forward_(Tensor x, Tensor input_norm_weight, Tensor q_packed, Tensor q_scales, Tensor "
      "q_gamma, Tensor k_packed, Tensor k_scales, Tensor k_gamma, Tensor v_packed, Tensor v_scales, Tensor v_gamma, "
      "Tensor q_norm_weight, Tensor k_norm_weight, Tensor o_packed, Tensor o_scales, Tensor o_gamma, Tensor(a!) "
      "k_cache, Tensor(b!) v_cache, int past_length, float rms_eps=1e-06, float rope_theta=10000.0) -> Tensor",
      TORCH_FN(forward_));
  m.def(
      "cuda_decoder_attention_forward_varlen_(Tensor x, Tensor input_norm_weight, Tensor q_packed, Tensor q_scales, "
      "Tensor q_gamma, Tensor k_packed, Tensor k_scales, Tensor k_gamma, Tensor v_packed, Tensor v_scales, Tensor "
      "v_gamma, Tensor q_norm_weight, Tensor k_norm_weight, Tensor o_packed, Tensor o_scales, Tensor o_gamma, "
      "Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor past_lengths, int max_past_length, float rms_eps=1e-06, float "
      "rope_theta=10000.0) -> Tensor",
      TORCH_FN(forward_varlen_));
  m.def("cuda_quantize_nvfp4(Tensor source) -> (Tensor, Tensor, Tensor)", TORCH_FN(quantize_nvfp4));
}
