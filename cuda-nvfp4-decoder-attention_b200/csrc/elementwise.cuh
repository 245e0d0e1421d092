// Standalone elementwise / row kernels behind the reference's modular ops:
// RMSNorm, adjacent-pair RoPE, KV-cache append, NVFP4 unpack / dequantize and
// the NVFP4 quantizer.  The fused decode step does not use these; they back
// the individual operators and the general-shape forward.
#pragma once

#include <float.h>
#include <math.h>

#include "common.cuh"

namespace nvfp4da {

// ------------------------------------------------------------------ RMSNorm
// reference/decoder_attention.py:117-140, src/rmsnorm.cu:34-87.
// One CTA per row; the sum of squares is accumulated exactly (FP64, every
// square of a BF16 value is exact in FP32) and rounded once to FP32.
constexpr int kNormThreads = 128;

__device__ __forceinline__ double block_sum_f64(double v, double* scratch /* [kNormThreads/32] */) {
  v = warp_sum_f64(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += scratch[w];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const uint16_t* x, const uint16_t* w,
                                                                uint16_t* out, int64_t cols, float eps) {
  __shared__ double scratch[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const uint16_t* xr = x + row * cols;
  double ss = 0.0;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = bf16_bits_to_f32(xr[c]);
    ss += static_cast<double>(v * v);
  }
  const float inv = rms_inverse(static_cast<float>(block_sum_f64(ss, scratch)), static_cast<float>(cols), eps);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = bf16_bits_to_f32(xr[c]);
    out[row * cols + c] = f32_to_bf16_bits(__fmul_rn(__fmul_rn(v, inv), bf16_bits_to_f32(w[c])));
  }
}

// ------------------------------------------------------------------ RoPE
// reference/decoder_attention.py:205-270, src/rope.cu:18-72.
// cos / sin of the FP32 angle p / theta^(2m/D) are evaluated in FP64 and
// rounded once to FP32 (the correctly rounded FP32 value); position 0 is an
// exact storage copy (keeps signed zeros).
__device__ __forceinline__ void rope_cos_sin(int64_t pos, int64_t pair, int64_t head_dim, float theta, float& c,
                                             float& s) {
  const float expo = __fdiv_rn(static_cast<float>(2 * pair), static_cast<float>(head_dim));
  const float denom = static_cast<float>(pow(static_cast<double>(theta), static_cast<double>(expo)));
  const float angle = __fdiv_rn(static_cast<float>(pos), denom);
  double sd, cd;
  sincos(static_cast<double>(angle), &sd, &cd);
  c = static_cast<float>(cd);
  s = static_cast<float>(sd);
}

// The same with theta^(2m/D) rounded to FP32 given (computed on the host with
// the arithmetic above): only the angle and its cos / sin on the device.
__device__ __forceinline__ void rope_cos_sin_denom(int64_t pos, float denom, float& c, float& s) {
  const float angle = __fdiv_rn(static_cast<float>(pos), denom);
  double sd, cd;
  sincos(static_cast<double>(angle), &sd, &cd);
  c = static_cast<float>(cd);
  s = static_cast<float>(sd);
}

__device__ __forceinline__ void rope_pair(float xe, float xo, float c, float s, uint16_t& ye, uint16_t& yo) {
  ye = f32_to_bf16_bits(__fsub_rn(__fmul_rn(xe, c), __fmul_rn(xo, s)));
  yo = f32_to_bf16_bits(__fadd_rn(__fmul_rn(xe, s), __fmul_rn(xo, c)));
}

// Positions P_b + t: P_b = past_lengths[b] when given (device int64 [B]),
// else past_length.
__global__ void rope_kernel(const uint16_t* x, uint16_t* out, int64_t total_pairs, int64_t tokens, int64_t heads,
                            int64_t head_dim, int64_t past_length, float theta,
                            const int64_t* past_lengths = nullptr) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total_pairs) return;
  const int64_t pairs = head_dim / 2;
  const int64_t row = i / pairs;  // ((b*T + t)*H + h)
  const int64_t m = i % pairs;
  const int64_t t = (row / heads) % tokens;
  const int64_t pos = (past_lengths ? past_lengths[row / heads / tokens] : past_length) + t;
  const int64_t off = row * head_dim + 2 * m;
  if (pos == 0) {
    out[off] = x[off];
    out[off + 1] = x[off + 1];
    return;
  }
  float c, s;
  rope_cos_sin(pos, m, head_dim, theta, c, s);
  rope_pair(bf16_bits_to_f32(x[off]), bf16_bits_to_f32(x[off + 1]), c, s, out[off], out[off + 1]);
}

// ------------------------------------------------------------------ KV append
// src/kv_cache.cu:18-57: cache[b, h, P_b + t, :] = new[b, t, h, :] (bit copy).
__global__ void kv_append_kernel(uint16_t* kc, uint16_t* vc, const uint16_t* nk, const uint16_t* nv, int64_t total,
                                 int64_t tokens, int64_t kv_heads, int64_t head_dim, int64_t capacity,
                                 int64_t past_length, const int64_t* past_lengths) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int64_t r = i;
  const int64_t d = r % head_dim;
  r /= head_dim;
  const int64_t h = r % kv_heads;
  r /= kv_heads;
  const int64_t t = r % tokens;
  const int64_t b = r / tokens;
  const int64_t p = past_lengths ? past_lengths[b] : past_length;
  if (p < 0 || p + t >= capacity) return;  // slot outside the cache: not written
  const int64_t dst = ((b * kv_heads + h) * capacity + p + t) * head_dim + d;
  kc[dst] = nk[i];
  vc[dst] = nv[i];
}

// ------------------------------------------------------------------ NVFP4 storage tools
// src/nvfp4.cu:60-112: unpack bytes to nibble codes; dequantize to FP32
// (q * beta) * gamma in that order (bit-exact with reference/nvfp4.py:539-554).
__global__ void unpack_kernel(const uint8_t* packed, uint8_t* codes, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t v = packed[i];
  codes[2 * i] = v & 0x0f;
  codes[2 * i + 1] = v >> 4;
}

__global__ void dequant_kernel(const uint8_t* packed, const uint8_t* scales, const float* gamma, float* out,
                               int64_t n_bytes, int64_t packed_cols) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_bytes) return;
  const int64_t row = i / packed_cols;
  const int64_t col = (i % packed_cols) * 2;  // logical k of the low nibble
  const float beta = decode_ue4m3(scales[row * (packed_cols / 8) + col / 16]);
  const float g = *gamma;
  const uint8_t v = packed[i];
  const int64_t o = row * packed_cols * 2 + col;
  out[o] = __fmul_rn(__fmul_rn(decode_e2m1_scalar(v & 0x0f), beta), g);
  out[o + 1] = __fmul_rn(__fmul_rn(decode_e2m1_scalar(v >> 4), beta), g);
}

// ------------------------------------------------------------------ quantizer
// reference/nvfp4.py:443-536, restated with the same FP32 operation order:
//   amax = max |x|; enc = amax == 0 ? 1 : min(2688 / amax, FLT_MAX);
//   gamma = amax * FP32(1/2688);
//   beta = UE4M3_RNE(block_amax * (enc * FP32(1/6)));
//   factor = beta > 0 ? min(1 / (beta * (1/enc)), FLT_MAX) : 0;
//   code = E2M1_RNE(x * factor)  (0 for beta == 0 blocks).
__device__ __forceinline__ float load_src(const void* src, int is_bf16, int64_t i) {
  return is_bf16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(src)[i]) : static_cast<const float*>(src)[i];
}

// amax bits accumulate with atomicMax on the unsigned pattern (|x| >= 0, so
// the integer order is the float order).
__global__ void quant_amax_kernel(const void* src, int is_bf16, int64_t n, unsigned* amax_bits) {
  float m = 0.0f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(load_src(src, is_bf16, i)));
  m = warp_max_f32(m);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

__device__ __forceinline__ uint32_t encode_e2m1_dev(float v) {
  const float a = fabsf(v);
  uint32_t code = 0x7;
  if (a <= 5.0f) code = 0x6;
  if (a < 3.5f) code = 0x5;
  if (a <= 2.5f) code = 0x4;
  if (a < 1.75f) code = 0x3;
  if (a <= 1.25f) code = 0x2;
  if (a < 0.75f) code = 0x1;
  if (a <= 0.25f) code = 0x0;
  return code | (signbit(v) ? 0x8u : 0x0u);
}

// Decoded UE4M3 value of canonical code c (0..126), FP32.
__device__ __forceinline__ float ue4m3_level(int c) { return decode_ue4m3(static_cast<uint32_t>(c)); }

__device__ __forceinline__ uint32_t encode_ue4m3_dev(float cand) {
  // first index i with level[i] >= cand (levels ascending, 127 entries)
  int lo = 0, hi = 127;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (ue4m3_level(mid) >= cand) hi = mid; else lo = mid + 1;
  }
  const int upper = lo > 0x7e ? 0x7e : lo;
  const int lower = (lo - 1) < 0 ? 0 : ((lo - 1) > 0x7e ? 0x7e : lo - 1);
  const float ud = fabsf(__fsub_rn(ue4m3_level(upper), cand));
  const float ld = fabsf(__fsub_rn(cand, ue4m3_level(lower)));
  const bool tie_up = (ud == ld) && ((upper & 1) == 0);
  return static_cast<uint32_t>((ud < ld || tie_up) ? upper : lower);
}

// One thread per 16-element block.
__global__ void quant_blocks_kernel(const void* src, int is_bf16, int64_t rows, int64_t cols,
                                    const unsigned* amax_bits, uint8_t* packed, uint8_t* scales, float* gamma) {
  const int64_t nblk = rows * (cols / 16);
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const float amax = __uint_as_float(*amax_bits);
  const float enc = (amax == 0.0f) ? 1.0f : fminf(__fdiv_rn(2688.0f, amax), FLT_MAX);
  if (i == 0) *gamma = __fmul_rn(amax, static_cast<float>(1.0 / 2688.0));
  if (i >= nblk) return;
  const int64_t base = i * 16;
  float v[16];
  float bmax = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    v[e] = load_src(src, is_bf16, base + e);
    bmax = fmaxf(bmax, fabsf(v[e]));
  }
  const float mult = __fmul_rn(enc, static_cast<float>(1.0 / 6.0));
  const uint32_t sc = encode_ue4m3_dev(__fmul_rn(bmax, mult));
  scales[i] = static_cast<uint8_t>(sc);
  const float beta = ue4m3_level(static_cast<int>(sc));
  uint8_t out[8];
  if (beta > 0.0f) {
    const float ginv = __fdiv_rn(1.0f, enc);
    const float factor = fminf(__fdiv_rn(1.0f, __fmul_rn(beta, ginv)), FLT_MAX);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t lo = encode_e2m1_dev(__fmul_rn(v[2 * e], factor));
      const uint32_t hi = encode_e2m1_dev(__fmul_rn(v[2 * e + 1], factor));
      out[e] = static_cast<uint8_t>(lo | (hi << 4));
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = 0;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) packed[i * 8 + e] = out[e];
}

}  // namespace nvfp4da
