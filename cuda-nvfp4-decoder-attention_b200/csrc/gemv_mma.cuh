// W4A16 decode GEMV on the tensor cores, operands decoded in registers.
//
// Semantics (reference/w4a16.py:11-59, src/w4a16.cu:79-151):
//   y[m, n] = BF16( sum_k FP32(x[m, k]) * W_hat[n, k] ),  W_hat = (q * beta) * gamma.
// Evaluated as  y = BF16( gamma * 2^-e_m * sum_k (q*beta)[n, k] * (x[m, k] * 2^e_m) )
// with one warp-level mma.m16n8k16 (FP32 accumulate) per 16 rows x 16 k:
//  * A = q * beta in f16: the E2M1 nibble pair is converted by the hardware
//    (cvt.rn.f16x2.e2m1x2, exact) and multiplied by the UE4M3 block scale in
//    f16 — exact, since q*beta has at most 6 significant bits and lies in
//    [2^-10, 2688];
//  * B = the activation row scaled by a power of two 2^e_m (chosen so its
//    largest element lands in [2^14, 2^15)) in f16 — used only when every
//    element converts exactly, which is checked; otherwise the same loop runs
//    with bf16 operands (x exactly, q*beta exactly in bf16 as well).
// Every product is therefore exact; only the FP32 summation order differs
// from the reference.
//
// k-permutation: the sum over k is order-free, so each lane's MMA "k slots"
// are fed from the physical k that one ldmatrix (A, 16 rows x 32 k = 16 B per
// row) and one 16-byte shared load (B) hand it: lane (g = lane/4, t = lane%4)
// holds physical k = 8t .. 8t+7 of a 32-wide k chunk; k 8t..8t+3 go to the
// first MMA's slots (2t, 2t+1, 2t+8, 2t+9) and 8t+4..8t+7 to the second's.
//
// Shared-memory layout (per CTA, R rows, up to MG <= 8 activation rows):
//   w_smem [R][K/2 + 16]   nibbles; 16 B padding per row so the 8 rows an
//                          ldmatrix reads fall into distinct banks
//   s_smem [R][K/16 + 16]  UE4M3 scale bytes, padded likewise
//   x_stage [MG][K] bf16   raw (or normalised) activation rows
//   x16     [MG][K] f16    power-of-two-scaled activations
//   red     [warps][16][8] FP32 partial tiles for the cross-warp k reduction
#pragma once

#include "common.cuh"

namespace nvfp4da {

constexpr int kMmaWarps = 8;
constexpr int kMmaThreads = kMmaWarps * kWarp;
constexpr int kMmaMaxM = 8;  // activation rows per MMA pass (the n dimension)

struct MmaGemvLayout {
  uint32_t w_stride, s_stride;  // padded row strides (bytes)
  uint32_t w_bytes, s_bytes, xs_bytes, x16_bytes, red_bytes;
  __host__ __device__ uint32_t w_off() const { return 0; }
  __host__ __device__ uint32_t s_off() const { return w_bytes; }
  __host__ __device__ uint32_t xs_off() const { return w_bytes + s_bytes; }
  __host__ __device__ uint32_t x16_off() const { return w_bytes + s_bytes + xs_bytes; }
  __host__ __device__ uint32_t red_off() const { return w_bytes + s_bytes + xs_bytes + x16_bytes; }
  __host__ __device__ uint32_t total() const { return red_off() + red_bytes; }
};

__host__ __device__ inline uint32_t r16(uint64_t v) { return static_cast<uint32_t>((v + 15) & ~uint64_t(15)); }

__host__ __device__ inline MmaGemvLayout mma_gemv_layout(int rows, int64_t k, int mg) {
  MmaGemvLayout l;
  l.w_stride = r16(static_cast<uint64_t>(k / 2)) + 16;
  l.s_stride = r16(static_cast<uint64_t>(k / 16)) + 16;
  const int tiles_rows = ((rows + 15) / 16) * 16;
  l.w_bytes = l.w_stride * tiles_rows;
  l.s_bytes = l.s_stride * tiles_rows;
  l.xs_bytes = r16(static_cast<uint64_t>(mg) * k * 2);
  l.x16_bytes = r16(static_cast<uint64_t>(mg) * k * 2);
  l.red_bytes = kMmaWarps * 16 * 8 * 4;
  return l;
}

// The tensor-core path handles K % 32 == 0; other K use the reference-order
// CUDA-core GEMV.
__host__ __device__ inline bool mma_gemv_supported(int64_t k) { return k >= 32 && k % 32 == 0; }

// ---------------------------------------------------------------- weight staging
// Bulk-copy rows [row0, row0 + rows) into the padded layout: one copy per row
// for the nibbles and one for the scales, all counted on `bar` (threads
// 0..rows-1 issue).  Rows at or past n_rows are zero-filled by the fallback
// and skipped (never stored) by the bulk path.  Fallback when an address or
// size is not 16-byte granular: cooperative byte copy + __syncthreads.
// Returns true when the bulk path was taken (caller waits on `bar`).
__device__ __forceinline__ bool mma_stage_weights(uint8_t* w_smem, uint8_t* s_smem, const MmaGemvLayout& L,
                                                  const uint8_t* packed, const uint8_t* scales, int64_t k,
                                                  int64_t row0, int rows, int64_t n_rows, uint64_t* bar) {
  const int64_t kb = k / 2, ks = k / 16;
  const bool bulk = (kb % 16 == 0) && (ks % 16 == 0) && aligned16(packed) && aligned16(scales);
  int64_t valid = n_rows - row0;
  valid = valid < 0 ? 0 : (valid > rows ? rows : valid);
  if (bulk) {
    if (threadIdx.x == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(valid * (kb + ks)));
    __syncthreads();  // expect_tx before any complete_tx can land
    if (threadIdx.x < valid) {
      const int r = threadIdx.x;
      bulk_g2s(w_smem + r * L.w_stride, packed + (row0 + r) * kb, static_cast<uint32_t>(kb), bar);
      bulk_g2s(s_smem + r * L.s_stride, scales + (row0 + r) * ks, static_cast<uint32_t>(ks), bar);
    }
    return true;
  }
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(rows) * kb; i += blockDim.x) {
    const int64_t r = i / kb, c = i % kb;
    w_smem[r * L.w_stride + c] = r < valid ? packed[(row0 + r) * kb + c] : uint8_t(0);
  }
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(rows) * ks; i += blockDim.x) {
    const int64_t r = i / ks, c = i % ks;
    s_smem[r * L.s_stride + c] = r < valid ? scales[(row0 + r) * ks + c] : uint8_t(0);
  }
  __syncthreads();
  return false;
}

// ---------------------------------------------------------------- activation prep
// From BF16 rows in x_stage ([mgv][K]) build the f16 operand rows in x16:
// x16[m][k] = f16(x[m][k] * 2^e_m) with e_m putting max|x[m]| in [2^14, 2^15).
// Returns (uniformly over the CTA) whether every element converted exactly;
// `escale[m]` receives 2^-e_m.  Must be called by all threads.
__device__ __forceinline__ bool mma_prepare_f16(const uint16_t* x_stage, __half* x16, int64_t k, int mgv,
                                                float* escale /* [kMmaMaxM] smem */,
                                                float* red /* >= kMmaMaxM * warps floats */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  // per-row amax
  for (int m = 0; m < mgv; ++m) {
    float mx = 0.0f;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) mx = fmaxf(mx, fabsf(bf16_bits_to_f32(x_stage[m * k + i])));
    mx = warp_max_f32(mx);
    if (lane == 0) red[m * nw + warp] = mx;
  }
  __syncthreads();
  if (threadIdx.x < mgv) {
    float mx = 0.0f;
    for (int w = 0; w < nw; ++w) mx = fmaxf(mx, red[threadIdx.x * nw + w]);
    // 2^e with mx * 2^e in [2^14, 2^15); exponent of mx from its bits.
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
      const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 127;  // floor(log2) for normals
      e = 14 - (ex < -126 ? -126 : ex);
      e = e > 126 ? 126 : (e < -126 ? -126 : e);
    }
    escale[threadIdx.x] = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);   // 2^e
  }
  __syncthreads();
  int inexact = 0;
  for (int m = 0; m < mgv; ++m) {
    const float sc = escale[m], inv = 1.0f / sc;  // powers of two: both exact
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
      const float x = bf16_bits_to_f32(x_stage[m * k + i]);
      const __half h = __float2half_rn(x * sc);
      inexact |= (__half2float(h) * inv != x);  // round trip must give x back
      x16[m * k + i] = h;
    }
  }
  __syncthreads();  // escale reads done before it is overwritten below
  if (threadIdx.x < mgv) escale[threadIdx.x] = 1.0f / escale[threadIdx.x];  // 2^-e, exact
  return __syncthreads_or(inexact) == 0;
}

// ---------------------------------------------------------------- MMA primitives
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t& r0, uint32_t& r1, const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(row_addr)));
}

// f16x2 (exact q*beta) -> bf16x2 (exact as well: <= 6 significant bits).
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
  const __half2 hv = *reinterpret_cast<const __half2*>(&h);
  const __nv_bfloat162 b = __floats2bfloat162_rn(__low2float(hv), __high2float(hv));
  return *reinterpret_cast<const uint32_t*>(&b);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// One warp: 16-row tile `tile_row0` (CTA-local) x k32 chunks [c0, c1),
// against activation rows (n = lane/4 < mgv) in `xop` (f16 or bf16 bits,
// [mgv][K]).  Accumulates into d[4] (rows g, g+8; n = 2t, 2t+1).
template <bool F16>
__device__ __forceinline__ void mma_tile_partial(const uint8_t* w_smem, const uint8_t* s_smem,
                                                 const MmaGemvLayout& L, const uint16_t* xop, int64_t k,
                                                 int tile_row0, int64_t c0, int64_t c1, int mgv, float (&d)[4]) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* arow = w_smem + (tile_row0 + (lane & 7) + ((lane >> 3) & 1) * 8) * L.w_stride;
  const uint8_t* s0 = s_smem + (tile_row0 + g) * L.s_stride + (t >> 1);
  const uint8_t* s1 = s0 + 8 * L.s_stride;
  const bool has_n = g < mgv;
  const uint16_t* xrow = xop + static_cast<int64_t>(has_n ? g : 0) * k + 8 * t;
#pragma unroll 2
  for (int64_t c = c0; c < c1; ++c) {
    uint32_t r0, r1;
    ldmatrix_x2(r0, r1, arow + c * 16);
    uint4 xb = make_uint4(0u, 0u, 0u, 0u);
    if (has_n) xb = *reinterpret_cast<const uint4*>(xrow + c * 32);
    const uint32_t sc0 = s0[2 * c], sc1 = s1[2 * c];
    // block scales as f16x2 (same value in both halves)
    uint32_t b2_0, b2_1;
    asm("{\n .reg .b16 lo;\n cvt.u16.u32 lo, %1;\n cvt.rn.f16x2.e4m3x2 %0, lo;\n}" : "=r"(b2_0) : "r"(sc0));
    asm("{\n .reg .b16 lo;\n cvt.u16.u32 lo, %1;\n cvt.rn.f16x2.e4m3x2 %0, lo;\n}" : "=r"(b2_1) : "r"(sc1));
    b2_0 = __byte_perm(b2_0, 0, 0x1010);
    b2_1 = __byte_perm(b2_1, 0, 0x1010);
    uint32_t q0[4], q1[4];  // row g / row g+8: nibble pairs (8t,8t+1) (8t+2,+3) (8t+4,+5) (8t+6,+7)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q0[i] = hmul2_u32(e2m1x2_to_f16x2(r0 >> (8 * i)), b2_0);
      q1[i] = hmul2_u32(e2m1x2_to_f16x2(r1 >> (8 * i)), b2_1);
    }
    if constexpr (F16) {
      const uint32_t a_lo[4] = {q0[0], q1[0], q0[1], q1[1]};
      const uint32_t a_hi[4] = {q0[2], q1[2], q0[3], q1[3]};
      mma_f16(d, a_lo, xb.x, xb.y);
      mma_f16(d, a_hi, xb.z, xb.w);
    } else {
      const uint32_t a_lo[4] = {f16x2_to_bf16x2(q0[0]), f16x2_to_bf16x2(q1[0]), f16x2_to_bf16x2(q0[1]),
                                f16x2_to_bf16x2(q1[1])};
      const uint32_t a_hi[4] = {f16x2_to_bf16x2(q0[2]), f16x2_to_bf16x2(q1[2]), f16x2_to_bf16x2(q0[3]),
                                f16x2_to_bf16x2(q1[3])};
      mma_bf16(d, a_lo, xb.x, xb.y);
      mma_bf16(d, a_hi, xb.z, xb.w);
    }
  }
}

// Full CTA GEMV pass for `rows` (<= 16 * tiles) rows and mgv activation rows.
// Warps are split as (tile, k-slice); partial tiles are summed through
// `red`.  On return, out[r * 8 + n] (r < rows, n < mgv) holds the FP32 sum
// for CTA-local row r and activation row n, before gamma and 2^-e scaling.
// Must be called by all kMmaWarps warps.
template <bool F16>
__device__ __forceinline__ void mma_gemv_pass(const uint8_t* w_smem, const uint8_t* s_smem, const MmaGemvLayout& L,
                                              const uint16_t* xop, int64_t k, int rows, int mgv, float* red,
                                              float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tiles = (rows + 15) / 16;
  const int ksplit = kMmaWarps / tiles;  // tiles in {1, 2, 4, 8}
  const int tile = warp / ksplit, ks = warp % ksplit;
  const int64_t nchunks = k / 32;
  const int64_t per = (nchunks + ksplit - 1) / ksplit;
  const int64_t c0 = ks * per;
  const int64_t c1 = (c0 + per < nchunks) ? c0 + per : nchunks;
  float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (c0 < c1) mma_tile_partial<F16>(w_smem, s_smem, L, xop, k, tile * 16, c0, c1, mgv, d);
  // partial tile -> red[warp][16][8]
  const int g = lane >> 2, t = lane & 3;
  float* rw = red + warp * 128;
  rw[g * 8 + 2 * t] = d[0];
  rw[g * 8 + 2 * t + 1] = d[1];
  rw[(g + 8) * 8 + 2 * t] = d[2];
  rw[(g + 8) * 8 + 2 * t + 1] = d[3];
  __syncthreads();
  for (int i = threadIdx.x; i < tiles * 128; i += blockDim.x) {
    const int tl = i / 128, e = i % 128;
    float s = 0.0f;
    for (int w = 0; w < ksplit; ++w) s += red[(tl * ksplit + w) * 128 + e];
    const int r = tl * 16 + e / 8;
    if (r < rows) out[r * 8 + (e % 8)] = s;
  }
  __syncthreads();
}

}  // namespace nvfp4da
