// W4A16 decode GEMV on the tensor cores, weights streamed straight from HBM
// into registers and decoded there.
//
// Semantics (reference/w4a16.py:11-59, src/w4a16.cu:79-151):
//   y[m, n] = BF16( sum_k FP32(x[m, k]) * W_hat[n, k] ),  W_hat = (q * beta) * gamma.
// Evaluated as  y = BF16( gamma * 2^-e_m * sum_k (q*beta)[n, k] * (x[m, k] * 2^e_m) )
// with warp-level mma.m16n8k16 (FP32 accumulate), 16 weight rows x 16 k each:
//  * A = q * beta in f16: the E2M1 nibble pair is converted by the hardware
//    (cvt.rn.f16x2.e2m1x2, exact) and multiplied by the UE4M3 block scale in
//    f16 — exact, since q*beta has at most 6 significant bits and lies in
//    [2^-10, 2688];
//  * B = the activation row scaled by a power of two 2^e_m (its largest
//    element lands in [2^14, 2^15)) in f16 — used only when every element
//    converts exactly, which is checked; otherwise the same loop runs with bf16
//    operands (x exactly, q*beta exactly in bf16 as well).
// Every product is exact; only the FP32 summation order differs from the
// reference.
//
// Data movement: a warp owns a 16-row tile and a slice of K.  K is walked in
// "steps" of 128 (64 bytes per row).  In a step, lane (g = lane/4, t = lane%4)
// loads 16 contiguous bytes — physical k = 128 s + 32 t .. +31 — of rows g and
// g+8 with one 16-byte global load each, so a quad reads 64 contiguous bytes
// of a row (whole sectors).  A warp issues the loads of a whole batch of steps
// before it waits on any, and the first batch is issued before the kernel's
// programmatic-dependency wait, so the CTA's slice is in flight at once.
// Because the sum over k is order-free, word p (0..3) of the lane's 16 bytes
// (k = 128 s + 32 t + 8 p .. +7) feeds MMA-pair p: k 8p+{0,1}, 8p+{2,3} go to
// the MMA slots (2t, 2t+1), (2t+8, 2t+9) of the first MMA and 8p+{4..7} to the
// second; the activation operand is read from shared memory at the same
// physical k.  Block scales (one byte per 16 k) come from one bulk copy of the
// CTA's rows.
#pragma once

#include "common.cuh"

namespace nvfp4da {

constexpr int kMmaWarps = 8;
constexpr int kMmaThreads = kMmaWarps * kWarp;
constexpr int kMmaMaxM = 8;  // activation rows per MMA pass (the n dimension)
constexpr int kStepK = 128;  // k per step

struct MmaGemvLayout {
  uint32_t s_bytes, xs_bytes, x16_bytes, red_bytes;
  __host__ __device__ uint32_t s_off() const { return 0; }
  __host__ __device__ uint32_t xs_off() const { return s_bytes; }
  __host__ __device__ uint32_t x16_off() const { return x16_bytes ? s_bytes + xs_bytes : s_bytes; }
  __host__ __device__ uint32_t red_off() const { return s_bytes + xs_bytes + x16_bytes; }
  __host__ __device__ uint32_t total() const { return red_off() + red_bytes; }
};

__host__ __device__ inline uint32_t r16(uint64_t v) { return static_cast<uint32_t>((v + 15) & ~uint64_t(15)); }

__host__ __device__ inline MmaGemvLayout mma_gemv_layout(int rows, int64_t k, int mg) {
  MmaGemvLayout l;
  const int tile_rows = ((rows + 15) / 16) * 16;
  l.s_bytes = r16(static_cast<uint64_t>(tile_rows) * (k / 16));
  l.xs_bytes = r16(static_cast<uint64_t>(mg) * k * 2);
  // Several rows on the warp-per-row path (K <= 4096) convert in place: no
  // separate f16 buffer.
  l.x16_bytes = (mg > 1 && k <= 4096) ? 0 : r16(static_cast<uint64_t>(mg) * k * 2);
  l.red_bytes = kMmaWarps * 16 * 8 * 4;
  return l;
}

// The tensor-core path needs K % 128 == 0 (whole steps); other K use the
// CUDA-core GEMV.
__host__ __device__ inline bool mma_gemv_supported(int64_t k) { return k >= kStepK && k % kStepK == 0; }

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

// Canonical UE4M3 byte -> f16x2 with the scale in both halves.
__device__ __forceinline__ uint32_t ue4m3_to_f16x2_dup(uint32_t code) {
  uint32_t h;
  asm("{\n .reg .b16 lo;\n cvt.u16.u32 lo, %1;\n cvt.rn.f16x2.e4m3x2 %0, lo;\n}" : "=r"(h) : "r"(code & 0xffu));
  return __byte_perm(h, 0, 0x1010);
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------- per-warp work
// Warp geometry for a CTA of `rows` weight rows (<= 16 * tiles, tiles in
// {1, 2, 4, 8}): warp w handles tile w / ksplit and steps [s0, s1).
struct WarpSlice {
  int tile;
  int s0, s1;
};

__device__ __forceinline__ WarpSlice warp_slice(int rows, int64_t k) {
  const int warp = threadIdx.x >> 5;
  const int tiles = (rows + 15) / 16;
  const int ksplit = kMmaWarps / tiles;
  const int steps = static_cast<int>(k / kStepK);
  const int per = (steps + ksplit - 1) / ksplit;
  WarpSlice w;
  w.tile = warp / ksplit;
  w.s0 = (warp % ksplit) * per;
  w.s1 = w.s0 + per < steps ? w.s0 + per : steps;
  return w;
}

// This lane's weight registers for up to NB steps of its warp slice (rows g
// and g+8 of the tile): the batch a warp keeps in flight at once.
template <int NB>
struct WeightRegs {
  uint4 lo[NB], hi[NB];
};

// Issue (no wait) the loads for steps [s, min(s + NB, s_end)).  Rows at or
// past `valid_rows` (CTA-local) read as zero.
template <int NB>
__device__ __forceinline__ void issue_weight_batch(WeightRegs<NB>& w, const uint8_t* packed_row0, int64_t k,
                                                   int tile, int s, int s_end, int valid_rows) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r_lo = tile * 16 + g, r_hi = r_lo + 8;
  const int64_t kb = k / 2;
  const uint8_t* plo = packed_row0 + r_lo * kb + 16 * t;
  const uint8_t* phi = packed_row0 + r_hi * kb + 16 * t;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int st = s + i;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    w.lo[i] = (st < s_end && r_lo < valid_rows) ? ldg_stream(plo + st * 64) : z;
    w.hi[i] = (st < s_end && r_hi < valid_rows) ? ldg_stream(phi + st * 64) : z;
  }
}

// Consume a batch: decode in registers, 8 MMAs per step.  `xop` is the
// activation operand ([mgv][K], f16 or bf16 bits) in shared memory; `s_smem`
// the CTA's scale rows ([rows][K/16]).
// `hi_rows`: whether rows g + 8 of the tile hold weights at all (warp-uniform);
// if not, their decode is skipped and they enter the MMA as zeros.
template <bool F16, int NB>
__device__ __forceinline__ void mma_batch(const WeightRegs<NB>& w, const uint8_t* s_smem, const uint16_t* xop,
                                          int64_t k, int tile, int s, int s_end, int mgv, float (&d)[4][4],
                                          bool hi_rows = true) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t ks = k / 16;
  const uint8_t* sc_lo = s_smem + (tile * 16 + g) * ks + 2 * t;
  const uint8_t* sc_hi = sc_lo + 8 * ks;
  const bool has_n = g < mgv;
  const uint16_t* xrow = xop + static_cast<int64_t>(has_n ? g : 0) * k + 32 * t;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int st = s + i;
    if (st >= s_end) break;
    // scales of blocks 8 st + 2 t (+1) for rows g and g+8
    const uint32_t s2lo = *reinterpret_cast<const uint16_t*>(sc_lo + 8 * st);
    const uint32_t s2hi = *reinterpret_cast<const uint16_t*>(sc_hi + 8 * st);
    const uint32_t blo[2] = {ue4m3_to_f16x2_dup(s2lo), ue4m3_to_f16x2_dup(s2lo >> 8)};
    const uint32_t bhi[2] = {ue4m3_to_f16x2_dup(s2hi), ue4m3_to_f16x2_dup(s2hi >> 8)};
    const uint32_t wl[4] = {w.lo[i].x, w.lo[i].y, w.lo[i].z, w.lo[i].w};
    const uint32_t wh[4] = {w.hi[i].x, w.hi[i].y, w.hi[i].z, w.hi[i].w};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      uint4 xb = make_uint4(0u, 0u, 0u, 0u);
      if (has_n) xb = *reinterpret_cast<const uint4*>(xrow + st * kStepK + 8 * p);
      uint32_t q0[4], q1[4];  // rows g / g+8: nibble pairs of word p
      e2m1x8_to_f16x2x4(wl[p], q0);
      if (hi_rows) e2m1x8_to_f16x2x4(wh[p], q1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q0[j] = hmul2_u32(q0[j], blo[p >> 1]);
        q1[j] = hi_rows ? hmul2_u32(q1[j], bhi[p >> 1]) : 0u;
      }
      if constexpr (F16) {
        const uint32_t a_lo[4] = {q0[0], q1[0], q0[1], q1[1]};
        const uint32_t a_hi[4] = {q0[2], q1[2], q0[3], q1[3]};
        mma_f16(d[p], a_lo, xb.x, xb.y);  // one accumulator per word p: four
        mma_f16(d[p], a_hi, xb.z, xb.w);  // independent MMA dependency chains
      } else {
        const uint32_t a_lo[4] = {f16x2_to_bf16x2(q0[0]), f16x2_to_bf16x2(q1[0]), f16x2_to_bf16x2(q0[1]),
                                  f16x2_to_bf16x2(q1[1])};
        const uint32_t a_hi[4] = {f16x2_to_bf16x2(q0[2]), f16x2_to_bf16x2(q1[2]), f16x2_to_bf16x2(q0[3]),
                                  f16x2_to_bf16x2(q1[3])};
        mma_bf16(d[p], a_lo, xb.x, xb.y);
        mma_bf16(d[p], a_hi, xb.z, xb.w);
      }
    }
  }
}

// Sum the warps' partial 16x8 tiles: out[r * 8 + n] for CTA-local row r.
__device__ __forceinline__ void reduce_tiles(const float (&d)[4], int rows, float* red, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int tiles = (rows + 15) / 16;
  const int ksplit = kMmaWarps / tiles;
  float* rw = red + warp * 128;
  rw[g * 8 + 2 * t] = d[0];
  rw[g * 8 + 2 * t + 1] = d[1];
  rw[(g + 8) * 8 + 2 * t] = d[2];
  rw[(g + 8) * 8 + 2 * t + 1] = d[3];
  __syncthreads();
  for (int i = threadIdx.x; i < tiles * 128; i += blockDim.x) {
    const int tl = i >> 7, e = i & 127;
    float s = 0.0f;
    for (int w = 0; w < ksplit; ++w) s += red[(tl * ksplit + w) * 128 + e];
    const int r = tl * 16 + (e >> 3);
    if (r < rows) out[r * 8 + (e & 7)] = s;
  }
  __syncthreads();
}

// One full pass: this warp's slice over all its steps (batches of NB, the
// first batch already issued into `w` by the caller), then the cross-warp
// reduction into out[r * 8 + n].
template <bool F16, int NB>
__device__ __forceinline__ void mma_gemv_pass(WeightRegs<NB>& w, const uint8_t* packed_row0, const uint8_t* s_smem,
                                              const uint16_t* xop, int64_t k, int rows, int valid_rows, int mgv,
                                              float* red, float* out) {
  const WarpSlice ws = warp_slice(rows, k);
  float d[4][4] = {};
  for (int s = ws.s0; s < ws.s1; s += NB) {
    if (s != ws.s0) issue_weight_batch<NB>(w, packed_row0, k, ws.tile, s, ws.s1, valid_rows);
    mma_batch<F16, NB>(w, s_smem, xop, k, ws.tile, s, ws.s1, mgv, d);
  }
  float dsum[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dsum[i] = (d[0][i] + d[1][i]) + (d[2][i] + d[3][i]);
  reduce_tiles(dsum, rows, red, out);
}

// The same pass with the CTA's weight rows already in shared memory
// (`w_smem`: rows x K/2 bytes, row-major as in global memory), for kernels
// that bulk-copy their whole weight slice at launch.
template <int NB>
__device__ __forceinline__ void load_weight_batch_smem(WeightRegs<NB>& w, const uint8_t* w_smem, int64_t k, int tile,
                                                       int s, int s_end) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t kb = k / 2;
  const uint8_t* plo = w_smem + (tile * 16 + g) * kb + 16 * t;
  const uint8_t* phi = plo + 8 * kb;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int st = s + i;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    w.lo[i] = st < s_end ? *reinterpret_cast<const uint4*>(plo + st * 64) : z;
    w.hi[i] = st < s_end ? *reinterpret_cast<const uint4*>(phi + st * 64) : z;
  }
}

// `rows` is tile-padded (16 x 1/2/4/8); tiles or tile halves at or past
// `valid_rows` are skipped (their outputs are undefined).
template <bool F16, int NB>
__device__ __forceinline__ void mma_gemv_pass_smem(const uint8_t* w_smem, const uint8_t* s_smem, const uint16_t* xop,
                                                   int64_t k, int rows, int valid_rows, int mgv, float* red,
                                                   float* out) {
  const WarpSlice ws = warp_slice(rows, k);
  float d[4][4] = {};
  if (ws.tile * 16 < valid_rows) {
    const bool hi = ws.tile * 16 + 8 < valid_rows;
#pragma unroll 1
    for (int s = ws.s0; s < ws.s1; s += NB) {
      WeightRegs<NB> w;
      load_weight_batch_smem<NB>(w, w_smem, k, ws.tile, s, ws.s1);
      mma_batch<F16, NB>(w, s_smem, xop, k, ws.tile, s, ws.s1, mgv, d, hi);
    }
  }
  float dsum[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dsum[i] = (d[0][i] + d[1][i]) + (d[2][i] + d[3][i]);
  reduce_tiles(dsum, rows, red, out);
}

// ---------------------------------------------------------------- scales
// Copy the CTA's scale rows ([rows][K/16], contiguous in global memory) into
// shared memory: one bulk copy on `bar` when 16-byte granular (returns true;
// the caller waits on `bar` phase 0), else a cooperative copy (returns false,
// the data is visible after the caller's next __syncthreads).  Rows at or past
// valid_rows are not copied.
__device__ __forceinline__ bool stage_scales(uint8_t* s_smem, const uint8_t* scales, int64_t k, int64_t row0,
                                             int valid_rows, uint64_t* bar) {
  const int64_t ks = k / 16;
  const uint32_t bytes = static_cast<uint32_t>(valid_rows * ks);
  const uint8_t* src = scales + row0 * ks;
  if (aligned16(src) && bytes % 16 == 0) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, bytes);
      if (bytes) bulk_g2s(s_smem, src, bytes, bar);
    }
    return true;
  }
  for (uint32_t i = threadIdx.x; i < bytes; i += blockDim.x) s_smem[i] = src[i];
  return false;
}

// ---------------------------------------------------------------- activations
// Global -> shared copy of n BF16 values with 16-byte loads (all threads).
__device__ __forceinline__ void load_rows_lsu(uint16_t* dst, const uint16_t* src, int64_t n) {
  if (aligned16(src) && n % 8 == 0) {
    const int64_t nv = n / 8;
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = *reinterpret_cast<const uint4*>(src + 8 * i);
  } else {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// From BF16 rows in x_stage ([mgv][K], K % 8 == 0) build the f16 operand rows
// in x16: x16[m][k] = f16(x[m][k] * 2^e_m) with e_m putting max|x[m]| in
// [2^14, 2^15).  Returns (uniformly over the CTA) whether every element
// converted exactly; `escale[m]` receives 2^-e_m.  Must be called by all
// threads; x_stage must be visible to all threads on entry.
__device__ __forceinline__ bool mma_prepare_f16(const uint16_t* x_stage, __half* x16, int64_t k, int mgv,
                                                float* escale /* [kMmaMaxM] smem */,
                                                float* red /* >= kMmaMaxM * warps floats */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int kv = static_cast<int>(k / 8);  // uint4 per row
  for (int m = 0; m < mgv; ++m) {
    const uint4* row = reinterpret_cast<const uint4*>(x_stage + m * k);
    float mx = 0.0f;
    for (int i = threadIdx.x; i < kv; i += blockDim.x) {
      const uint4 v = row[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(w[j] << 16)), fabsf(__uint_as_float(w[j] & 0xffff0000u))));
    }
    mx = warp_max_f32(mx);
    if (lane == 0) red[m * nw + warp] = mx;
  }
  __syncthreads();
  if (threadIdx.x < mgv) {
    float mx = 0.0f;
    for (int w = 0; w < nw; ++w) mx = fmaxf(mx, red[threadIdx.x * nw + w]);
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
      const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 127;  // floor(log2) for normals
      e = 14 - (ex < -126 ? -126 : ex);
      e = e > 126 ? 126 : (e < -126 ? -126 : e);
    }
    escale[threadIdx.x] = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);  // 2^e
  }
  __syncthreads();
  int inexact = 0;
  for (int m = 0; m < mgv; ++m) {
    const float sc = escale[m], inv = 1.0f / sc;  // powers of two: both exact
    const uint4* row = reinterpret_cast<const uint4*>(x_stage + m * k);
    uint4* orow = reinterpret_cast<uint4*>(x16 + m * k);
    for (int i = threadIdx.x; i < kv; i += blockDim.x) {
      const uint4 v = row[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = __uint_as_float(w[j] << 16), b = __uint_as_float(w[j] & 0xffff0000u);
        const __half2 h = __floats2half2_rn(a * sc, b * sc);
        inexact |= (__low2float(h) * inv != a) | (__high2float(h) * inv != b);  // round trip gives x back
        o[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      orow[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();  // escale reads done before it is overwritten below
  if (threadIdx.x < mgv) escale[threadIdx.x] = 1.0f / escale[threadIdx.x];  // 2^-e, exact
  return __syncthreads_or(inexact) == 0;
}

// ---------------------------------------------------------------- register path
// Activation rows straight from global memory through registers, for
// K <= 8 * kMmaThreads * NCH: optional RMSNorm (reference
// decoder_attention.py:117-140; the gain's 8-element chunks `gch` already in
// registers), then the power-of-two f16 operand.  Per row: one block
// reduction for the sum of squares (FP64, exact), one for the max.  Writes the
// BF16 row to x_stage (the bf16 fallback operand and, if `dbg`, the stage
// output) and the f16 row to x16; escale[m] = 2^-e_m.  Returns, uniformly over
// the CTA, whether every conversion was exact (then x16 is the operand).
// `x` must be readable coherently: written by an earlier kernel, or (with
// L2_ONLY, which reads through L2 only) by another CTA of this kernel before a
// release/acquire handshake.
template <int NCH, bool NORM, bool L2_ONLY = false>
__device__ __forceinline__ bool prep_rows_regs(const uint16_t* x, int64_t k, int mgv, const uint4 (&gch)[NCH],
                                               float eps, uint16_t* x_stage, __half* x16, float* escale,
                                               float* redf /* 2 * warps */, double* redd /* 2 * warps */,
                                               uint16_t* dbg) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kv8 = static_cast<int>(k / 8);
  int inexact = 0;
  for (int m = 0; m < mgv; ++m) {
    const int buf = (m & 1) * kMmaWarps;
    uint4 v[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int idx = threadIdx.x + c * kMmaThreads;
      const uint4* src = reinterpret_cast<const uint4*>(x + m * k + 8 * idx);
      if (idx >= kv8)
        v[c] = make_uint4(0u, 0u, 0u, 0u);
      else if constexpr (L2_ONLY)
        v[c] = __ldcg(src);  // rows written by other CTAs of the same kernel
      else
        v[c] = *src;
    }
    if constexpr (NORM) {
      double ss = 0.0;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const uint32_t wv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = __uint_as_float(wv[j] << 16), b = __uint_as_float(wv[j] & 0xffff0000u);
          ss += static_cast<double>(a * a) + static_cast<double>(b * b);
        }
      }
      ss = warp_sum_f64(ss);
      if (lane == 0) redd[buf + warp] = ss;
      __syncthreads();
      double tot = 0.0;
#pragma unroll
      for (int w = 0; w < kMmaWarps; ++w) tot += redd[buf + w];
      const float inv = rms_inverse(static_cast<float>(tot), static_cast<float>(k), eps);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const uint32_t wv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
        const uint32_t wg[4] = {gch[c].x, gch[c].y, gch[c].z, gch[c].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t lo = f32_to_bf16_bits(
              __fmul_rn(__fmul_rn(__uint_as_float(wv[j] << 16), inv), __uint_as_float(wg[j] << 16)));
          const uint32_t hi = f32_to_bf16_bits(
              __fmul_rn(__fmul_rn(__uint_as_float(wv[j] & 0xffff0000u), inv), __uint_as_float(wg[j] & 0xffff0000u)));
          o[j] = lo | (hi << 16);
        }
        v[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    float mx = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int idx = threadIdx.x + c * kMmaThreads;
      if (idx < kv8) {
        reinterpret_cast<uint4*>(x_stage + m * k)[idx] = v[c];
        if (dbg) reinterpret_cast<uint4*>(dbg + m * k)[idx] = v[c];
      }
      const uint32_t wv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(wv[j] << 16)), fabsf(__uint_as_float(wv[j] & 0xffff0000u))));
    }
    mx = warp_max_f32(mx);
    if (lane == 0) redf[buf + warp] = mx;
    __syncthreads();
    mx = 0.0f;
#pragma unroll
    for (int w = 0; w < kMmaWarps; ++w) mx = fmaxf(mx, redf[buf + w]);
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
      const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 127;  // floor(log2) for normals
      e = 14 - (ex < -126 ? -126 : ex);
      e = e > 126 ? 126 : (e < -126 ? -126 : e);
    }
    const float sc = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);   // 2^e
    const float isc = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
    if (threadIdx.x == 0) escale[m] = isc;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int idx = threadIdx.x + c * kMmaThreads;
      if (idx >= kv8) continue;
      const uint32_t wv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = __uint_as_float(wv[j] << 16), b = __uint_as_float(wv[j] & 0xffff0000u);
        const __half2 h = __floats2half2_rn(a * sc, b * sc);
        inexact |= (__low2float(h) * isc != a) | (__high2float(h) * isc != b);  // round trip gives x back
        o[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      reinterpret_cast<uint4*>(x16 + m * k)[idx] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  return __syncthreads_or(inexact) == 0;
}

// Several activation rows at once (mgv >= 2): warp w prepares row w (and
// w + 8, ...) alone, in place in its x_stage row -- the same per-row
// arithmetic as prep_rows_regs (optional RMSNorm with the FP64 sum of squares,
// exact in any order, then the power-of-two f16 operand) with warp reductions
// only, so the rows proceed in parallel and the CTA meets one barrier in all.
// Each lane only rereads the 16-byte chunks it wrote itself.  `g` is the norm
// gain, in shared or global memory (every warp reads the same chunks).
// Same outputs as prep_rows_regs; with x16 == x_stage the two share one
// buffer (see below).
template <bool NORM, bool L2_ONLY = false>
__device__ __forceinline__ bool prep_rows_warp(const uint16_t* x, const uint16_t* g, int64_t k, int mgv, float eps,
                                               uint16_t* x_stage, __half* x16, float* escale, uint16_t* dbg) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kv8 = static_cast<int>(k / 8);
  // x16 == x_stage: one buffer, the f16 operand written over the BF16 rows
  // only once every row is known to convert exactly (else the BF16 rows stay).
  const bool in_place = reinterpret_cast<const void*>(x16) == reinterpret_cast<const void*>(x_stage);
  int inexact = 0;
  for (int m = warp; m < mgv; m += kMmaWarps) {
    uint4* row = reinterpret_cast<uint4*>(x_stage + m * k);  // this warp's row, staged in shared memory
    const uint4* src = reinterpret_cast<const uint4*>(x + m * k);
    // Four FP64 partial sums (the squares of BF16 values are exact in FP32 and
    // their FP64 sum is exact, so the order does not change the result).
    double ssp[4] = {0.0, 0.0, 0.0, 0.0};
    constexpr int kBatch = 6;  // loads in flight per lane (two rounds at K = 3072)
    for (int idx0 = lane; idx0 < kv8; idx0 += 32 * kBatch) {
      uint4 v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int idx = idx0 + 32 * j;
        v[j] = idx < kv8 ? (L2_ONLY ? __ldcg(src + idx) : src[idx]) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int idx = idx0 + 32 * j;
        if (idx < kv8) row[idx] = v[j];
        if constexpr (NORM) {
          const uint32_t wv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a = __uint_as_float(wv[q] << 16), b = __uint_as_float(wv[q] & 0xffff0000u);
            ssp[q] += static_cast<double>(a * a) + static_cast<double>(b * b);
          }
        }
      }
    }
    double ss = (ssp[0] + ssp[1]) + (ssp[2] + ssp[3]);
    float mx = 0.0f;
    if constexpr (NORM) {
      ss = warp_sum_f64(ss);  // also orders the row's shared-memory writes before the reads below
      const float inv = rms_inverse(static_cast<float>(ss), static_cast<float>(k), eps);
      for (int idx0 = lane; idx0 < kv8; idx0 += 32 * kBatch) {
       uint4 gb[kBatch];
#pragma unroll
       for (int j = 0; j < kBatch; ++j) {
         const int idx = idx0 + 32 * j;
         gb[j] = idx < kv8 ? reinterpret_cast<const uint4*>(g)[idx] : make_uint4(0u, 0u, 0u, 0u);
       }
#pragma unroll
       for (int j = 0; j < kBatch; ++j) {
        const int idx = idx0 + 32 * j;
        if (idx >= kv8) break;
        const uint4 v = row[idx], gg = gb[j];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w}, wg[4] = {gg.x, gg.y, gg.z, gg.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = __fmul_rn(__fmul_rn(__uint_as_float(wv[q] << 16), inv), __uint_as_float(wg[q] << 16));
          const float hi =
              __fmul_rn(__fmul_rn(__uint_as_float(wv[q] & 0xffff0000u), inv), __uint_as_float(wg[q] & 0xffff0000u));
          o[q] = static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
          mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(o[q] << 16)), fabsf(__uint_as_float(o[q] & 0xffff0000u))));
        }
        const uint4 nv = make_uint4(o[0], o[1], o[2], o[3]);
        row[idx] = nv;
        if (dbg) reinterpret_cast<uint4*>(dbg + m * k)[idx] = nv;
       }
      }
    } else {
      for (int idx = lane; idx < kv8; idx += 32) {
        const uint4 v = row[idx];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(wv[q] << 16)), fabsf(__uint_as_float(wv[q] & 0xffff0000u))));
        if (dbg) reinterpret_cast<uint4*>(dbg + m * k)[idx] = v;
      }
    }
    mx = warp_max_f32(mx);  // each lane reads back only what it wrote, so no other ordering is needed
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
      const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 127;  // floor(log2) for normals
      e = 14 - (ex < -126 ? -126 : ex);
      e = e > 126 ? 126 : (e < -126 ? -126 : e);
    }
    const float sc = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);   // 2^e
    const float isc = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
    if (lane == 0) escale[m] = isc;
    for (int idx = lane; idx < kv8; idx += 32) {
      const uint4 v = row[idx];
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = __uint_as_float(wv[q] << 16), b = __uint_as_float(wv[q] & 0xffff0000u);
        const __half2 h = __floats2half2_rn(a * sc, b * sc);
        inexact |= (__low2float(h) * isc != a) | (__high2float(h) * isc != b);  // round trip gives x back
        o[q] = *reinterpret_cast<const uint32_t*>(&h);
      }
      if (!in_place) reinterpret_cast<uint4*>(x16 + m * k)[idx] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  const bool exact = __syncthreads_or(inexact) == 0;
  if (in_place && exact) {
    // Every row converts exactly: overwrite the BF16 rows with the f16
    // operand (each lane converts the chunks it owns).
    for (int m = warp; m < mgv; m += kMmaWarps) {
      const float sc = 1.0f / escale[m];  // a power of two: exact
      uint4* row = reinterpret_cast<uint4*>(x_stage + m * k);
      for (int idx = lane; idx < kv8; idx += 32) {
        const uint4 v = row[idx];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __half2 h = __floats2half2_rn(__uint_as_float(wv[q] << 16) * sc, __uint_as_float(wv[q] & 0xffff0000u) * sc);
          o[q] = *reinterpret_cast<const uint32_t*>(&h);
        }
        row[idx] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncthreads();
  }
  return exact;
}

}  // namespace nvfp4da
