// W4A16 GEMV core: a CTA owns `rows` consecutive weight rows (resident in
// shared memory) and produces them for a group of up to MG activation rows.
//
// Semantics (reference/w4a16.py:11-59, src/w4a16.cu:79-151):
//   y[m, n] = BF16( sum_k FP32(x[m, k]) * W_hat[n, k] ),  W_hat = (q * beta) * gamma
// evaluated as  BF16( gamma * sum_blocks beta_b * sum_{k in b} q_k * x_k )  in FP32.
// Each q_k * x_k is exact in FP32 (2 x 8 significant bits), so the only
// differences from the reference are FP32 reassociation roundings.
//
// Shared-memory layout per CTA:
//   w_smem  [rows][K/2]   packed nibbles, copied verbatim from global
//   s_smem  [rows][K/16]  UE4M3 scale bytes
//   x_smem  float4[MG][4][K/16]  activations as FP32, quad-interleaved: quad q
//           of 16-element chunk c of row m sits at (m*4 + q)*NC + c, so lanes
//           reading consecutive chunks hit consecutive 16-byte words.
#pragma once

#include "common.cuh"

namespace nvfp4da {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * kWarp;

struct GemvSmemLayout {
  uint32_t w_bytes;   // rows * K/2, rounded up to 16
  uint32_t s_bytes;   // rows * K/16, rounded up to 16
  uint32_t x_bytes;   // MG * K * 4   (FP32, quad-interleaved)
  uint32_t xs_bytes;  // MG * K * 2   (BF16 staging of the raw activation rows)
  __host__ __device__ uint32_t w_off() const { return 0; }
  __host__ __device__ uint32_t s_off() const { return w_bytes; }
  __host__ __device__ uint32_t x_off() const { return w_bytes + s_bytes; }
  __host__ __device__ uint32_t xs_off() const { return w_bytes + s_bytes + x_bytes; }
  __host__ __device__ uint32_t total() const { return w_bytes + s_bytes + x_bytes + xs_bytes; }
};

__host__ __device__ inline uint32_t round16(uint64_t v) { return static_cast<uint32_t>((v + 15) & ~uint64_t(15)); }

__host__ __device__ inline GemvSmemLayout gemv_layout(int rows, int64_t k, int mg) {
  GemvSmemLayout l;
  l.w_bytes = round16(static_cast<uint64_t>(rows) * (k / 2));
  l.s_bytes = round16(static_cast<uint64_t>(rows) * (k / 16));
  l.x_bytes = static_cast<uint32_t>(static_cast<uint64_t>(mg) * k * 4);
  l.xs_bytes = round16(static_cast<uint64_t>(mg) * k * 2);
  return l;
}

// Whether this CTA's slice can be moved with bulk async copies: every warp
// sub-slice (including a partial last one) must start 16-byte aligned and span
// a multiple of 16 bytes, which holds when both row strides K/2 and K/16 are
// multiples of 16 (K % 256 == 0) and the bases are 16-byte aligned.
__device__ __forceinline__ bool gemv_bulk_ok(const uint8_t* packed, const uint8_t* scales, int64_t k) {
  return ((k / 2) % 16 == 0) && ((k / 16) % 16 == 0) && aligned16(packed) && aligned16(scales);
}

// Stage this CTA's weight rows into shared memory.  Bulk path: thread 0 arms
// one mbarrier per warp and issues two bulk copies per warp sub-slice (rows
// beyond n_rows are not copied; their smem is never read).  Fallback path:
// a cooperative byte copy finished by __syncthreads (then bars are unused).
// Must be called by all threads; bars are initialised by the caller.
__device__ __forceinline__ void gemv_stage_weights(uint8_t* w_smem, uint8_t* s_smem, const uint8_t* packed,
                                                   const uint8_t* scales, int64_t k, int64_t row0,
                                                   int rows, int64_t n_rows, bool bulk, uint64_t* bars) {
  const int64_t kb = k / 2, ks = k / 16;
  const int rpw = rows / kGemvWarps;
  if (bulk) {
    if (threadIdx.x < kGemvWarps) {
      const int w = threadIdx.x;
      const int64_t r0 = row0 + static_cast<int64_t>(w) * rpw;
      int64_t valid = n_rows - r0;
      valid = valid < 0 ? 0 : (valid > rpw ? rpw : valid);
      const uint32_t wb = static_cast<uint32_t>(valid * kb);
      const uint32_t sb = static_cast<uint32_t>(valid * ks);
      mbar_arrive_expect_tx(&bars[w], wb + sb);
      if (wb) bulk_g2s(w_smem + static_cast<int64_t>(w) * rpw * kb, packed + r0 * kb, wb, &bars[w]);
      if (sb) bulk_g2s(s_smem + static_cast<int64_t>(w) * rpw * ks, scales + r0 * ks, sb, &bars[w]);
    }
  } else {
    int64_t valid = n_rows - row0;
    valid = valid < 0 ? 0 : (valid > rows ? rows : valid);
    const int64_t wb = valid * kb, sb = valid * ks;
    for (int64_t i = threadIdx.x; i < wb; i += blockDim.x) w_smem[i] = packed[row0 * kb + i];
    for (int64_t i = threadIdx.x; i < sb; i += blockDim.x) s_smem[i] = scales[row0 * ks + i];
    __syncthreads();
  }
}

// Accumulate rows [warp*RPW, warp*RPW+RPW) of the CTA slice against MGV
// activation rows held in x_smem.  Returns, in every lane, the warp-reduced
// FP32 sums acc[r][m] (before the gamma scale).
template <int RPW, int MG>
__device__ __forceinline__ void gemv_warp_rows(const uint8_t* w_smem, const uint8_t* s_smem,
                                               const float4* x_smem, int64_t k, int mgv,
                                               float (&acc)[RPW][MG]) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t nc = k / 16;
  const int64_t kb = k / 2;
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 0; m < MG; ++m) acc[r][m] = 0.0f;

  const uint8_t* wrow = w_smem + static_cast<int64_t>(warp) * RPW * kb;
  const uint8_t* srow = s_smem + static_cast<int64_t>(warp) * RPW * nc;
  for (int64_t c = lane; c < nc; c += kWarp) {
    float x[MG][16];
#pragma unroll
    for (int m = 0; m < MG; ++m) {
      if (m < mgv) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = x_smem[(static_cast<int64_t>(m) * 4 + q) * nc + c];
          x[m][4 * q + 0] = v.x;
          x[m][4 * q + 1] = v.y;
          x[m][4 * q + 2] = v.z;
          x[m][4 * q + 3] = v.w;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const uint2 wv = *reinterpret_cast<const uint2*>(wrow + r * kb + c * 8);
      const float beta = decode_ue4m3(srow[r * nc + c]);
      float q[16];
      float lo[8], hi[8];
      decode8_e2m1(wv.x, lo);
      decode8_e2m1(wv.y, hi);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[i] = lo[i];
        q[8 + i] = hi[i];
      }
#pragma unroll
      for (int m = 0; m < MG; ++m) {
        if (m < mgv) {
          float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            s0 = fmaf(q[i], x[m][i], s0);
            s1 = fmaf(q[i + 1], x[m][i + 1], s1);
          }
          acc[r][m] = fmaf(s0 + s1, beta, acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 0; m < MG; ++m) acc[r][m] = warp_sum_f32(acc[r][m]);
}

// Store activation row (FP32 value per element) into the quad-interleaved layout.
__device__ __forceinline__ void x_smem_store(float4* x_smem, int64_t nc, int m, int64_t kidx, float v) {
  const int64_t c = kidx >> 4;
  const int e = static_cast<int>(kidx & 15);
  float* base = reinterpret_cast<float*>(&x_smem[(static_cast<int64_t>(m) * 4 + (e >> 2)) * nc + c]);
  base[e & 3] = v;
}

}  // namespace nvfp4da
