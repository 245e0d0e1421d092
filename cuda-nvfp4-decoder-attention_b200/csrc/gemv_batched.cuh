// Batched decode projections: W4A16 with 2 <= M <= 64 activation rows.
//
// Same semantics as the decode GEMV (reference/w4a16.py:11-59,
// src/w4a16.cu:79-151): y[m, n] = BF16(gamma * sum_k x[m, k] * (q * beta)[n, k]),
// every product exact in FP32 (q * beta has at most 6 significant bits, so
// it is exact in BF16 as well), only the FP32 summation order differs.
//
// Why a separate kernel: the decode GEMV puts the activation rows on the
// n = 8 side of mma.m16n8k16 and walks the weights once per 8 rows, so at
// M = 64 every CTA re-streams and re-decodes its weight slice eight times and
// redoes the row preparation each time.  Here a weight fragment is decoded
// once and multiplied into all M rows (NT n-tiles of 8 rows):
//  * a 4-CTA cluster owns 128 weight rows; CTA q of the cluster takes the
//    K-quarter q of them, so each CTA reads only a quarter of the activation
//    rows (every CTA reading whole rows made the activations' L2 lines the
//    bottleneck: 144 CTAs x 384 KB at M = 64);
//  * at launch, before the programmatic-dependency wait, the CTA copies its
//    128 x K/4 weight block and its scale block into shared memory; after
//    the wait, its K-quarter of every activation row (row stride K/2 + 32
//    bytes, so the 16-byte operand loads of a warp hit distinct banks);
//  * warp w takes tiles 2 (w % 4) and 2 (w % 4) + 1 (32 weight rows) and the
//    128-k steps s = w / 4 (mod 2) of the quarter: per step it decodes its
//    weight block once (hardware E2M1/UE4M3 conversions) and issues
//    4 * 2 * NT BF16 MMAs;
//  * the two step-halves are summed in the CTA, then the four K-quarters
//    through distributed shared memory, always in the same order, so results
//    are deterministic.  CTA q finishes rows [32 q, 32 q + 32) of the block.
// The k-permutation: lane (g, t) holds 16 contiguous weight bytes (k = 128 s
// + 32 t .. + 31), word p of them (8 k) feeding MMA pair p.  Lanes with
// t >= 2 take their words in the order 1, 0, 3, 2 (A and B alike), which
// moves their operand loads to other shared-memory banks; every physical k
// still meets the same activation k exactly once.
//
// The fused front half (qkv_batched_kernel, one cluster per head of D = 128)
// keeps the decode chain's stage order -- input RMSNorm (bat_norm_kernel,
// once per row), Q/K/V projection, per-head RMSNorm, RoPE, cache append; the
// O projection (o_batched_kernel) writes BF16 rows.
#pragma once

#include <cooperative_groups.h>

#include "attention_prefill.cuh"  // cp_async16
#include "elementwise.cuh"
#include "gemv_kernel.cuh"
#include "gemv_mma.cuh"
#include "qkv_fused.cuh"

namespace nvfp4da {

constexpr int kBatMinM = 2;           // one row: the decode GEMV (latency-bound, no row reuse)
constexpr int kBatMaxM = 64;
constexpr int kBatCluster = 4;        // K-quarters
constexpr int kBatRows = 128;         // weight rows per cluster
constexpr int kBatRowsPerCta = kBatRows / kBatCluster;
constexpr int kBatThreads = 256;

// Dynamic shared memory of one CTA (K-quarter kq = K / 4): scales [128][kq/16],
// weights [128][kq/2, row stride bat_wrow_stride], the activation rows [MP][kq * 2 + 32 bytes] (which the
// step-half partials [128][MP] FP32 and then the CTA's results [32][MP]
// overlay once the MMAs are done), and the inbox [4 quarters][32][MP] FP32
// that the cluster's CTAs write their partials of this CTA's rows into.
__host__ __device__ inline int64_t bat_quarter(int64_t k) { return k / kBatCluster; }
__host__ __device__ inline uint32_t bat_row_stride(int64_t k) { return static_cast<uint32_t>(bat_quarter(k) * 2 + 32); }
__host__ __device__ inline uint32_t bat_scale_bytes(int64_t k) { return static_cast<uint32_t>(kBatRows * (bat_quarter(k) / 16)); }
// Staged weight rows: K/8 bytes, padded to 64 mod 128 so that the two rows
// a quarter-warp reads at once (g, g + 1) fall in different banks.
__host__ __device__ inline uint32_t bat_wrow_stride(int64_t k) {
  const uint32_t kb = static_cast<uint32_t>(bat_quarter(k) / 2);
  return kb + ((64u - kb % 128u) + 128u) % 128u;
}
__host__ __device__ inline uint32_t bat_weight_bytes(int64_t k) { return kBatRows * bat_wrow_stride(k); }
__host__ __device__ inline uint32_t bat_act_off(int64_t k) { return bat_scale_bytes(k) + bat_weight_bytes(k); }
__host__ __device__ inline uint32_t bat_act_bytes(int64_t k, int mpad) {
  const uint32_t rows = static_cast<uint32_t>(mpad) * bat_row_stride(k);
  const uint32_t red = kBatRows * static_cast<uint32_t>(mpad) * 4u;
  return rows > red ? rows : red;
}
__host__ __device__ inline uint32_t bat_inbox_bytes(int mpad) {
  return static_cast<uint32_t>(kBatCluster * kBatRowsPerCta * mpad * 4);
}
__host__ __device__ inline uint32_t bat_smem_bytes(int64_t k, int mpad) {
  return bat_act_off(k) + bat_act_bytes(k, mpad) + bat_inbox_bytes(mpad);
}
// K a multiple of 1024: each quarter whole 128-k steps and 16-byte multiples
// of scale bytes per row (bulk-copy sizes).
__host__ __device__ inline bool bat_shape_ok(int64_t m, int64_t n, int64_t k) {
  return m >= kBatMinM && m <= kBatMaxM && k >= 1024 && k % 1024 == 0 && n % kBatRows == 0;
}

// The CTA's blocks are strided in global memory (a K-quarter of each row),
// so they are staged with 16-byte asynchronous copies from every thread:
// hundreds of small bulk copies per CTA measured several microseconds of
// issue time alone.
__device__ __forceinline__ void bat_cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bat_cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// All threads: copy the CTA's scale and weight blocks (rows row0 .. row0 +
// 127, K-quarter q) and commit them as one group.
__device__ __forceinline__ void bat_stage_weights(uint8_t* smem, const uint8_t* scales, const uint8_t* packed,
                                                  int64_t row0, int64_t k, int q) {
  const int64_t kq = bat_quarter(k);
  const int sc = static_cast<int>(kq / 256), wc = static_cast<int>(kq / 32);  // 16-byte chunks per row
  const uint32_t sbase = smem_u32(smem), wbase = smem_u32(smem + bat_scale_bytes(k)), ws = bat_wrow_stride(k);
  for (int i = threadIdx.x; i < kBatRows * sc; i += kBatThreads) {
    const int r = i / sc, c = i % sc;
    cp_async16(sbase + r * sc * 16 + c * 16, scales + (row0 + r) * (k / 16) + q * (kq / 16) + c * 16, true);
  }
  for (int i = threadIdx.x; i < kBatRows * wc; i += kBatThreads) {
    const int r = i / wc, c = i % wc;
    cp_async16(wbase + r * ws + c * 16, packed + (row0 + r) * (k / 2) + q * (kq / 2) + c * 16, true);
  }
  bat_cp_async_commit();
}

// All threads: copy K-quarter q of activation rows [0, m) and commit.
__device__ __forceinline__ void bat_stage_rows(uint8_t* dst, const uint16_t* xrows, int64_t k, int m, int q) {
  const int64_t kq = bat_quarter(k);
  const int xc = static_cast<int>(kq / 8);
  const uint32_t base = smem_u32(dst), rs = bat_row_stride(k);
  for (int i = threadIdx.x; i < m * xc; i += kBatThreads) {
    const int r = i / xc, c = i % xc;
    cp_async16(base + r * rs + c * 16, xrows + static_cast<int64_t>(r) * k + q * kq + c * 8, true);
  }
  bat_cp_async_commit();
}

// The cluster's 128 rows x M outputs: CTA q returns rows [32 q, 32 q + 32)
// (before gamma) as [32][MP] FP32 in its own shared memory (the pointer
// returned).  All threads of every CTA of the cluster call it after the
// programmatic-dependency wait; the weight copies were issued
// (bat_stage_weights) before it.  After it returns no CTA touches another's
// shared memory.
template <int NT, unsigned PHASE_BASE>
__device__ __forceinline__ const float* bat_pass(uint8_t* smem, const uint16_t* xrows, int64_t k, int m) {
  [[maybe_unused]] constexpr unsigned kPhaseBase = PHASE_BASE;
  constexpr int MP = NT * 8;
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int q = static_cast<int>(cluster.block_rank());
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int tp = warp & 3, sh = warp >> 2;  // tile pair, step parity
  const int64_t kq = bat_quarter(k);
  const int steps = static_cast<int>(kq / 128);
  const uint32_t ks = static_cast<uint32_t>(kq / 16), kb = bat_wrow_stride(k), rs = bat_row_stride(k);
  const uint8_t* s_smem = smem;
  const uint8_t* w_smem = smem + bat_scale_bytes(k);
  uint8_t* act = smem + bat_act_off(k);
  bat_stage_rows(act, xrows, k, m, q);
  // lane's bytes: rows 32 tp + g + 8 r (r = 0..3: tiles 2 tp, 2 tp + 1, lower / upper half)
  const uint8_t* wl0 = w_smem + (32 * tp + g) * kb + 16 * t;
  const uint8_t* sc0 = s_smem + (32 * tp + g) * ks + 2 * t;
  // operand byte offset of (row g, lane t) in the staged rows; word p at + 16 (p ^ (t >> 1))
  const uint8_t* xs0 = act + g * rs + t * 64;
  const uint32_t pswap = (t >> 1) & 1;
  float d[2][NT][4];
#pragma unroll
  for (int tl = 0; tl < 2; ++tl)
#pragma unroll
    for (int n = 0; n < NT; ++n) d[tl][n][0] = d[tl][n][1] = d[tl][n][2] = d[tl][n][3] = 0.0f;
  NVFP4DA_PHASE(3);
  bat_cp_async_wait_all();
  __syncthreads();  // every thread's copies have landed
  NVFP4DA_PHASE(4);
  for (int s = sh; s < steps; s += 2) {
    uint4 wv[4];
    uint32_t bs[4][2];  // block scales (f16x2) of rows g + 8 r, blocks 2 t and 2 t + 1 of step s
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      wv[r] = *reinterpret_cast<const uint4*>(wl0 + 8 * r * kb + s * 64);
      if (t & 2) wv[r] = make_uint4(wv[r].y, wv[r].x, wv[r].w, wv[r].z);
      const uint32_t s2 = *reinterpret_cast<const uint16_t*>(sc0 + 8 * r * ks + 8 * s);
      bs[r][0] = ue4m3_to_f16x2_dup(s2);
      bs[r][1] = ue4m3_to_f16x2_dup(s2 >> 8);
    }
    const uint8_t* xs = xs0 + s * 256;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      // register word p is physical word p ^ pswap; its scale block is the same (p >> 1)
      uint32_t a[2][2][4];  // [tile][k half][fragment]
#pragma unroll
      for (int tl = 0; tl < 2; ++tl) {
        const uint4 lo = wv[2 * tl], hi = wv[2 * tl + 1];
        const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w};
        const uint32_t wh[4] = {hi.x, hi.y, hi.z, hi.w};
        uint32_t q0[4], q1[4];
        e2m1x8_to_f16x2x4(wl[p], q0);
        e2m1x8_to_f16x2x4(wh[p], q1);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          q0[i] = f16x2_to_bf16x2(hmul2_u32(q0[i], bs[2 * tl][p >> 1]));
          q1[i] = f16x2_to_bf16x2(hmul2_u32(q1[i], bs[2 * tl + 1][p >> 1]));
        }
        a[tl][0][0] = q0[0], a[tl][0][1] = q1[0], a[tl][0][2] = q0[1], a[tl][0][3] = q1[1];
        a[tl][1][0] = q0[2], a[tl][1][1] = q1[2], a[tl][1][2] = q0[3], a[tl][1][3] = q1[3];
      }
      const uint32_t wo = 16u * (static_cast<uint32_t>(p) ^ pswap);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4 xb = *reinterpret_cast<const uint4*>(xs + n * 8 * rs + wo);
#pragma unroll
        for (int tl = 0; tl < 2; ++tl) {
          mma_bf16(d[tl][n], a[tl][0], xb.x, xb.y);
          mma_bf16(d[tl][n], a[tl][1], xb.z, xb.w);
        }
      }
    }
  }
  NVFP4DA_PHASE(5);
  __syncthreads();  // every warp is done with the activation rows
  // Step-half 1 leaves its partials in shared memory; step-half 0 adds its
  // own and writes the sums of rows [32 tp, 32 tp + 32) straight into the
  // inbox of cluster CTA tp (slot q), which owns those rows.
  float* half = reinterpret_cast<float*>(act);  // [128][MP]
  if (sh == 1) {
#pragma unroll
    for (int tl = 0; tl < 2; ++tl)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        float* rw = half + (32 * tp + 16 * tl + g) * MP + n * 8 + 2 * t;
        rw[0] = d[tl][n][0];
        rw[1] = d[tl][n][1];
        rw[8 * MP] = d[tl][n][2];
        rw[8 * MP + 1] = d[tl][n][3];
      }
  }
  __syncthreads();
  float* inbox = reinterpret_cast<float*>(act + bat_act_bytes(k, MP));  // [4][32][MP]
  if (sh == 0) {
    float* dst = cluster.map_shared_rank(inbox, tp) + q * kBatRowsPerCta * MP;
#pragma unroll
    for (int tl = 0; tl < 2; ++tl)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int r = 16 * tl + g, col = n * 8 + 2 * t;
        const float* hr = half + (32 * tp + r) * MP + col;
        float* o = dst + r * MP + col;
        *reinterpret_cast<float2*>(o) = make_float2(d[tl][n][0] + hr[0], d[tl][n][1] + hr[1]);
        *reinterpret_cast<float2*>(o + 8 * MP) = make_float2(d[tl][n][2] + hr[8 * MP], d[tl][n][3] + hr[8 * MP + 1]);
      }
  }
  cluster.sync();  // every quarter's partials of every CTA's rows have landed
  NVFP4DA_PHASE(6);
  // This CTA's rows: the four quarters in cluster-rank order.
  float* out = reinterpret_cast<float*>(act);  // [32][MP] (the step-half partials are consumed)
  for (int i = threadIdx.x; i < kBatRowsPerCta * MP; i += kBatThreads) {
    const float* v = inbox + i;
    out[i] = ((v[0] + v[kBatRowsPerCta * MP]) + v[2 * kBatRowsPerCta * MP]) + v[3 * kBatRowsPerCta * MP];
  }
  __syncthreads();
  NVFP4DA_PHASE(7);
  return out;
}

// ---------------------------------------------------------------- input RMSNorm + RoPE table
// One CTA per activation row (kNormThreads threads): the row's RMSNorm
// (reference/decoder_attention.py:117-140, the arithmetic of rms_norm_kernel)
// into p.xn, and the row's RoPE (cos, sin) at its position into p.rope_tab
// [M][D/2] with the arithmetic of the fused kernel's table (host values for
// scalar positions, else FP32 angle with a double sincos rounded once).
__global__ void __launch_bounds__(kNormThreads) bat_norm_kernel(const __grid_constant__ QkvParams p) {
  __shared__ double scratch[kNormThreads / 32];
  [[maybe_unused]] constexpr unsigned kPhaseBase = 3584;
  NVFP4DA_PHASE(0);
  pdl_launch_dependents();  // the projection kernel may stage its weights meanwhile
  const int64_t row = blockIdx.x, k = p.hidden;
  // 16-byte chunks, up to kB per thread, all in flight at once (the gain
  // never depends on an earlier kernel, so it is requested before the wait).
  constexpr int kB = 8;  // K <= 8 * 8 * kNormThreads (checked by the host)
  const int kv8 = static_cast<int>(k / 8);
  const uint4* gr = reinterpret_cast<const uint4*>(p.g_in);
  uint4 v[kB], gg[kB];
#pragma unroll
  for (int i = 0; i < kB; ++i) {
    const int idx = threadIdx.x + i * kNormThreads;
    gg[i] = idx < kv8 ? gr[idx] : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  NVFP4DA_PHASE(1);
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + row * k);
#pragma unroll
  for (int i = 0; i < kB; ++i) {
    const int idx = threadIdx.x + i * kNormThreads;
    v[i] = idx < kv8 ? xr[idx] : make_uint4(0u, 0u, 0u, 0u);
  }
  // The row's RoPE table while the loads are in flight.
  const int64_t b = row / p.tokens, t = row % p.tokens;
  const int64_t pos = (p.past_lengths ? p.past_lengths[b] : p.past_length) + t;
  const int64_t pairs = p.head_dim / 2;
  for (int64_t pr = threadIdx.x; pr < pairs; pr += blockDim.x) {
    float c = 1.0f, sn = 0.0f;
    if (t < p.rope_rows) {
      c = p.rope_host[t][pr].x;
      sn = p.rope_host[t][pr].y;
    } else if (pos != 0) {
      rope_cos_sin_denom(pos, p.rope_denom[pr], c, sn);
    }
    p.rope_tab[row * pairs + pr] = make_float2(c, sn);
  }
  NVFP4DA_PHASE(3);
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < kB; ++i) {
    const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = __uint_as_float(wv[q] << 16), c = __uint_as_float(wv[q] & 0xffff0000u);
      ss += static_cast<double>(a * a) + static_cast<double>(c * c);
    }
  }
  const double tot = block_sum_f64(ss, scratch);
  NVFP4DA_PHASE(4);
  const float inv = rms_inverse(static_cast<float>(tot), static_cast<float>(k), p.eps);
  uint4* xo = reinterpret_cast<uint4*>(p.xn + row * k);
  uint4* dbg = p.dbg_xnorm ? reinterpret_cast<uint4*>(p.dbg_xnorm + row * k) : nullptr;
#pragma unroll
  for (int i = 0; i < kB; ++i) {
    const int idx = threadIdx.x + i * kNormThreads;
    if (idx >= kv8) break;
    const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w}, wg[4] = {gg[i].x, gg[i].y, gg[i].z, gg[i].w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = __fmul_rn(__fmul_rn(__uint_as_float(wv[q] << 16), inv), __uint_as_float(wg[q] << 16));
      const float hi =
          __fmul_rn(__fmul_rn(__uint_as_float(wv[q] & 0xffff0000u), inv), __uint_as_float(wg[q] & 0xffff0000u));
      o[q] = static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
    }
    const uint4 nv = make_uint4(o[0], o[1], o[2], o[3]);
    xo[idx] = nv;
    if (dbg) dbg[idx] = nv;
  }
  NVFP4DA_PHASE(2);
}

// ---------------------------------------------------------------- fused front half, D = 128
template <int NT>
__global__ void __cluster_dims__(kBatCluster, 1, 1) __launch_bounds__(kBatThreads, 1)
    qkv_batched_kernel(const __grid_constant__ QkvParams p) {
  constexpr int MP = NT * 8;
  constexpr int D = kBatRows;  // one head per cluster
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ __align__(16) uint16_t head_out[MP][D];
  [[maybe_unused]] constexpr unsigned kPhaseBase = 0;
  NVFP4DA_PHASE(0);
  pdl_launch_dependents();

  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t unit = blockIdx.x / kBatCluster;
  const int64_t k = p.hidden;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = static_cast<int>(p.m);
  int mat;
  int64_t head;
  if (unit < p.q_heads) {
    mat = 0;
    head = unit;
  } else if (unit < p.q_heads + p.kv_heads) {
    mat = 1;
    head = unit - p.q_heads;
  } else {
    mat = 2;
    head = unit - p.q_heads - p.kv_heads;
  }
  const int64_t row0 = head * D;

  bat_stage_weights(smem, p.scales[mat], p.packed[mat], row0, k, rank);
  const float gamma = *p.gamma[mat];
  NVFP4DA_PHASE(1);

  pdl_wait();
  NVFP4DA_PHASE(2);
  if (blockIdx.x == 0)
    for (int64_t i = threadIdx.x; i < p.n_zero_words; i += blockDim.x) p.zero_words[i] = 0u;
  const float* outv = bat_pass<NT, 0>(smem, p.xn, k, m);

  uint16_t* leader_out = cluster.map_shared_rank(&head_out[0][0], 0);
  for (int i = threadIdx.x; i < kBatRowsPerCta * m; i += kBatThreads) {
    const int n = i / kBatRowsPerCta, r = i % kBatRowsPerCta;
    leader_out[n * D + rank * kBatRowsPerCta + r] = f32_to_bf16_bits(__fmul_rn(outv[r * MP + n], gamma));
  }
  cluster.sync();
  NVFP4DA_PHASE(8);
  if (rank != 0) return;

  // ---- head epilogue (the leader): activation row mrow per warp
  const int64_t hq = p.q_heads, hkv = p.kv_heads;
  for (int mrow = warp; mrow < m; mrow += kBatThreads / 32) {
    const int64_t b = mrow / p.tokens, t = mrow % p.tokens;
    const int64_t pos = (p.past_lengths ? p.past_lengths[b] : p.past_length) + t;
    // A slot outside [0, C) (a device-side length breaking the caller's
    // contract) is not written.
    const int64_t slot = pos - p.slot_offset;
    const bool slot_ok = slot >= 0 && slot < p.capacity;
    const uint16_t* y = head_out[mrow];
    if (mat == 2) {
      uint32_t* dst = slot_ok ? reinterpret_cast<uint32_t*>(p.v_cache + ((b * hkv + head) * p.capacity + slot) * D)
                              : nullptr;
      for (int e2 = lane; e2 < D / 2; e2 += 32) {
        const uint32_t v = reinterpret_cast<const uint32_t*>(y)[e2];
        if (dst) dst[e2] = v;
        if (p.dbg_v) reinterpret_cast<uint32_t*>(p.dbg_v + mrow * hkv * D + head * D)[e2] = v;
      }
      continue;
    }
    const uint16_t* gsrc = mat == 0 ? p.g_q : p.g_k;
    double ss = 0.0;
    for (int e = lane; e < D; e += 32) {
      const float v = bf16_bits_to_f32(y[e]);
      ss += static_cast<double>(v * v);
    }
    ss = warp_sum_f64(ss);
    const float inv = rms_inverse(static_cast<float>(ss), static_cast<float>(D), p.eps);
    const int64_t heads = mat == 0 ? hq : hkv;
    uint16_t* dbg_proj = mat == 0 ? p.dbg_q : p.dbg_k;
    uint16_t* dbg_norm = mat == 0 ? p.dbg_qn : p.dbg_kn;
    uint16_t* dst = mat == 0 ? p.q_out + (mrow * hq + head) * D
                    : slot_ok ? p.k_cache + ((b * hkv + head) * p.capacity + slot) * D
                              : nullptr;
    const float2* cs_row = p.rope_tab + static_cast<int64_t>(mrow) * (D / 2);
    for (int pr = lane; pr < D / 2; pr += 32) {
      const int e = 2 * pr;
      const uint16_t n0 = f32_to_bf16_bits(__fmul_rn(__fmul_rn(bf16_bits_to_f32(y[e]), inv), bf16_bits_to_f32(gsrc[e])));
      const uint16_t n1 =
          f32_to_bf16_bits(__fmul_rn(__fmul_rn(bf16_bits_to_f32(y[e + 1]), inv), bf16_bits_to_f32(gsrc[e + 1])));
      if (dbg_proj) {
        dbg_proj[mrow * heads * D + head * D + e] = y[e];
        dbg_proj[mrow * heads * D + head * D + e + 1] = y[e + 1];
      }
      if (dbg_norm) {
        dbg_norm[mrow * heads * D + head * D + e] = n0;
        dbg_norm[mrow * heads * D + head * D + e + 1] = n1;
      }
      uint16_t r0 = n0, r1 = n1;
      if (pos != 0) {
        const float2 cs = cs_row[pr];
        rope_pair(bf16_bits_to_f32(n0), bf16_bits_to_f32(n1), cs.x, cs.y, r0, r1);
      }
      if (dst) {
        dst[e] = r0;
        dst[e + 1] = r1;
      }
    }
  }
}

// ---------------------------------------------------------------- O projection (any W4A16 linear)
template <int NT>
__global__ void __cluster_dims__(kBatCluster, 1, 1) __launch_bounds__(kBatThreads, 1)
    o_batched_kernel(const __grid_constant__ GemvParams p) {
  constexpr int MP = NT * 8;
  extern __shared__ __align__(16) uint8_t smem[];
  namespace cg = cooperative_groups;
  const int rank = static_cast<int>(cg::this_cluster().block_rank());
  const int64_t k = p.k;
  const int m = static_cast<int>(p.m);
  const int64_t row0 = static_cast<int64_t>(blockIdx.x / kBatCluster) * kBatRows;
  [[maybe_unused]] constexpr unsigned kPhaseBase = 2048;
  NVFP4DA_PHASE(0);
  bat_stage_weights(smem, p.scales, p.packed, row0, k, rank);
  const float gamma = *p.gamma;
  NVFP4DA_PHASE(1);
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  NVFP4DA_PHASE(2);
  const float* outv = bat_pass<NT, 2048>(smem, p.x, k, m);
  const int64_t r0 = row0 + rank * kBatRowsPerCta;
  for (int i = threadIdx.x; i < kBatRowsPerCta * m; i += kBatThreads) {
    const int n = i / kBatRowsPerCta, r = i % kBatRowsPerCta;
    p.y[n * p.n + r0 + r] = f32_to_bf16_bits(__fmul_rn(outv[r * MP + n], gamma));
  }
}

}  // namespace nvfp4da
