// Batched decode projections: W4A16 with 8 < M <= 64 activation rows.
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
// once and multiplied into all M rows (NT = ceil(M / 8) n-tiles of 8 rows):
//  * a CTA owns 32 weight rows (two 16-row tiles) over the whole K; its
//    packed rows and scale rows (contiguous in the portable layout) are
//    bulk-copied into shared memory at launch, before the programmatic-
//    dependency wait;
//  * the activation rows stream through a shared-memory ring (2-4 stages)
//    in chunks of 512 k (one bulk copy per row and chunk, row stride 1,056
//    bytes so the 16-byte operand loads of a warp hit distinct banks);
//  * warp w takes the 128-k step w % 4 of every chunk and half of the
//    n-tiles (w / 4): per chunk it decodes its 32 x 128 weight block
//    (hardware E2M1/UE4M3 conversions) and issues 8 * NT BF16 MMAs; each
//    activation operand is read from shared memory once per CTA;
//  * the four step-warps are summed in a fixed order, so results are
//    deterministic.
// The k-permutation: lane (g, t) holds 16 contiguous weight bytes (k = 128 s
// + 32 t .. + 31), word p of them (8 k) feeding MMA pair p.  Lanes with
// t >= 2 take their words in the order 1, 0, 3, 2 (A and B alike), which
// moves their operand loads to other shared-memory banks; every physical k
// still meets the same activation k exactly once.
//
// The fused front half (qkv_batched_kernel) keeps the decode chain's stage
// order -- input RMSNorm (bat_norm_kernel, once per row instead of once per
// CTA), Q/K/V projection, per-head RMSNorm, RoPE, cache append -- with one
// 4-CTA cluster per head as in qkv_fused_kernel; the O projection
// (o_batched_kernel) writes BF16 rows.
#pragma once

#include <cooperative_groups.h>

#include "elementwise.cuh"
#include "gemv_kernel.cuh"
#include "gemv_mma.cuh"
#include "qkv_fused.cuh"

namespace nvfp4da {

constexpr int kBatMinM = 9;           // below this the decode GEMV is the better kernel
constexpr int kBatMaxM = 64;
constexpr int kBatRows = 32;          // weight rows per CTA
constexpr int kBatChunkK = 512;       // k per activation chunk (4 steps of 128)
constexpr int kBatRowStride = kBatChunkK * 2 + 32;  // bytes per activation row in a ring stage
constexpr int kBatThreads = 256;

__host__ __device__ inline uint32_t bat_stage_bytes(int mpad) {
  return static_cast<uint32_t>(mpad) * kBatRowStride;
}
// Ring stages: as many as fit beside the staged weights (a chunk of 64 rows
// takes 66 KB).
__host__ __device__ constexpr int bat_stages(int mpad) { return mpad >= 64 ? 2 : (mpad >= 32 ? 3 : 4); }
// Dynamic shared memory: scales [32][K/16], packed weights [32][K/2], then
// two ring stages.
__host__ __device__ inline uint32_t bat_scale_bytes(int64_t k) { return r16(static_cast<uint64_t>(kBatRows) * (k / 16)); }
__host__ __device__ inline uint32_t bat_weight_bytes(int64_t k) { return r16(static_cast<uint64_t>(kBatRows) * (k / 2)); }
__host__ __device__ inline uint32_t bat_ring_off(int64_t k) { return bat_scale_bytes(k) + bat_weight_bytes(k); }
__host__ __device__ inline uint32_t bat_smem_bytes(int64_t k, int mpad) {
  return bat_ring_off(k) + bat_stages(mpad) * bat_stage_bytes(mpad);
}

// Thread 0: bulk-copy the CTA's scale and packed rows (completion on `bar`).
__device__ __forceinline__ void bat_stage_weights(uint8_t* smem, const uint8_t* scales, const uint8_t* packed,
                                                  int64_t row0, int64_t k, uint64_t* bar) {
  const uint32_t sbytes = static_cast<uint32_t>(kBatRows * (k / 16));
  const uint32_t wbytes = static_cast<uint32_t>(kBatRows * (k / 2));
  mbar_arrive_expect_tx(bar, sbytes + wbytes);
  bulk_g2s(smem, scales + row0 * (k / 16), sbytes, bar);
  bulk_g2s(smem + bat_scale_bytes(k), packed + row0 * (k / 2), wbytes, bar);
}
__host__ __device__ inline bool bat_shape_ok(int64_t m, int64_t n, int64_t k) {
  return m >= kBatMinM && m <= kBatMaxM && k >= kBatChunkK && k % kBatChunkK == 0 && n % kBatRows == 0;
}

// Issue the bulk copies of activation chunk c (rows [0, m) of xrows [M][K])
// into ring stage c % S (warp 0 calls; lane 0 posts the byte count first).
__device__ __forceinline__ void bat_issue_chunk(const uint16_t* xrows, int64_t k, int m, int c, int S, uint8_t* ring,
                                                uint32_t stage_bytes, uint64_t* full) {
  const int lane = threadIdx.x & 31;
  const int st = c % S;
  if (lane == 0) mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(m) * (kBatChunkK * 2));
  __syncwarp();
  for (int r = lane; r < m; r += 32)
    bulk_g2s(ring + st * stage_bytes + r * kBatRowStride, xrows + static_cast<int64_t>(r) * k + c * kBatChunkK,
             kBatChunkK * 2, &full[st]);
}

// This lane's weight bytes of chunk c (rows g and g + 8 of its tile, step
// 4 c + j) from the staged rows, words swapped pairwise for lanes t >= 2
// (see the header).
__device__ __forceinline__ void bat_load_weights(const uint8_t* w_smem, int64_t k, int tile, int j, int c,
                                                 uint4& lo, uint4& hi) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t kb = k / 2;
  const int s = c * 4 + j;
  const uint8_t* plo = w_smem + static_cast<int64_t>(tile * 16 + g) * kb + s * 64 + 16 * t;
  lo = *reinterpret_cast<const uint4*>(plo);
  hi = *reinterpret_cast<const uint4*>(plo + 8 * kb);
  if (t & 2) {
    lo = make_uint4(lo.y, lo.x, lo.w, lo.z);
    hi = make_uint4(hi.y, hi.x, hi.w, hi.z);
  }
}

// The CTA's 32 rows x M outputs (before gamma) into out[r * MP + m], MP = 8 NT.
// Called by all threads after the programmatic-dependency wait (xrows may be
// an earlier kernel's output).  `smem` holds the staged scale and weight rows
// (bat_stage_weights, completion on wbar) and the ring.  Bounded waits: a
// timeout is recorded in *err (when given) and the pass carries on with
// whatever the buffers hold.
template <int NT, unsigned PHASE_BASE>
__device__ __forceinline__ void bat_pass(uint8_t* smem, uint64_t* wbar, const uint16_t* xrows, int64_t k, int m,
                                         uint64_t* full, unsigned* err, float* out) {
  [[maybe_unused]] constexpr unsigned kPhaseBase = PHASE_BASE;
  constexpr int MP = NT * 8;
  constexpr int S = bat_stages(MP);
  constexpr int NH = NT / 2;  // n-tiles per warp
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int j = warp & 3, nh = warp >> 2;
  const uint32_t sb = bat_stage_bytes(MP);
  const int chunks = static_cast<int>(k / kBatChunkK);
  const int64_t ks = k / 16;
  const uint8_t* s_smem = smem;
  const uint8_t* w_smem = smem + bat_scale_bytes(k);
  uint8_t* ring = smem + bat_ring_off(k);
  if (warp == 0)
    for (int c = 0; c < S && c < chunks; ++c) bat_issue_chunk(xrows, k, m, c, S, ring, sb, full);
  mbar_wait_bounded(wbar, 0, err);
  NVFP4DA_PHASE(3);
  uint4 w[2][2];  // [tile][lo / hi rows]
#pragma unroll
  for (int tl = 0; tl < 2; ++tl) bat_load_weights(w_smem, k, tl, j, 0, w[tl][0], w[tl][1]);
  const uint8_t* sc0 = s_smem + g * ks + 2 * t;  // rows g, g + 8, g + 16, g + 24
  // operand byte offset of (row g of n-tile nh * NH, step j, lane t) inside a
  // stage; word p at + 16 (p ^ (t >> 1))
  const uint32_t xoff = (nh * NH * 8 + g) * kBatRowStride + j * 256 + t * 64;
  const uint32_t pswap = (t >> 1) & 1;
  float d[2][NH][4];
#pragma unroll
  for (int tl = 0; tl < 2; ++tl)
#pragma unroll
    for (int n = 0; n < NH; ++n) d[tl][n][0] = d[tl][n][1] = d[tl][n][2] = d[tl][n][3] = 0.0f;
  for (int c = 0; c < chunks; ++c) {
    const int st = c % S;
    uint4 wn[2][2];
#pragma unroll
    for (int tl = 0; tl < 2; ++tl) {
      wn[tl][0] = w[tl][0];
      wn[tl][1] = w[tl][1];
      if (c + 1 < chunks) bat_load_weights(w_smem, k, tl, j, c + 1, wn[tl][0], wn[tl][1]);
    }
    const int s = c * 4 + j;
    uint32_t bs[4][2];  // block scales (f16x2) of rows g + 8 r, blocks 2 t and 2 t + 1 of step s
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t s2 = *reinterpret_cast<const uint16_t*>(sc0 + 8 * r * ks + 8 * s);
      bs[r][0] = ue4m3_to_f16x2_dup(s2);
      bs[r][1] = ue4m3_to_f16x2_dup(s2 >> 8);
    }
    mbar_wait_bounded(&full[st], static_cast<uint32_t>(c / S) & 1u, err);
    const uint8_t* xs = ring + st * sb + xoff;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      // register word p is physical word p ^ pswap; its scale block is the same (p >> 1)
      uint32_t a[2][2][4];  // [tile][k half][fragment]
#pragma unroll
      for (int tl = 0; tl < 2; ++tl) {
        const uint32_t wl[4] = {w[tl][0].x, w[tl][0].y, w[tl][0].z, w[tl][0].w};
        const uint32_t wh[4] = {w[tl][1].x, w[tl][1].y, w[tl][1].z, w[tl][1].w};
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
      for (int n = 0; n < NH; ++n) {
        const uint4 xb = *reinterpret_cast<const uint4*>(xs + n * 8 * kBatRowStride + wo);
#pragma unroll
        for (int tl = 0; tl < 2; ++tl) {
          mma_bf16(d[tl][n], a[tl][0], xb.x, xb.y);
          mma_bf16(d[tl][n], a[tl][1], xb.z, xb.w);
        }
      }
    }
#pragma unroll
    for (int tl = 0; tl < 2; ++tl) {
      w[tl][0] = wn[tl][0];
      w[tl][1] = wn[tl][1];
    }
    __syncthreads();  // every warp is done with stage st
    if (warp == 0 && c + S < chunks) bat_issue_chunk(xrows, k, m, c + S, S, ring, sb, full);
  }
  NVFP4DA_PHASE(4);
  // Sum the four step-warps in step order (stage 0 holds the partials: its
  // last chunk has been consumed, and no copy is in flight).
  float* red = reinterpret_cast<float*>(ring);  // [j][32 rows][MP]
  float* rw = red + j * kBatRows * MP;
#pragma unroll
  for (int tl = 0; tl < 2; ++tl)
#pragma unroll
    for (int n = 0; n < NH; ++n) {
      const int col = (nh * NH + n) * 8 + 2 * t, r0 = tl * 16 + g;
      rw[r0 * MP + col] = d[tl][n][0];
      rw[r0 * MP + col + 1] = d[tl][n][1];
      rw[(r0 + 8) * MP + col] = d[tl][n][2];
      rw[(r0 + 8) * MP + col + 1] = d[tl][n][3];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < kBatRows * MP; i += kBatThreads) {
    float v = 0.0f;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) v += red[jj * kBatRows * MP + i];
    out[i] = v;
  }
  __syncthreads();
  NVFP4DA_PHASE(5);
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
  pdl_wait();
  NVFP4DA_PHASE(1);
  const int64_t row = blockIdx.x, k = p.hidden;
  // 16-byte chunks, eight per thread in flight (K % 512 == 0 here).
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + row * k);
  const uint4* gr = reinterpret_cast<const uint4*>(p.g_in);
  const int kv8 = static_cast<int>(k / 8);
  constexpr int kB = 8;
  double ss = 0.0;
  for (int base = threadIdx.x; base < kv8; base += kB * kNormThreads) {
    uint4 v[kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int idx = base + i * kNormThreads;
      v[i] = idx < kv8 ? xr[idx] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = __uint_as_float(wv[q] << 16), c = __uint_as_float(wv[q] & 0xffff0000u);
        ss += static_cast<double>(a * a) + static_cast<double>(c * c);
      }
    }
  }
  NVFP4DA_PHASE(3);
  const double tot = block_sum_f64(ss, scratch);
  NVFP4DA_PHASE(4);
  const float inv = rms_inverse(static_cast<float>(tot), static_cast<float>(k), p.eps);
  NVFP4DA_PHASE(5);
  uint4* xo = reinterpret_cast<uint4*>(p.xn + row * k);
  uint4* dbg = p.dbg_xnorm ? reinterpret_cast<uint4*>(p.dbg_xnorm + row * k) : nullptr;
  for (int base = threadIdx.x; base < kv8; base += kB * kNormThreads) {
    uint4 v[kB], gg[kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int idx = base + i * kNormThreads;
      v[i] = idx < kv8 ? xr[idx] : make_uint4(0u, 0u, 0u, 0u);
      gg[i] = idx < kv8 ? gr[idx] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int idx = base + i * kNormThreads;
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
  }
  NVFP4DA_PHASE(6);
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
  NVFP4DA_PHASE(2);
}

// ---------------------------------------------------------------- fused front half, D = 128
template <int NT>
__global__ void __cluster_dims__(kQkvCluster, 1, 1) __launch_bounds__(kBatThreads, 1)
    qkv_batched_kernel(const __grid_constant__ QkvParams p) {
  constexpr int MP = NT * 8;
  constexpr int D = 4 * kBatRows;  // one head per cluster
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t sbar, full[4];
  __shared__ __align__(16) uint16_t head_out[MP][D];
  [[maybe_unused]] constexpr unsigned kPhaseBase = 0;
  NVFP4DA_PHASE(0);
  pdl_launch_dependents();

  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t unit = blockIdx.x / kQkvCluster;
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
  const int64_t row0 = head * D + static_cast<int64_t>(rank) * kBatRows;
  float* outv = reinterpret_cast<float*>(smem + bat_ring_off(k) + bat_stage_bytes(MP));  // [32][MP], after the pass

  if (threadIdx.x == 0) {
    mbar_init(&sbar, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    bat_stage_weights(smem, p.scales[mat], p.packed[mat], row0, k, &sbar);
  }
  const float gamma = *p.gamma[mat];
  __syncthreads();  // the barriers are initialised
  NVFP4DA_PHASE(1);

  pdl_wait();
  NVFP4DA_PHASE(2);
  if (blockIdx.x == 0)
    for (int64_t i = threadIdx.x; i < p.n_zero_words; i += blockDim.x) p.zero_words[i] = 0u;
  bat_pass<NT, 0>(smem, &sbar, p.xn, k, m, full, p.err, outv);
  NVFP4DA_PHASE(6);

  uint16_t* leader_out = cluster.map_shared_rank(&head_out[0][0], 0);
  for (int i = threadIdx.x; i < kBatRows * m; i += kBatThreads) {
    const int n = i / kBatRows, r = i % kBatRows;
    leader_out[n * D + rank * kBatRows + r] = f32_to_bf16_bits(__fmul_rn(outv[r * MP + n], gamma));
  }
  cluster.sync();
  NVFP4DA_PHASE(7);
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
__global__ void __launch_bounds__(kBatThreads, 1) o_batched_kernel(const __grid_constant__ GemvParams p) {
  constexpr int MP = NT * 8;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t sbar, full[4];
  const int64_t k = p.k;
  const int m = static_cast<int>(p.m);
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kBatRows;
  float* outv = reinterpret_cast<float*>(smem + bat_ring_off(k) + bat_stage_bytes(MP));
  [[maybe_unused]] constexpr unsigned kPhaseBase = 2048;
  NVFP4DA_PHASE(0);
  if (threadIdx.x == 0) {
    mbar_init(&sbar, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    bat_stage_weights(smem, p.scales, p.packed, row0, k, &sbar);
  }
  const float gamma = *p.gamma;
  __syncthreads();
  NVFP4DA_PHASE(1);
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  NVFP4DA_PHASE(2);
  bat_pass<NT, 2048>(smem, &sbar, p.x, k, m, full, p.err, outv);
  NVFP4DA_PHASE(6);
  for (int i = threadIdx.x; i < kBatRows * m; i += kBatThreads) {
    const int n = i / kBatRows, r = i % kBatRows;
    p.y[n * p.n + row0 + r] = f32_to_bf16_bits(__fmul_rn(outv[r * MP + n], gamma));
  }
}

}  // namespace nvfp4da
