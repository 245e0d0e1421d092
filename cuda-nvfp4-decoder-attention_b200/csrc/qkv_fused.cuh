// Fused decode-step front half: input RMSNorm -> W4A16 Q/K/V projection ->
// per-head Q/K RMSNorm -> adjacent-pair RoPE -> K/V cache append.
//
// Reference stages (decoder_attention_cuda.py:273-395): cuda_rms_norm,
// 3x cuda_w4a16_linear, 2x cuda_rms_norm, 2x cuda_apply_rope and
// cuda_kv_cache_append_ — nine launches there, one here.
//
// Decomposition: one thread-block cluster of 4 CTAs per "head unit" (Hq query
// heads, then Hkv key heads, then Hkv value heads).  Each CTA owns D/4
// consecutive weight rows of that head (32 rows for D = 128), bulk-copies them
// (K/2 + K/16 bytes per row) into shared memory at kernel start, recomputes the
// input RMSNorm of the activation rows itself (the x row is tiny and L2-hot),
// and reduces its rows.  The BF16 projections are written into the cluster
// leader's shared memory through distributed shared memory; after a cluster
// barrier the leader owns the whole head and applies the head epilogue.
#pragma once

#include <cooperative_groups.h>

#include "elementwise.cuh"
#include "gemv_core.cuh"
#include "gemv_mma.cuh"

namespace nvfp4da {

namespace cg = cooperative_groups;

constexpr int kQkvCluster = 4;
constexpr int kMaxHeadDim = 256;
constexpr int kMaxRopeRows = 8;

struct QkvParams {
  const uint16_t* x;     // [M, H] bf16, M = B*T
  const uint16_t* g_in;  // [H]
  const uint8_t* packed[3];  // q, k, v
  const uint8_t* scales[3];
  const float* gamma[3];
  const uint16_t* g_q;  // [D]
  const uint16_t* g_k;  // [D]
  uint16_t* q_out;      // [M, Hq, D]
  uint16_t* k_cache;    // [B, Hkv, C, D]
  uint16_t* v_cache;
  int64_t m, tokens, hidden, q_heads, kv_heads, head_dim, capacity;
  int64_t past_length;
  const int64_t* past_lengths;
  float eps, theta;
  // Optional stage outputs (nullptr = skip), for stage-by-stage parity checks.
  uint16_t* dbg_xnorm;  // [M, H]
  uint16_t* dbg_q;      // [M, Hq*D]
  uint16_t* dbg_k;      // [M, Hkv*D]
  uint16_t* dbg_v;      // [M, Hkv*D]
  uint16_t* dbg_qn;     // [M, Hq*D]
  uint16_t* dbg_kn;     // [M, Hkv*D]
  unsigned* zero_words;  // cleared by CTA 0 (attention split counters)
  int64_t n_zero_words;
  unsigned* err;
  int pdl;
  // KV-length sharding: the caches hold positions [slot_offset, slot_offset +
  // capacity); a position outside that range is not appended here (RoPE still
  // uses the global position).
  int64_t slot_offset;
  // RoPE cos/sin per token index t < rope_rows, computed on the host when the
  // positions are the scalar past_length + t (rope_rows == 0: on the device).
  int rope_rows;
  float2 rope_host[kMaxRopeRows][kMaxHeadDim / 2];
  // theta^(2m/D) rounded to FP32, from the host, for positions read on the device.
  float rope_denom[kMaxHeadDim / 2];
  // Batched front half (gemv_batched.cuh): the normalised activation rows
  // [M, H] and the RoPE (cos, sin) of every row [M, D/2], written by
  // bat_norm_kernel and read by qkv_batched_kernel.
  uint16_t* xn;
  float2* rope_tab;
};

// Dynamic shared memory of the fused kernel: the MMA-GEMV layout followed by
// the input-norm gain [K] and the two head-norm gains [D] (BF16).
struct QkvSmemLayout {
  MmaGemvLayout g;
  uint32_t gin_bytes, gh_bytes;
  __host__ __device__ uint32_t gin_off() const { return g.total(); }
  __host__ __device__ uint32_t gq_off() const { return g.total() + gin_bytes; }
  __host__ __device__ uint32_t gk_off() const { return g.total() + gin_bytes + gh_bytes; }
  __host__ __device__ uint32_t total() const { return g.total() + gin_bytes + 2 * gh_bytes; }
};

__host__ __device__ inline QkvSmemLayout qkv_layout(int rows, int64_t k, int64_t d, int mg) {
  QkvSmemLayout l;
  l.g = mma_gemv_layout(rows, k, mg);
  l.gin_bytes = r16(static_cast<uint64_t>(k) * 2);
  l.gh_bytes = r16(static_cast<uint64_t>(d) * 2);
  return l;
}

// ROWS = D / 4 weight rows per CTA (the 4 CTAs of a cluster cover one head).
template <int ROWS>
__global__ void __cluster_dims__(kQkvCluster, 1, 1) __launch_bounds__(kMmaThreads, 2)
    qkv_fused_kernel(QkvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t sbar, gbar;
  __shared__ uint16_t head_out[kMmaMaxM][kMaxHeadDim];
  __shared__ float2 rope_cs[kMmaMaxM][kMaxHeadDim / 2];
  __shared__ double red[kMmaWarps];
  __shared__ float escale[kMmaMaxM];
  __shared__ float red_small[kMmaMaxM * kMmaWarps];
  __shared__ float outv[ROWS * 8];
  __shared__ float redf[2 * kMmaWarps];
  __shared__ double redd[2 * kMmaWarps];
  [[maybe_unused]] constexpr unsigned kPhaseBase = 0;
  NVFP4DA_PHASE(0);
  // Nothing the dependent attention kernel reads before its own dependency
  // wait (cache rows below P_b, past lengths) is written here, so let it
  // launch at once and prefetch while this kernel streams its weights.
  if (p.pdl) pdl_launch_dependents();

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t unit = blockIdx.x / kQkvCluster;
  const int64_t d = p.head_dim, k = p.hidden;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

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
  const int64_t n_rows = (mat == 0 ? p.q_heads : p.kv_heads) * d;
  const int64_t row0 = head * d + static_cast<int64_t>(rank) * ROWS;
  const int valid_rows = static_cast<int>((n_rows - row0) < ROWS ? (n_rows - row0) : ROWS);
  const bool leader = (rank == 0);
  const int mg = static_cast<int>(p.m < kMmaMaxM ? p.m : kMmaMaxM);
  const uint8_t* packed_row0 = p.packed[mat] + row0 * (k / 2);

  const QkvSmemLayout lay = qkv_layout(ROWS, k, d, mg);
  uint8_t* s_smem = smem + lay.g.s_off();
  uint16_t* x_stage = reinterpret_cast<uint16_t*>(smem + lay.g.xs_off());
  __half* x16 = reinterpret_cast<__half*>(smem + lay.g.x16_off());
  const bool aliased = reinterpret_cast<const void*>(x16) == reinterpret_cast<const void*>(x_stage);
  float* mred = reinterpret_cast<float*>(smem + lay.g.red_off());
  uint16_t* gin_s = reinterpret_cast<uint16_t*>(smem + lay.gin_off());
  uint16_t* gq_s = reinterpret_cast<uint16_t*>(smem + lay.gq_off());
  uint16_t* gk_s = reinterpret_cast<uint16_t*>(smem + lay.gk_off());

  if (threadIdx.x == 0) {
    mbar_init(&sbar, 1);
    mbar_init(&gbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- Before the programmatic-dependency wait: everything that no earlier
  // kernel writes.  Gains (needed first) and scales by bulk copy, the first
  // batch of weight bytes into registers, gamma, and the RoPE table when the
  // positions are a host scalar.
  const bool gains_bulk = aligned16(p.g_in) && aligned16(p.g_q) && aligned16(p.g_k) && (k * 2) % 16 == 0 &&
                          (d * 2) % 16 == 0;
  if (gains_bulk && threadIdx.x == 0) {
    mbar_arrive_expect_tx(&gbar, static_cast<uint32_t>(k * 2 + 2 * d * 2));
    bulk_g2s(gin_s, p.g_in, static_cast<uint32_t>(k * 2), &gbar);
    bulk_g2s(gq_s, p.g_q, static_cast<uint32_t>(d * 2), &gbar);
    bulk_g2s(gk_s, p.g_k, static_cast<uint32_t>(d * 2), &gbar);
  }
  const bool sbulk = stage_scales(s_smem, p.scales[mat], k, row0, valid_rows, &sbar);
  const WarpSlice wsl = warp_slice(ROWS, k);
  constexpr int NB = 6;  // weight steps in flight per warp
  WeightRegs<NB> w;
  issue_weight_batch<NB>(w, packed_row0, k, wsl.tile, wsl.s0, wsl.s1, valid_rows);
  NVFP4DA_PHASE(1);
  const float gamma = *p.gamma[mat];
  const bool table_early = leader && mat < 2 && p.past_lengths == nullptr;
  auto fill_rope_table = [&](int64_t m0, int mgv) {
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(mgv) * (d / 2); i += blockDim.x) {
      const int m = static_cast<int>(i / (d / 2));
      const int64_t pr = i % (d / 2);
      const int64_t mrow = m0 + m;
      const int64_t b = mrow / p.tokens, t = mrow % p.tokens;
      const int64_t pos = (p.past_lengths ? p.past_lengths[b] : p.past_length) + t;
      float c = 1.0f, sn = 0.0f;
      if (t < p.rope_rows) {
        const float2 cs = p.rope_host[t][pr];
        c = cs.x;
        sn = cs.y;
      } else if (pos != 0) {
        rope_cos_sin_denom(pos, p.rope_denom[pr], c, sn);
      }
      rope_cs[m][pr] = make_float2(c, sn);
    }
  };
  if (table_early) fill_rope_table(0, mg);
  // Register path for the activation rows (K <= 4096): the gain's chunks
  // are constants, so load them now.
  constexpr int NCH = 2;
  const bool reg_path = (k / 8) <= NCH * kMmaThreads && aligned16(p.x) && aligned16(p.g_in);
  uint4 gch[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int idx = threadIdx.x + c * kMmaThreads;
    gch[c] = (reg_path && idx < k / 8) ? ldg_stream(p.g_in + 8 * idx) : make_uint4(0u, 0u, 0u, 0u);
  }
  NVFP4DA_PHASE(2);

  if (p.pdl) pdl_wait();
  if (blockIdx.x == 0)
    for (int64_t i = threadIdx.x; i < p.n_zero_words; i += blockDim.x) p.zero_words[i] = 0u;
  bool ok = true;
  if (!gains_bulk) {
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) gin_s[i] = p.g_in[i];
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
      gq_s[i] = p.g_q[i];
      gk_s[i] = p.g_k[i];
    }
  }
  bool gains_ready = !gains_bulk;
  bool scales_ready = !sbulk;
  uint16_t* leader_out = cluster.map_shared_rank(&head_out[0][0], 0);
  NVFP4DA_PHASE(3);

  const int kv8 = static_cast<int>(k / 8);
  for (int64_t m0 = 0; m0 < p.m; m0 += kMmaMaxM) {
    const int mgv = static_cast<int>((p.m - m0) < kMmaMaxM ? (p.m - m0) : kMmaMaxM);
    __syncthreads();  // staging buffers (and the RoPE table) are free again
    if (m0 > 0) issue_weight_batch<NB>(w, packed_row0, k, wsl.tile, wsl.s0, wsl.s1, valid_rows);
    if (leader && mat < 2 && !(table_early && m0 == 0)) fill_rope_table(m0, mgv);
    bool f16;
    if (reg_path) {
      if (!gains_ready) {
        ok = mbar_wait_bounded(&gbar, 0, p.err) && ok;
        gains_ready = true;
      }
      NVFP4DA_PHASE(4);
      f16 = (mgv > 1 || aliased) ? prep_rows_warp<true>(p.x + m0 * k, gin_s, k, mgv, p.eps, x_stage, x16, escale,
                                           (p.dbg_xnorm && blockIdx.x == 0) ? p.dbg_xnorm + m0 * k : nullptr)
                    : prep_rows_regs<NCH, true>(p.x + m0 * k, k, mgv, gch, p.eps, x_stage, x16, escale, redf, redd,
                                      (p.dbg_xnorm && blockIdx.x == 0) ? p.dbg_xnorm + m0 * k : nullptr);
    } else {
      load_rows_lsu(x_stage, p.x + m0 * k, static_cast<int64_t>(mgv) * k);
      if (!gains_ready) {
        ok = mbar_wait_bounded(&gbar, 0, p.err) && ok;
        gains_ready = true;
      }
      __syncthreads();
      NVFP4DA_PHASE(4);
      // ---- input RMSNorm (reference/decoder_attention.py:117-140), in place in x_stage
      for (int m = 0; m < mgv; ++m) {
        uint4* xr = reinterpret_cast<uint4*>(x_stage + static_cast<int64_t>(m) * k);
        double ss = 0.0;
        for (int i = threadIdx.x; i < kv8; i += blockDim.x) {
          const uint4 v = xr[i];
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a = __uint_as_float(wv[j] << 16), b = __uint_as_float(wv[j] & 0xffff0000u);
            ss += static_cast<double>(a * a) + static_cast<double>(b * b);
          }
        }
        ss = warp_sum_f64(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int ww = 0; ww < kMmaWarps; ++ww) tot += red[ww];
        const float inv = rms_inverse(static_cast<float>(tot), static_cast<float>(k), p.eps);
        const uint4* gv = reinterpret_cast<const uint4*>(gin_s);
        for (int i = threadIdx.x; i < kv8; i += blockDim.x) {
          const uint4 v = xr[i], gg = gv[i];
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w}, wg[4] = {gg.x, gg.y, gg.z, gg.w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t lo = f32_to_bf16_bits(__fmul_rn(__fmul_rn(__uint_as_float(wv[j] << 16), inv),
                                                           __uint_as_float(wg[j] << 16)));
            const uint32_t hi = f32_to_bf16_bits(__fmul_rn(__fmul_rn(__uint_as_float(wv[j] & 0xffff0000u), inv),
                                                           __uint_as_float(wg[j] & 0xffff0000u)));
            o[j] = lo | (hi << 16);
          }
          const uint4 nv = make_uint4(o[0], o[1], o[2], o[3]);
          xr[i] = nv;
          if (p.dbg_xnorm && blockIdx.x == 0) reinterpret_cast<uint4*>(p.dbg_xnorm + (m0 + m) * k)[i] = nv;
        }
        __syncthreads();
      }
      // With one staging buffer the f16 operand would overwrite the BF16 rows
      // before their exactness is known: the BF16 operand then.
      f16 = aliased ? false : mma_prepare_f16(x_stage, x16, k, mgv, escale, red_small);
    }
    NVFP4DA_PHASE(5);
    if (!scales_ready) {
      ok = mbar_wait_bounded(&sbar, 0, p.err) && ok;
      scales_ready = true;
    }
    NVFP4DA_PHASE(6);
    if (f16)
      mma_gemv_pass<true, NB>(w, packed_row0, s_smem, reinterpret_cast<const uint16_t*>(x16), k, ROWS, valid_rows,
                              mgv, mred, outv);
    else
      mma_gemv_pass<false, NB>(w, packed_row0, s_smem, x_stage, k, ROWS, valid_rows, mgv, mred, outv);
    for (int i = threadIdx.x; i < ROWS * mgv; i += blockDim.x) {
      const int n = i / ROWS, r = i % ROWS;
      const float v = f16 ? outv[r * 8 + n] * escale[n] : outv[r * 8 + n];
      leader_out[n * kMaxHeadDim + rank * ROWS + r] = ok ? f32_to_bf16_bits(__fmul_rn(v, gamma)) : uint16_t(0x7fc0);
    }
    NVFP4DA_PHASE(7);
    cluster.sync();
    NVFP4DA_PHASE(8);

    if (leader && warp < mgv) {
      // ---- head epilogue for activation row m0 + warp
      const int64_t mrow = m0 + warp;
      const int64_t b = mrow / p.tokens, t = mrow % p.tokens;
      const int64_t pos = (p.past_lengths ? p.past_lengths[b] : p.past_length) + t;
      // A per-sequence length read from device memory cannot be checked on the
      // host: a slot outside [0, C) is not written (the caller's contract is
      // 0 <= P_b and P_b + T <= C).
      const int64_t slot = pos - p.slot_offset;  // cache slot of this position in this shard
      const bool slot_ok = slot >= 0 && slot < p.capacity;
      const uint16_t* y = head_out[warp];
      if (mat == 2) {
        uint16_t* dst = slot_ok ? p.v_cache + ((b * p.kv_heads + head) * p.capacity + slot) * d : nullptr;
        for (int64_t e = lane; e < d; e += 32) {
          if (dst) dst[e] = y[e];
          if (p.dbg_v) p.dbg_v[mrow * p.kv_heads * d + head * d + e] = y[e];
        }
      } else {
        const uint16_t* g = (mat == 0) ? gq_s : gk_s;
        double ss = 0.0;
        for (int64_t e = lane; e < d; e += 32) {
          const float v = bf16_bits_to_f32(y[e]);
          ss += static_cast<double>(v * v);
        }
        ss = warp_sum_f64(ss);
        const float inv = rms_inverse(static_cast<float>(ss), static_cast<float>(d), p.eps);
        const int64_t heads = (mat == 0) ? p.q_heads : p.kv_heads;
        uint16_t* dbg_proj = (mat == 0) ? p.dbg_q : p.dbg_k;
        uint16_t* dbg_norm = (mat == 0) ? p.dbg_qn : p.dbg_kn;
        uint16_t* dst = (mat == 0) ? p.q_out + (mrow * p.q_heads + head) * d
                        : slot_ok  ? p.k_cache + ((b * p.kv_heads + head) * p.capacity + slot) * d
                                   : nullptr;
        for (int64_t pr = lane; pr < d / 2; pr += 32) {
          const int64_t e = 2 * pr;
          const uint16_t n0 = f32_to_bf16_bits(
              __fmul_rn(__fmul_rn(bf16_bits_to_f32(y[e]), inv), bf16_bits_to_f32(g[e])));
          const uint16_t n1 = f32_to_bf16_bits(
              __fmul_rn(__fmul_rn(bf16_bits_to_f32(y[e + 1]), inv), bf16_bits_to_f32(g[e + 1])));
          if (dbg_proj) {
            dbg_proj[mrow * heads * d + head * d + e] = y[e];
            dbg_proj[mrow * heads * d + head * d + e + 1] = y[e + 1];
          }
          if (dbg_norm) {
            dbg_norm[mrow * heads * d + head * d + e] = n0;
            dbg_norm[mrow * heads * d + head * d + e + 1] = n1;
          }
          uint16_t r0 = n0, r1 = n1;
          if (pos != 0) {
            const float2 cs = rope_cs[warp][pr];
            rope_pair(bf16_bits_to_f32(n0), bf16_bits_to_f32(n1), cs.x, cs.y, r0, r1);
          }
          if (dst) {
            dst[e] = r0;
            dst[e + 1] = r1;
          }
        }
      }
    }
    NVFP4DA_PHASE(9);
    // head_out is reused by the next activation group.  After the last group
    // nothing reads another CTA's shared memory any more, so no barrier.
    if (m0 + kMmaMaxM < p.m) cluster.sync();
    NVFP4DA_PHASE(10);
  }
}

}  // namespace nvfp4da
