// Split-KV flash-decoding causal GQA over the physical BF16 cache [B, Hkv, C, D].
//
// Semantics (reference/decoder_attention.py:273-381, src/gqa_attention_cached.cu):
//   query head h reads KV head h / (Hq/Hkv); token t of sequence b sees keys
//   j <= P_b + t; score = FP32(q . k) * FP32(1/sqrt(D)); softmax in FP32;
//   context = BF16(sum_j p_j v_j).  K/V rows are addressed with the physical
//   capacity C as the head stride; slots beyond P_b + t are never read.
//
// Work decomposition: one CTA per (split, kv head x head group, b*T + t).  The
// CTA's GH query heads share every K/V row it loads.  Four warps walk the
// split's positions in chunks of NPOS = min(8, 32/GH) rows; lane l holds
// elements [l*EPL, l*EPL+EPL) of q, k and v.  Per chunk the NPOS x GH partial
// dot products are summed across lanes with a butterfly reduce-scatter (31
// shuffles), after which lane l owns the score of (row l/GH, head l%GH).
// Softmax is online (running max and sum per head, FP32).  Splits combine
// with the log-sum-exp rule in one of two ways: when a (b, t, head group) has
// at most 16 splits they form one thread-block cluster and combine through
// distributed shared memory after a cluster barrier; otherwise every split
// writes (m, l, o) to the workspace and the last CTA to finish — detected with
// an atomic counter, no waiting — combines them.  No score or probability
// tensor is materialised.
#pragma once

#include <math.h>

#include <cooperative_groups.h>

#include "common.cuh"

namespace nvfp4da {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * kWarp;

struct AttnParams {
  const uint16_t* q;        // [B, T, Hq, D]
  const uint16_t* k_cache;  // [B, Hkv, C, D]
  const uint16_t* v_cache;
  uint16_t* ctx;  // [B, T, Hq, D]
  int64_t batch, tokens, q_heads, kv_heads, capacity, head_dim;
  int64_t past_length;          // used when past_lengths == nullptr
  const int64_t* past_lengths;  // optional device [B]
  int64_t split_len;            // positions per split (multiple of 32)
  int splits;
  int head_groups;  // (Hq/Hkv) / GH
  float scale;      // FP32(1/sqrt(D))
  float* partials;  // [B*T*Hq][splits][D + 2]  (o[D], m, l)   (global combine only)
  unsigned* counters;  // [B*T*Hkv*head_groups], zero on entry, left zero on exit
  int pdl;
  int cluster_combine;  // 1: the `splits` CTAs of a (b, t, head group) form one
                        // thread-block cluster and combine through DSMEM
  // KV-length sharding: the caches hold global positions [pos_offset,
  // pos_offset + capacity) of each sequence; a query at global position P_b + t
  // sees the local slots below P_b + t + 1 - pos_offset.  With out_partial set,
  // the result is this shard's log-sum-exp partial instead of the context:
  // out_partial[row][0..D) = sum_j exp(s_j - m) v_j (unnormalised), [D] = m,
  // [D + 1] = l = sum_j exp(s_j - m); a shard with no visible key gives
  // m = -inf, l = 0, o = 0.
  int64_t pos_offset;
  float* out_partial;  // [B*T*Hq][D + 2] or nullptr
};

// Final write of one (row, element): the BF16 context, or the shard partial.
__device__ __forceinline__ void attn_store(const AttnParams& p, int64_t row, int64_t e, float o, float m, float l) {
  if (p.out_partial) {
    float* dst = p.out_partial + row * (p.head_dim + 2);
    dst[e] = o;
    if (e == 0) {
      dst[p.head_dim] = m;
      dst[p.head_dim + 1] = l;
    }
  } else {
    p.ctx[row * p.head_dim + e] = f32_to_bf16_bits(__fdiv_rn(o, l));
  }
}

template <int EPL>
__device__ __forceinline__ void load_row(const uint16_t* row, int lane, int64_t d, float (&out)[EPL]) {
  if (lane * EPL < d) {
    const uint16_t* p = row + lane * EPL;
    if constexpr (EPL == 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(p);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else if constexpr (EPL == 4) {
      const uint2 v = *reinterpret_cast<const uint2*>(p);
      out[0] = __uint_as_float(v.x << 16);
      out[1] = __uint_as_float(v.x & 0xffff0000u);
      out[2] = __uint_as_float(v.y << 16);
      out[3] = __uint_as_float(v.y & 0xffff0000u);
    } else if constexpr (EPL == 2) {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
      out[0] = __uint_as_float(v << 16);
      out[1] = __uint_as_float(v & 0xffff0000u);
    } else {
      out[0] = bf16_bits_to_f32(*p);
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = 0.0f;
  }
}

// Butterfly reduce-scatter of 32 per-lane values: afterwards lane l holds the
// sum over all lanes of v[l].
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = upper ? v[i] : v[i + s];
      const float keep = upper ? v[i + s] : v[i];
      v[i] = keep + __shfl_xor_sync(kFull, send, s);
    }
  }
  return v[0];
}

__device__ __forceinline__ int64_t seq_past(const AttnParams& p, int64_t b) {
  return p.past_lengths ? p.past_lengths[b] : p.past_length;
}

template <int EPL, int GH>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnParams p) {
  // Rows per warp chunk; NPOS * GH <= 32 dot products go through one
  // butterfly (unused slots are zero).  Capped at 8 rows to bound registers.
  constexpr int NPOS = (32 / GH) > 8 ? 8 : (32 / GH);
  constexpr int NDOT = NPOS * GH;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.head_groups;
  const int hg = blockIdx.y % p.head_groups;
  const int64_t bt = blockIdx.z;
  const int64_t b = bt / p.tokens;
  const int64_t t = bt % p.tokens;
  const int64_t d = p.head_dim;
  const int64_t group = p.q_heads / p.kv_heads;
  const int64_t h0 = static_cast<int64_t>(kvh) * group + static_cast<int64_t>(hg) * GH;

  // This kernel reads nothing before its dependency wait that its dependent
  // (the O projection, which prefetches only weights) writes, so it lets the
  // dependent launch at once.
  [[maybe_unused]] constexpr unsigned kPhaseBase = 1024;
  NVFP4DA_PHASE(0);
  if (p.pdl) pdl_launch_dependents();

  // Keys 0 .. P_b + t; never read beyond the physical capacity, whatever a
  // device-side length says.
  const int64_t pb = seq_past(p, b) - p.pos_offset;  // this shard's slot of position P_b
  int64_t visible = pb + t + 1;
  if (visible > p.capacity) visible = p.capacity;
  const int64_t s0 = static_cast<int64_t>(split) * p.split_len;
  int64_t s1 = s0 + p.split_len;
  if (s1 > visible) s1 = visible;

  const uint16_t* kbase = p.k_cache + (b * p.kv_heads + kvh) * p.capacity * d;
  const uint16_t* vbase = p.v_cache + (b * p.kv_heads + kvh) * p.capacity * d;

  // Before waiting on the kernel that produced q (the fused QKV kernel, which
  // writes only slots >= P_b), prefetch this warp's first chunk of cache rows
  // below P_b.  Rows at or above P_b are loaded after the wait.
  float kr[NPOS][EPL], vr[NPOS][EPL];
  int64_t c0 = s0 + static_cast<int64_t>(warp) * NPOS;
#pragma unroll
  for (int j = 0; j < NPOS; ++j) {
    const int64_t pos = c0 + j;
    if (pos < s1 && pos < pb) {
      load_row<EPL>(kbase + pos * d, lane, d, kr[j]);
      load_row<EPL>(vbase + pos * d, lane, d, vr[j]);
    } else {
#pragma unroll
      for (int e = 0; e < EPL; ++e) kr[j][e] = vr[j][e] = 0.0f;
    }
  }
  NVFP4DA_PHASE(1);
  if (p.pdl) pdl_wait();
  NVFP4DA_PHASE(2);

  // q for GH heads, this lane's slice.
  float q[GH][EPL];
#pragma unroll
  for (int g = 0; g < GH; ++g) load_row<EPL>(p.q + ((bt * p.q_heads) + h0 + g) * d, lane, d, q[g]);

  float m_run[GH], l_run[GH], acc[GH][EPL];
#pragma unroll
  for (int g = 0; g < GH; ++g) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[g][e] = 0.0f;
  }

  for (bool first = true; c0 < s1; c0 += kAttnWarps * NPOS, first = false) {
#pragma unroll
    for (int j = 0; j < NPOS; ++j) {
      const int64_t pos = c0 + j;
      const bool need = pos < s1 && (!first || pos >= pb);
      if (need) {
        load_row<EPL>(kbase + pos * d, lane, d, kr[j]);
        load_row<EPL>(vbase + pos * d, lane, d, vr[j]);
      } else if (!first) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) kr[j][e] = vr[j][e] = 0.0f;
      }
    }
    float dots[32];
#pragma unroll
    for (int i = NDOT; i < 32; ++i) dots[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < NPOS; ++j)
#pragma unroll
      for (int g = 0; g < GH; ++g) {
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) s = fmaf(q[g][e], kr[j][e], s);
        dots[j * GH + g] = s;
      }
    const float dot = reduce_scatter32(dots, lane);
    const int my_j = lane / GH;
    const int my_g = lane % GH;
    const bool valid = lane < NDOT && (c0 + my_j) < s1;
    const float score = valid ? __fmul_rn(dot, p.scale) : -INFINITY;
    // chunk max per head (lanes sharing my_g)
    float cmax = score;
#pragma unroll
    for (int o = GH; o < 32; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(kFull, cmax, o));
    float m_old_mine = m_run[0];
#pragma unroll
    for (int g = 1; g < GH; ++g)
      if (my_g == g) m_old_mine = m_run[g];
    const float m_new_mine = fmaxf(m_old_mine, cmax);  // finite: chunk has >= 1 valid row
    const float pexp = valid ? expf(score - m_new_mine) : 0.0f;
    float psum = pexp;
#pragma unroll
    for (int o = GH; o < 32; o <<= 1) psum += __shfl_xor_sync(kFull, psum, o);
    const float alpha_mine = (m_old_mine == -INFINITY) ? 0.0f : expf(m_old_mine - m_new_mine);
#pragma unroll
    for (int g = 0; g < GH; ++g) {
      const float alpha = __shfl_sync(kFull, alpha_mine, g);
      const float mnew = __shfl_sync(kFull, m_new_mine, g);
      const float ps = __shfl_sync(kFull, psum, g);
      m_run[g] = mnew;
      l_run[g] = fmaf(l_run[g], alpha, ps);
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] *= alpha;
    }
#pragma unroll
    for (int j = 0; j < NPOS; ++j)
#pragma unroll
      for (int g = 0; g < GH; ++g) {
        const float pj = __shfl_sync(kFull, pexp, j * GH + g);
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(pj, vr[j][e], acc[g][e]);
      }
  }

  NVFP4DA_PHASE(3);
  // ---- combine the four warps of this CTA
  __shared__ float sm_m[kAttnWarps][GH], sm_l[kAttnWarps][GH];
  __shared__ float sm_o[kAttnWarps][GH][32 * EPL];
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GH; ++g) {
      sm_m[warp][g] = m_run[g];
      sm_l[warp][g] = l_run[g];
    }
  }
#pragma unroll
  for (int g = 0; g < GH; ++g)
#pragma unroll
    for (int e = 0; e < EPL; ++e) sm_o[warp][g][lane * EPL + e] = acc[g][e];
  __syncthreads();

  // Per-head rescale factors of the four warps, computed once.
  __shared__ float wf[kAttnWarps][GH], cta_m[GH], cta_l[GH];
  if (threadIdx.x < GH) {
    const int g = threadIdx.x;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, sm_m[w][g]);
    float l = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = (sm_m[w][g] == -INFINITY) ? 0.0f : expf(sm_m[w][g] - mx);
      wf[w][g] = f;
      l = fmaf(sm_l[w][g], f, l);
    }
    cta_m[g] = mx;
    cta_l[g] = l;
  }
  __syncthreads();

  // thread i handles element i of head g for i < d (loop over heads)
  float* part_base = p.partials;
  const bool single = (p.splits == 1);
  __shared__ float cta_o[GH][32 * EPL];
  for (int idx = threadIdx.x; idx < GH * 32 * EPL; idx += kAttnThreads) {
    const int g = idx / (32 * EPL);
    const int e = idx % (32 * EPL);
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) o = fmaf(sm_o[w][g][e], wf[w][g], o);
    if (p.cluster_combine) {
      cta_o[g][e] = o;
      continue;
    }
    if (e >= d) continue;
    const int64_t row = bt * p.q_heads + h0 + g;
    if (single) {
      attn_store(p, row, e, o, cta_m[g], cta_l[g]);
    } else {
      float* dst = part_base + (row * p.splits + split) * (d + 2);
      dst[e] = o;
      if (e == 0) {
        dst[d] = cta_m[g];
        dst[d + 1] = cta_l[g];
      }
    }
  }
  if (single) return;

  if (p.cluster_combine) {
    // ---- the splits of this (b, t, head group) are one cluster: combine the
    // CTAs' (m, l, o) through distributed shared memory.  Every CTA first
    // gathers all ranks' (m, l) (independent remote loads), turns them into
    // rescale weights, then finalises its slice of the GH x D outputs with one
    // independent remote load per rank and element.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int ns = static_cast<int>(cluster.num_blocks());
    const int rank = static_cast<int>(cluster.block_rank());
    __shared__ float rw[16][GH], rl[16][GH], head_inv_l[GH], head_mx[GH];
    NVFP4DA_PHASE(4);
    cluster.sync();
    NVFP4DA_PHASE(5);
    for (int i = threadIdx.x; i < ns * GH; i += kAttnThreads) {
      const int r = i / GH, g = i % GH;
      rw[r][g] = *cluster.map_shared_rank(&cta_m[g], r);
      rl[r][g] = *cluster.map_shared_rank(&cta_l[g], r);
    }
    __syncthreads();
    if (threadIdx.x < GH) {
      const int g = threadIdx.x;
      float mx = -INFINITY;
      for (int r = 0; r < ns; ++r) mx = fmaxf(mx, rw[r][g]);
      float l = 0.0f;
      for (int r = 0; r < ns; ++r) {
        const float f = (rw[r][g] == -INFINITY) ? 0.0f : expf(rw[r][g] - mx);
        rw[r][g] = f;
        l = fmaf(rl[r][g], f, l);
      }
      head_inv_l[g] = l;
      head_mx[g] = mx;
    }
    __syncthreads();
    const int total = GH * static_cast<int>(d);
    const int per = (total + ns - 1) / ns;
    for (int idx = rank * per + threadIdx.x; idx < total && idx < (rank + 1) * per; idx += kAttnThreads) {
      const int g = idx / static_cast<int>(d);
      const int e = idx % static_cast<int>(d);
      float vals[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) vals[r] = r < ns ? *cluster.map_shared_rank(&cta_o[g][e], r) : 0.0f;
      float o = 0.0f;
#pragma unroll
      for (int r = 0; r < 16; ++r)
        if (r < ns) o = fmaf(vals[r], rw[r][g], o);
      attn_store(p, bt * p.q_heads + h0 + g, e, o, head_mx[g], head_inv_l[g]);
    }
    NVFP4DA_PHASE(6);
    cluster.sync();  // keep this CTA's shared memory alive until its peers are done
    NVFP4DA_PHASE(7);
    return;
  }

  // ---- last CTA of this (b, t, head group) combines all splits.
  __shared__ unsigned s_last;
  __shared__ float head_l[GH], head_m[GH];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned idx = static_cast<unsigned>(bt * (p.kv_heads * p.head_groups) + blockIdx.y);
    const unsigned prev = atomicAdd(&p.counters[idx], 1u);
    s_last = (prev == static_cast<unsigned>(p.splits - 1)) ? 1u : 0u;
    if (s_last) p.counters[idx] = 0u;  // leave zero for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Stage every split's (m, l) for the GH heads in shared memory (sm_o is free
  // now; the host caps splits at 64 * EPL so 2 * GH * splits floats fit), then
  // turn m into the rescale weights exp(m_s - M).
  const int ns = p.splits;
  float* sw = &sm_o[0][0][0];
  float* sl = sw + GH * ns;
  for (int i = threadIdx.x; i < GH * ns; i += kAttnThreads) {
    const int g = i / ns, sp = i % ns;
    const float* src = part_base + ((bt * p.q_heads + h0 + g) * ns + sp) * (d + 2);
    sw[i] = __ldcg(src + d);
    sl[i] = __ldcg(src + d + 1);
  }
  __syncthreads();
  for (int g = warp; g < GH; g += kAttnWarps) {
    float mx = -INFINITY;
    for (int sp = lane; sp < ns; sp += 32) mx = fmaxf(mx, sw[g * ns + sp]);
    mx = warp_max_f32(mx);
    float l = 0.0f;
    for (int sp = lane; sp < ns; sp += 32) {
      const float ms = sw[g * ns + sp];
      const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
      sw[g * ns + sp] = f;
      l = fmaf(sl[g * ns + sp], f, l);
    }
    l = warp_sum_f32(l);
    if (lane == 0) {
      head_l[g] = l;
      head_m[g] = mx;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < GH * d; idx += kAttnThreads) {
    const int g = static_cast<int>(idx / d);
    const int64_t e = idx % d;
    const int64_t row = bt * p.q_heads + h0 + g;
    const float* src = part_base + row * ns * (d + 2) + e;
    float o = 0.0f;
#pragma unroll 8
    for (int sp = 0; sp < ns; ++sp) o = fmaf(__ldcg(src + sp * (d + 2)), sw[g * ns + sp], o);
    attn_store(p, row, e, o, head_m[g], head_l[g]);
  }
}

// Log-sum-exp combine of the per-shard partials of KV-length-sharded
// attention: partials [G][rows][D + 2] (o unnormalised, m, l) ->
// ctx[rows][D] = BF16( sum_r o_r e^(m_r - M) / sum_r l_r e^(m_r - M) ),
// shards in order.  One warp per row.
__global__ void attn_combine_kernel(const float* partials, int shards, int64_t rows, int64_t d, uint16_t* ctx) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t stride = rows * (d + 2);
  float mx = -INFINITY;
  for (int r = 0; r < shards; ++r) mx = fmaxf(mx, partials[r * stride + row * (d + 2) + d]);
  float l = 0.0f;
  for (int r = 0; r < shards; ++r) {
    const float* src = partials + r * stride + row * (d + 2);
    const float f = (src[d] == -INFINITY) ? 0.0f : expf(src[d] - mx);
    l = fmaf(src[d + 1], f, l);
  }
  for (int64_t e = lane; e < d; e += 32) {
    float o = 0.0f;
    for (int r = 0; r < shards; ++r) {
      const float* src = partials + r * stride + row * (d + 2);
      const float f = (src[d] == -INFINITY) ? 0.0f : expf(src[d] - mx);
      o = fmaf(src[e], f, o);
    }
    ctx[row * d + e] = f32_to_bf16_bits(__fdiv_rn(o, l));
  }
}

}  // namespace nvfp4da
