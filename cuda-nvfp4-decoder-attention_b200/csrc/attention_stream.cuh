// Long-context split-KV decode attention: a persistent, TMA-fed tensor-core
// kernel that streams the physical BF16 cache [B, Hkv, C, D] at HBM rate.
//
// Semantics are those of attn_split_kernel (reference
// reference/decoder_attention.py:273-381, src/gqa_attention_cached.cu:93-337):
// query head h reads KV head h / group; token t of sequence b sees the keys
// j <= P_b + t; score = FP32(q . k) * FP32(1/sqrt(D)); softmax in FP32 with a
// log-sum-exp combine of the pieces; context = BF16(sum_j p_j v_j / sum_j p_j).
//
// Work decomposition.  Every (sequence b, KV head) pair owns ceil(S_b / 64)
// tiles of 64 positions (S_b = the positions any of its queries sees).  All
// pairs' tiles are laid end to end (b-major, then KV head, then position) and
// the grid -- one CTA per SM -- cuts that line into equal contiguous ranges, so
// every SM streams the same number of bytes whatever the per-sequence lengths.
// A CTA walks its range as segments (the part of one pair inside it); the
// (pair p, CTA c) segment writes its log-sum-exp partial to slot p + c, which
// is unique (the boundaries of pairs and of CTAs interleave).  The last CTA
// of a pair to finish -- an atomic counter, no waiting -- combines its pair's
// partials in CTA order.
//
// Per CTA: warp 8 (one lane) issues the TMA loads of K and V tiles (64 rows x
// 64 elements per box, 128-byte swizzle, so ldmatrix reads are conflict-free)
// into a ring of kStages stages, running ahead across segment boundaries;
// two groups of four consumer warps take alternate tiles (the CTA's n-th tile
// goes to group n % 2), each warp 16 positions of its group's tiles.  With
// one group the per-tile dependency chain (S^T MMAs, softmax, PV MMAs) set
// the pace below the HBM rate.  One KV head's queries
// (group x T <= 8 rows) are the N = 8 side of the tensor-core tiles:
//   S^T[pos, q]  = K[pos, :] . Q^T      mma.m16n8k16, BF16 x BF16 -> FP32
//   O^T[d, q]   += V^T[d, pos] P^T      P split as BF16 hi + lo (two MMAs),
// so every product is exact in FP32 and P keeps ~16 significant bits; the
// online softmax runs on the accumulator fragments (the layouts of the two
// MMAs line up through one movmatrix.trans per 8 x 8 block of P).  No score or
// probability tensor is materialised.
//
// Waits are bounded: a stage barrier that does not complete within 2^22 tries
// records kErrBarrierTimeout in *err and the kernel stops waiting (its results
// are then garbage; the GPU stays usable).
#pragma once

#include <cuda.h>
#include <math.h>

#include "attention_prefill.cuh"  // ldsm_x4, ldsm_x4_t, mma_bf16_16816
#include "common.cuh"
#include "prefill_gemm.cuh"  // tma_load_2d, mbar_arrive

namespace nvfp4da {

constexpr int kAsTile = 64;            // positions per stage
constexpr int kAsGroupWarps = 4;       // 16 positions of a tile each
constexpr int kAsConsumerWarps = 8;    // two groups, alternate tiles
constexpr int kAsThreads = (kAsConsumerWarps + 1) * 32;
constexpr int kAsRows = 8;             // query rows per KV head (the MMA's N)
constexpr uint32_t kAsBox = kAsTile * 128;  // one 64-row x 64-element box: 8 KB
constexpr int kAsMaxBatch = 1024;

template <int D>
struct AsCfg {
  static_assert(D == 64 || D == 128 || D == 256, "head_dim 64, 128 or 256");
  static constexpr int kBoxes = D / 64;                     // boxes per K (or V) tile
  static constexpr uint32_t kStage = 2 * kBoxes * kAsBox;   // K + V bytes per stage
  static constexpr uint32_t kComb = kAsConsumerWarps * kAsRows * D * 4;  // per-warp O^T for the combine
  // Stages in flight: what is left of 217 KB after the combine area (the
  // rest holds the alignment slack and up to kAsMaxBatch sequences' prefix).
  static constexpr int kStagesFit = static_cast<int>((217u * 1024 - kComb) / kStage);
  // An even count: the CTA's n-th tile goes to stage n % kStages and consumer
  // group n % 2, so every stage serves one group only.  (With an odd count a
  // group one ring ahead of the other would wait on a stage whose previous
  // phase -- the other group's tile, still landing -- already reads as
  // complete: the parity wait cannot tell the two apart.)
  static constexpr int kStages = (kStagesFit > 12 ? 12 : kStagesFit) & ~1;  // 12, 4 or 2
  static_assert(kStages >= 2, "two stages at least");
  static constexpr uint32_t kRing = kStages * kStage;
  // ring (1024-aligned) + combine + m/l + barriers; the per-sequence tile
  // prefix (int64 [B + 1]) follows.
  static constexpr uint32_t kOffComb = kRing;
  static constexpr uint32_t kOffMl = kOffComb + kComb;                       // [2][warps][rows] f32
  static constexpr uint32_t kOffBar = kOffMl + 2 * kAsConsumerWarps * kAsRows * 4;
  static constexpr uint32_t kOffPrefix = kOffBar + 2 * kStages * 8 + 64;
  static constexpr uint32_t bytes(int batch) { return kOffPrefix + 8u * (batch + 1) + 1024; }
};

struct StreamAttnParams {
  const uint16_t* q;      // [B, T, Hq, D]
  uint16_t* ctx;          // [B, T, Hq, D] (context mode)
  float* out_partial;     // [B*T*Hq][D + 2] (shard-partial mode) or nullptr
  int batch, tokens, q_heads, kv_heads, group;
  int64_t capacity;       // physical positions per (b, KV head) in the cache tensor
  int64_t past_length;    // used when past_lengths == nullptr
  const int64_t* past_lengths;
  int64_t pos_offset;     // global position of the cache's slot 0 (KV-length sharding)
  float scale;            // FP32(1/sqrt(D))
  float* partials;        // [(pairs + grid) slots][kAsRows][D + 2]
  unsigned* counters;     // [pairs], zero on entry, left zero on exit
  unsigned* err;
  int pdl;
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// BF16 pair (lo in the low half) of two FP32 values, round to nearest even.
__device__ __forceinline__ uint32_t as_pack_bf16(float lo, float hi) {
  return static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
}

// Local positions [0, limit) of pair's cache that query token t sees.
__device__ __forceinline__ int64_t as_limit(int64_t pb, int t, int64_t off, int64_t cap) {
  int64_t l = pb + t + 1 - off;
  return l < 0 ? 0 : (l > cap ? cap : l);
}

// The walk over one CTA's range [x, x_end) of the flattened tile line.
struct AsWalk {
  const long long* prefix;  // [B + 1]: tiles before sequence b (all its KV heads)
  int batch, hkv;
  long long x, x_end;
  int b, kvh;
  int t0, t1, nt;  // this segment's tiles [t0, t1) of nt in the pair
  __device__ bool begin(const long long* pre, int nb, int nh, long long x0, long long x1) {
    prefix = pre;
    batch = nb;
    hkv = nh;
    x = x0;
    x_end = x1;
    if (x >= x_end) return false;
    int lo = 0, hi = batch - 1;  // largest b with prefix[b] <= x
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= x) lo = mid;
      else hi = mid - 1;
    }
    b = lo;
    nt = static_cast<int>((prefix[b + 1] - prefix[b]) / hkv);
    const long long within = x - prefix[b];
    kvh = static_cast<int>(within / nt);
    t0 = static_cast<int>(within % nt);
    t1 = static_cast<int>(min(static_cast<long long>(nt), t0 + (x_end - x)));
    return true;
  }
  __device__ bool next() {
    x += t1 - t0;
    if (x >= x_end) return false;
    if (++kvh == hkv) {
      kvh = 0;
      do {
        ++b;
      } while (prefix[b + 1] == prefix[b]);
      nt = static_cast<int>((prefix[b + 1] - prefix[b]) / hkv);
    }
    t0 = 0;
    t1 = static_cast<int>(min(static_cast<long long>(nt), x_end - x));
    return true;
  }
};

// CTA (of G over N tiles, CTA c owning [c*N/G, (c+1)*N/G)) that holds tile x.
__device__ __forceinline__ int as_cta_of(long long x, long long n, int g) {
  return static_cast<int>(((x + 1) * g - 1) / n);
}

template <int D>
__global__ void __launch_bounds__(kAsThreads, 1)
    attn_stream_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const StreamAttnParams p) {
  using Cfg = AsCfg<D>;
  constexpr int KS = D / 16;  // MMA k-steps of QK, d m-tiles of PV
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* so = reinterpret_cast<float*>(smem + Cfg::kOffComb);            // [warp][row][D]
  float* sm_m = reinterpret_cast<float*>(smem + Cfg::kOffMl);            // [warp][row]
  float* sm_l = sm_m + kAsConsumerWarps * kAsRows;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty = full + Cfg::kStages;
  unsigned* s_flag = reinterpret_cast<unsigned*>(empty + Cfg::kStages);
  long long* prefix = reinterpret_cast<long long*>(smem + Cfg::kOffPrefix);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int T = p.tokens, hkv = p.kv_heads, group = p.group, nq = group * T;
  const int64_t cap = p.capacity, off = p.pos_offset;

  if (p.pdl) pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kAsGroupWarps);
    }
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_k)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_v)) : "memory");
  }
  // Tiles per sequence (all its KV heads), then the prefix over sequences.
  // The lengths are inputs of the step (not written by the kernel before this
  // one), so they are read before the dependency wait.
  for (int b = threadIdx.x; b < p.batch; b += blockDim.x) {
    const int64_t pb = p.past_lengths ? p.past_lengths[b] : p.past_length;
    const int64_t vis = as_limit(pb, T - 1, off, cap);
    prefix[b + 1] = ((vis + kAsTile - 1) / kAsTile) * hkv;
  }
  __syncthreads();
  if (warp == 0) {
    long long carry = 0;
    for (int base = 0; base < p.batch; base += 32) {
      const int b = base + lane;
      long long v = b < p.batch ? prefix[b + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long u = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += u;
      }
      if (b < p.batch) prefix[b + 1] = carry + v;
      carry += __shfl_sync(kFull, v, 31);
    }
    if (lane == 0) prefix[0] = 0;
  }
  __syncthreads();
  const long long n_tiles = prefix[p.batch];
  // With fewer tiles than CTAs only the first n_tiles CTAs take part, so that
  // every CTA between a pair's first and last holds at least one of its tiles
  // (the combine counts arrivals over that CTA range).
  const int G = n_tiles < gridDim.x ? static_cast<int>(n_tiles) : static_cast<int>(gridDim.x);
  const long long x0 = cta < G ? n_tiles * cta / G : 0, x1 = cta < G ? n_tiles * (cta + 1) / G : 0;

  // Shard-partial mode: sequences with no visible key in this shard still get
  // their (m = -inf, l = 0, o = 0) rows.
  if (p.out_partial && warp < kAsConsumerWarps) {
    for (int b = cta; b < p.batch; b += gridDim.x) {
      if (prefix[b + 1] != prefix[b]) continue;
      const int64_t rows = static_cast<int64_t>(T) * p.q_heads;
      for (int64_t i = threadIdx.x; i < rows * (D + 2); i += kAsConsumerWarps * 32) {
        const int64_t e = i % (D + 2);
        p.out_partial[static_cast<int64_t>(b) * rows * (D + 2) + i] = e == D ? -INFINITY : 0.0f;
      }
    }
  }

  if (warp == kAsConsumerWarps) {
    // ---------------------------------------------------------------- producer
    if (lane != 0) return;
    AsWalk w;
    bool more = w.begin(prefix, p.batch, hkv, x0, x1);
    bool waited = !p.pdl;
    bool dead = false;
    int stage = 0;
    uint32_t phase = 0;
    long long it = 0;
    while (more && !dead) {
      const int64_t pb = p.past_lengths ? p.past_lengths[w.b] : p.past_length;
      const int64_t row0 = (static_cast<int64_t>(w.b) * hkv + w.kvh) * cap;
      for (int t = w.t0; t < w.t1; ++t, ++it) {
        // Rows at or above P_b are written by the kernel before this one (the
        // K/V append): wait for it before the first such tile.
        if (!waited && static_cast<int64_t>(t + 1) * kAsTile > pb - off) {
          pdl_wait();
          waited = true;
        }
        if (it >= Cfg::kStages && !mbar_wait_bounded(&empty[stage], phase ^ 1u, p.err)) {
          dead = true;
          break;
        }
        uint8_t* st = smem + stage * Cfg::kStage;
        mbar_arrive_expect_tx(&full[stage], Cfg::kStage);
        const int r = static_cast<int>(row0 + static_cast<int64_t>(t) * kAsTile);
#pragma unroll
        for (int bx = 0; bx < Cfg::kBoxes; ++bx) {
          tma_load_2d(st + bx * kAsBox, &tm_k, bx * 64, r, &full[stage]);
          tma_load_2d(st + (Cfg::kBoxes + bx) * kAsBox, &tm_v, bx * 64, r, &full[stage]);
        }
        if (++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      more = w.next();
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  if (p.pdl) pdl_wait();  // q comes from the kernel before this one
  const int g = lane >> 2, tq = lane & 3;  // fragment row group / column pair
  const int grp = warp / kAsGroupWarps, wq = warp % kAsGroupWarps;
  AsWalk w;
  bool more = w.begin(prefix, p.batch, hkv, x0, x1);
  bool dead = false;
  long long it = 0;  // the CTA's tile counter, as the producer counts
  while (more) {
    const int b = w.b, kvh = w.kvh;
    const int64_t pb = p.past_lengths ? p.past_lengths[b] : p.past_length;
    const int64_t vis = as_limit(pb, T - 1, off, cap);
    // Query row n = t * group + j of this KV head (n < nq): lane's B-fragment
    // rows are n = g; its score columns are n = 2 tq, 2 tq + 1.
    uint32_t qb[KS][2];
    {
      const int n = g;
      const int64_t row = n < nq ? (static_cast<int64_t>(b) * T + n / group) * p.q_heads +
                                       static_cast<int64_t>(kvh) * group + n % group
                                 : 0;
      const uint32_t* qr = reinterpret_cast<const uint32_t*>(p.q + row * D);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qb[ks][0] = n < nq ? qr[ks * 8 + tq] : 0u;
        qb[ks][1] = n < nq ? qr[ks * 8 + 4 + tq] : 0u;
      }
    }
    int64_t lim[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int n = 2 * tq + c;
      lim[c] = n < nq ? as_limit(pb, n / group, off, cap) : 0;
    }
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    float acc[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

    for (int t = w.t0; t < w.t1; ++t, ++it) {
      if ((it & 1) != grp) continue;
      const int stage = static_cast<int>(it % Cfg::kStages);
      const uint32_t phase = static_cast<uint32_t>(it / Cfg::kStages) & 1u;
      if (!dead && !mbar_wait_bounded(&full[stage], phase, p.err)) dead = true;
      const uint8_t* kt = smem + stage * Cfg::kStage;
      const uint8_t* vt = kt + Cfg::kBoxes * kAsBox;
      const int64_t pos0 = static_cast<int64_t>(t) * kAsTile + wq * 16;  // this warp's first position
      if (!dead && pos0 < vis) {
        if (pos0 + 16 > vis) {
          // The sequence ends inside this warp's rows: rows at or past it may
          // hold anything (unwritten slots, the next head's rows) -- zero
          // their V so that p = 0 times them stays 0.
          for (int i = lane; i < 16 * Cfg::kBoxes * 8; i += 32) {
            const int r = i / (Cfg::kBoxes * 8);
            if (pos0 + r >= vis) {
              const int bx = (i / 8) % Cfg::kBoxes, c = i % 8;
              *reinterpret_cast<uint4*>(const_cast<uint8_t*>(vt) + bx * kAsBox + (wq * 16 + r) * 128 + c * 16) =
                  make_uint4(0u, 0u, 0u, 0u);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        // ---- S^T = K Q^T for this warp's 16 positions (two accumulators)
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const int mat = lane >> 3, r = wq * 16 + (mat & 1) * 8 + (lane & 7);
          const uint32_t rbase = smem_u32(kt) + r * 128;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            const int c = (ks & 3) * 2 + (mat >> 1);
            uint32_t a0, a1, a2, a3;
            ldsm_x4(rbase + (ks >> 2) * kAsBox + ((c ^ (lane & 7)) << 4), a0, a1, a2, a3);
            if (ks & 1) mma_bf16_16816(s1, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
            else mma_bf16_16816(s0, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
          }
        }
        // s[i]: position pos0 + g (+8 for i >= 2), column 2 tq + (i & 1)
        float sc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int64_t pos = pos0 + g + (i >= 2 ? 8 : 0);
          const float v = __fmul_rn(__fadd_rn(s0[i], s1[i]), p.scale);
          sc[i] = pos < lim[i & 1] ? v : -INFINITY;
        }
        float alpha[2], pr[4];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float mx = fmaxf(sc[c], sc[c + 2]);
          mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
          const float m_new = fmaxf(m_run[c], mx);
          alpha[c] = m_run[c] == -INFINITY ? 0.0f : expf(m_run[c] - m_new);
          pr[c] = sc[c] == -INFINITY ? 0.0f : expf(sc[c] - m_new);
          pr[c + 2] = sc[c + 2] == -INFINITY ? 0.0f : expf(sc[c + 2] - m_new);
          l_run[c] = fmaf(l_run[c], alpha[c], pr[c] + pr[c + 2]);
          m_run[c] = m_new;
        }
#pragma unroll
        for (int i = 0; i < KS; ++i) {
          acc[i][0] *= alpha[0];
          acc[i][1] *= alpha[1];
          acc[i][2] *= alpha[0];
          acc[i][3] *= alpha[1];
        }
        // ---- P^T as B fragments: hi = BF16(p), lo = BF16(p - hi)
        const uint32_t h01 = as_pack_bf16(pr[0], pr[1]), h23 = as_pack_bf16(pr[2], pr[3]);
        const uint32_t l01 = as_pack_bf16(pr[0] - __uint_as_float(h01 << 16), pr[1] - __uint_as_float(h01 & 0xffff0000u));
        const uint32_t l23 = as_pack_bf16(pr[2] - __uint_as_float(h23 << 16), pr[3] - __uint_as_float(h23 & 0xffff0000u));
        const uint32_t bh0 = movmatrix_trans(h01), bh1 = movmatrix_trans(h23);
        const uint32_t bl0 = movmatrix_trans(l01), bl1 = movmatrix_trans(l23);
        // ---- O^T += V^T P^T
        {
          const int mat = lane >> 3, r = wq * 16 + (mat >> 1) * 8 + (lane & 7);
          const uint32_t rbase = smem_u32(vt) + r * 128;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            const int c = (mt & 3) * 2 + (mat & 1);
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(rbase + (mt >> 2) * kAsBox + ((c ^ (lane & 7)) << 4), a0, a1, a2, a3);
            mma_bf16_16816(acc[mt], a0, a1, a2, a3, bh0, bh1);
            mma_bf16_16816(acc[mt], a0, a1, a2, a3, bl0, bl1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }

    // ---- this segment's (m, l, o): combine the eight warps
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      l_run[c] += __shfl_xor_sync(kFull, l_run[c], 4);
      l_run[c] += __shfl_xor_sync(kFull, l_run[c], 8);
      l_run[c] += __shfl_xor_sync(kFull, l_run[c], 16);
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      const int d0 = mt * 16 + g;
      float* o0 = so + (warp * kAsRows + 2 * tq) * D;
      float* o1 = o0 + D;
      o0[d0] = acc[mt][0];
      o1[d0] = acc[mt][1];
      o0[d0 + 8] = acc[mt][2];
      o1[d0 + 8] = acc[mt][3];
    }
    if (g == 0) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        sm_m[warp * kAsRows + 2 * tq + c] = m_run[c];
        sm_l[warp * kAsRows + 2 * tq + c] = l_run[c];
      }
    }
    named_bar_sync(1, kAsConsumerWarps * 32);

    const int64_t pair = static_cast<int64_t>(b) * hkv + kvh;
    const long long a = prefix[b] + static_cast<long long>(kvh) * w.nt;  // the pair's first tile
    const int c_first = as_cta_of(a, n_tiles, G), c_last = as_cta_of(a + w.nt - 1, n_tiles, G);
    const bool whole = c_first == c_last;
    float* slot = p.partials + (pair + cta) * kAsRows * (D + 2);
    const int tid = threadIdx.x;
    for (int i = tid; i < nq * D; i += kAsConsumerWarps * 32) {
      const int n = i / D, e = i % D;
      float mx = -INFINITY;
#pragma unroll
      for (int u = 0; u < kAsConsumerWarps; ++u) mx = fmaxf(mx, sm_m[u * kAsRows + n]);
      float o = 0.0f, l = 0.0f;
#pragma unroll
      for (int u = 0; u < kAsConsumerWarps; ++u) {
        const float mu = sm_m[u * kAsRows + n];
        const float f = mu == -INFINITY ? 0.0f : expf(mu - mx);
        o = fmaf(so[(u * kAsRows + n) * D + e], f, o);
        l = fmaf(sm_l[u * kAsRows + n], f, l);
      }
      const int64_t row = (static_cast<int64_t>(b) * T + n / group) * p.q_heads +
                          static_cast<int64_t>(kvh) * group + n % group;
      if (whole) {
        if (p.out_partial) {
          float* dst = p.out_partial + row * (D + 2);
          dst[e] = o;
          if (e == 0) {
            dst[D] = mx;
            dst[D + 1] = l;
          }
        } else {
          p.ctx[row * D + e] = f32_to_bf16_bits(__fdiv_rn(o, l));
        }
      } else {
        float* dst = slot + n * (D + 2);
        dst[e] = o;
        if (e == 0) {
          dst[D] = mx;
          dst[D + 1] = l;
        }
      }
    }
    if (!whole) {
      __threadfence();
      named_bar_sync(1, kAsConsumerWarps * 32);
      if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counters[pair], 1u);
        const bool last = prev == static_cast<unsigned>(c_last - c_first);
        if (last) p.counters[pair] = 0u;  // zero for the next launch
        *s_flag = last ? 1u : 0u;
      }
      named_bar_sync(1, kAsConsumerWarps * 32);
      if (*s_flag) {
        __threadfence();
        // Weights exp(m_c - M) of the pair's partials (CTA order), in `so`.
        const int ncov = c_last - c_first + 1;
        float* wts = so;                 // [nq][ncov]
        float* tot = so + kAsRows * ncov;  // [nq]: l, then M
        const float* base = p.partials + (pair + c_first) * kAsRows * (D + 2);
        for (int n = warp; n < nq; n += kAsConsumerWarps) {
          float mx = -INFINITY;
          for (int c = lane; c < ncov; c += 32) mx = fmaxf(mx, __ldcg(base + (c * kAsRows + n) * (D + 2) + D));
          mx = warp_max_f32(mx);
          float l = 0.0f;
          for (int c = lane; c < ncov; c += 32) {
            const float* src = base + (c * kAsRows + n) * (D + 2);
            const float mc = __ldcg(src + D);
            const float f = mc == -INFINITY ? 0.0f : expf(mc - mx);
            wts[n * ncov + c] = f;
            l = fmaf(__ldcg(src + D + 1), f, l);
          }
          l = warp_sum_f32(l);
          if (lane == 0) {
            tot[n] = l;
            tot[kAsRows + n] = mx;
          }
        }
        named_bar_sync(1, kAsConsumerWarps * 32);
        for (int i = tid; i < nq * D; i += kAsConsumerWarps * 32) {
          const int n = i / D, e = i % D;
          float o = 0.0f;
          for (int c = 0; c < ncov; ++c) o = fmaf(__ldcg(base + (c * kAsRows + n) * (D + 2) + e), wts[n * ncov + c], o);
          const int64_t row = (static_cast<int64_t>(b) * T + n / group) * p.q_heads +
                              static_cast<int64_t>(kvh) * group + n % group;
          if (p.out_partial) {
            float* dst = p.out_partial + row * (D + 2);
            dst[e] = o;
            if (e == 0) {
              dst[D] = tot[kAsRows + n];
              dst[D + 1] = tot[n];
            }
          } else {
            p.ctx[row * D + e] = f32_to_bf16_bits(__fdiv_rn(o, tot[n]));
          }
        }
      }
    }
    named_bar_sync(1, kAsConsumerWarps * 32);  // `so` and the flags are reused by the next segment
    more = w.next();
  }
}

}  // namespace nvfp4da
