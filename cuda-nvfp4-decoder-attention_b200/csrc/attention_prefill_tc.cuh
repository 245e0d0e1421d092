// Causal GQA prefill attention on the 5th-generation tensor cores (T >= 64,
// head_dim 128): tcgen05.mma with TMA-loaded operands and FP32 accumulators
// in tensor memory.
//
// Semantics (reference/decoder_attention.py:273-381, src/gqa_attention_cached.cu
// :93-248): query token t of sequence b (position P_b + t) and head h attends
// to keys j <= P_b + t of KV head h / (Hq / Hkv) in the physical cache
// [B, Hkv, C, D]; score = FP32(q . k) * FP32(1/sqrt(D)); FP32 softmax;
// context = BF16(sum_j p_j v_j / sum_j p_j).  No score or probability tensor
// is materialised.
//
// One CTA: 128 query rows of one (sequence, head), key tiles of 64.  Roles:
//  * warp 0 (one lane): TMA loads -- the Q tile once (two 64-wide column
//    panels, 128-byte swizzle), then K and V tiles into a 3-stage ring;
//  * warp 1 (one lane): the MMAs.  S_j = Q K_j^T (M 128, N 64) as two
//    partial sums over the halves of d, each in its own tensor-memory
//    accumulator; O_j = P_j Vt_j (M 128, N 128) as two 32-key blocks, each in
//    its own accumulator, P in three BF16 terms (six chained MMAs per block);
//  * warps 2-9: softmax.  Warp w reads tensor-memory lanes 32 (w % 4) .. +31;
//    each query row is split between two threads (warps w and w + 4), one
//    per half of the keys of a tile and of the output columns, exchanging
//    only the row maximum once per tile: the score is the FP32 round-to-nearest sum of
//    the two partials (short accumulation chains keep the tensor cores'
//    internal rounding small), online max / sum in FP32, P = exp(s - m) split
//    into BF16 hi + mid + lo (each the residual of the previous rounding:
//    ~24 bits, every product exact) written to shared memory in the MMA's
//    operand layout; then O_{j-1} is folded into an FP32 register accumulator
//    (rescale, then each 32-key block added with round-to-nearest);
//  * warps 10-11: transpose V_j into Vt_j ([d][key], the K-major B operand of
//    the PV MMA) with ldmatrix.trans / stmatrix, zeroing keys past the last
//    one any row of the tile sees (the cache may hold anything there).
// Every operand is K-major with the 128-byte swizzle: 128-byte rows, 8-row
// atoms of 1024 bytes, +32 bytes per 16-element k step inside an atom.
// Waits are bounded (one second, shared give-up flag); tensor memory is freed
// on every path.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "attention_prefill.cuh"  // pack_bf16
#include "prefill_gemm.cuh"       // tcgen05 / TMA primitives, pg_wait, mbar_arrive

namespace nvfp4da {

constexpr int kPtRows = 128;   // query rows per CTA
constexpr int kPtKeys = 64;    // keys per tile
constexpr int kPtD = 128;      // head dim
constexpr int kPtStages = 3;   // K/V ring
constexpr int kPtSoftmaxWarps = 8;  // two per tensor-memory lane quadrant: each row split in halves
constexpr int kPtThreads = (2 + kPtSoftmaxWarps + 2) * 32;
constexpr uint32_t kPtPanel = kPtRows * 128;          // 128 rows x 64 elements: 16 KB
constexpr uint32_t kPtKv = kPtKeys * 128;             // 64 rows x 64 elements: 8 KB
// shared memory (offsets from a 1024-aligned base)
constexpr uint32_t kPtOffQ = 0;                                  // 2 panels
constexpr uint32_t kPtOffK = kPtOffQ + 2 * kPtPanel;             // stages x 2 panels
constexpr uint32_t kPtOffV = kPtOffK + kPtStages * 2 * kPtKv;    // stages x 2 panels
constexpr uint32_t kPtOffVt = kPtOffV + kPtStages * 2 * kPtKv;   // 2 buffers of [128 d][64 keys]
constexpr uint32_t kPtOffP = kPtOffVt + 2 * kPtPanel;            // hi, mid, lo: [128 rows][64 keys] each
constexpr uint32_t kPtSmem = kPtOffP + 3 * kPtPanel + 1024;
constexpr int kPtSChains = 2;        // score accumulators: one per 64-wide half of d
constexpr int kPtOBlockKeys = 32;    // keys per output accumulator
constexpr uint32_t kPtTmemCols = 512;  // S: 2 buffers x 2 chains x 64 columns; O: 2 blocks x 128 columns
constexpr uint32_t kPtTmemS = kPtSChains * kPtKeys;  // columns per S buffer
constexpr uint32_t kPtTmemO = 2 * kPtTmemS;

struct PrefillTcParams {
  uint16_t* ctx;  // [B, T, Hq, D]
  int batch, tokens, q_heads, kv_heads;
  int64_t capacity;
  int64_t past_length;
  const int64_t* past_lengths;
  float scale;
  unsigned* err;
};

__device__ __forceinline__ void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// 16 columns of this warp's 32 tensor-memory lanes into registers, without
// waiting: several loads share one tcgen05.wait::ld.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of (row r, 16-byte chunk c) in a 128-byte-row swizzled tile.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kPtThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, PrefillTcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_q, bar_kv_full[kPtStages], bar_kv_empty[kPtStages], bar_vt_full[2], bar_vt_empty[2],
      bar_s_full[2], bar_s_empty[2], bar_p_full, bar_o_full[2], bar_o_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ float s_rowmax[2][2][kPtRows];  // [tile parity][half][row]: partial row maxima
  __shared__ float s_rowl[2][kPtRows];       // [half][row]: partial row sums, at the end
  __shared__ uint64_t bar_mx[2], bar_l;
  __shared__ volatile unsigned s_bad;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Query tiles longest first (the causal triangle).
  const int ntile = (p.tokens + kPtRows - 1) / kPtRows;
  const int qt = ntile - 1 - static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int group = p.q_heads / p.kv_heads, kvh = h / group;
  const int64_t pb = p.past_lengths ? p.past_lengths[b] : p.past_length;
  const int t0 = qt * kPtRows;
  const int rows_valid = min(kPtRows, p.tokens - t0);
  // Keys the tile's rows see: 0 .. P_b + t0 + rows_valid - 1 (never past C).
  int64_t klim = pb + t0 + rows_valid;
  if (klim > p.capacity) klim = p.capacity;
  const int nkt = static_cast<int>((klim + kPtKeys - 1) / kPtKeys);

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kPtTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(&bar_q, 1);
    for (int s = 0; s < kPtStages; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 3);  // the S MMA's commit and both transpose warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_vt_full[i], 2);   // both transpose warps
      mbar_init(&bar_vt_empty[i], 1);  // PV commit
      mbar_init(&bar_s_full[i], 1);    // S commit
      mbar_init(&bar_s_empty[i], kPtSoftmaxWarps);
      mbar_init(&bar_o_full[i], 1);    // PV commit
      mbar_init(&bar_o_empty[i], kPtSoftmaxWarps);
    }
    mbar_init(&bar_p_full, kPtSoftmaxWarps);
    mbar_init(&bar_mx[0], kPtSoftmaxWarps);
    mbar_init(&bar_mx[1], kPtSoftmaxWarps);
    mbar_init(&bar_l, kPtSoftmaxWarps);
    fence_mbar_init();
    s_bad = 0u;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  const int64_t kv_row0 = (static_cast<int64_t>(b) * p.kv_heads + kvh) * p.capacity;

  if (warp == 0) {
    // ---------------------------------------------------------------- loads
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar_q, 2 * kPtPanel);
      for (int pn = 0; pn < 2; ++pn)
        tma_load_3d(smem + kPtOffQ + pn * kPtPanel, &tm_q, pn * 64, h, b * p.tokens + t0, &bar_q);
      for (int j = 0; j < nkt; ++j) {
        const int s = j % kPtStages;
        if (j >= kPtStages && !pg_wait(&bar_kv_empty[s], ((j / kPtStages) - 1) & 1, &s_bad, p.err)) break;
        mbar_arrive_expect_tx(&bar_kv_full[s], 4 * kPtKv);
        const int row = static_cast<int>(kv_row0 + static_cast<int64_t>(j) * kPtKeys);
        for (int pn = 0; pn < 2; ++pn) {
          tma_load_2d(smem + kPtOffK + (s * 2 + pn) * kPtKv, &tm_k, pn * 64, row, &bar_kv_full[s]);
          tma_load_2d(smem + kPtOffV + (s * 2 + pn) * kPtKv, &tm_v, pn * 64, row, &bar_kv_full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMAs
    if (lane == 0) {
      constexpr uint32_t kIdescS = umma_idesc_bf16(kPtRows, kPtKeys);
      constexpr uint32_t kIdescO = umma_idesc_bf16(kPtRows, kPtD);
      bool ok = pg_wait(&bar_q, 0, &s_bad, p.err);
      // S_j for j = 0 .. nkt-1 and O_{j-1} after it, so that the softmax of
      // tile j overlaps the PV MMA of tile j - 1.  S is double-buffered (S_j
      // waits until the softmax has read S_{j-2}); O is one buffer (O_i waits
      // until the softmax has folded O_{i-1}).
      for (int j = 0; ok && j <= nkt; ++j) {
        if (j < nkt) {
          const int s = j % kPtStages, sb = j & 1;
          ok = pg_wait(&bar_kv_full[s], (j / kPtStages) & 1, &s_bad, p.err) &&
               (j < 2 || pg_wait(&bar_s_empty[sb], ((j >> 1) - 1) & 1, &s_bad, p.err));
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
          for (int pn = 0; pn < kPtSChains; ++pn) {  // half pn of d: its own accumulator
            const uint64_t ad = umma_desc_sw128(smem_u32(smem + kPtOffQ + pn * kPtPanel));
            const uint64_t bd = umma_desc_sw128(smem_u32(smem + kPtOffK + (s * 2 + pn) * kPtKv));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(tmem + sb * kPtTmemS + static_cast<uint32_t>(pn * kPtKeys), ad + 2 * kk, bd + 2 * kk, kIdescS,
                        kk ? 1u : 0u);
          }
          umma_commit(&bar_s_full[sb]);
          umma_commit(&bar_kv_empty[s]);  // K_j consumed (the transposers release V_j)
        }
        if (j >= 1) {
          const int i = j - 1, vb = i & 1;
          ok = pg_wait(&bar_p_full, i & 1, &s_bad, p.err) && pg_wait(&bar_vt_full[vb], (i >> 1) & 1, &s_bad, p.err) &&
               (i < 1 || pg_wait(&bar_o_empty[0], (i - 1) & 1, &s_bad, p.err));
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + kPtOffVt + vb * kPtPanel));
#pragma unroll
          for (int ob = 0; ob < kPtKeys / kPtOBlockKeys; ++ob) {  // 32-key block ob: its own accumulator
            const uint32_t oacc = tmem + kPtTmemO + static_cast<uint32_t>(ob * kPtD);
#pragma unroll
            for (int kk = 0; kk < kPtOBlockKeys / 16; ++kk) {
              const int ks = ob * (kPtOBlockKeys / 16) + kk;
#pragma unroll
              for (int term = 0; term < 3; ++term) {
                const uint64_t ad = umma_desc_sw128(smem_u32(smem + kPtOffP + term * kPtPanel));
                umma_bf16(oacc, ad + 2 * ks, bd + 2 * ks, kIdescO, (term | kk) ? 1u : 0u);
              }
            }
          }
          umma_commit(&bar_o_full[0]);
          umma_commit(&bar_vt_empty[vb]);
        }
      }
    }
    __syncwarp();
  } else if (warp >= 2 + kPtSoftmaxWarps) {
    // ---------------------------------------------------------------- V transpose
    // 128 8x8 blocks per tile (8 key blocks x 16 d blocks), 4 per x4
    // instruction, 16 instructions per warp.
    const int tw = warp - 2 - kPtSoftmaxWarps;
    for (int j = 0; j < nkt; ++j) {
      const int s = j % kPtStages, vb = j & 1;
      bool ok = pg_wait(&bar_kv_full[s], (j / kPtStages) & 1, &s_bad, p.err) &&
                (j < 2 || pg_wait(&bar_vt_empty[vb], ((j >> 1) - 1) & 1, &s_bad, p.err));
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint8_t* vsrc = smem + kPtOffV + s * 2 * kPtKv;
      uint8_t* vdst = smem + kPtOffVt + vb * kPtPanel;
      const int64_t key0 = static_cast<int64_t>(j) * kPtKeys;
      const int mat = lane >> 3, r8 = lane & 7;
      const int t = lane & 3;
#pragma unroll 4
      for (int it = 0; it < 16; ++it) {
        // instruction it of warp tw: blocks q = 4 * (tw * 16 + it) + mat
        const int q = 4 * (tw * 16 + it) + mat;
        const int kb = q & 7, db = q >> 3;  // key block 0..7, d block 0..15
        const int key = kb * 8 + r8, dch = db & 7, pn = db >> 3;
        uint32_t r[4];
        ldsm_x4_t(smem_u32(vsrc + pn * kPtKv + sw128(key, dch)), r[0], r[1], r[2], r[3]);
        // r[i] (block 4 * (tw * 16 + it) + i): this lane holds d = 8 db_i + lane / 4,
        // keys 8 kb_i + 2 (lane % 4), + 1.  Zero keys at or past klim.
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int qi = 4 * (tw * 16 + it) + i;
          const int64_t k0 = key0 + (qi & 7) * 8 + 2 * t;
          if (k0 >= klim) r[i] = 0u;
          else if (k0 + 1 >= klim) r[i] &= 0xffffu;
        }
        // rows of Vt: d = 8 db + r8 for the address this lane supplies
        const int d = db * 8 + r8;
        stsm_x4(smem_u32(vdst + sw128(d, kb)), r[0], r[1], r[2], r[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar_vt_full[vb]);
        mbar_arrive(&bar_kv_empty[s]);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    constexpr int kHalfD = kPtD / 2, kHalfKeys = kPtKeys / 2;
    const int quad = warp & 3, row = quad * 32 + lane;
    const int half = (warp - 2) / 4;  // keys [32 half, +32) of each tile, output columns [64 half, +64)
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int64_t pos = pb + t0 + row;  // this row's position (rows past T are computed, not stored)
    constexpr float kLog2e = 1.4426950408889634f;
    float m_run = -INFINITY, ml_run = 0.0f, l_run = 0.0f, alpha_prev = 1.0f;
    float o[kHalfD];
#pragma unroll
    for (int i = 0; i < kHalfD; ++i) o[i] = 0.0f;
    bool ok = true;
    // Fold O_i (scaled to m_i) into the register accumulator: o = o * a +
    // (first 32-key block), one rounding, then the second block added with
    // round-to-nearest; a = exp(m_{i-1} - m_i).
    auto fold = [&](int i, float a) -> bool {
      const bool good = pg_wait(&bar_o_full[0], i & 1, &s_bad, p.err);
      if (!__all_sync(0xffffffffu, good)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int ob = 0; ob < kPtKeys / kPtOBlockKeys; ++ob) {  // this half's 64 columns: four loads, one wait
        uint32_t v[4][16];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          tmem_ld16_nowait(tmem + lane_base + kPtTmemO + static_cast<uint32_t>(ob * kPtD + half * kHalfD + 16 * q),
                           v[q]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < 16; ++e)
            o[16 * q + e] = ob == 0 ? fmaf(o[16 * q + e], a, __uint_as_float(v[q][e]))
                                    : __fadd_rn(o[16 * q + e], __uint_as_float(v[q][e]));
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_o_empty[0]);
      return true;
    };
    for (int j = 0; j < nkt && ok; ++j) {
      const int sb = j & 1;
      const uint32_t sbase = sb * kPtTmemS;
      ok = pg_wait(&bar_s_full[sb], (j >> 1) & 1, &s_bad, p.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // Score of key e (16 at a time): the two half-d partials added with
      // round-to-nearest, scaled, causally masked.  Read twice from tensor
      // memory (max, then exponentials) instead of holding 64 in registers.
      const int64_t key0 = static_cast<int64_t>(j) * kPtKeys;
      // Keys key0 + e with e < vis are visible to this row (causal bound and
      // the tile's key limit).
      const int64_t vis64 = min(pos + 1, klim) - key0;
      const int vis = vis64 < 0 ? 0 : (vis64 > kPtKeys ? kPtKeys : static_cast<int>(vis64));
      auto scores32 = [&](int c, float (&sc)[32]) {  // keys c .. c + 31: four loads, one wait
        uint32_t a[2][16], bq[2][16];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          tmem_ld16_nowait(tmem + lane_base + sbase + static_cast<uint32_t>(c + 16 * q), a[q]);
          tmem_ld16_nowait(tmem + lane_base + sbase + static_cast<uint32_t>(kPtKeys + c + 16 * q), bq[q]);
        }
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          sc[e] = (c + e < vis)
                      ? __fmul_rn(__fadd_rn(__uint_as_float(a[e >> 4][e & 15]), __uint_as_float(bq[e >> 4][e & 15])),
                                  p.scale)
                      : -INFINITY;
      };
      float sc[kHalfKeys];  // this half's 32 keys
      scores32(half * kHalfKeys, sc);
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < kHalfKeys; ++e) mx = fmaxf(mx, sc[e]);
      // The row maximum: exchange with the other half through shared memory
      // and an mbarrier of the softmax warps (bounded wait).  The buffer of
      // tile j is next written at tile j + 2, after the partner has read it.
      s_rowmax[j & 1][half][row] = mx;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_mx[j & 1]);
      ok = pg_wait(&bar_mx[j & 1], (j >> 1) & 1, &s_bad, p.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      mx = fmaxf(mx, s_rowmax[j & 1][half ^ 1][row]);
      const float m_new = fmaxf(m_run, mx);
      // exp(s - m) as 2^(s log2(e) - m log2(e)) with one rounding in the
      // exponent: the rounding of m log2(e) is the same for every term of
      // the row and for alpha, so it cancels in sum(p v) / sum(p).
      const float ml_new = m_new == -INFINITY ? 0.0f : __fmul_rn(m_new, kLog2e);
      const float alpha = m_run == -INFINITY ? 0.0f : exp2f(__fsub_rn(ml_run, ml_new));
      // The P buffers are free once PV_{j-1} is done, which the fold of
      // O_{j-1} waits for.
      if (j >= 1 && !(ok = fold(j - 1, alpha_prev))) break;
      alpha_prev = alpha;  // O_j is scaled to m_j
      float lsum = 0.0f;
      {
        const int c = half * kHalfKeys;
#pragma unroll
        for (int h8 = 0; h8 < 4; ++h8) {  // 16-byte chunk (c + 8 h8) / 8 of each term
          uint32_t w[3][4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float s0 = sc[8 * h8 + 2 * e], s1 = sc[8 * h8 + 2 * e + 1];
            float r0 = s0 == -INFINITY ? 0.0f : exp2f(fmaf(s0, kLog2e, -ml_new));
            float r1 = s1 == -INFINITY ? 0.0f : exp2f(fmaf(s1, kLog2e, -ml_new));
            lsum += r0 + r1;
#pragma unroll
            for (int term = 0; term < 3; ++term) {
              const uint32_t both = pack_bf16(r0, r1);  // one conversion for the pair
              w[term][e] = both;
              if (term < 2) {
                r0 -= __uint_as_float(both << 16);  // exact residuals
                r1 -= __uint_as_float(both & 0xffff0000u);
              }
            }
          }
#pragma unroll
          for (int term = 0; term < 3; ++term)
            *reinterpret_cast<uint4*>(smem + kPtOffP + term * kPtPanel + sw128(row, c / 8 + h8)) =
                make_uint4(w[term][0], w[term][1], w[term][2], w[term][3]);
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_s_empty[sb]);
      l_run = fmaf(l_run, alpha, lsum);
      m_run = m_new;
      ml_run = ml_new;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p_full);
    }
    if (ok && nkt > 0) ok = fold(nkt - 1, alpha_prev);
    // The row's sum: this half's l plus the other half's (same running max).
    s_rowl[half][row] = l_run;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_l);
    if (ok) ok = pg_wait(&bar_l, 0, &s_bad, p.err);
    l_run = __fadd_rn(s_rowl[0][row], s_rowl[1][row]);
    if (ok && !s_bad && row < rows_valid) {
      uint16_t* dst = p.ctx + ((static_cast<int64_t>(b) * p.tokens + t0 + row) * p.q_heads + h) * kPtD + half * kHalfD;
#pragma unroll
      for (int c = 0; c < kHalfD; c += 8) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[e] = static_cast<uint32_t>(f32_to_bf16_bits(__fdiv_rn(o[c + 2 * e], l_run))) |
                 (static_cast<uint32_t>(f32_to_bf16_bits(__fdiv_rn(o[c + 2 * e + 1], l_run))) << 16);
        *reinterpret_cast<uint4*>(dst + c) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPtTmemCols) : "memory");
}

}  // namespace nvfp4da
