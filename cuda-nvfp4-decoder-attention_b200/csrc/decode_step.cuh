// The whole T = 1 decode step as one persistent cooperative kernel.
//
// Same results as the three-kernel chain (qkv_fused -> attn_split ->
// mma_gemv), i.e. the reference's composed forward
// (decoder_attention_cuda.py:149-417): input RMSNorm, W4A16 Q/K/V projection,
// per-head Q/K RMSNorm, adjacent-pair RoPE, K/V cache append, causal GQA over
// the cache, W4A16 O projection.
//
// Why one kernel: at decode sizes every stage moves a few MB and is bound by
// latency (launch, first bytes from HBM, reductions), not bandwidth.  None of
// the step's big inputs -- Q/K/V/O weights and the cache rows below P_b --
// depends on any stage, so every CTA issues bulk copies of ALL of its slices
// (its QKV weight rows, its O weight rows, its attention unit's K/V tile) the
// moment it starts; the whole step's HBM traffic is in flight at once, and the
// stages then run out of shared memory, ordered by counters instead of kernel
// boundaries.
//
// Work per CTA (grid = one CTA per SM, all co-resident: cooperative launch):
//  * QKV block c: concatenated rows [c*RQ, c*RQ + RQ) of [Wq; Wk; Wv]
//    (RQ divides D, so a block lies in one head).  Each CTA recomputes the
//    input RMSNorm of the activation rows itself (tiny, L2-resident), runs the
//    tensor-core GEMV from shared memory and writes the raw BF16 projections
//    to the workspace, then bumps its head's counter.
//  * Attention unit (b, kv head, split j): positions [j*L, j*L + L) of
//    sequence b.  Waits for the counters of its GH query heads and its K and V
//    head, applies the per-head RMSNorm + RoPE to those rows itself, appends
//    the new K/V row to the cache (the split holding position P_b), runs the
//    online-softmax loop over its K/V tile, and leaves (m, l, o) partials.
//  * O block c: 8-row multiples of Wo (the rows spread over all CTAs).  When
//    every split's partials fit in shared memory (o_combine) each O CTA
//    bulk-copies all of them once every unit has signalled and does the
//    log-sum-exp combine itself -- no extra hand-off; otherwise the last split
//    of each (b, kv head) to arrive combines them into a BF16 context buffer
//    that the O CTAs read.
//
// Synchronisation state lives in a slot of library-owned device memory (one
// slot per stream), zero between launches: the last CTA to leave clears it.
// Every wait is bounded by a time limit; on expiry the kernel records
// kErrBarrierTimeout in the slot and carries on (results are then garbage, the
// GPU stays usable).
#pragma once

#include "attention.cuh"
#include "elementwise.cuh"
#include "gemv_mma.cuh"
#include "qkv_fused.cuh"  // kMaxHeadDim

namespace nvfp4da {

constexpr int kStepThreads = kMmaThreads;
constexpr int kStepWarps = kMmaWarps;
constexpr int kStepMaxRows = 128;    // RQ / RO rows per CTA (tile-padded)
constexpr int kStepSyncWords = 2048;  // one slot
// Slot layout (32-bit words).
constexpr int kSyncExit = 0, kSyncCtxDone = 1, kSyncErr = 2, kSyncHeads = 16;

struct StepParams {
  const uint16_t* x;     // [B, H]
  const uint16_t* g_in;  // [H]
  const uint8_t* packed[4];  // q, k, v, o
  const uint8_t* scales[4];
  const float* gamma[4];
  const uint16_t* g_q;  // [D]
  const uint16_t* g_k;  // [D]
  uint16_t* k_cache;    // [B, Hkv, C, D]
  uint16_t* v_cache;
  uint16_t* out;  // [B, H]
  int64_t batch, hidden, q_heads, kv_heads, head_dim, capacity;
  int64_t past_length;
  const int64_t* past_lengths;
  float eps, theta, scale;
  // plan
  int rq, n_qkv_blocks;                        // QKV rows per block (divides D)
  int o_rows_big, o_n_big, o_rows_small, o_tile_rows;  // O rows per CTA: big for CTAs < o_n_big
  int splits, split_len;
  int o_combine;  // 1: O CTAs combine the split partials themselves
  // workspace
  uint16_t* proj;    // [B, (Hq + 2 Hkv) D] raw projections
  uint16_t* ctx;     // [B, H]            (o_combine == 0)
  float* part_o;     // [B * Hq, splits, D]
  float* part_ml;    // [B * Hq, splits, 4]  (m, l, -, -)
  unsigned* sync;    // slot
  unsigned long long timeout_ns;
  // When the K/V tile and the O rows are requested: 0 at launch, 1 once the
  // QKV rows have landed, 2 the K/V tile then and the O rows after the
  // attention unit.
  int sched;
  // dynamic shared-memory layout (byte offsets); qs/qw/kv/q and comb overlay
  uint32_t off_qs, off_qw, off_kv, off_q, off_comb, off_os, off_ow, off_xs, off_x16, off_red;
  // cos/sin of RoPE at position past_length (rope_host_ok), else computed on the device
  int rope_host_ok;
  float2 rope_host[kMaxHeadDim / 2];
};

// ---------------------------------------------------------------- sync primitives
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Publish this CTA's global writes, then add 1 to *ctr.  All threads call.
// The barrier orders every thread's writes before thread 0's release, and a
// release is cumulative over what its thread has observed.
__device__ __forceinline__ void cta_signal(unsigned* ctr) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

// Returns the counter's previous value (acquire + release: the caller sees
// the writes of every CTA that added before it).
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* ctr, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(ctr), "r"(v) : "memory");
  return old;
}

// Wait (all threads call; warp 0 polls) until ctr[idx[i]] >= target for the n
// (<= 32) counters listed, then make the producers' writes visible to the CTA.
// Bounded: gives up after timeout_ns, recording the timeout in *err.
__device__ __forceinline__ void cta_wait(const unsigned* ctr, const int* idx, int n, unsigned target,
                                         unsigned* err, unsigned long long timeout_ns) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const unsigned* mine = lane < n ? ctr + idx[lane] : nullptr;
    const unsigned long long t0 = global_ns();
    for (;;) {
      const bool ok = !mine || ld_acquire_u32(mine) >= target;
      if (__all_sync(kFull, ok)) break;
      if (global_ns() - t0 > timeout_ns) {
        if (lane == 0) atomicOr(err, static_cast<unsigned>(kErrBarrierTimeout));
        break;
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- the kernel
template <int EPL, int GH>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t bar_qkv, bar_kv, bar_o, bar_c;
  __shared__ float redf[2 * kStepWarps];
  __shared__ double redd[2 * kStepWarps];
  __shared__ float escale[kMmaMaxM];
  __shared__ float red_small[kMmaMaxM * kStepWarps];
  __shared__ float outv[kStepMaxRows * 8];
  __shared__ float sm_m[kStepWarps][GH], sm_l[kStepWarps][GH], wf[kStepWarps][GH], cta_m[GH], cta_l[GH];
  __shared__ unsigned s_flag;
  [[maybe_unused]] constexpr unsigned kPhaseBase = 3072;
  constexpr int PPL = EPL / 2;  // RoPE pairs per lane (D = 32 * EPL)
  NVFP4DA_PHASE(0);
#ifdef NVFP4DA_PHASES
  if (p.sched & 32) {  // diagnostic: touch every line of the parameter block at once
    constexpr int kLines = (sizeof(StepParams) + 127) / 128;
    if (threadIdx.x < kLines) {
      const uint32_t v = reinterpret_cast<const uint32_t*>(&p)[threadIdx.x * 32];
      asm volatile("" ::"r"(v));
    }
  }
#endif

  const int cta = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t k = p.hidden, d = p.head_dim, nb = p.batch;
  const int mrows = static_cast<int>(nb);  // T = 1: one activation row per sequence
  const int64_t hq = p.q_heads, hkv = p.kv_heads;
  const int64_t nqkv = (hq + 2 * hkv) * d;
  const int ns = p.splits;
  unsigned* sync = p.sync;
  unsigned* err = sync + kSyncErr;
  unsigned* head_done = sync + kSyncHeads;        // [Hq + 2 Hkv]
  unsigned* arrive = head_done + (hq + 2 * hkv);  // [B * Hkv]

  uint8_t* qs_smem = smem + p.off_qs;
  uint8_t* qw_smem = smem + p.off_qw;
  uint8_t* os_smem = smem + p.off_os;
  uint8_t* ow_smem = smem + p.off_ow;
  uint16_t* kv_k = reinterpret_cast<uint16_t*>(smem + p.off_kv);
  uint16_t* kv_v = kv_k + static_cast<int64_t>(p.split_len) * d;
  float* qf = reinterpret_cast<float*>(smem + p.off_q);  // [GH][D]
  uint16_t* x_stage = reinterpret_cast<uint16_t*>(smem + p.off_xs);
  __half* x16 = reinterpret_cast<__half*>(smem + p.off_x16);
  float* mred = reinterpret_cast<float*>(smem + p.off_red);

  // ---- roles
  const bool has_qkv = cta < p.n_qkv_blocks;
  const int n_units = static_cast<int>(nb * hkv) * ns;
  const bool has_attn = cta < n_units;
  int64_t orow0;
  int o_rows;
  if (cta < p.o_n_big) {
    o_rows = p.o_rows_big;
    orow0 = static_cast<int64_t>(cta) * p.o_rows_big;
  } else {
    o_rows = p.o_rows_small;
    orow0 = static_cast<int64_t>(p.o_n_big) * p.o_rows_big + static_cast<int64_t>(cta - p.o_n_big) * p.o_rows_small;
  }
  const int o_valid = orow0 < k ? static_cast<int>((k - orow0) < o_rows ? (k - orow0) : o_rows) : 0;
  const bool has_o = o_valid > 0;

  const int64_t qrow0 = static_cast<int64_t>(cta) * p.rq;  // concatenated QKV row
  const int mat = qrow0 < hq * d ? 0 : (qrow0 < (hq + hkv) * d ? 1 : 2);
  const int64_t mat_row0 = qrow0 - (mat == 0 ? 0 : (mat == 1 ? hq * d : (hq + hkv) * d));

  const int split = has_attn ? cta % ns : 0;
  const int64_t bh = has_attn ? cta / ns : 0;
  const int64_t b = bh / hkv, kvh = bh % hkv;
  const int64_t pb = has_attn ? (p.past_lengths ? p.past_lengths[b] : p.past_length) : 0;
  const int64_t s0 = static_cast<int64_t>(split) * p.split_len;
  // Keys 0 .. P_b; never beyond the physical capacity, whatever a device-side
  // length says.
  int64_t s_end = pb + 1 < p.capacity ? pb + 1 : p.capacity;
  if (s_end > s0 + p.split_len) s_end = s0 + p.split_len;
  const int64_t cache_end = pb < s_end ? pb : s_end;  // rows [s0, cache_end) come from the cache
  const int64_t n_cache = cache_end > s0 ? cache_end - s0 : 0;
  const bool owns_new = has_attn && pb >= 0 && pb < p.capacity && pb >= s0 && pb < s0 + p.split_len;
  const uint16_t* kbase = p.k_cache + (b * hkv + kvh) * p.capacity * d;
  const uint16_t* vbase = p.v_cache + (b * hkv + kvh) * p.capacity * d;

  // ---- the activation rows and the input-norm gain first: they head the
  // critical path, so their requests go out before any bulk traffic.
  constexpr int NCH = 2;
  uint4 gch[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int idx = threadIdx.x + c * kStepThreads;
    gch[c] = idx < k / 8 ? ldg_stream(p.g_in + 8 * idx) : make_uint4(0u, 0u, 0u, 0u);
    if (idx < k / 8)
      for (int m = 0; m < mrows; ++m) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.x + m * k + 8 * idx));
  }

  if (threadIdx.x == 0) {
    mbar_init(&bar_qkv, 1);
    mbar_init(&bar_kv, 1);
    mbar_init(&bar_o, 1);
    mbar_init(&bar_c, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- input slices of this CTA (none is written by the step): the QKV
  // rows now, the K/V tile and the O rows later (p.sched), so that they do
  // not queue ahead of the critical path.
  const int64_t ks = k / 16, kb = k / 2;
  auto issue_kv = [&]() {
    if (n_cache > 0) {
      const uint32_t tb = static_cast<uint32_t>(n_cache * d * 2);
      mbar_arrive_expect_tx(&bar_kv, 2 * tb);
      bulk_g2s(kv_k, kbase + s0 * d, tb, &bar_kv);
      bulk_g2s(kv_v, vbase + s0 * d, tb, &bar_kv);
    }
  };
  auto issue_o = [&]() {
    if (has_o) {
      const uint32_t sb = static_cast<uint32_t>(o_valid * ks), wb = static_cast<uint32_t>(o_valid * kb);
      mbar_arrive_expect_tx(&bar_o, sb + wb);
      bulk_g2s(os_smem, p.scales[3] + orow0 * ks, sb, &bar_o);
      bulk_g2s(ow_smem, p.packed[3] + orow0 * kb, wb, &bar_o);
    }
  };
  if (threadIdx.x == 0) {
    if (has_qkv) {
      const uint32_t sb = static_cast<uint32_t>(p.rq * ks), wb = static_cast<uint32_t>(p.rq * kb);
      mbar_arrive_expect_tx(&bar_qkv, sb + wb);
      bulk_g2s(qs_smem, p.scales[mat] + mat_row0 * ks, sb, &bar_qkv);
      bulk_g2s(qw_smem, p.packed[mat] + mat_row0 * kb, wb, &bar_qkv);
    }
    if ((p.sched & 7) == 0 || !has_qkv) {
      issue_kv();
      issue_o();
    }
  }
  NVFP4DA_PHASE(1);

  // ---- input RMSNorm of the activation rows -> MMA operand, QKV GEMV
  if (has_qkv) {
    bool f16 = prep_rows_regs<NCH, true>(p.x, k, mrows, gch, p.eps, x_stage, x16, escale, redf, redd, nullptr);
    NVFP4DA_PHASE(2);
    mbar_wait_bounded(&bar_qkv, 0, err);
    if (threadIdx.x == 0 && (p.sched & 7) != 0) {
      issue_kv();
      if ((p.sched & 7) == 1 || !has_attn) issue_o();
    }
    NVFP4DA_PHASE(3);
#ifdef NVFP4DA_PHASES
    if (p.sched & 16) {  // diagnostic: one step per loop iteration (small loop body)
      if (f16)
        mma_gemv_pass_smem<true, 1>(qw_smem, qs_smem, reinterpret_cast<const uint16_t*>(x16), k, p.rq, p.rq, mrows,
                                    mred, outv);
      else
        mma_gemv_pass_smem<false, 1>(qw_smem, qs_smem, x_stage, k, p.rq, p.rq, mrows, mred, outv);
    } else
#endif
    if (f16)
      mma_gemv_pass_smem<true, 4>(qw_smem, qs_smem, reinterpret_cast<const uint16_t*>(x16), k, p.rq, p.rq, mrows,
                                  mred, outv);
    else
      mma_gemv_pass_smem<false, 4>(qw_smem, qs_smem, x_stage, k, p.rq, p.rq, mrows, mred, outv);
    NVFP4DA_PHASE(13);
    const float gamma = *p.gamma[mat];
    for (int i = threadIdx.x; i < p.rq * mrows; i += kStepThreads) {
      const int n = i / p.rq, r = i % p.rq;
      const float v = f16 ? outv[r * 8 + n] * escale[n] : outv[r * 8 + n];
      p.proj[n * nqkv + qrow0 + r] = f32_to_bf16_bits(__fmul_rn(v, gamma));
    }
    cta_signal(&head_done[qrow0 / d]);
    NVFP4DA_PHASE(4);
  }

  // ---- attention unit
  if (has_attn) {
    {
      __shared__ int widx[GH + 2];
      if (threadIdx.x < GH) widx[threadIdx.x] = static_cast<int>(kvh * GH + threadIdx.x);
      if (threadIdx.x == GH) widx[GH] = static_cast<int>(hq + kvh);
      if (threadIdx.x == GH + 1) widx[GH + 1] = static_cast<int>(hq + hkv + kvh);
      __syncthreads();
      cta_wait(head_done, widx, GH + 2, static_cast<unsigned>(d / p.rq), err, p.timeout_ns);
    }
    NVFP4DA_PHASE(5);
    // Per-head RMSNorm + RoPE of this unit's query heads (and, for the split
    // holding position P_b, of the new key; the new value is the raw
    // projection) -- the arithmetic of the fused QKV epilogue.  Lane l owns
    // element pairs l, l + 32, ...: one read of the projection row.
    const int64_t nslot = pb - s0;
    for (int item = warp; item < GH + 2; item += kStepWarps) {
      const bool is_q = item < GH;
      if (!is_q && !owns_new) continue;
      const int64_t col = is_q ? (kvh * GH + item) * d : (item == GH ? (hq + kvh) * d : (hq + hkv + kvh) * d);
      const uint32_t* y2 = reinterpret_cast<const uint32_t*>(p.proj + b * nqkv + col);
      uint32_t pr2[PPL];
#pragma unroll
      for (int j = 0; j < PPL; ++j) pr2[j] = __ldcg(y2 + lane + 32 * j);
      if (item == GH + 1) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(p.v_cache + ((b * hkv + kvh) * p.capacity + pb) * d);
        uint32_t* tile = reinterpret_cast<uint32_t*>(kv_v + nslot * d);
#pragma unroll
        for (int j = 0; j < PPL; ++j) {
          tile[lane + 32 * j] = pr2[j];
          dst[lane + 32 * j] = pr2[j];
        }
        continue;
      }
      double ss = 0.0;
#pragma unroll
      for (int j = 0; j < PPL; ++j) {
        const float a = __uint_as_float(pr2[j] << 16), c = __uint_as_float(pr2[j] & 0xffff0000u);
        ss += static_cast<double>(a * a) + static_cast<double>(c * c);
      }
      ss = warp_sum_f64(ss);
      const float inv = rms_inverse(static_cast<float>(ss), static_cast<float>(d), p.eps);
      const uint32_t* g2 = reinterpret_cast<const uint32_t*>(is_q ? p.g_q : p.g_k);
      uint32_t* kdst =
          is_q ? nullptr : reinterpret_cast<uint32_t*>(p.k_cache + ((b * hkv + kvh) * p.capacity + pb) * d);
#pragma unroll
      for (int j = 0; j < PPL; ++j) {
        const int pr = lane + 32 * j;
        const uint32_t gg = g2[pr];
        const uint16_t n0 = f32_to_bf16_bits(
            __fmul_rn(__fmul_rn(__uint_as_float(pr2[j] << 16), inv), __uint_as_float(gg << 16)));
        const uint16_t n1 = f32_to_bf16_bits(
            __fmul_rn(__fmul_rn(__uint_as_float(pr2[j] & 0xffff0000u), inv), __uint_as_float(gg & 0xffff0000u)));
        uint16_t r0 = n0, r1 = n1;
        if (pb != 0) {
          float c, sn;
          if (p.rope_host_ok) {
            c = p.rope_host[pr].x;
            sn = p.rope_host[pr].y;
          } else {
            rope_cos_sin(pb, pr, d, p.theta, c, sn);
          }
          rope_pair(bf16_bits_to_f32(n0), bf16_bits_to_f32(n1), c, sn, r0, r1);
        }
        if (is_q) {
          qf[item * d + 2 * pr] = bf16_bits_to_f32(r0);
          qf[item * d + 2 * pr + 1] = bf16_bits_to_f32(r1);
        } else {
          const uint32_t both = static_cast<uint32_t>(r0) | (static_cast<uint32_t>(r1) << 16);
          reinterpret_cast<uint32_t*>(kv_k + nslot * d)[pr] = both;
          kdst[pr] = both;
        }
      }
    }
    if (n_cache > 0) mbar_wait_bounded(&bar_kv, 0, err);
    __syncthreads();
    NVFP4DA_PHASE(6);

    // Online softmax over the tile (the loop of attn_split_kernel, reading
    // shared memory): warp w takes chunks of NPOS positions.
    constexpr int NPOS = (32 / GH) > 8 ? 8 : (32 / GH);
    constexpr int NDOT = NPOS * GH;
    float q[GH][EPL];
#pragma unroll
    for (int g = 0; g < GH; ++g)
#pragma unroll
      for (int e = 0; e < EPL; ++e) q[g][e] = qf[g * d + lane * EPL + e];
    float m_run[GH], l_run[GH], acc[GH][EPL];
#pragma unroll
    for (int g = 0; g < GH; ++g) {
      m_run[g] = -INFINITY;
      l_run[g] = 0.0f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] = 0.0f;
    }
    for (int64_t c0 = s0 + warp * NPOS; c0 < s_end; c0 += kStepWarps * NPOS) {
      float kr[NPOS][EPL], vr[NPOS][EPL];
#pragma unroll
      for (int j = 0; j < NPOS; ++j) {
        if (c0 + j < s_end) {
          load_row<EPL>(kv_k + (c0 + j - s0) * d, lane, d, kr[j]);
          load_row<EPL>(kv_v + (c0 + j - s0) * d, lane, d, vr[j]);
        } else {
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
      const int my_j = lane / GH, my_g = lane % GH;
      const bool valid = lane < NDOT && (c0 + my_j) < s_end;
      const float score = valid ? __fmul_rn(dot, p.scale) : -INFINITY;
      float cmax = score;
#pragma unroll
      for (int o = GH; o < 32; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(kFull, cmax, o));
      float m_old_mine = m_run[0];
#pragma unroll
      for (int g = 1; g < GH; ++g)
        if (my_g == g) m_old_mine = m_run[g];
      const float m_new_mine = fmaxf(m_old_mine, cmax);
      const float pexp = valid ? expf(score - m_new_mine) : 0.0f;
      float psum = pexp;
#pragma unroll
      for (int o = GH; o < 32; o <<= 1) psum += __shfl_xor_sync(kFull, psum, o);
      const float alpha_mine = (m_old_mine == -INFINITY) ? 0.0f : expf(m_old_mine - m_new_mine);
#pragma unroll
      for (int g = 0; g < GH; ++g) {
        const float alpha = __shfl_sync(kFull, alpha_mine, g);
        m_run[g] = __shfl_sync(kFull, m_new_mine, g);
        l_run[g] = fmaf(l_run[g], alpha, __shfl_sync(kFull, psum, g));
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
    NVFP4DA_PHASE(7);

    // ---- combine the eight warps (their o vectors reuse the K/V tile) and
    // leave this split's (m, l, o) in the workspace
    __syncthreads();  // every warp is done with the tile
    float* sm_o = reinterpret_cast<float*>(smem + p.off_kv);  // [warps][GH][D]
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
      for (int e = 0; e < EPL; ++e) sm_o[(warp * GH + g) * 32 * EPL + lane * EPL + e] = acc[g][e];
    __syncthreads();
    if (threadIdx.x < GH) {
      const int g = threadIdx.x;
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) mx = fmaxf(mx, sm_m[w][g]);
      float l = 0.0f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) {
        const float f = (sm_m[w][g] == -INFINITY) ? 0.0f : expf(sm_m[w][g] - mx);
        wf[w][g] = f;
        l = fmaf(sm_l[w][g], f, l);
      }
      cta_m[g] = mx;
      cta_l[g] = l;
      float* ml = p.part_ml + ((b * hq + kvh * GH + g) * ns + split) * 4;
      ml[0] = mx;
      ml[1] = l;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < GH * d; idx += kStepThreads) {
      const int g = static_cast<int>(idx / d);
      const int64_t e = idx % d;
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) o = fmaf(sm_o[(w * GH + g) * 32 * EPL + e], wf[w][g], o);
      p.part_o[((b * hq + kvh * GH + g) * ns + split) * d + e] = o;
    }
    if (p.o_combine) {
      cta_signal(&sync[kSyncCtxDone]);  // counts units
    } else {
      // The last split of (b, kv head) to arrive combines all of them.
      __syncthreads();
      if (threadIdx.x == 0) {
        const unsigned prev = atom_add_acq_rel(&arrive[bh], 1u);
        s_flag = prev == static_cast<unsigned>(ns - 1) ? 1u : 0u;
      }
      __syncthreads();
      if (s_flag) {
        NVFP4DA_PHASE(8);
        float* sw = sm_o;  // free again: weights exp(m_s - M)
        for (int g = warp; g < GH; g += kStepWarps) {
          const float* ml = p.part_ml + (b * hq + kvh * GH + g) * ns * 4;
          float mx = -INFINITY;
          for (int sp = lane; sp < ns; sp += 32) mx = fmaxf(mx, __ldcg(ml + sp * 4));
          mx = warp_max_f32(mx);
          float l = 0.0f;
          for (int sp = lane; sp < ns; sp += 32) {
            const float ms = __ldcg(ml + sp * 4);
            const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
            sw[g * ns + sp] = f;
            l = fmaf(__ldcg(ml + sp * 4 + 1), f, l);
          }
          l = warp_sum_f32(l);
          if (lane == 0) cta_l[g] = l;
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < GH * d; idx += kStepThreads) {
          const int g = static_cast<int>(idx / d);
          const int64_t e = idx % d;
          const int64_t row = b * hq + kvh * GH + g;
          const float* src = p.part_o + row * ns * d + e;
          float o = 0.0f;
#pragma unroll 8
          for (int sp = 0; sp < ns; ++sp) o = fmaf(__ldcg(src + sp * d), sw[g * ns + sp], o);
          p.ctx[row * d + e] = f32_to_bf16_bits(__fdiv_rn(o, cta_l[g]));
        }
        cta_signal(&sync[kSyncCtxDone]);  // counts (b, kv head) groups
      }
    }
    if (threadIdx.x == 0 && (p.sched & 7) == 2 && has_qkv) issue_o();
    NVFP4DA_PHASE(9);
  }

  // ---- O projection
  if (has_o) {
    {
      const int idx0 = kSyncCtxDone;
      const unsigned target = p.o_combine ? static_cast<unsigned>(n_units) : static_cast<unsigned>(nb * hkv);
      cta_wait(sync, &idx0, 1, target, err, p.timeout_ns);
    }
    NVFP4DA_PHASE(10);
    bool f16;
    if (p.o_combine) {
      // Every split's partials in one bulk copy (the QKV/KV region is dead),
      // then the log-sum-exp combine of reference decoder_attention.py's
      // softmax, split by split in order, per (row, head) item.
      float* co = reinterpret_cast<float*>(smem + p.off_comb);
      const int64_t items = nb * hq;
      float* cml = co + items * ns * d;
      if (threadIdx.x == 0) {
        const uint32_t ob = static_cast<uint32_t>(items * ns * d * 4), mb = static_cast<uint32_t>(items * ns * 16);
        asm volatile("fence.proxy.async.global;" ::: "memory");  // acquired generic writes -> bulk reads
        mbar_arrive_expect_tx(&bar_c, ob + mb);
        bulk_g2s(co, p.part_o, ob, &bar_c);
        bulk_g2s(cml, p.part_ml, mb, &bar_c);
      }
      mbar_wait_bounded(&bar_c, 0, err);
      for (int64_t it = warp; it < items; it += kStepWarps) {
        const float* ml = cml + it * ns * 4;
        float mx = -INFINITY;
        for (int sp = 0; sp < ns; ++sp) mx = fmaxf(mx, ml[sp * 4]);
        float l = 0.0f, o[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
        const float* ob = co + it * ns * d + lane * EPL;
        for (int sp = 0; sp < ns; ++sp) {
          const float ms = ml[sp * 4];
          const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
          l = fmaf(ml[sp * 4 + 1], f, l);
#pragma unroll
          for (int e = 0; e < EPL; ++e) o[e] = fmaf(ob[sp * d + e], f, o[e]);
        }
        const int64_t m = it / hq, h = it % hq;
        uint16_t* dst = x_stage + m * k + h * d + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[e] = f32_to_bf16_bits(__fdiv_rn(o[e], l));
      }
      __syncthreads();
      NVFP4DA_PHASE(14);
      f16 = mma_prepare_f16(x_stage, x16, k, mrows, escale, red_small);
    } else {
      const uint4 none[NCH] = {};
      f16 = prep_rows_regs<NCH, false, true>(p.ctx, k, mrows, none, 0.0f, x_stage, x16, escale, redf, redd, nullptr);
    }
    mbar_wait_bounded(&bar_o, 0, err);
    NVFP4DA_PHASE(11);
    if (f16)
      mma_gemv_pass_smem<true, 4>(ow_smem, os_smem, reinterpret_cast<const uint16_t*>(x16), k, p.o_tile_rows,
                                  o_valid, mrows, mred, outv);
    else
      mma_gemv_pass_smem<false, 4>(ow_smem, os_smem, x_stage, k, p.o_tile_rows, o_valid, mrows, mred, outv);
    const float gamma = *p.gamma[3];
    for (int i = threadIdx.x; i < o_valid * mrows; i += kStepThreads) {
      const int n = i / o_valid, r = i % o_valid;
      const float v = f16 ? outv[r * 8 + n] * escale[n] : outv[r * 8 + n];
      p.out[n * k + orow0 + r] = f32_to_bf16_bits(__fmul_rn(v, gamma));
    }
    NVFP4DA_PHASE(12);
  }

  // ---- leave; the last CTA out clears the slot's counters for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atom_add_acq_rel(&sync[kSyncExit], 1u);
    s_flag = prev == gridDim.x - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (s_flag) {
    const int64_t words = (hq + 2 * hkv) + nb * hkv;
    for (int64_t i = threadIdx.x; i < words; i += kStepThreads) head_done[i] = 0u;
    if (threadIdx.x == 0) {
      sync[kSyncCtxDone] = 0u;
      sync[kSyncExit] = 0u;
    }
  }
}

}  // namespace nvfp4da
