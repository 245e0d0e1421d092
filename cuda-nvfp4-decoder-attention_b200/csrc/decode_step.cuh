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
//    online-softmax loop over its K/V tile, and leaves (m, l, o) partials; the
//    last split to arrive combines them into the BF16 context.
//  * O block c: rows [c*RO, c*RO + RO) of Wo, after every context row is done.
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
  int rq, rq_rows, n_qkv_blocks;  // rows per QKV block, tile-padded rows
  int ro, ro_rows, n_o_blocks;
  int splits, split_len;
  // workspace
  uint16_t* proj;   // [B, (Hq + 2 Hkv) D] raw projections
  uint16_t* ctx;    // [B, H]
  float* partials;  // [B * Hq, splits, D + 2]
  unsigned* sync;   // slot
  unsigned long long timeout_ns;
  // dynamic shared-memory layout (byte offsets)
  uint32_t off_qs, off_qw, off_os, off_ow, off_kv, off_q, off_xs, off_x16, off_red;
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
__device__ __forceinline__ void cta_signal(unsigned* ctr) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
  }
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
    __threadfence();
  }
  __syncthreads();
}

// ---------------------------------------------------------------- the kernel
template <int EPL, int GH>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t bar_qkv, bar_kv, bar_o;
  __shared__ float redf[2 * kStepWarps];
  __shared__ double redd[2 * kStepWarps];
  __shared__ float escale[kMmaMaxM];
  __shared__ float outv[kStepMaxRows * 8];
  __shared__ float sm_m[kStepWarps][GH], sm_l[kStepWarps][GH], wf[kStepWarps][GH], cta_m[GH], cta_l[GH];
  __shared__ unsigned s_flag;
  [[maybe_unused]] constexpr unsigned kPhaseBase = 3072;
  NVFP4DA_PHASE(0);

  const int cta = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t k = p.hidden, d = p.head_dim, nb = p.batch;
  const int mrows = static_cast<int>(nb);  // T = 1: one activation row per sequence
  const int64_t hq = p.q_heads, hkv = p.kv_heads;
  const int64_t nqkv = (hq + 2 * hkv) * d;
  unsigned* sync = p.sync;
  unsigned* err = sync + kSyncErr;
  unsigned* head_done = sync + kSyncHeads;                 // [Hq + 2 Hkv]
  unsigned* arrive = head_done + (hq + 2 * hkv);           // [B * Hkv]

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
  const bool has_o = cta < p.n_o_blocks;
  const int n_units = static_cast<int>(nb * hkv) * p.splits;
  const bool has_attn = cta < n_units;

  const int64_t qrow0 = static_cast<int64_t>(cta) * p.rq;  // concatenated QKV row
  const int mat = qrow0 < hq * d ? 0 : (qrow0 < (hq + hkv) * d ? 1 : 2);
  const int64_t mat_row0 = qrow0 - (mat == 0 ? 0 : (mat == 1 ? hq * d : (hq + hkv) * d));
  const int64_t orow0 = static_cast<int64_t>(cta) * p.ro;
  const int o_valid = has_o ? static_cast<int>((k - orow0) < p.ro ? (k - orow0) : p.ro) : 0;

  const int split = has_attn ? cta % p.splits : 0;
  const int64_t bh = has_attn ? cta / p.splits : 0;
  const int64_t b = bh / hkv, kvh = bh % hkv;
  const int64_t pb = has_attn ? (p.past_lengths ? p.past_lengths[b] : p.past_length) : 0;
  const int64_t s0 = static_cast<int64_t>(split) * p.split_len;
  // Keys 0 .. P_b; never beyond the physical capacity, whatever a device-side
  // length says.
  int64_t s_end = pb + 1 < p.capacity ? pb + 1 : p.capacity;
  if (s_end > s0 + p.split_len) s_end = s0 + p.split_len;
  int64_t cache_end = pb < s_end ? pb : s_end;  // rows [s0, cache_end) come from the cache
  const int64_t n_cache = cache_end > s0 ? cache_end - s0 : 0;
  const bool owns_new = has_attn && pb >= 0 && pb < p.capacity && pb >= s0 && pb < s0 + p.split_len;
  const uint16_t* kbase = p.k_cache + (b * hkv + kvh) * p.capacity * d;
  const uint16_t* vbase = p.v_cache + (b * hkv + kvh) * p.capacity * d;

  if (threadIdx.x == 0) {
    mbar_init(&bar_qkv, 1);
    mbar_init(&bar_kv, 1);
    mbar_init(&bar_o, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- put every input slice of this CTA in flight (none is written by the step)
  if (threadIdx.x == 0) {
    const int64_t ks = k / 16, kb = k / 2;
    if (has_qkv) {
      const uint32_t sb = static_cast<uint32_t>(p.rq * ks), wb = static_cast<uint32_t>(p.rq * kb);
      mbar_arrive_expect_tx(&bar_qkv, sb + wb);
      bulk_g2s(qs_smem, p.scales[mat] + mat_row0 * ks, sb, &bar_qkv);
      bulk_g2s(qw_smem, p.packed[mat] + mat_row0 * kb, wb, &bar_qkv);
    }
    if (n_cache > 0) {
      const uint32_t tb = static_cast<uint32_t>(n_cache * d * 2);
      mbar_arrive_expect_tx(&bar_kv, 2 * tb);
      bulk_g2s(kv_k, kbase + s0 * d, tb, &bar_kv);
      bulk_g2s(kv_v, vbase + s0 * d, tb, &bar_kv);
    }
    if (has_o) {
      const uint32_t sb = static_cast<uint32_t>(o_valid * ks), wb = static_cast<uint32_t>(o_valid * kb);
      mbar_arrive_expect_tx(&bar_o, sb + wb);
      bulk_g2s(os_smem, p.scales[3] + orow0 * ks, sb, &bar_o);
      bulk_g2s(ow_smem, p.packed[3] + orow0 * kb, wb, &bar_o);
    }
  }
  NVFP4DA_PHASE(1);

  // ---- input RMSNorm of the activation rows -> MMA operand (every CTA)
  constexpr int NCH = 2;
  uint4 gch[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int idx = threadIdx.x + c * kStepThreads;
    gch[c] = idx < k / 8 ? ldg_stream(p.g_in + 8 * idx) : make_uint4(0u, 0u, 0u, 0u);
  }
  if (has_qkv) {
    bool f16 = prep_rows_regs<NCH, true>(p.x, k, mrows, gch, p.eps, x_stage, x16, escale, redf, redd, nullptr);
    NVFP4DA_PHASE(2);
    mbar_wait_bounded(&bar_qkv, 0, err);
    NVFP4DA_PHASE(3);
    if (f16)
      mma_gemv_pass_smem<true, 4>(qw_smem, qs_smem, reinterpret_cast<const uint16_t*>(x16), k, p.rq_rows, mrows,
                                  mred, outv);
    else
      mma_gemv_pass_smem<false, 4>(qw_smem, qs_smem, x_stage, k, p.rq_rows, mrows, mred, outv);
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
    // projection) -- the arithmetic of the fused QKV epilogue.
    const int64_t nslot = pb - s0;
    for (int item = warp; item < GH + 2; item += kStepWarps) {
      const bool is_q = item < GH;
      if (!is_q && !owns_new) continue;
      const int64_t col = is_q ? (kvh * GH + item) * d : (item == GH ? (hq + kvh) * d : (hq + hkv + kvh) * d);
      const uint16_t* y = p.proj + b * nqkv + col;
      if (item == GH + 1) {
        uint16_t* dst = p.v_cache + ((b * hkv + kvh) * p.capacity + pb) * d;
        for (int64_t e = lane; e < d; e += 32) {
          const uint16_t v = __ldcg(y + e);
          kv_v[nslot * d + e] = v;
          dst[e] = v;
        }
        continue;
      }
      double ss = 0.0;
      for (int64_t e = lane; e < d; e += 32) {
        const float v = bf16_bits_to_f32(__ldcg(y + e));
        ss += static_cast<double>(v * v);
      }
      ss = warp_sum_f64(ss);
      const float inv = rms_inverse(static_cast<float>(ss), static_cast<float>(d), p.eps);
      const uint16_t* g = is_q ? p.g_q : p.g_k;
      uint16_t* kdst = is_q ? nullptr : p.k_cache + ((b * hkv + kvh) * p.capacity + pb) * d;
      for (int64_t pr = lane; pr < d / 2; pr += 32) {
        const int64_t e = 2 * pr;
        const uint16_t n0 =
            f32_to_bf16_bits(__fmul_rn(__fmul_rn(bf16_bits_to_f32(__ldcg(y + e)), inv), bf16_bits_to_f32(g[e])));
        const uint16_t n1 = f32_to_bf16_bits(
            __fmul_rn(__fmul_rn(bf16_bits_to_f32(__ldcg(y + e + 1)), inv), bf16_bits_to_f32(g[e + 1])));
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
          qf[item * d + e] = bf16_bits_to_f32(r0);
          qf[item * d + e + 1] = bf16_bits_to_f32(r1);
        } else {
          kv_k[nslot * d + e] = r0;
          kv_k[nslot * d + e + 1] = r1;
          kdst[e] = r0;
          kdst[e + 1] = r1;
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

    // ---- combine the eight warps (their o vectors reuse the K/V tile)
    __syncthreads();  // every warp is done with the tile
    float* sm_o = reinterpret_cast<float*>(smem + p.off_kv);  // [warps][GH][32 * EPL]
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
    }
    __syncthreads();
    const int ns = p.splits;
    for (int idx = threadIdx.x; idx < GH * d; idx += kStepThreads) {
      const int g = static_cast<int>(idx / d);
      const int64_t e = idx % d;
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) o = fmaf(sm_o[(w * GH + g) * 32 * EPL + e], wf[w][g], o);
      const int64_t row = b * hq + kvh * GH + g;
      if (ns == 1) {
        p.ctx[row * d + e] = f32_to_bf16_bits(__fdiv_rn(o, cta_l[g]));
      } else {
        float* dst = p.partials + (row * ns + split) * (d + 2);
        dst[e] = o;
        if (e == 0) {
          dst[d] = cta_m[g];
          dst[d + 1] = cta_l[g];
        }
      }
    }
    bool combine = ns == 1;
    if (ns > 1) {
      // The last split of (b, kv head) to arrive combines all of them.
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&arrive[bh], 1u);
        s_flag = prev == static_cast<unsigned>(ns - 1) ? 1u : 0u;
        __threadfence();
      }
      __syncthreads();
      combine = s_flag != 0;
      if (combine) {
        NVFP4DA_PHASE(8);
        // (m, l) of every split -> weights exp(m_s - M); sm_o is free again.
        float* sw = sm_o;
        float* sl = sw + GH * ns;
        for (int i = threadIdx.x; i < GH * ns; i += kStepThreads) {
          const int g = i / ns, sp = i % ns;
          const float* src = p.partials + ((b * hq + kvh * GH + g) * ns + sp) * (d + 2);
          sw[i] = __ldcg(src + d);
          sl[i] = __ldcg(src + d + 1);
        }
        __syncthreads();
        for (int g = warp; g < GH; g += kStepWarps) {
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
          if (lane == 0) cta_l[g] = l;
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < GH * d; idx += kStepThreads) {
          const int g = static_cast<int>(idx / d);
          const int64_t e = idx % d;
          const int64_t row = b * hq + kvh * GH + g;
          const float* src = p.partials + row * ns * (d + 2) + e;
          float o = 0.0f;
#pragma unroll 8
          for (int sp = 0; sp < ns; ++sp) o = fmaf(__ldcg(src + sp * (d + 2)), sw[g * ns + sp], o);
          p.ctx[row * d + e] = f32_to_bf16_bits(__fdiv_rn(o, cta_l[g]));
        }
      }
    }
    if (combine) cta_signal(&sync[kSyncCtxDone]);
    NVFP4DA_PHASE(9);
  }

  // ---- O projection
  if (has_o) {
    {
      const int zero = kSyncCtxDone;
      cta_wait(sync, &zero, 1, static_cast<unsigned>(nb * hkv), err, p.timeout_ns);
    }
    NVFP4DA_PHASE(10);
    const uint4 none[NCH] = {};
    const bool f16 =
        prep_rows_regs<NCH, false, true>(p.ctx, k, mrows, none, 0.0f, x_stage, x16, escale, redf, redd, nullptr);
    mbar_wait_bounded(&bar_o, 0, err);
    NVFP4DA_PHASE(11);
    if (f16)
      mma_gemv_pass_smem<true, 4>(ow_smem, os_smem, reinterpret_cast<const uint16_t*>(x16), k, p.ro_rows, mrows,
                                  mred, outv);
    else
      mma_gemv_pass_smem<false, 4>(ow_smem, os_smem, x_stage, k, p.ro_rows, mrows, mred, outv);
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
    __threadfence();
    const unsigned prev = atomicAdd(&sync[kSyncExit], 1u);
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
