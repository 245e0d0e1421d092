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
//    tensor-core GEMV from shared memory and publishes the raw BF16
//    projections.
//  * Attention unit (b, kv head, split j): positions [j*L, j*L + L) of
//    sequence b.  Takes the projections of its GH query heads and its K and V
//    head as they are published, applies the per-head RMSNorm + RoPE to those
//    rows itself, appends the new K/V row to the cache (the split holding
//    position P_b), runs the online-softmax loop over its K/V tile and
//    publishes (m, l, o) partials.  Then the splits of (b, kv head) combine
//    together: split j takes every split's partials for its share of the
//    GH x D context and publishes that share as BF16.
//  * O block c: 8-row multiples of Wo (the rows spread over all CTAs): takes
//    the context as it is published and runs the O GEMV.
//
// Hand-offs between CTAs carry their own validity: every published value is
// a 64-bit word (32 bits of data, 32 bits of tag) stored and polled with
// relaxed gpu-scope accesses, which are single-copy atomic.  The words live
// in the stream's slot of library-owned device memory, written only by this
// stream's step launches; the tag is the launch's epoch (kept in the slot,
// advanced by the last CTA to leave), so no value of an earlier launch
// passes for this launch's.  One round trip through L2 per hand-off: no
// separate counter to release and acquire.  Every wait is bounded by a time
// limit; on expiry the kernel records kErrBarrierTimeout in the slot and
// carries on (results are then garbage, the GPU stays usable).
#pragma once

#include "attention.cuh"
#include "attention_prefill.cuh"  // ldsm_x4
#include "elementwise.cuh"
#include "gemv_mma.cuh"
#include "qkv_fused.cuh"  // kMaxHeadDim

namespace nvfp4da {

constexpr int kStepThreads = kMmaThreads;
constexpr int kStepWarps = kMmaWarps;
constexpr int kStepMaxRows = 128;    // RQ / RO rows per CTA (tile-padded)
constexpr int kStepSyncWords = 2048;  // one slot
// Slot layout (32-bit words).
constexpr int kSyncExit = 0, kSyncEpoch = 1, kSyncErr = 2;
constexpr size_t kStepTagWords = 65536;  // hand-off words per slot (512 KB)

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
  // the slot's hand-off region: tagged words (low 32 bits data, high 32 bits tag)
  unsigned long long* proj;     // [B, (Hq + 2 Hkv) D / 2] raw projections, BF16 pairs
  unsigned long long* ctx;      // [B, H / 2]              context, BF16 pairs
  unsigned long long* part_o;   // [B * Hq, splits, D]     FP32
  unsigned long long* part_ml;  // [B * Hq, splits, 2]     FP32 (m, l)
  unsigned long long* xin;      // [B, H / 2]              activation rows read from host memory, BF16 pairs
  // Activation rows in page-locked host memory mapped into the device's
  // address space, or nullptr (then x).  Each CTA reads a slice of them over
  // the host link once and publishes it as tagged words (xin); the QKV CTAs
  // poll the whole rows from L2.  One host read per byte, no copy engine.
  const uint16_t* x_mapped;
  size_t tag_words;             // the region's size, cleared when the epoch wraps
  unsigned* sync;    // slot
  unsigned long long timeout_ns;
  // dynamic shared-memory layout (byte offsets); qs/qw/kv/q and comb overlay
  uint32_t off_qs, off_qw, off_kv, off_q, off_os, off_ow, off_xs, off_x16, off_red;
  // O rows decoded ahead into f16 rows at off_od (stride od_ld halves), which
  // overlays the QKV rows, the K/V tile and q once they are consumed.
  int o_predecode;
  uint32_t off_od;
  int od_ld;
  // RoPE: rope_host_ok == 1: (cos, sin) at position past_length; == 2: .x holds
  // theta^(2m/D) in FP32 and the angle and its cos / sin come from the device
  // (per-sequence lengths read on the device).
  int rope_host_ok;
  float2 rope_host[kMaxHeadDim / 2];
};

// The launch's parameter block.  With XI the activation rows travel inside
// it (the host-buffer entry point copies them there on the host), so a step
// whose input starts in host memory needs no copy-engine transfer before the
// kernel: the rows reach every SM through the constant cache with the launch.
constexpr int kStepInlineX = 3072;  // activation elements (6 KB; a 16 KB block measured 2 us slower)
template <bool XI>
struct StepLaunch {
  StepParams p;
};
template <>
struct StepLaunch<true> {
  StepParams p;
  uint4 x[kStepInlineX / 8];
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

// Wait for an mbarrier phase with the non-suspending test_wait, bounded by the
// launch's deadline: a suspended try_wait can sleep past the phase flip, and
// these waits sit on the critical path.
__device__ __forceinline__ void mbar_spin_until(uint64_t* bar, uint32_t parity, unsigned long long deadline,
                                                unsigned* err) {
  for (uint32_t i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return;
    if ((i & 255u) == 255u && global_ns() > deadline) {
      atomicOr(err, static_cast<unsigned>(kErrBarrierTimeout));
      return;
    }
  }
}

// Tagged words: 32 bits of data (low) and the launch's tag (high).
__device__ __forceinline__ void st_tagged(unsigned long long* p, uint32_t v, uint32_t tag) {
  const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | v;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Poll N tagged words of this thread at once until all carry `tag` or the
// deadline passes (then the timeout is recorded in *err and the last values
// read are returned).  Each round costs one L2 round trip for all N.
template <int N>
__device__ __forceinline__ void poll_tagged(const unsigned long long* const (&src)[N], uint32_t (&out)[N],
                                            uint32_t tag, unsigned long long deadline, unsigned* err) {
  static_assert(N >= 1 && N <= 32, "at most 32 words per poll");
  constexpr uint32_t kAll = N == 32 ? 0xFFFFFFFFu : (1u << (N & 31)) - 1u;
  uint32_t have = 0;
  for (;;) {
    unsigned long long w[N];
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (!(have >> i & 1u)) w[i] = ld_tagged(src[i]);
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (!(have >> i & 1u) && static_cast<uint32_t>(w[i] >> 32) == tag) {
        out[i] = static_cast<uint32_t>(w[i]);
        have |= 1u << i;
      }
    if (have == kAll) return;
    if (global_ns() > deadline) {
      atomicOr(err, static_cast<unsigned>(kErrBarrierTimeout));
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (!(have >> i & 1u)) out[i] = static_cast<uint32_t>(w[i]);
      return;
    }
  }
}

// ---------------------------------------------------------------- O rows decoded ahead
// Decode `rows` weight rows (packed [rows][K/2], scales [rows][K/16], both in
// shared memory) into f16 rows of stride `ld` halves: (q * beta) exactly, in
// natural k order.  Called by every thread; the caller synchronises.
__device__ __forceinline__ void predecode_rows_f16(const uint8_t* w_smem, const uint8_t* s_smem, int64_t k, int rows,
                                                   __half* dst, int ld) {
  const int chunks = static_cast<int>(k / 32);  // 16 packed bytes = 32 k = two scale blocks
  const int64_t kb = k / 2, ks = k / 16;
  for (int i = threadIdx.x; i < rows * chunks; i += blockDim.x) {
    const int r = i / chunks, c = i % chunks;
    const uint4 w = *reinterpret_cast<const uint4*>(w_smem + r * kb + 16 * c);
    const uint32_t s2 = *reinterpret_cast<const uint16_t*>(s_smem + r * ks + 2 * c);
    const uint32_t sc[2] = {ue4m3_to_f16x2_dup(s2), ue4m3_to_f16x2_dup(s2 >> 8)};
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    uint4* o = reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * ld + 32 * c);
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // word q: k = 32 c + 8 q .. + 7 (block 2 c + q / 2)
      uint32_t h[4];
      e2m1x8_to_f16x2x4(wv[q], h);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = hmul2_u32(h[j], sc[q >> 1]);
      o[q] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
}

// The O pass over rows decoded ahead: A fragments by ldmatrix from the f16
// rows (stride `ld` halves), B from the activation operand rows (f16, or
// bf16 with A converted -- exact either way), 16 k per MMA, four accumulator
// chains; then the cross-warp reduction into out[r * 8 + n].  `rows` is
// tile-padded; rows at or past `valid_rows` are never read (a tile's upper
// half past them re-reads its lower half) and their outputs are discarded.
template <bool F16>
__device__ __forceinline__ void mma_pass_decoded(const __half* a_smem, int ld, const uint16_t* xop, int64_t k,
                                                 int rows, int valid_rows, int mgv, float* red, float* out) {
  const WarpSlice ws = warp_slice(rows, k);
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float d[4][4] = {};
  if (ws.tile * 16 < valid_rows) {
    const bool hi = ws.tile * 16 + 8 < valid_rows;
    const int mat = lane >> 3;
    const int row = ws.tile * 16 + (lane & 7) + ((mat & 1) && hi ? 8 : 0);
    const uint32_t abase = smem_u32(a_smem) + static_cast<uint32_t>((row * ld + (mat >> 1) * 8) * 2);
    const bool has_n = g < mgv;
    const uint16_t* xrow = xop + static_cast<int64_t>(has_n ? g : 0) * k + 2 * t;
#pragma unroll 1
    for (int s = ws.s0; s < ws.s1; ++s) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k0 = s * kStepK + 16 * j;
        uint32_t a[4];
        ldsm_x4(abase + k0 * 2, a[0], a[1], a[2], a[3]);
        const uint32_t b0 = has_n ? *reinterpret_cast<const uint32_t*>(xrow + k0) : 0u;
        const uint32_t b1 = has_n ? *reinterpret_cast<const uint32_t*>(xrow + k0 + 8) : 0u;
        if constexpr (F16) {
          mma_f16(d[j & 3], a, b0, b1);
        } else {
          const uint32_t ab[4] = {f16x2_to_bf16x2(a[0]), f16x2_to_bf16x2(a[1]), f16x2_to_bf16x2(a[2]),
                                  f16x2_to_bf16x2(a[3])};
          mma_bf16(d[j & 3], ab, b0, b1);
        }
      }
    }
  }
  float dsum[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dsum[i] = (d[0][i] + d[1][i]) + (d[2][i] + d[3][i]);
  reduce_tiles(dsum, rows, red, out);
}

// ---------------------------------------------------------------- the kernel
template <int EPL, int GH, bool XI>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepLaunch<XI> launch) {
  const StepParams& p = launch.p;
  // Activation rows: global memory, or (XI) the parameter block itself, read
  // with generic loads through the parameter space's address.
  const uint16_t* xin;
  if constexpr (XI)
    xin = reinterpret_cast<const uint16_t*>(launch.x);
  else
    xin = p.x;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t bar_qkv, bar_kv, bar_o;
  __shared__ float redf[2 * kStepWarps];
  __shared__ double redd[2 * kStepWarps];
  __shared__ float escale[kMmaMaxM];
  __shared__ float red_small[kMmaMaxM * kStepWarps];
  __shared__ float outv[kStepMaxRows * 8];
  __shared__ float sm_m[kStepWarps][GH], sm_l[kStepWarps][GH], cta_l[GH];
  __shared__ unsigned s_flag;
  [[maybe_unused]] constexpr unsigned kPhaseBase = 3072;
  constexpr int PPL = EPL / 2;  // RoPE pairs per lane (D = 32 * EPL)
  NVFP4DA_PHASE(0);

  const int cta = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t k = p.hidden, d = p.head_dim, nb = p.batch;
  const int mrows = static_cast<int>(nb);  // T = 1: one activation row per sequence
  const int64_t hq = p.q_heads, hkv = p.kv_heads;
  const int64_t nqkv = (hq + 2 * hkv) * d;
  const int ns = p.splits;
  unsigned* sync = p.sync;
  unsigned* err = sync + kSyncErr;

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
  // O rows: the o_n_big CTAs at the end of the grid take o_rows_big rows,
  // the others o_rows_small (the attention units sit at the start).
  int64_t orow0;
  int o_rows;
  const int o_n_small = static_cast<int>(gridDim.x) - p.o_n_big;
  if (cta < o_n_small) {
    o_rows = p.o_rows_small;
    orow0 = static_cast<int64_t>(cta) * p.o_rows_small;
  } else {
    o_rows = p.o_rows_big;
    orow0 = static_cast<int64_t>(o_n_small) * p.o_rows_small + static_cast<int64_t>(cta - o_n_small) * p.o_rows_big;
  }
  const int o_valid = orow0 < k ? static_cast<int>((k - orow0) < o_rows ? (k - orow0) : o_rows) : 0;
  const bool has_o = o_valid > 0;

  const int64_t qrow0 = static_cast<int64_t>(cta) * p.rq;  // concatenated QKV row
  const int mat = qrow0 < hq * d ? 0 : (qrow0 < (hq + hkv) * d ? 1 : 2);
  const int64_t mat_row0 = qrow0 - (mat == 0 ? 0 : (mat == 1 ? hq * d : (hq + hkv) * d));
  const int64_t ks = k / 16, kb = k / 2;
  // The QKV slice heads the critical path: thread 0 requests it before
  // anything else (the barrier below publishes the initialised mbarriers to
  // the other threads before they wait on them).
  if (threadIdx.x == 0) {
    mbar_init(&bar_qkv, 1);
    mbar_init(&bar_kv, 1);
    mbar_init(&bar_o, 1);
    fence_mbar_init();
    if (has_qkv) {
      const uint32_t sb = static_cast<uint32_t>(p.rq * ks), wb = static_cast<uint32_t>(p.rq * kb);
      mbar_arrive_expect_tx(&bar_qkv, sb + wb);
      bulk_g2s(qs_smem, p.scales[mat] + mat_row0 * ks, sb, &bar_qkv);
      bulk_g2s(qw_smem, p.packed[mat] + mat_row0 * kb, wb, &bar_qkv);
    }
  }

  const int split = has_attn ? cta % ns : 0;
  const int64_t bh = has_attn ? cta / ns : 0;
  const int64_t b = static_cast<int>(bh) / static_cast<int>(hkv), kvh = static_cast<int>(bh) % static_cast<int>(hkv);
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

  // This launch's tag (1 .. 2^32 - 1): every thread loads the epoch word now
  // and first uses it microseconds later, so the load's latency is hidden.
  uint32_t epoch;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(epoch) : "l"(sync + kSyncEpoch) : "memory");
  const uint32_t tag = epoch + 1u;
  // ---- activation rows from host memory: this CTA's 16-byte chunks, read by
  // the last warp (warp 0's thread 0 has the bulk copies to issue).
  if (p.x_mapped != nullptr && warp == kStepWarps - 1) {
    const int64_t n16 = nb * k / 8;
    const int64_t per = (n16 + gridDim.x - 1) / gridDim.x;
    const int64_t c_end = (cta + 1) * per < n16 ? (cta + 1) * per : n16;
    for (int64_t c = cta * per + lane; c < c_end; c += 32) {
      const uint4 v = reinterpret_cast<const uint4*>(p.x_mapped)[c];
      st_tagged(p.xin + 4 * c + 0, v.x, tag);
      st_tagged(p.xin + 4 * c + 1, v.y, tag);
      st_tagged(p.xin + 4 * c + 2, v.z, tag);
      st_tagged(p.xin + 4 * c + 3, v.w, tag);
    }
  }
  // ---- the activation rows and the input-norm gain first: they head the
  // critical path, so their requests go out before any bulk traffic.
  constexpr int NCH = 2;
  uint4 gch[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int idx = threadIdx.x + c * kStepThreads;
    gch[c] = idx < k / 8 ? ldg_stream(p.g_in + 8 * idx) : make_uint4(0u, 0u, 0u, 0u);
    if (!XI && p.x_mapped == nullptr && idx < k / 8)
      for (int m = 0; m < mrows; ++m) asm volatile("prefetch.global.L2 [%0];" ::"l"(xin + m * k + 8 * idx));
  }

  __syncthreads();
  const unsigned long long deadline = global_ns() + p.timeout_ns;

  // ---- input slices of this CTA (none is written by the step): the QKV
  // rows now, the K/V tile and the O rows once the QKV rows have landed, so
  // that they do not queue ahead of the critical path (CTAs without QKV
  // rows request them at once).
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
  if (threadIdx.x == 0 && !has_qkv) {
    issue_kv();
    issue_o();
  }
  NVFP4DA_PHASE(1);
  // Small inputs read late on the critical path (the projections' global
  // scales, the per-head norm gains): loaded now, used microseconds later.
  const float gamma_qkv = has_qkv ? __ldg(p.gamma[mat]) : 0.0f;
  const float gamma_o = has_o ? __ldg(p.gamma[3]) : 0.0f;
  uint32_t gq2[PPL], gk2[PPL];
#pragma unroll
  for (int j = 0; j < PPL; ++j) {
    gq2[j] = has_attn ? __ldg(reinterpret_cast<const uint32_t*>(p.g_q) + lane + 32 * j) : 0u;
    gk2[j] = has_attn ? __ldg(reinterpret_cast<const uint32_t*>(p.g_k) + lane + 32 * j) : 0u;
  }


  // ---- input RMSNorm of the activation rows -> MMA operand, QKV GEMV
  if (has_qkv) {
    if (p.x_mapped != nullptr) {
      // Every CTA's published slice of the rows, into x_stage (the prep
      // functions below read their input before writing x_stage).
      const int pairs = static_cast<int>(nb * k / 2);
      uint32_t* xs2 = reinterpret_cast<uint32_t*>(x_stage);
      for (int i0 = threadIdx.x; i0 < pairs; i0 += 8 * kStepThreads) {
        const unsigned long long* src[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j * kStepThreads;
          src[j] = p.xin + (i < pairs ? i : i0);
        }
        uint32_t v[8];
        poll_tagged<8>(src, v, tag, deadline, err);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j * kStepThreads < pairs) xs2[i0 + j * kStepThreads] = v[j];
      }
      __syncthreads();
      xin = x_stage;
    }
    bool f16 = mrows > 1 ? prep_rows_warp<true>(xin, p.g_in, k, mrows, p.eps, x_stage, x16, escale, nullptr)
                         : prep_rows_regs<NCH, true>(xin, k, mrows, gch, p.eps, x_stage, x16, escale, redf, redd, nullptr);
    NVFP4DA_PHASE(2);
    mbar_spin_until(&bar_qkv, 0, deadline, err);
    if (threadIdx.x == 0) {
      issue_kv();
      issue_o();
    }
    NVFP4DA_PHASE(3);
    if (f16)
      mma_gemv_pass_smem<true, 4>(qw_smem, qs_smem, reinterpret_cast<const uint16_t*>(x16), k, p.rq, p.rq, mrows,
                                  mred, outv);
    else
      mma_gemv_pass_smem<false, 4>(qw_smem, qs_smem, x_stage, k, p.rq, p.rq, mrows, mred, outv);
    NVFP4DA_PHASE(13);
    const float gamma = gamma_qkv;
    const int rq2 = p.rq / 2;  // BF16 pairs (RQ and the row offsets are even)
    for (int i = threadIdx.x; i < rq2 * mrows; i += kStepThreads) {
      const int n = i / rq2, r = 2 * (i % rq2);
      const float v0 = f16 ? outv[r * 8 + n] * escale[n] : outv[r * 8 + n];
      const float v1 = f16 ? outv[(r + 1) * 8 + n] * escale[n] : outv[(r + 1) * 8 + n];
      const uint32_t pair = f32_to_bf16_bits(__fmul_rn(v0, gamma)) |
                            (static_cast<uint32_t>(f32_to_bf16_bits(__fmul_rn(v1, gamma))) << 16);
      st_tagged(p.proj + (n * nqkv + qrow0 + r) / 2, pair, tag);
    }
    NVFP4DA_PHASE(4);
  }

  // ---- attention unit
  if (has_attn) {
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
      const unsigned long long* y2 = p.proj + (b * nqkv + col) / 2;
      const unsigned long long* src[PPL];
#pragma unroll
      for (int j = 0; j < PPL; ++j) src[j] = y2 + lane + 32 * j;
      uint32_t pr2[PPL];
      poll_tagged<PPL>(src, pr2, tag, deadline, err);
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
      uint32_t* kdst =
          is_q ? nullptr : reinterpret_cast<uint32_t*>(p.k_cache + ((b * hkv + kvh) * p.capacity + pb) * d);
#pragma unroll
      for (int j = 0; j < PPL; ++j) {
        const int pr = lane + 32 * j;
        const uint32_t gg = is_q ? gq2[j] : gk2[j];
        const uint16_t n0 = f32_to_bf16_bits(
            __fmul_rn(__fmul_rn(__uint_as_float(pr2[j] << 16), inv), __uint_as_float(gg << 16)));
        const uint16_t n1 = f32_to_bf16_bits(
            __fmul_rn(__fmul_rn(__uint_as_float(pr2[j] & 0xffff0000u), inv), __uint_as_float(gg & 0xffff0000u)));
        uint16_t r0 = n0, r1 = n1;
        if (pb != 0) {
          float c, sn;
          if (p.rope_host_ok == 1) {
            c = p.rope_host[pr].x;
            sn = p.rope_host[pr].y;
          } else {
            rope_cos_sin_denom(pb, p.rope_host[pr].x, c, sn);
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
    NVFP4DA_PHASE(18);
    if (n_cache > 0) mbar_spin_until(&bar_kv, 0, deadline, err);
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
    NVFP4DA_PHASE(16);
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
    // One thread per (head, warp) computes that warp's weight exp(m_w - M);
    // then every item is an 8-term FMA chain in warp order, and one thread per
    // head publishes (M, l).
    float* wsm = reinterpret_cast<float*>(outv);  // [GH][warps], free until the O pass
    if (threadIdx.x < GH * kStepWarps) {
      const int g = threadIdx.x / kStepWarps, w = threadIdx.x % kStepWarps;
      float mx = -INFINITY;
#pragma unroll
      for (int u = 0; u < kStepWarps; ++u) mx = fmaxf(mx, sm_m[u][g]);
      wsm[threadIdx.x] = (sm_m[w][g] == -INFINITY) ? 0.0f : expf(sm_m[w][g] - mx);
      if (w == 0) cta_l[g] = mx;
    }
    __syncthreads();
    const int di = static_cast<int>(d);
    for (int idx = threadIdx.x; idx < GH * di; idx += kStepThreads) {
      const int g = idx / di, e = idx % di;
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) o = fmaf(sm_o[(w * GH + g) * 32 * EPL + e], wsm[g * kStepWarps + w], o);
      const int64_t row = b * hq + kvh * GH + g;
      st_tagged(p.part_o + (row * ns + split) * d + e, __float_as_uint(o), tag);
      if (e == 0) {
        float l = 0.0f;
#pragma unroll
        for (int w = 0; w < kStepWarps; ++w) l = fmaf(sm_l[w][g], wsm[g * kStepWarps + w], l);
        unsigned long long* ml = p.part_ml + (row * ns + split) * 2;
        st_tagged(ml, __float_as_uint(cta_l[g]), tag);
        st_tagged(ml + 1, __float_as_uint(l), tag);
      }
    }
    NVFP4DA_PHASE(8);
    const int pairs = GH * static_cast<int>(d) / 2;
    const int share = (pairs + ns - 1) / ns;
    const int lo = split * share, hi = lo + share < pairs ? lo + share : pairs;
    if (ns <= 8) {
      // Every split's (m, l) and o for this thread's pair in one poll: one
      // round trip once the slowest split has published.
      for (int pi = lo + threadIdx.x; pi < hi; pi += kStepThreads) {
        const int g = (2 * pi) / static_cast<int>(d);
        const int64_t e = (2 * pi) % static_cast<int>(d);
        const int64_t row = b * hq + kvh * GH + g;
        const unsigned long long* src[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int sp = j < ns ? j : ns - 1;
          src[4 * j] = p.part_ml + (row * ns + sp) * 2;
          src[4 * j + 1] = src[4 * j] + 1;
          src[4 * j + 2] = p.part_o + (row * ns + sp) * d + e;
          src[4 * j + 3] = src[4 * j + 2] + 1;
        }
        uint32_t v[32];
        poll_tagged<32>(src, v, tag, deadline, err);
        NVFP4DA_PHASE(14);
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < ns) mx = fmaxf(mx, __uint_as_float(v[4 * j]));
        float l = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < ns) {
            const float ms = __uint_as_float(v[4 * j]);
            const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
            l = fmaf(__uint_as_float(v[4 * j + 1]), f, l);
            o0 = fmaf(__uint_as_float(v[4 * j + 2]), f, o0);
            o1 = fmaf(__uint_as_float(v[4 * j + 3]), f, o1);
          }
        const uint32_t pair = f32_to_bf16_bits(__fdiv_rn(o0, l)) |
                              (static_cast<uint32_t>(f32_to_bf16_bits(__fdiv_rn(o1, l))) << 16);
        st_tagged(p.ctx + (b * k + (kvh * GH + g) * d + e) / 2, pair, tag);
      }
    } else {
      float* sw = sm_o;  // [GH][ns] weights exp(m_s - M); the o vectors are consumed
      __syncthreads();
      for (int it = threadIdx.x; it < GH * ns; it += kStepThreads) {
        const int g = it / ns, sp = it % ns;
        const unsigned long long* mlp = p.part_ml + ((b * hq + kvh * GH + g) * ns + sp) * 2;
        const unsigned long long* src[2] = {mlp, mlp + 1};
        uint32_t v[2];
        poll_tagged<2>(src, v, tag, deadline, err);
        sw[it] = __uint_as_float(v[0]);               // m_s
        sw[GH * ns + it] = __uint_as_float(v[1]);     // l_s
      }
      __syncthreads();
      if (threadIdx.x < GH) {
        const int g = threadIdx.x;
        float mx = -INFINITY;
        for (int sp = 0; sp < ns; ++sp) mx = fmaxf(mx, sw[g * ns + sp]);
        float l = 0.0f;
        for (int sp = 0; sp < ns; ++sp) {
          const float ms = sw[g * ns + sp];
          const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
          sw[g * ns + sp] = f;
          l = fmaf(sw[GH * ns + g * ns + sp], f, l);
        }
        cta_l[g] = l;
      }
      __syncthreads();
      for (int pi = lo + threadIdx.x; pi < hi; pi += kStepThreads) {
        const int g = (2 * pi) / static_cast<int>(d);
        const int64_t e = (2 * pi) % static_cast<int>(d);
        const int64_t row = b * hq + kvh * GH + g;
        float o0 = 0.0f, o1 = 0.0f;
        for (int sp0 = 0; sp0 < ns; sp0 += 4) {
          const unsigned long long* src[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int sp = sp0 + j < ns ? sp0 + j : ns - 1;
            src[2 * j] = p.part_o + (row * ns + sp) * d + e;
            src[2 * j + 1] = src[2 * j] + 1;
          }
          uint32_t v[8];
          poll_tagged<8>(src, v, tag, deadline, err);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (sp0 + j < ns) {
              const float f = sw[g * ns + sp0 + j];
              o0 = fmaf(__uint_as_float(v[2 * j]), f, o0);
              o1 = fmaf(__uint_as_float(v[2 * j + 1]), f, o1);
            }
        }
        const uint32_t pair = f32_to_bf16_bits(__fdiv_rn(o0, cta_l[g])) |
                              (static_cast<uint32_t>(f32_to_bf16_bits(__fdiv_rn(o1, cta_l[g]))) << 16);
        st_tagged(p.ctx + (b * k + (kvh * GH + g) * d + e) / 2, pair, tag);
      }
    }
    NVFP4DA_PHASE(9);
  }

  // ---- O projection
  if (has_o) {
    // Decode the O rows into f16 while the context is still being computed
    // (every thread; the weight decode leaves the critical path).
    __half* od = reinterpret_cast<__half*>(smem + p.off_od);
    if (p.o_predecode) {
      // The decoded rows overlay the K/V tile region, which the attention
      // unit's combine may still be reading in other warps.
      if (has_attn) __syncthreads();
      mbar_spin_until(&bar_o, 0, deadline, err);
      predecode_rows_f16(ow_smem, os_smem, k, o_valid, od, p.od_ld);
      NVFP4DA_PHASE(19);
    }
    // The context, as the splits publish it, into the BF16 operand rows.
    bool o_f16;
    {
      const int pairs = static_cast<int>(nb * k / 2);
      uint32_t* xs2 = reinterpret_cast<uint32_t*>(x_stage);
      float rmax = 0.0f;  // |x| maximum of this thread's pairs (used when B = 1)
      for (int i0 = threadIdx.x; i0 < pairs; i0 += 8 * kStepThreads) {  // one round trip per 2,048 pairs
        const unsigned long long* src[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j * kStepThreads;
          src[j] = p.ctx + (i < pairs ? i : i0);
        }
        uint32_t v[8];
        poll_tagged<8>(src, v, tag, deadline, err);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j * kStepThreads < pairs) {
            xs2[i0 + j * kStepThreads] = v[j];
            rmax = fmaxf(rmax, fmaxf(fabsf(__uint_as_float(v[j] << 16)), fabsf(__uint_as_float(v[j] & 0xffff0000u))));
          }
      }
      NVFP4DA_PHASE(17);
      if (mrows == 1) {
        // One row: the maximum from the polled values, then each thread
        // converts its own pairs (the rule of mma_prepare_f16: row maximum to
        // 2^14..2^15, exact or the BF16 path) -- one barrier instead of four.
        rmax = warp_max_f32(rmax);
        if (lane == 0) red_small[warp] = rmax;
        __syncthreads();
        float mx = 0.0f;
#pragma unroll
        for (int w = 0; w < kStepWarps; ++w) mx = fmaxf(mx, red_small[w]);
        int e = 0;
        if (mx > 0.0f && isfinite(mx)) {
          const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xff) - 127;  // floor(log2) for normals
          e = 14 - (ex < -126 ? -126 : ex);
          e = e > 126 ? 126 : (e < -126 ? -126 : e);
        }
        const float sc = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);   // 2^e
        const float isc = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
        uint32_t* x162 = reinterpret_cast<uint32_t*>(x16);
        int inexact = 0;
        for (int i = threadIdx.x; i < pairs; i += kStepThreads) {
          const uint32_t w = xs2[i];
          const float a = __uint_as_float(w << 16), c = __uint_as_float(w & 0xffff0000u);
          const __half2 h = __floats2half2_rn(a * sc, c * sc);
          inexact |= (__low2float(h) * isc != a) | (__high2float(h) * isc != c);  // round trip gives x back
          x162[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        if (threadIdx.x == 0) escale[0] = isc;
        o_f16 = __syncthreads_or(inexact) == 0;
      } else {
        __syncthreads();
        o_f16 = mma_prepare_f16(x_stage, x16, k, mrows, escale, red_small);
      }
    }
    NVFP4DA_PHASE(10);
    const bool f16 = o_f16;
    if (p.o_predecode) {
      NVFP4DA_PHASE(11);
      if (f16)
        mma_pass_decoded<true>(od, p.od_ld, reinterpret_cast<const uint16_t*>(x16), k, p.o_tile_rows, o_valid, mrows,
                               mred, outv);
      else
        mma_pass_decoded<false>(od, p.od_ld, x_stage, k, p.o_tile_rows, o_valid, mrows, mred, outv);
    } else {
      mbar_spin_until(&bar_o, 0, deadline, err);
      NVFP4DA_PHASE(11);
      if (f16)
        mma_gemv_pass_smem<true, 4>(ow_smem, os_smem, reinterpret_cast<const uint16_t*>(x16), k, p.o_tile_rows,
                                    o_valid, mrows, mred, outv);
      else
        mma_gemv_pass_smem<false, 4>(ow_smem, os_smem, x_stage, k, p.o_tile_rows, o_valid, mrows, mred, outv);
    }
    const float gamma = gamma_o;
    // Eight rows per 16-byte store (o_valid and orow0 are multiples of 8).
    const int o_oct = o_valid / 8;
    for (int i = threadIdx.x; i < o_oct * mrows; i += kStepThreads) {
      const int n = i / o_oct, r0 = (i % o_oct) * 8;
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v0 = outv[(r0 + 2 * j) * 8 + n], v1 = outv[(r0 + 2 * j + 1) * 8 + n];
        if (f16) {
          v0 *= escale[n];
          v1 *= escale[n];
        }
        w[j] = static_cast<uint32_t>(f32_to_bf16_bits(__fmul_rn(v0, gamma))) |
               (static_cast<uint32_t>(f32_to_bf16_bits(__fmul_rn(v1, gamma))) << 16);
      }
      *reinterpret_cast<uint4*>(p.out + n * k + orow0 + r0) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    NVFP4DA_PHASE(12);
  }

  // ---- leave; the last CTA out resets the exit counter and advances the epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atom_add_acq_rel(&sync[kSyncExit], 1u);
    s_flag = prev == gridDim.x - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (s_flag) {
    // Tags run 1, 2, ..., 2^32 - 1 (the region starts zeroed, and 0 is never
    // a tag); before they wrap, the region is cleared so that no word of an
    // old launch can carry a reused tag.
    if (tag == 0xFFFFFFFFu) {
      unsigned long long* region = p.proj;  // the region's first word
      for (size_t i = threadIdx.x; i < p.tag_words; i += kStepThreads) region[i] = 0ull;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      sync[kSyncExit] = 0u;
      sync[kSyncEpoch] = tag == 0xFFFFFFFFu ? 0u : tag;  // the next launch tags with epoch + 1
    }
  }
}

}  // namespace nvfp4da
