// W4A16 dense projection for prefill-sized M on the 5th-generation tensor
// cores: y[M, N] = BF16( gamma * sum_k x[m, k] * (q * beta)[n, k] ).
//
// Semantics: reference/w4a16.py:11-59 (x @ W_hat.T with W_hat = (q*beta)*gamma,
// FP32 accumulation, BF16 output).  q*beta has at most 6 significant bits and
// lies in [2^-10, 2688], so it is exact in BF16; BF16 x BF16 products are exact
// in the FP32 accumulator, and gamma is applied once in the epilogue.
//
// One CTA computes a 128 x BN tile (BN = 128 or 256) of y with tcgen05.mma
// (kind::f16, BF16 operands, FP32 accumulators in tensor memory), K in steps
// of 64, as a warp-specialised pipeline on mbarriers:
//  * warp 0 (one lane) streams, kStages steps ahead, the x tile [128 rows x
//    64 k] by TMA with 128-byte swizzle (the canonical K-major SW128 operand
//    layout) and the packed weight tile [BN x 32 bytes]; every fourth step
//    also the scale tile [BN x 16 bytes] that covers four steps;
//  * warps 2.. decode the weight tile (two threads per row, 32 k each) into
//    one of kDec BF16 buffers in the SW128 K-major layout: E2M1 -> BF16 by
//    byte permutes from two 8-entry tables (sign from the nibble's top bit),
//    times the UE4M3 block scale in BF16, all exact;
//  * warp 1 (one lane) issues the four K=16 MMAs of a step once its x tile and
//    decoded buffer are ready, and commits them to one barrier that frees the
//    load stage and the decoded buffer;
//  * epilogue: the decode warps (warp w on the 32-lane quarter w % 4 of tensor
//    memory, 64 columns each) read the accumulators with tcgen05.ld, scale by
//    gamma and store BF16.
// Every wait is bounded (one second); on expiry the kernel records
// kErrBarrierTimeout, skips the remaining work, and still frees its tensor
// memory.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace nvfp4da {

constexpr int kPgBM = 128;
constexpr int kPgBK = 64;
// Per tile width BN: the decode warps (two threads per weight row), the
// accumulators and the buffers.  K steps go round-robin to kAcc accumulators
// (TMEM column blocks, 512 columns in all) that the epilogue adds in FP32:
// shorter accumulation chains keep the tensor cores' internal rounding within
// one BF16 step of the correctly rounded sum.
template <int BN>
struct PgCfg {
  // Warp roles: warp 0 issues the TMA loads, warp 1 the MMAs, warps 2.. decode
  // and then run the epilogue (a warp may only read tensor-memory lane
  // quarter warp % 4; each takes 64 of the BN columns).
  static constexpr int kDecodeWarps = BN / 16;
  static constexpr int kThreads = 64 + 32 * kDecodeWarps;
  static constexpr int kAcc = 512 / BN;
  static constexpr int kStages = BN == 128 ? 8 : 6;  // x + packed-weight load stages in flight
  static constexpr int kDec = 2;                     // decoded weight buffers
  static constexpr int kScaleSlots = 3;              // scale tiles, one per 4 K steps
};

struct PgParams {
  int64_t m, n, k;
  const float* gamma;
  uint16_t* y;  // [M, N]
  unsigned* err;
};

// Shared-memory layout of one CTA (byte offsets from a 1024-aligned base).
template <int BN>
struct PgLayout {
  using C = PgCfg<BN>;
  static constexpr uint32_t kA = kPgBM * kPgBK * 2;  // 16 KB per stage
  static constexpr uint32_t kW = BN * kPgBK / 2;     // packed weight tile per stage
  static constexpr uint32_t kB = BN * kPgBK * 2;     // decoded weight tile per buffer
  static constexpr uint32_t kS = BN * 16;            // scale bytes of 4 K steps per slot
  __host__ __device__ static constexpr uint32_t a(int s) { return s * kA; }
  __host__ __device__ static constexpr uint32_t b(int d) { return C::kStages * kA + d * kB; }
  __host__ __device__ static constexpr uint32_t w(int s) { return C::kStages * kA + C::kDec * kB + s * kW; }
  __host__ __device__ static constexpr uint32_t sc(int g) {
    return C::kStages * (kA + kW) + C::kDec * kB + g * kS;
  }
  // + 1024 alignment slack.  One CTA per SM: it holds all 512 tensor-memory
  // columns.
  __host__ __device__ static constexpr uint32_t total() {
    return C::kStages * (kA + kW) + C::kDec * kB + C::kScaleSlots * kS + 1024;
  }
  static_assert(C::kStages * (kA + kW) + C::kDec * kB + C::kScaleSlots * kS + 1024 <= 227u * 1024,
                "shared memory per CTA");
};

// ---------------------------------------------------------------- tcgen05 / TMA primitives
// Shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// start address >> 4 (bits 0-13), leading byte offset (unused for swizzled
// K-major, 16 B), stride byte offset 1024 B = 8 rows x 128 B (bits 32-45),
// descriptor version 1 (bits 46-47), swizzle mode 2 = 128 B (bits 61-63).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor, kind::f16: FP32 D (bits 4-5 = 1), BF16 A and B
// (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// Sum of accumulators [a, a + n) of 16 columns, pairwise (n a power of two);
// accumulators at or past `used` (never written) count as zero.
template <int N>
__device__ __forceinline__ void tmem_sum_x16(uint32_t base, uint32_t stride, int a, int used, float (&out)[16]) {
  if constexpr (N == 1) {
    if (a < used) {
      tmem_ld_32x32b_x16(base + a * stride, out);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = 0.0f;
    }
  } else {
    float r[16];
    tmem_sum_x16<N / 2>(base, stride, a, used, out);
    tmem_sum_x16<N / 2>(base, stride, a + N / 2, used, r);
#pragma unroll
    for (int j = 0; j < 16; ++j) out[j] = __fadd_rn(out[j], r[j]);
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Eight E2M1 nibbles (nibble i = element i, low nibble first) -> four BF16x2,
// exact, with integer byte permutes only.  The magnitude code (e1 e0 m) picks
// the low and high byte of the BF16 value from two 8-entry tables:
//   code      0    1    2    3    4    5    6    7
//   value     0   0.5   1   1.5   2    3    4    6
//   BF16   0000 3F00 3F80 3FC0 4000 4040 4080 40C0
// and the nibble's sign bit becomes bit 15 of its BF16 half.
__device__ __forceinline__ void e2m1x8_to_bf16x2x4(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t m = w & 0x77777777u;
  const uint32_t lo0 = __byte_perm(0xC0800000u, 0xC0804000u, m);
  const uint32_t hi0 = __byte_perm(0x3F3F3F00u, 0x40404040u, m);
  const uint32_t lo1 = __byte_perm(0xC0800000u, 0xC0804000u, m >> 16);
  const uint32_t hi1 = __byte_perm(0x3F3F3F00u, 0x40404040u, m >> 16);
  const uint32_t mag[4] = {__byte_perm(lo0, hi0, 0x5140), __byte_perm(lo0, hi0, 0x7362),
                           __byte_perm(lo1, hi1, 0x5140), __byte_perm(lo1, hi1, 0x7362)};
  // Byte j of w holds the signs of elements 2j (bit 3) and 2j+1 (bit 7):
  // byte j of (w << 4) into result byte 1 puts the first at bit 15, byte j of
  // w into result byte 3 puts the second at bit 31.
  const uint32_t w4 = w << 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sg = __byte_perm(w4, w, static_cast<uint32_t>(((4 + j) << 12) | (j << 4)));
    o[j] = mag[j] | (sg & 0x80008000u);
  }
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Exact f16x2 -> bf16x2 for the decoded weights (at most 6 significant bits).
__device__ __forceinline__ uint32_t f16x2_to_bf16x2_exact(uint32_t h) {
  float lo, hi;
  asm("{\n .reg .b16 l, u;\n mov.b32 {l, u}, %2;\n cvt.f32.f16 %0, l;\n cvt.f32.f16 %1, u;\n}"
      : "=f"(lo), "=f"(hi)
      : "r"(h));
  uint32_t out;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
  return out;
}

// ---------------------------------------------------------------- the kernel
// Bounded wait of the GEMM pipeline: try_wait until the phase with `parity`
// completes; gives up (returns false) when another role already gave up
// (`bad`) or after one second, recording kErrBarrierTimeout in `err`.
__device__ __forceinline__ bool pg_wait(uint64_t* bar, uint32_t parity, volatile unsigned* bad, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*bad) return false;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 1000000000ull) {
        if (err) atomicOr(err, static_cast<unsigned>(kErrBarrierTimeout));
        *bad = 1u;
        return false;
      }
    }
  }
}

// Pipeline (step kt = K columns [64 kt, 64 kt + 64)):
//   full[s]   x tile + packed weights of step kt landed (s = kt % kStages);
//   sfull[g]  scale tile of steps [4 g', 4 g' + 4) landed (g = g' % kScaleSlots);
//   dfull[d]  every decode warp wrote decoded buffer d = kt % kDec;
//   empty[s]  the MMAs of step kt are done (one tcgen05.commit per step): frees
//             load stage s and decoded buffer kt % kDec, and, kStages steps on,
//             the scale slot read four groups earlier;
//   acc       every MMA is done (the epilogue may read tensor memory).
// Every waiter is within one phase of the barrier it waits on: a later phase
// needs work that itself waits for the waiter.
template <int BN>
__global__ void __launch_bounds__(PgCfg<BN>::kThreads, 1)
    w4a16_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_s, PgParams p) {
  static_assert(BN == 128 || BN == 256, "N = 128 or 256 per MMA");
  using L = PgLayout<BN>;
  using C = PgCfg<BN>;
  constexpr int kSt = C::kStages, kDec = C::kDec, kAcc = C::kAcc, kSl = C::kScaleSlots;
  static_assert(kSt > kDec && kSt <= 8, "stage reuse order");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_full[kSt], bar_empty[kSt], bar_sfull[kSl], bar_dfull[kDec], bar_acc;
  __shared__ uint32_t tmem_base;
  __shared__ volatile unsigned s_bad;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * kPgBM, n0 = blockIdx.x * BN;
  const int nk = static_cast<int>(p.k / kPgBK);

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(BN * kAcc)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kSt; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int g = 0; g < kSl; ++g) mbar_init(&bar_sfull[g], 1);
    for (int d = 0; d < kDec; ++d) mbar_init(&bar_dfull[d], C::kDecodeWarps);
    mbar_init(&bar_acc, 1);
    fence_mbar_init();
    s_bad = 0u;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---- producer.  Stage kt % kSt is refilled once the MMAs of step kt - kSt
    // are done; scale slot (kt / 4) % kSl was last read by step kt - 9 at the
    // latest, whose decode finished before MMA(kt - 9) was issued.
    if (lane == 0) {
      for (int kt = 0; kt < nk; ++kt) {
        const int st = kt % kSt;
        if (kt >= kSt && !pg_wait(&bar_empty[st], ((kt / kSt) - 1) & 1, &s_bad, p.err)) break;
        if ((kt & 3) == 0) {
          const int g = kt >> 2;
          mbar_arrive_expect_tx(&bar_sfull[g % kSl], L::kS);
          tma_load_2d(smem + L::sc(g % kSl), &tm_s, g * 16, n0, &bar_sfull[g % kSl]);
        }
        mbar_arrive_expect_tx(&bar_full[st], L::kA + L::kW);
        tma_load_2d(smem + L::a(st), &tm_x, kt * kPgBK, m0, &bar_full[st]);
        tma_load_2d(smem + L::w(st), &tm_w, kt * (kPgBK / 2), n0, &bar_full[st]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: K steps go round-robin to the kAcc accumulators.
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_bf16(kPgBM, BN);
      for (int kt = 0; kt < nk; ++kt) {
        const int st = kt % kSt, db = kt % kDec;
        if (!pg_wait(&bar_full[st], (kt / kSt) & 1, &s_bad, p.err) ||
            !pg_wait(&bar_dfull[db], (kt / kDec) & 1, &s_bad, p.err))
          break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t ad = umma_desc_sw128(smem_u32(smem + L::a(st)));
        const uint64_t bd = umma_desc_sw128(smem_u32(smem + L::b(db)));
        const uint32_t acc = tmem + static_cast<uint32_t>((kt % kAcc) * BN);
#pragma unroll
        for (int kk = 0; kk < kPgBK / 16; ++kk)  // +32 bytes of K per MMA inside the swizzle atom
          umma_bf16(acc, ad + 2 * kk, bd + 2 * kk, kIdesc, (kt >= kAcc || kk > 0) ? 1u : 0u);
        umma_commit(&bar_empty[st]);
      }
      umma_commit(&bar_acc);  // arrives once every MMA issued above is done
    }
    __syncwarp();
  } else {
    // ---- decoders: thread t of 2 * BN decodes k [32 (t & 1), +32) of row t >> 1.
    const int dt = tid - 64, row = dt >> 1, half = dt & 1;
    for (int kt = 0; kt < nk; ++kt) {
      const int st = kt % kSt, db = kt % kDec, g = kt >> 2;
      bool ok = pg_wait(&bar_full[st], (kt / kSt) & 1, &s_bad, p.err) &&
                pg_wait(&bar_sfull[g % kSl], (g / kSl) & 1, &s_bad, p.err);
      // Decoded buffer db is free once the MMAs of step kt - kDec are done.
      if (ok && kt >= kDec) ok = pg_wait(&bar_empty[(kt - kDec) % kSt], ((kt - kDec) / kSt) & 1, &s_bad, p.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint4 wv = *reinterpret_cast<const uint4*>(smem + L::w(st) + row * (kPgBK / 2) + half * 16);
      const uint32_t sc2 =
          *reinterpret_cast<const uint16_t*>(smem + L::sc(g % kSl) + row * 16 + (kt & 3) * 4 + half * 2);
      // The two block scales as BF16 (exact: UE4M3 has at most 4 significant bits).
      uint32_t bh;
      asm("{\n .reg .b16 lo;\n cvt.u16.u32 lo, %1;\n cvt.rn.f16x2.e4m3x2 %0, lo;\n}" : "=r"(bh) : "r"(sc2));
      const uint32_t beta2 = f16x2_to_bf16x2_exact(bh);
      const uint32_t beta[2] = {__byte_perm(beta2, 0, 0x1010), __byte_perm(beta2, 0, 0x3232)};
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
      uint8_t* brow = smem + L::b(db) + row * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 16-byte chunk half * 4 + c = 8 k = word c
        uint32_t q[4];
        e2m1x8_to_bf16x2x4(words[c], q);
        const uint32_t bt = beta[c >> 1];
        // q * beta has at most 6 significant bits: the BF16 product is exact.
        const int chunk = half * 4 + c;
        *reinterpret_cast<uint4*>(brow + ((chunk ^ (row & 7)) << 4)) =
            make_uint4(bf16x2_mul(q[0], bt), bf16x2_mul(q[1], bt), bf16x2_mul(q[2], bt), bf16x2_mul(q[3], bt));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_dfull[db]);
    }

    // ---- epilogue (all decode warps): warp w reads tensor-memory lanes
    // 32 * (w % 4) and 64 of the BN columns.
    {
      const int quad = warp & 3, cbase = ((warp - 2) >> 2) * 64;
      const bool ok = nk > 0 && pg_wait(&bar_acc, 0, &s_bad, p.err) && !s_bad;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (__all_sync(0xffffffffu, ok)) {
        const float gamma = *p.gamma;
        const int64_t grow = m0 + quad * 32 + lane;
        const uint32_t base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
        for (int c0 = cbase; c0 < cbase + 64; c0 += 32) {
          // The accumulators that received K steps, added pairwise.
          uint32_t v[32];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float f[16];
            tmem_sum_x16<kAcc>(base + c0 + 16 * hh, BN, 0, nk, f);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[16 * hh + j] = __float_as_uint(f[j]);
          }
          if (grow < p.m) {
            uint16_t* dst = p.y + grow * p.n + n0 + c0;
            const int64_t cols = p.n - (n0 + c0);
            if (cols >= 32 && (p.n % 8) == 0) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t pk[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t lo = f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[8 * q + 2 * j]), gamma));
                  const uint32_t hi = f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[8 * q + 2 * j + 1]), gamma));
                  pk[j] = lo | (hi << 16);
                }
                reinterpret_cast<uint4*>(dst)[q] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            } else {
              for (int j = 0; j < 32 && j < cols; ++j)
                dst[j] = f32_to_bf16_bits(__fmul_rn(__uint_as_float(v[j]), gamma));
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN * kAcc) : "memory");
}

}  // namespace nvfp4da
