// Causal GQA attention for prefill-sized T on the tensor cores.
//
// Semantics (reference/decoder_attention.py:273-381): query token t of
// sequence b (position P_b + t) attends to cache slots j <= P_b + t of KV head
// h / (Hq/Hkv); score = FP32(q.k) * FP32(1/sqrt(D)); softmax in FP32;
// context = BF16(sum_j p_j v_j).
//
// One CTA = one (b, query head, tile of 64 query tokens); four warps own 16
// query rows each.  K/V tiles of 64 positions are double-buffered in shared
// memory with cp.async (16-byte chunks XOR-swizzled by row so ldmatrix is
// conflict-free).  S = Q K^T with mma.m16n8k16 BF16 (exact products, FP32
// accumulation per 16-wide step, steps added with FP32 round-to-nearest);
// online softmax in registers; O += P V with P split into three BF16 terms
// (each the residual of the previous rounding), so the probabilities keep ~24
// bits and every product is exact.
#pragma once

#include "common.cuh"

namespace nvfp4da {

constexpr int kPaRows = 64;  // query tokens per CTA
constexpr int kPaKeys = 64;  // positions per K/V tile
constexpr int kPaD = 128;    // head dimension covered
constexpr int kPaThreads = 128;

struct PrefillAttnParams {
  const uint16_t* q;        // [B, T, Hq, D]
  const uint16_t* k_cache;  // [B, Hkv, C, D]
  const uint16_t* v_cache;
  uint16_t* ctx;  // [B, T, Hq, D]
  int64_t batch, tokens, q_heads, kv_heads, capacity;
  int64_t past_length;
  const int64_t* past_lengths;
  float scale;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Byte offset of 16-byte chunk c (0..15) of row r in a [rows x 256 B] tile.
__device__ __forceinline__ uint32_t pa_off(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

constexpr uint32_t kPaSmem = (kPaRows + 4 * kPaKeys) * 256;  // Q tile + double-buffered K and V

__global__ void __launch_bounds__(kPaThreads) attn_prefill_kernel(PrefillAttnParams p) {
  extern __shared__ __align__(128) uint8_t pa_smem[];
  uint8_t* sq = pa_smem;
  uint8_t* sk[2] = {pa_smem + kPaRows * 256, pa_smem + (kPaRows + kPaKeys) * 256};
  uint8_t* sv[2] = {pa_smem + (kPaRows + 2 * kPaKeys) * 256, pa_smem + (kPaRows + 3 * kPaKeys) * 256};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kPaRows;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t group = p.q_heads / p.kv_heads;
  const int64_t kvh = h / group;
  const int64_t pb = p.past_lengths ? p.past_lengths[b] : p.past_length;
  const int64_t T = p.tokens;
  // Keys visible to the last row of the tile; never beyond the capacity.
  int64_t kend = pb + (t0 + kPaRows < T ? t0 + kPaRows : T);
  if (kend > p.capacity) kend = p.capacity;
  const uint16_t* kbase = p.k_cache + (b * p.kv_heads + kvh) * p.capacity * kPaD;
  const uint16_t* vbase = p.v_cache + (b * p.kv_heads + kvh) * p.capacity * kPaD;

  // ---- Q tile (rows beyond T read as zeros) and the first K/V tile
  for (int i = tid; i < kPaRows * 16; i += kPaThreads) {
    const int r = i >> 4, c = i & 15;
    const int64_t t = t0 + r;
    cp_async16(smem_u32(sq + pa_off(r, c)), p.q + ((b * T + (t < T ? t : 0)) * p.q_heads + h) * kPaD + c * 8, t < T);
  }
  auto load_kv = [&](int buf, int64_t j0) {
    for (int i = tid; i < kPaKeys * 16; i += kPaThreads) {
      const int r = i >> 4, c = i & 15;
      const int64_t j = j0 + r;
      const bool ok = j < kend;
      cp_async16(smem_u32(sk[buf] + pa_off(r, c)), kbase + (ok ? j : 0) * kPaD + c * 8, ok);
      cp_async16(smem_u32(sv[buf] + pa_off(r, c)), vbase + (ok ? j : 0) * kPaD + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_kv(0, 0);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  // Q fragments of this warp's 16 rows: 8 k-steps of 16 (A operand, row-major).
  uint32_t qf[8][4];
  {
    const int r = warp * 16 + (lane & 15);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c = ks * 2 + (lane >> 4);
      ldsm_x4(smem_u32(sq + pa_off(r, c)), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
    }
  }

  float o[16][4];  // 16 rows x 128 dims: 16 n-tiles of 8
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};  // rows lane/4 and lane/4 + 8
  const int64_t row_t[2] = {t0 + warp * 16 + (lane >> 2), t0 + warp * 16 + (lane >> 2) + 8};
  const int64_t lim[2] = {pb + row_t[0], pb + row_t[1]};  // last visible key of each row

  const int ntiles = static_cast<int>((kend + kPaKeys - 1) / kPaKeys);
  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    const int64_t j0 = static_cast<int64_t>(it) * kPaKeys;
    if (it + 1 < ntiles) load_kv(buf ^ 1, j0 + kPaKeys);
    // ---- S = Q K^T for 64 keys: 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
    // Each 16-wide k-step starts from zero and is added in FP32 with
    // round-to-nearest, so the tensor cores' accumulation rounding does not
    // compound along D.
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // two n-tiles (16 keys) per ldmatrix.x4
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(sk[buf] + pa_off(r, c)), b0, b1, b2, b3);
        float t0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, t1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_bf16_16816(t0, qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
        mma_bf16_16816(t1, qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[2 * np][e] = __fadd_rn(s[2 * np][e], t0[e]);
          s[2 * np + 1][e] = __fadd_rn(s[2 * np + 1][e], t1[e]);
        }
      }
    }
    // ---- scale, causal mask, online softmax (rows lane/4 and lane/4 + 8)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const int64_t j = j0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        const float v = (j <= lim[hr] && j < kend) ? __fmul_rn(s[nt][e], p.scale) : -INFINITY;
        s[nt][e] = v;
        mx[hr] = fmaxf(mx[hr], v);
      }
    float alpha[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(kFull, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(kFull, mx[hr], 2));
      const float mnew = fmaxf(m_run[hr], mx[hr]);
      alpha[hr] = (m_run[hr] == -INFINITY) ? 0.0f : expf(m_run[hr] - mnew);
      m_run[hr] = mnew;
    }
    float psum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const float pe = (s[nt][e] == -INFINITY) ? 0.0f : expf(s[nt][e] - m_run[hr]);
        s[nt][e] = pe;
        psum[hr] += pe;
      }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      psum[hr] += __shfl_xor_sync(kFull, psum[hr], 1);
      psum[hr] += __shfl_xor_sync(kFull, psum[hr], 2);
      l_run[hr] = fmaf(l_run[hr], alpha[hr], psum[hr]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // ---- O += P V: P as A fragments in three BF16 terms (hi + mid + lo, ~24
    // significant bits), V^T by ldmatrix.trans; each 16-key step starts from
    // zero and is added to O in FP32 with round-to-nearest.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
      const float* f0 = s[2 * kk];
      const float* f1 = s[2 * kk + 1];
      const float pv[8] = {f0[0], f0[1], f0[2], f0[3], f1[0], f1[1], f1[2], f1[3]};
      float t1[8], t2[8], t3[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        t1[i] = __bfloat162float(__float2bfloat16_rn(pv[i]));
        const float r1 = pv[i] - t1[i];  // exact
        t2[i] = __bfloat162float(__float2bfloat16_rn(r1));
        t3[i] = __bfloat162float(__float2bfloat16_rn(r1 - t2[i]));
      }
      // A layout: a0 = (row r, keys 2t..2t+1), a1 = (row r+8, ...), a2 = (row r, keys 2t+8..), a3 = (row r+8, ...)
      const uint32_t ph[4] = {pack_bf16(t1[0], t1[1]), pack_bf16(t1[2], t1[3]), pack_bf16(t1[4], t1[5]),
                              pack_bf16(t1[6], t1[7])};
      const uint32_t pm[4] = {pack_bf16(t2[0], t2[1]), pack_bf16(t2[2], t2[3]), pack_bf16(t2[4], t2[5]),
                              pack_bf16(t2[6], t2[7])};
      const uint32_t pl[4] = {pack_bf16(t3[0], t3[1]), pack_bf16(t3[2], t3[3]), pack_bf16(t3[4], t3[5]),
                              pack_bf16(t3[6], t3[7])};
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // two d n-tiles (16 dims) per ldmatrix.x4.trans
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(sv[buf] + pa_off(r, c)), b0, b1, b2, b3);
        float u0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, u1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_bf16_16816(u0, pl[0], pl[1], pl[2], pl[3], b0, b1);
        mma_bf16_16816(u0, pm[0], pm[1], pm[2], pm[3], b0, b1);
        mma_bf16_16816(u0, ph[0], ph[1], ph[2], ph[3], b0, b1);
        mma_bf16_16816(u1, pl[0], pl[1], pl[2], pl[3], b2, b3);
        mma_bf16_16816(u1, pm[0], pm[1], pm[2], pm[3], b2, b3);
        mma_bf16_16816(u1, ph[0], ph[1], ph[2], ph[3], b2, b3);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[2 * dp][e] = __fadd_rn(o[2 * dp][e], u0[e]);
          o[2 * dp + 1][e] = __fadd_rn(o[2 * dp + 1][e], u1[e]);
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
  }

  // ---- context = BF16(O / l)
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int64_t t = row_t[hr];
    if (t >= T) continue;
    uint16_t* dst = p.ctx + ((b * T + t) * p.q_heads + h) * kPaD + 2 * (lane & 3);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t v = pack_bf16(__fdiv_rn(o[i][2 * hr], l_run[hr]), __fdiv_rn(o[i][2 * hr + 1], l_run[hr]));
      *reinterpret_cast<uint32_t*>(dst + i * 8) = v;
    }
  }
}

}  // namespace nvfp4da
