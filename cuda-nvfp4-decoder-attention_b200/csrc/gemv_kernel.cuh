// Standalone W4A16 GEMV kernel: y[M, N] = x[M, K] @ W_hat[N, K]^T (BF16 out).
// Backs `cuda_w4a16_linear` and the O projection of the decode step.
#pragma once

#include "gemv_core.cuh"
#include "gemv_mma.cuh"

namespace nvfp4da {

struct GemvParams {
  const uint16_t* x;  // [M, K] bf16
  int64_t m;
  const uint8_t* packed;  // [N, K/2]
  const uint8_t* scales;  // [N, K/16]
  const float* gamma;
  uint16_t* y;  // [M, N] bf16
  int64_t n, k;
  unsigned* err;
  int pdl;
};

// One CTA = 8*RPW weight rows, all M activation rows (in groups of MG).
// Weights are bulk-copied into shared memory first (before the PDL wait, since
// they never depend on an earlier kernel), then activations are staged per
// group as FP32.
template <int RPW, int MG>
__global__ void __launch_bounds__(kGemvThreads) w4a16_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t bars[kGemvWarps];
  __shared__ uint64_t xbar;
  constexpr int kRows = kGemvWarps * RPW;
  const int64_t k = p.k, nc = k / 16;
  const GemvSmemLayout lay = gemv_layout(kRows, k, MG);
  uint8_t* w_smem = smem + lay.w_off();
  uint8_t* s_smem = smem + lay.s_off();
  float4* x_smem = reinterpret_cast<float4*>(smem + lay.x_off());
  uint16_t* x_stage = reinterpret_cast<uint16_t*>(smem + lay.xs_off());
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  [[maybe_unused]] constexpr unsigned kPhaseBase = 2048;
  NVFP4DA_PHASE(0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemvWarps; ++i) mbar_init(&bars[i], 1);
    mbar_init(&xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights never depend on an earlier kernel: start streaming them before
  // the programmatic-dependency wait.
  const bool bulk = gemv_bulk_ok(p.packed, p.scales, k);
  gemv_stage_weights(w_smem, s_smem, p.packed, p.scales, k, row0, kRows, p.n, bulk, bars);
  const float gamma = *p.gamma;
  NVFP4DA_PHASE(1);
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  bool waited = !bulk;
  int group = 0;
  for (int64_t m0 = 0; m0 < p.m; m0 += MG, ++group) {
    const int mgv = static_cast<int>((p.m - m0) < MG ? (p.m - m0) : MG);
    __syncthreads();  // staging buffers are free again
    if (!stage_to_smem(x_stage, p.x + m0 * k, static_cast<uint32_t>(mgv * k * 2), &xbar, group & 1, p.err))
      return;
    NVFP4DA_PHASE(2);
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(mgv) * k; i += blockDim.x)
      x_smem_store(x_smem, nc, static_cast<int>(i / k), i % k, bf16_bits_to_f32(x_stage[i]));
    __syncthreads();
    NVFP4DA_PHASE(3);
    if (!waited) {
      if (!mbar_wait_bounded(&bars[warp], 0, p.err)) return;
      waited = true;
    }
    NVFP4DA_PHASE(4);
    float acc[RPW][MG];
    gemv_warp_rows<RPW, MG>(w_smem, s_smem, x_smem, k, mgv, acc);
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int m = 0; m < MG; ++m) {
        const int64_t row = row0 + warp * RPW + r;
        if (lane == ((r * MG + m) & 31) && m < mgv && row < p.n)
          p.y[(m0 + m) * p.n + row] = f32_to_bf16_bits(__fmul_rn(acc[r][m], gamma));
      }
  }
  NVFP4DA_PHASE(5);
}

// Tensor-core decode GEMV (K % 128 == 0): one CTA = ROWS weight rows, all M
// activation rows in groups of up to 8 (the MMA's n dimension).  Weights go
// from HBM straight into registers (issued before the dependency wait); the
// scales take one bulk copy; activations are loaded after the wait.
template <int ROWS>
__global__ void __launch_bounds__(kMmaThreads, 2) mma_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t sbar;
  __shared__ float redf[2 * kMmaWarps];
  __shared__ double redd[2 * kMmaWarps];
  __shared__ float escale[kMmaMaxM];
  __shared__ float red_small[kMmaMaxM * kMmaWarps];
  __shared__ float outv[ROWS * 8];
  [[maybe_unused]] constexpr unsigned kPhaseBase = 2048;
  NVFP4DA_PHASE(0);
  const int64_t k = p.k;
  const int mg = static_cast<int>(p.m < kMmaMaxM ? p.m : kMmaMaxM);
  const MmaGemvLayout L = mma_gemv_layout(ROWS, k, mg);
  uint8_t* s_smem = smem + L.s_off();
  uint16_t* x_stage = reinterpret_cast<uint16_t*>(smem + L.xs_off());
  __half* x16 = reinterpret_cast<__half*>(smem + L.x16_off());
  const bool aliased = reinterpret_cast<const void*>(x16) == reinterpret_cast<const void*>(x_stage);
  float* red = reinterpret_cast<float*>(smem + L.red_off());
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * ROWS;
  const int valid_rows = static_cast<int>((p.n - row0) < ROWS ? (p.n - row0) : ROWS);
  const uint8_t* packed_row0 = p.packed + row0 * (k / 2);

  if (threadIdx.x == 0) {
    mbar_init(&sbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights and scales never depend on an earlier kernel: put this CTA's
  // slice in flight before the programmatic-dependency wait.
  const bool sbulk = stage_scales(s_smem, p.scales, k, row0, valid_rows, &sbar);
  const WarpSlice wsl = warp_slice(ROWS, k);
  constexpr int NB = 4;  // weight steps in flight per warp
  WeightRegs<NB> w;
  issue_weight_batch<NB>(w, packed_row0, k, wsl.tile, wsl.s0, wsl.s1, valid_rows);
  const float gamma = *p.gamma;
  NVFP4DA_PHASE(1);
  if (p.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  bool scales_ready = !sbulk;
  for (int64_t m0 = 0; m0 < p.m; m0 += kMmaMaxM) {
    const int mgv = static_cast<int>((p.m - m0) < kMmaMaxM ? (p.m - m0) : kMmaMaxM);
    __syncthreads();  // staging buffers are free again
    if (m0 > 0) issue_weight_batch<NB>(w, packed_row0, k, wsl.tile, wsl.s0, wsl.s1, valid_rows);
    NVFP4DA_PHASE(2);
    bool f16;
    constexpr int NCH = 2;  // register path for K <= 4096
    if ((k / 8) <= NCH * kMmaThreads && aligned16(p.x)) {
      const uint4 none[NCH] = {};
      f16 = (mgv > 1 || aliased) ? prep_rows_warp<false>(p.x + m0 * k, nullptr, k, mgv, 0.0f, x_stage, x16, escale, nullptr)
                    : prep_rows_regs<NCH, false>(p.x + m0 * k, k, mgv, none, 0.0f, x_stage, x16, escale, redf, redd,
                                                 nullptr);
    } else {
      load_rows_lsu(x_stage, p.x + m0 * k, static_cast<int64_t>(mgv) * k);
      __syncthreads();
      // With one staging buffer the f16 operand would overwrite the BF16 rows
      // before their exactness is known: the BF16 operand then.
      f16 = aliased ? false : mma_prepare_f16(x_stage, x16, k, mgv, escale, red_small);
    }
    NVFP4DA_PHASE(3);
    if (!scales_ready) {
      if (!mbar_wait_bounded(&sbar, 0, p.err)) return;
      scales_ready = true;
    }
    NVFP4DA_PHASE(4);
    if (f16)
      mma_gemv_pass<true, NB>(w, packed_row0, s_smem, reinterpret_cast<const uint16_t*>(x16), k, ROWS, valid_rows,
                              mgv, red, outv);
    else
      mma_gemv_pass<false, NB>(w, packed_row0, s_smem, x_stage, k, ROWS, valid_rows, mgv, red, outv);
    for (int i = threadIdx.x; i < ROWS * mgv; i += blockDim.x) {
      const int n = i / ROWS, r = i % ROWS;
      if (r < valid_rows) {
        const float v = f16 ? outv[r * 8 + n] * escale[n] : outv[r * 8 + n];
        p.y[(m0 + n) * p.n + row0 + r] = f32_to_bf16_bits(__fmul_rn(v, gamma));
      }
    }
  }
  NVFP4DA_PHASE(5);
}

}  // namespace nvfp4da
