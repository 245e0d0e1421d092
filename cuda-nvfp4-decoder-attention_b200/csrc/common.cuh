// Shared device helpers for the sm_100a NVFP4-W4A16 decoder-attention kernels.
//
// Storage contract (reference docs/NUMERICS.md:441-468, reference/nvfp4.py:56-71):
//   packed_values  uint8 [N, K/2]   even k in the low nibble, odd k in the high nibble
//   block_scales   uint8 [N, K/16]  canonical UE4M3 (0x00..0x7e), row-local
//   global_decode_scale  float32 scalar (gamma)
//   W_hat[n, k] = (e2m1(q) * ue4m3(beta)) * gamma
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4da {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// Device-side error word (bit set per failure kind); read back by the host
// only in debug/diagnostic paths.  Waits never spin forever: every mbarrier
// wait is bounded and reports here.
enum DeviceError : unsigned {
  kErrNone = 0,
  kErrBarrierTimeout = 1u,
};

// ------------------------------------------------------------------ phase timing
// Diagnostic build only (-DNVFP4DA_PHASES): thread 0 of each CTA records
// clock64() at numbered points into a device table, read back by the debug
// entry nvfp4da_debug_phases().  Compiled out of the normal library.
#ifdef NVFP4DA_PHASES
constexpr int kPhaseSlots = 32;  // the last slot: clock64() at phase 0
constexpr int kPhaseCtas = 4096;  // table rows; each kernel writes rows kPhaseBase + cta
__device__ unsigned long long g_phase_table[kPhaseCtas * kPhaseSlots];
#define NVFP4DA_PHASE(i)                                                                               \
  do {                                                                                                 \
    const unsigned cta_ = kPhaseBase + blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z); \
    if (threadIdx.x == 0 && cta_ < kPhaseCtas) {                                                       \
      unsigned long long t_;                                                                           \
      if ((i) == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); else t_ = clock64();        \
      g_phase_table[cta_ * kPhaseSlots + (i)] = t_;                                                    \
      if ((i) == 0) g_phase_table[cta_ * kPhaseSlots + kPhaseSlots - 1] = clock64();                                \
    }                                                                                                  \
  } while (0)
#else
#define NVFP4DA_PHASE(i) \
  do {                   \
  } while (0)
#endif

// ------------------------------------------------------------------ BF16
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Round-to-nearest-even FP32 -> BF16 bits (NaN kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// ------------------------------------------------------------------ decode
// Two E2M1 nibbles (one packed byte, even element low) -> exact f16x2 via the
// sm_100a hardware conversion.  E2M1 values {0,.5,1,1.5,2,3,4,6} and their
// negatives (code 0x8 = -0) are all exact in f16.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte_in_low_bits) {
  uint32_t out;
  asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}"
      : "=r"(out) : "r"(byte_in_low_bits));
  return out;
}

// Four packed bytes -> four f16x2 (byte j -> out[j], low nibble in the low
// half).  The bytes are unpacked by one mov, so no shifts are issued.
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

// Decode four packed bytes (eight nibbles, k = 0..7 in order) to FP32.
__device__ __forceinline__ void decode8_e2m1(uint32_t word, float (&out)[8]) {
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t h2 = e2m1x2_to_f16x2(word >> (8 * b));
    const __half2 hv = *reinterpret_cast<const __half2*>(&h2);
    out[2 * b] = __low2float(hv);      // low nibble = even k
    out[2 * b + 1] = __high2float(hv); // high nibble = odd k
  }
}

// Canonical UE4M3 byte -> FP32.  A canonical UE4M3 byte (bit 7 clear, not 0x7f)
// is bit-identical to a positive E4M3 value (4 exponent bits, bias 7, 3 mantissa
// bits, subnormals m*2^-9), so the hardware e4m3 -> f16 conversion decodes it
// exactly: every value lies in [2^-9, 448], normal in f16.
__device__ __forceinline__ float decode_ue4m3(uint32_t code) {
  uint32_t out;
  asm("{\n .reg .b16 s;\n cvt.u16.u32 s, %1;\n cvt.rn.f16x2.e4m3x2 %0, s;\n}"
      : "=r"(out) : "r"(code & 0xffu));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(out & 0xffffu)));
}

// Scalar E2M1 decode with the sign applied to the bit pattern (keeps -0).
__device__ __forceinline__ float decode_e2m1_scalar(uint32_t code) {
  const uint32_t h2 = e2m1x2_to_f16x2(code & 0xfu);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffffu)));
}

// ------------------------------------------------------------------ sums
// FP32 value of an exactly accumulated sum: accumulate in FP64 (every term
// here is an FP32 value), round once.  Used for RMSNorm sums of squares.
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// RMSNorm scale 1 / sqrt(mean + eps) with IEEE-rounded sqrt and division,
// matching FP32 `torch.rsqrt` on the CPU (1 / sqrt, two roundings).
__device__ __forceinline__ float rms_inverse(float sum_sq, float count, float eps) {
  const float mean = __fdiv_rn(sum_sq, count);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// ------------------------------------------------------------------ PTX: shared memory, mbarrier, bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: each try_wait suspends for a hardware time slice; after
// `max_tries` unsuccessful tries the wait gives up, records the failure in
// `err` and returns false so the kernel can exit instead of hanging.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err,
                                                  uint32_t max_tries = (1u << 22)) {
  for (uint32_t i = 0; i < max_tries; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (err) atomicOr(err, static_cast<unsigned>(kErrBarrierTimeout));
  return false;
}

// Bulk async copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes.  Requires 16-byte aligned addresses and a size that is a
// multiple of 16 (checked by callers).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: allow the next kernel in the stream to begin
// launching, and wait until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Copy `bytes` from global to this CTA's shared memory.  If both ends are
// 16-byte aligned and the size is a multiple of 16, thread 0 issues one bulk
// async copy on `bar` and every thread waits on `parity`; otherwise all threads
// copy with plain loads.  Must be called by every thread of the CTA; ends with
// the data visible to the whole CTA.  Returns false if the bounded wait gave up.
__device__ __forceinline__ bool stage_to_smem(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint32_t parity, unsigned* err) {
  if (bytes == 0) return true;
  const bool bulk = aligned16(dst) && aligned16(src) && (bytes % 16 == 0);
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, bytes);
      bulk_g2s(dst, src, bytes, bar);
    }
    return mbar_wait_bounded(bar, parity, err);
  }
  uint8_t* d = static_cast<uint8_t*>(dst);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  for (uint32_t i = threadIdx.x; i < bytes; i += blockDim.x) d[i] = s[i];
  __syncthreads();
  return true;
}

// Issue (thread 0) a bulk copy whose completion is awaited later with
// mbar_wait_bounded(bar, parity); returns false (nothing issued) when the
// addresses or size do not allow a bulk copy.
__device__ __forceinline__ bool bulk_prefetch(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  if (!(aligned16(dst) && aligned16(src) && (bytes % 16 == 0))) return false;
  if (threadIdx.x == 0 && bytes) {
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(dst, src, bytes, bar);
  }
  return true;
}

}  // namespace nvfp4da
