/*
 * C ABI of the B200 (sm_100a) NVFP4-W4A16 decoder-attention library
 * (libnvfp4da.so).  Plain pointers and sizes only; every pointer is CUDA
 * device memory on the current device unless stated otherwise; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  BF16 tensors are passed as
 * uint16_t bit patterns, contiguous, row-major.  No function synchronises the
 * stream or reads device memory back to the host.
 *
 * Each entry point below names the reference interface it replaces
 * (PatrickZChen/cuda-nvfp4-decoder-attention, path:line).  Functions return
 * NVFP4DA_OK or an error code; nvfp4da_last_error() then gives a message
 * (thread-local).  Validation happens before any launch, so a rejected call
 * leaves every buffer untouched.
 *
 * Alignment: every device pointer must be 16-byte aligned (torch allocations
 * are), except that weights whose packed or scale row strides are not
 * multiples of 16 bytes take a slower staging path.
 */
#ifndef NVFP4_DECODER_ATTENTION_H_
#define NVFP4_DECODER_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4DA_OK 0
#define NVFP4DA_ERR_INVALID_ARGUMENT 1
#define NVFP4DA_ERR_UNSUPPORTED 2
#define NVFP4DA_ERR_WORKSPACE 3
#define NVFP4DA_ERR_CUDA 4

/* Message of the last failed call on this host thread ("" if none). */
const char* nvfp4da_last_error(void);

/* ABI version (bumped on any signature change). */
int nvfp4da_abi_version(void);

/* One portable NVFP4 matrix W[N, K] (reference reference/nvfp4.py:56-71,
 * docs/NUMERICS.md:441-468): packed_values uint8 [N, K/2] with the even k in
 * the low nibble; block_scales uint8 [N, K/16] canonical UE4M3 (0x00..0x7e);
 * global_decode_scale one float32 in device memory.  K % 16 == 0. */
typedef struct nvfp4da_weight {
  const uint8_t* packed_values;
  const uint8_t* block_scales;
  const float* global_decode_scale;
  int64_t rows; /* N */
  int64_t cols; /* K */
} nvfp4da_weight;

/* Replaces launch_unpack_e2m1_codes_cuda (include/nvfp4.h:16-18; op
 * src/bindings.cpp:113-122): codes[r, 2j] = low nibble, codes[r, 2j+1] = high
 * nibble of packed[r, j]. */
int nvfp4da_unpack_e2m1_codes(const uint8_t* packed_values, uint8_t* codes, int64_t rows,
                              int64_t packed_cols, void* stream);

/* Replaces launch_dequantize_nvfp4_cuda (include/nvfp4.h:20-24; op
 * src/bindings.cpp:124-198): out[N, K] float32 = (e2m1 * ue4m3) * gamma,
 * bit-exact with reference/nvfp4.py:539-554. */
int nvfp4da_dequantize_nvfp4(const nvfp4da_weight* w, float* out, void* stream);

/* Device quantizer, byte-exact with quantize_nvfp4_reference
 * (reference/nvfp4.py:500-536).  source: float32 [rows, cols] (or BF16 bits
 * if source_is_bf16), finite.  Writes packed_values [rows, cols/2],
 * block_scales [rows, cols/16] and *global_decode_scale.  Needs a workspace
 * of nvfp4da_quantize_workspace_size() bytes. */
size_t nvfp4da_quantize_workspace_size(int64_t rows, int64_t cols);
int nvfp4da_quantize_nvfp4(const void* source, int source_is_bf16, int64_t rows, int64_t cols,
                           uint8_t* packed_values, uint8_t* block_scales, float* global_decode_scale,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Replaces launch_rms_norm_cuda (include/rmsnorm.h:12-16; op
 * src/bindings.cpp:438-486): out = BF16(x * rsqrt(mean(x^2) + eps) * weight)
 * over the last dimension; x is [rows, cols]. */
int nvfp4da_rms_norm(const uint16_t* x, const uint16_t* weight, uint16_t* out, int64_t rows, int64_t cols,
                     float eps, void* stream);

/* Replaces launch_rope_cuda (include/rope.h:16-20; op src/bindings.cpp:488-532):
 * adjacent-pair RoPE on x [B, T, H, D] at positions past_length + t. */
int nvfp4da_apply_rope(const uint16_t* x, uint16_t* out, int64_t batch, int64_t tokens, int64_t heads,
                       int64_t head_dim, int64_t past_length, float rope_theta, void* stream);

/* Replaces launch_w4a16_linear_cuda (include/w4a16.h:15-20; op
 * src/bindings.cpp:200-317) and launch_w4a16_linear_grouped_decode_cuda
 * (include/w4a16_grouped.h:15-20): y[M, N] = BF16(x[M, K] @ W_hat^T). */
int nvfp4da_w4a16_linear(const uint16_t* x, int64_t m, const nvfp4da_weight* w, uint16_t* y, void* stream);

/* The same projection forced onto the tcgen05 tensor-core GEMM (BF16
 * operands from the in-shared-memory dequantization, FP32 accumulator in
 * tensor memory).  nvfp4da_w4a16_linear takes it by itself for M >= 64.  Needs
 * K % 256 == 0; NVFP4DA_ERR_UNSUPPORTED otherwise.  Replaces
 * launch_w4a16_linear_cuda (include/w4a16.h:15-20) for prefill-sized M. */
int nvfp4da_w4a16_gemm(const uint16_t* x, int64_t m, const nvfp4da_weight* w, uint16_t* y, void* stream);
/* Replaces launch_kv_cache_append_cuda (include/kv_cache.h:18-25; op
 * src/bindings.cpp:784-884): cache[b, h, P_b + t, :] = new[b, t, h, :] for K and V.
 * P_b = past_lengths[b] when past_lengths (device int64 [B]) is not NULL,
 * else past_length.  Caller guarantees P_b + T <= capacity. */
int nvfp4da_kv_cache_append(uint16_t* k_cache, uint16_t* v_cache, const uint16_t* new_k, const uint16_t* new_v,
                            int64_t batch, int64_t kv_heads, int64_t capacity, int64_t head_dim, int64_t tokens,
                            int64_t past_length, const int64_t* past_lengths, void* stream);

/* Replaces launch_gqa_attention_cached_cuda (include/gqa_attention_cached.h:17-25;
 * op src/bindings.cpp:653-782) and, with capacity == past_length + tokens,
 * launch_gqa_attention_cuda (include/gqa_attention.h:17-25): causal GQA of
 * q [B, T, Hq, D] over caches [B, Hkv, C, D]; context [B, T, Hq, D].
 * max_past_length bounds every P_b (== past_length when past_lengths is NULL).
 * head_dim <= 256.  Workspace: nvfp4da_gqa_attention_workspace_size() bytes;
 * its counter words are cleared by the call itself. */
size_t nvfp4da_gqa_attention_workspace_size(int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads,
                                            int64_t head_dim, int64_t max_past_length);
int nvfp4da_gqa_attention_cached(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                 uint16_t* context, int64_t batch, int64_t tokens, int64_t q_heads,
                                 int64_t kv_heads, int64_t capacity, int64_t head_dim, int64_t past_length,
                                 const int64_t* past_lengths, int64_t max_past_length, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Optional per-stage outputs of the forward (NULL entries are skipped), in the
 * reference's stage layout (reference/decoder_attention_nvfp4.py:20-31). */
typedef struct nvfp4da_forward_stages {
  uint16_t* input_normalized; /* [B, T, H] */
  uint16_t* q_projected;      /* [B, T, Hq*D] */
  uint16_t* k_projected;      /* [B, T, Hkv*D] */
  uint16_t* v_projected;      /* [B, T, Hkv*D] */
  uint16_t* q_normalized;     /* [B, T, Hq, D] */
  uint16_t* k_normalized;     /* [B, T, Hkv, D] */
  uint16_t* q_rope;           /* [B, T, Hq, D] */
  uint16_t* context;          /* [B, T, Hq, D] */
} nvfp4da_forward_stages;

typedef struct nvfp4da_forward_args {
  const uint16_t* x;                 /* [B, T, H] */
  const uint16_t* input_norm_weight; /* [H] */
  nvfp4da_weight q_weight;           /* [H, H] */
  nvfp4da_weight k_weight;           /* [Hkv*D, H] */
  nvfp4da_weight v_weight;           /* [Hkv*D, H] */
  nvfp4da_weight out_weight;         /* [H, H] */
  const uint16_t* q_norm_weight;     /* [D] */
  const uint16_t* k_norm_weight;     /* [D] */
  uint16_t* k_cache;                 /* [B, Hkv, C, D], slots P_b..P_b+T-1 written */
  uint16_t* v_cache;
  uint16_t* output; /* [B, T, H] */
  int64_t batch, tokens, hidden, kv_heads, head_dim, capacity;
  int64_t past_length;         /* used when past_lengths == NULL */
  const int64_t* past_lengths; /* optional device int64 [B] */
  int64_t max_past_length;     /* >= every P_b */
  float rms_eps;
  float rope_theta;
  const nvfp4da_forward_stages* stages; /* optional, host struct */
} nvfp4da_forward_args;

/* Replaces the composed forward cuda_decoder_attention_forward_
 * (decoder_attention_cuda.py:149-417: 13 launches).  A T = 1 decode step that
 * the one-kernel step covers runs as one cooperative launch; other shapes run
 * three kernels chained by programmatic dependent launch (fused QKV with the
 * norms, RoPE and append; split-KV attention; O projection), or for
 * B*T >= 128 the modular chain on the tensor-core GEMM.  Mutates the caches
 * in place. */
size_t nvfp4da_forward_workspace_size(const nvfp4da_forward_args* args);
int nvfp4da_decoder_attention_forward(const nvfp4da_forward_args* args, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* Forward with an explicit kernel path.  NVFP4DA_PATH_AUTO (what
 * nvfp4da_decoder_attention_forward uses) takes the faster path for the call
 * as measured on B200 (the one-kernel step where it applies: same device
 * time as the chain, one launch instead of three);
 * NVFP4DA_PATH_CHAIN always takes the chain; NVFP4DA_PATH_STEP takes the
 * one-kernel decode step or fails with NVFP4DA_ERR_UNSUPPORTED.  Same results within the numerics policy (the
 * FP32 summation order of the projections and of the attention splits
 * differs).  The one-kernel step covers T == 1, B <= 8, hidden % 256 == 0,
 * hidden <= 4096, head_dim in {64, 128, 256}, 1/2/4/8 query heads per KV head,
 * no stage outputs, and a K/V tile per split that fits in shared memory.  It
 * is a cooperative launch whose phases hand data to one another through a
 * library-owned region of the stream it is launched on (64 slots of 512 KB
 * per device, one per stream, never released; configurations whose hand-off
 * words do not fit, and streams beyond the 64th, take the chain under AUTO):
 * a graph that captured it must not be replayed concurrently with other
 * forwards issued to the capturing stream.  No counterpart in the reference
 * (its forward is always the modular chain). */
#define NVFP4DA_PATH_AUTO 0
#define NVFP4DA_PATH_CHAIN 1
#define NVFP4DA_PATH_STEP 2
int nvfp4da_decoder_attention_forward_path(const nvfp4da_forward_args* args, void* workspace, size_t workspace_bytes,
                                           void* stream, int path);
/* The forward with host buffers, for hosts that keep activations in host
 * memory: x_host ([B, T, H] BF16) in, output_host out, all enqueued on
 * `stream` (the caller synchronises before reading output_host).
 * Input: when the one-kernel step runs, rows of up to 6 KB travel in the
 * kernel's parameter block (x_host is read during the call and may be reused
 * at once; any host memory); larger rows in page-locked memory the device can
 * address (cudaHostAlloc / cudaHostRegister, as torch's pin_memory()) are
 * read by the kernel itself; otherwise x_host is copied into args->x on the
 * stream (and must stay valid until the stream gets there).  Output: into
 * such page-locked memory the forward writes directly and args->output is
 * not written; otherwise args->output is copied to output_host.  Replaces
 * the host-side sequence around cuda_decoder_attention_forward_
 * (decoder_attention_cuda.py:149-417: the caller's x.to(device) and y.cpu())
 * with one call. */
int nvfp4da_decoder_attention_forward_hostio(const nvfp4da_forward_args* args, const uint16_t* x_host,
                                             uint16_t* output_host, void* workspace, size_t workspace_bytes,
                                             void* stream);
/* 1 if the one-kernel decode step covers args, else 0. */
int nvfp4da_forward_step_supported(const nvfp4da_forward_args* args);
/* Error flags recorded by one-kernel steps on `stream` (bit 0: a bounded wait
 * timed out); synchronises the stream; clears them if `clear`.  No
 * counterpart in the reference. */
int nvfp4da_forward_sync_status(void* stream, unsigned* flags, int clear);
/* Self-test of the bounded wait used by the one-kernel step: one CTA waits on
 * a counter that nothing sets, gives up after timeout_ns and reports the
 * timeout in *flags (bit 0).  Synchronises the stream. */
int nvfp4da_debug_wait_timeout(void* stream, unsigned long long timeout_ns, unsigned* flags);
/* The fused front half of the forward on its own: input RMSNorm, Q/K/V
 * projection, per-head Q/K RMSNorm, RoPE and the K/V append, one kernel.
 * Replaces the reference's chain cuda_rms_norm -> 3x cuda_w4a16_linear ->
 * 2x cuda_rms_norm -> 2x cuda_apply_rope -> cuda_kv_cache_append_
 * (decoder_attention_cuda.py:273-395).  Writes q after RoPE to q_rope_out
 * [B, T, Hq, D] and the new K/V into the caches; args->out_weight and
 * args->output are not used.  Needs head_dim % 32 == 0 and head_dim <= 256. */
int nvfp4da_qkv_rope_append(const nvfp4da_forward_args* args, uint16_t* q_rope_out, void* stream);

/* ---- KV-length sharding (long-context decode over several GPUs).  Each
 * GPU holds the positions [shard_start, shard_start + shard_capacity) of every
 * sequence's cache ([B, Hkv, shard_capacity, D]).  One step:
 *   1. nvfp4da_qkv_rope_append_shard on every GPU (replicated projections;
 *      only the GPU whose shard holds slot P_b + t appends it);
 *   2. nvfp4da_gqa_attention_partials: this shard's log-sum-exp partials;
 *   3. an all-gather of the partials between the GPUs (the host's NCCL
 *      communicator), then nvfp4da_attention_combine -> context;
 *   4. nvfp4da_w4a16_linear with the O weight.
 * Replaces the single-GPU cuda_gqa_attention_cached path for caches split by
 * position; the reference has no multi-GPU path. */
/* Step 1: as nvfp4da_qkv_rope_append, with args->k_cache / v_cache this
 * shard's caches and args->capacity the shard capacity; positions are checked
 * against global_capacity; RoPE uses the global position. */
int nvfp4da_qkv_rope_append_shard(const nvfp4da_forward_args* args, int64_t shard_start, int64_t global_capacity,
                                  uint16_t* q_rope_out, void* workspace, size_t workspace_bytes, void* stream);
/* Workspace of nvfp4da_qkv_rope_append_shard (256-byte aligned): the
 * normalised activation rows and RoPE table of the batched front half, used
 * for 2..64 rows of D = 128; 0 where the shape takes the decode kernel (a
 * NULL workspace is then accepted). */
size_t nvfp4da_qkv_rope_append_shard_workspace_size(const nvfp4da_forward_args* args);
/* Step 2: partials [B*T*Hq][D + 2] float32: o (unnormalised), m, l per query
 * row; a shard with no visible key gives m = -inf, l = 0, o = 0. */
size_t nvfp4da_gqa_attention_partials_workspace_size(int64_t batch, int64_t tokens, int64_t q_heads,
                                                     int64_t kv_heads, int64_t head_dim, int64_t shard_start,
                                                     int64_t shard_capacity, int64_t max_past_length);
int nvfp4da_gqa_attention_partials(const uint16_t* q, const uint16_t* k_shard, const uint16_t* v_shard,
                                   float* partials, int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads,
                                   int64_t shard_capacity, int64_t head_dim, int64_t shard_start,
                                   int64_t past_length, const int64_t* past_lengths, int64_t max_past_length,
                                   void* workspace, size_t workspace_bytes, void* stream);
/* Step 3: partials [shards][rows][D + 2] (shard order) -> BF16 context
 * [rows][D], rows = B*T*Hq. */
int nvfp4da_attention_combine(const float* partials, int shards, int64_t rows, int64_t head_dim, uint16_t* ctx,
                              void* stream);
/* Allocation-free forward.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory (a fixed HBM budget reserved up
 * front, a host whose allocator owns all device memory, or a context where an
 * allocation would stall the stream).  Same arguments and results as
 * nvfp4da_decoder_attention_forward, but the scratch memory comes from one
 * NVFP4DA_NOALLOC_SCRATCH_BYTES (8 MiB) array built into the library, resident
 * on every GPU that loads it until the process exits.  Calls needing more
 * scratch than that are rejected with NVFP4DA_ERR_WORKSPACE before any launch.
 * The first call on a device looks up that device's copy of the array
 * (cudaGetSymbolAddress) with the device current; make that first call before
 * any stream capture.  Allocates nothing.  All calls share the one array and
 * it keeps the last call's contents, so calls that overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller.
 * The looked-up address is kept for the life of the process: resetting a
 * device (cudaDeviceReset) after its first call is not supported. */
#define NVFP4DA_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
int nvfp4da_decoder_attention_forward_noalloc(const nvfp4da_forward_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_DECODER_ATTENTION_H_ */
