// C ABI of libnvfp4da.so: validation, launch planning and kernel launches.
// Declarations and reference citations: include/nvfp4_decoder_attention.h.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/nvfp4_decoder_attention.h"
#include "attention.cuh"
#include "attention_stream.cuh"
#include "attention_prefill.cuh"
#include "attention_prefill_tc.cuh"
#include "elementwise.cuh"
#include "gemv_batched.cuh"
#include "gemv_kernel.cuh"
#include "prefill_gemm.cuh"
#include "decode_step.cuh"
#include "qkv_fused.cuh"

namespace nvfp4da {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear a non-sticky launch error so later calls start clean
  return fail(NVFP4DA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define NVFP4DA_CHECK_LAUNCH(what)                       \
  do {                                                   \
    cudaError_t e_ = cudaGetLastError();                 \
    if (e_ != cudaSuccess) return cuda_fail(e_, what);   \
  } while (0)

constexpr int kMaxDevices = 64;
constexpr uint32_t kMaxDynSmem = 227 * 1024;

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int sm_count() {
  static int cached[kMaxDevices] = {0};
  const int dev = current_device();
  if (dev < kMaxDevices && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < kMaxDevices) cached[dev] = n;
  return n;
}

// Raise the dynamic shared-memory limit of `fn` on the current device once
// (cached per kernel and device; all instantiations of one kernel template
// share a function type, so the key is the function address).
std::mutex g_smem_mutex;
std::map<std::pair<const void*, int>, uint32_t> g_smem_set;

template <typename F>
cudaError_t ensure_smem(F* fn, uint32_t bytes) {
  const void* key = reinterpret_cast<const void*>(fn);
  const int dev = current_device();
  // Each host thread remembers its last answer: a serving loop launches the
  // same kernels with the same sizes on every call.
  struct Hit {
    const void* key = nullptr;
    int dev = -1;
    uint32_t bytes = 0;
  };
  thread_local Hit hits[8];
  for (const Hit& h : hits)
    if (h.key == key && h.dev == dev && h.bytes >= bytes) return cudaSuccess;
  thread_local int next_hit = 0;
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  auto it = g_smem_set.find({key, dev});
  if (it != g_smem_set.end() && it->second >= bytes) return cudaSuccess;
  // Prefer the largest shared-memory carve-out so that several CTAs (of this
  // kernel and of the kernels chained after it) fit on one SM.
  cudaError_t e = cudaFuncSetAttribute(key, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       static_cast<int>(cudaSharedmemCarveoutMaxShared));
  // The opt-in is needed whenever static + dynamic shared memory passes 48 KB,
  // not only when the dynamic part alone does, so always declare it.
  if (e == cudaSuccess && bytes > 0)
    e = cudaFuncSetAttribute(key, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) {
    g_smem_set[{key, dev}] = bytes;
    hits[next_hit] = {key, dev, bytes};
    next_hit = (next_hit + 1) % 8;
  }
  return e;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           bool pdl, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                   Args&&... args) {
  return launch_cluster(kernel, grid, block, smem, stream, pdl, 1u, std::forward<Args>(args)...);
}

// Allow cluster sizes above the portable 8 for `fn` on the current device once.
std::map<std::pair<const void*, int>, bool> g_cluster_set;

template <typename F>
cudaError_t ensure_big_clusters(F* fn) {
  const void* key = reinterpret_cast<const void*>(fn);
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  if (g_cluster_set.count({key, dev})) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(key, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) g_cluster_set[{key, dev}] = true;
  return e;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int check_weight(const nvfp4da_weight* w, const char* name) {
  if (!w) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "%s is NULL", name);
  if (!w->packed_values || !w->block_scales || !w->global_decode_scale)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "%s has a NULL field", name);
  if (w->rows <= 0 || w->cols <= 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "%s dimensions must be positive", name);
  if (w->cols < 16 || w->cols % 16 != 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "logical K must be a positive multiple of 16, got %lld",
                static_cast<long long>(w->cols));
  return NVFP4DA_OK;
}

bool gemm_tc_supported(const uint16_t* x, int64_t m, const nvfp4da_weight& w, const uint16_t* y);
int run_gemm_tc(const uint16_t* x, int64_t m, const nvfp4da_weight& w, uint16_t* y, cudaStream_t s);
constexpr int64_t kGemmMinMDecl = 64;  // at and above this M the tensor-core GEMM replaces the GEMV
constexpr int64_t kPrefillMinM = 128;  // at and above this M the forward takes the modular chain
constexpr int64_t kPrefillAttnMinT = 64;  // at and above this T attention runs on the tensor cores

// ---------------------------------------------------------------- GEMV plan
struct GemvPlan {
  bool mma;      // tensor-core path (K % 32 == 0)
  int rows;      // mma path: rows per CTA (16 or 32)
  int rpw, mg;   // CUDA-core path
  uint32_t smem;
  int64_t ctas;
};

bool plan_gemv(int64_t m, int64_t n, int64_t k, GemvPlan& pl) {
  const int sms = sm_count();
  if (mma_gemv_supported(k)) {
    const int mg = static_cast<int>(m < kMmaMaxM ? m : kMmaMaxM);
    const int rows = (ceil_div(n, 32) >= 2 * sms) ? 32 : 16;
    const uint32_t bytes = mma_gemv_layout(rows, k, mg).total();
    if (bytes <= kMaxDynSmem - 8 * 1024) {
      pl = {true, rows, 0, 0, bytes, ceil_div(n, rows)};
      return true;
    }
  }
  int rpw = 1;
  for (int r : {4, 2}) {
    if (ceil_div(n, kGemvWarps * r) >= sms) {
      rpw = r;
      break;
    }
  }
  int mg = m <= 1 ? 1 : (m == 2 ? 2 : 4);
  for (;;) {
    const uint32_t bytes = gemv_layout(kGemvWarps * rpw, k, mg).total();
    if (bytes <= kMaxDynSmem) {
      pl = {false, 0, rpw, mg, bytes, ceil_div(n, kGemvWarps * rpw)};
      return true;
    }
    if (mg > 1) mg >>= 1;
    else if (rpw > 1) rpw >>= 1;
    else return false;
  }
}

template <int RPW, int MG>
cudaError_t launch_gemv_t(const GemvParams& p, const GemvPlan& pl, cudaStream_t s, bool pdl) {
  auto* k = w4a16_gemv_kernel<RPW, MG>;
  cudaError_t e = ensure_smem(k, pl.smem);
  if (e != cudaSuccess) return e;
  return launch(k, dim3(static_cast<unsigned>(pl.ctas)), dim3(kGemvThreads), pl.smem, s, pdl, p);
}

template <int ROWS>
cudaError_t launch_mma_gemv_t(const GemvParams& p, const GemvPlan& pl, cudaStream_t s, bool pdl) {
  auto* k = mma_gemv_kernel<ROWS>;
  cudaError_t e = ensure_smem(k, pl.smem);
  if (e != cudaSuccess) return e;
  return launch(k, dim3(static_cast<unsigned>(pl.ctas)), dim3(kMmaThreads), pl.smem, s, pdl, p);
}

cudaError_t launch_gemv(const GemvParams& p, const GemvPlan& pl, cudaStream_t s, bool pdl) {
  if (pl.mma) return pl.rows == 32 ? launch_mma_gemv_t<32>(p, pl, s, pdl) : launch_mma_gemv_t<16>(p, pl, s, pdl);
#define NVFP4DA_GEMV_CASE(R, M) \
  if (pl.rpw == R && pl.mg == M) return launch_gemv_t<R, M>(p, pl, s, pdl);
  NVFP4DA_GEMV_CASE(1, 1)
  NVFP4DA_GEMV_CASE(1, 2)
  NVFP4DA_GEMV_CASE(1, 4)
  NVFP4DA_GEMV_CASE(2, 1)
  NVFP4DA_GEMV_CASE(2, 2)
  NVFP4DA_GEMV_CASE(2, 4)
  NVFP4DA_GEMV_CASE(4, 1)
  NVFP4DA_GEMV_CASE(4, 2)
  NVFP4DA_GEMV_CASE(4, 4)
#undef NVFP4DA_GEMV_CASE
  return cudaErrorInvalidConfiguration;
}

// ---------------------------------------------------------------- batched decode projections (8 < M <= 64)
int bat_tiles(int64_t m) { return m <= 8 ? 1 : (m <= 16 ? 2 : (m <= 32 ? 4 : 8)); }

template <int NT>
cudaError_t launch_o_batched_t(const GemvParams& p, cudaStream_t s, bool pdl) {
  auto* k = o_batched_kernel<NT>;
  const uint32_t smem = bat_smem_bytes(p.k, NT * 8);
  cudaError_t e = ensure_smem(k, smem);
  if (e != cudaSuccess) return e;
  return launch(k, dim3(static_cast<unsigned>(p.n / kBatRows * kBatCluster)), dim3(kBatThreads), smem, s, pdl, p);
}

bool bat_linear_ok(const uint16_t* x, int64_t m, const nvfp4da_weight& w) {
  return bat_shape_ok(m, w.rows, w.cols) && aligned(x, 16) && aligned(w.packed_values, 16) &&
         aligned(w.block_scales, 16) && bat_smem_bytes(w.cols, 64) <= kMaxDynSmem &&
         w.rows / kBatRows <= std::numeric_limits<int32_t>::max();
}

int run_gemv(const uint16_t* x, int64_t m, const nvfp4da_weight& w, uint16_t* y, cudaStream_t s, bool pdl) {
  // Up to 8 rows the decode GEMV (one pass, 192 CTAs of 16 rows) measured
  // faster than the batched kernel (96 CTAs); from 9 rows it re-decodes.
  if (m > kMmaMaxM && bat_linear_ok(x, m, w)) {
    GemvParams p{x, m, w.packed_values, w.block_scales, w.global_decode_scale, y, w.rows, w.cols, nullptr, pdl ? 1 : 0};
    const int nt = bat_tiles(m);
    cudaError_t e = nt == 1 ? launch_o_batched_t<1>(p, s, pdl)
                    : nt == 2 ? launch_o_batched_t<2>(p, s, pdl)
                    : nt == 4 ? launch_o_batched_t<4>(p, s, pdl)
                              : launch_o_batched_t<8>(p, s, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "batched w4a16 launch");
    return NVFP4DA_OK;
  }
  if (m >= kGemmMinMDecl && gemm_tc_supported(x, m, w, y)) return run_gemm_tc(x, m, w, y, s);
  GemvPlan pl;
  if (!plan_gemv(m, w.rows, w.cols, pl))
    return fail(NVFP4DA_ERR_UNSUPPORTED, "K=%lld is too large for the shared-memory GEMV", static_cast<long long>(w.cols));
  if (pl.ctas > std::numeric_limits<int32_t>::max())
    return fail(NVFP4DA_ERR_UNSUPPORTED, "N is too large for a one-dimensional grid");
  GemvParams p{x, m, w.packed_values, w.block_scales, w.global_decode_scale, y, w.rows, w.cols, nullptr, pdl ? 1 : 0};
  cudaError_t e = launch_gemv(p, pl, s, pdl);
  if (e != cudaSuccess) return cuda_fail(e, "w4a16 gemv launch");
  return NVFP4DA_OK;
}

// ---------------------------------------------------------------- tensor-core GEMM (prefill-sized M)
// 128 x 256 tiles: half the x traffic of 128 x 128 per FLOP and full-rate
// N=256 MMAs; two accumulators of 256 columns fill the tensor memory.
constexpr int kPgBN = 256;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    cudaGetLastError();
  });
  return fn;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor-core path needs whole 64-wide K steps and 16-byte TMA row
// strides for the scales (K % 256 == 0), and 16-byte aligned bases.
bool gemm_tc_supported(const uint16_t* x, int64_t m, const nvfp4da_weight& w, const uint16_t* y) {
  return w.cols >= 256 && w.cols % 256 == 0 && m > 0 && aligned(x, 16) && aligned(y, 2) &&
         aligned(w.packed_values, 16) && aligned(w.block_scales, 16) && m <= (int64_t(1) << 31) &&
         w.rows <= (int64_t(1) << 31) && tensor_map_encoder() != nullptr;
}

int run_gemm_tc(const uint16_t* x, int64_t m, const nvfp4da_weight& w, uint16_t* y, cudaStream_t s) {
  const int64_t n = w.rows, k = w.cols;
  CUtensorMap tx, tw, ts;
  if (!make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, k, m, k * 2, kPgBK, kPgBM,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed_values, k / 2, n, k / 2, kPgBK / 2, kPgBN,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.block_scales, k / 16, n, k / 16, 16, kPgBN,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(NVFP4DA_ERR_CUDA, "tensor map encoding failed for the tensor-core GEMM");
  PgParams p{m, n, k, w.global_decode_scale, y, nullptr};
  auto* kern = w4a16_gemm_tc_kernel<kPgBN>;
  const uint32_t smem = PgLayout<kPgBN>::total();
  cudaError_t e = ensure_smem(kern, smem);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM shared-memory opt-in");
  const dim3 grid(static_cast<unsigned>(ceil_div(n, kPgBN)), static_cast<unsigned>(ceil_div(m, kPgBM)));
  if (grid.y > 65535) return fail(NVFP4DA_ERR_UNSUPPORTED, "M too large for the tensor-core GEMM grid");
  kern<<<grid, PgCfg<kPgBN>::kThreads, smem, s>>>(tx, tw, ts, p);
  NVFP4DA_CHECK_LAUNCH("tensor-core GEMM launch");
  return NVFP4DA_OK;
}

// ---------------------------------------------------------------- attention plan
// Two decode-attention kernels share one workspace layout (the partials at
// the start, the counter words at partial_bytes, both sized for the larger of
// the two plans), so a call planned for one can run the other:
//  * attn_split_kernel: splits of a fixed length, CUDA-core loop from global
//    memory, cluster (DSMEM) combine up to 16 splits -- lowest latency for
//    short caches;
//  * attn_stream_kernel: one persistent CTA per SM over the flattened tile
//    line of all (sequence, KV head) pairs, TMA-fed tensor-core loop -- HBM
//    rate for long caches (visible length >= kStreamMinVisible).
struct AttnPlan {
  int epl, gh, head_groups, splits;
  int64_t split_len;
  bool cluster;  // splits combine through DSMEM as one cluster (2..16 splits)
  bool stream;   // attn_stream_kernel applies (it is still skipped for unaligned or huge caches)
  int stream_grid;
  uint32_t stream_smem;
  size_t partial_bytes, counter_bytes;
};

constexpr int kMaxAttnCluster = 16;
constexpr int64_t kStreamMinVisible = 2048;

uint32_t stream_smem_bytes(int64_t head_dim, int64_t batch) {
  switch (head_dim) {
    case 64: return AsCfg<64>::bytes(static_cast<int>(batch));
    case 128: return AsCfg<128>::bytes(static_cast<int>(batch));
    case 256: return AsCfg<256>::bytes(static_cast<int>(batch));
    default: return 0;
  }
}

bool plan_attention(int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                    int64_t max_past, AttnPlan& pl) {
  if (head_dim <= 0 || head_dim > 256) return false;
  int epl = head_dim <= 32 ? 1 : head_dim <= 64 ? 2 : head_dim <= 128 ? 4 : 8;
  if (head_dim % epl != 0) return false;
  const int64_t group = q_heads / kv_heads;
  int gh = 1;
  for (int g : {8, 4, 2}) {
    if (group % g == 0) {
      gh = g;
      break;
    }
  }
  const int64_t ng = group / gh;
  const int64_t chunk = kAttnWarps * std::min<int64_t>(8, 32 / gh);
  const int64_t visible = max_past + tokens;
  const int64_t base = batch * tokens * kv_heads * ng;
  int64_t splits = ceil_div(8LL * sm_count(), base);
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, ceil_div(visible, chunk)));
  int64_t split_len = ceil_div(ceil_div(visible, splits), chunk) * chunk;
  splits = ceil_div(visible, split_len);
  // The last-CTA combine stages 2 * GH * splits floats in the CTA's
  // 4 * GH * 32 * EPL-float output buffer: at most 64 * EPL splits.
  const int64_t max_splits = 64LL * epl;
  if (splits > max_splits) {
    splits = max_splits;
    split_len = ceil_div(ceil_div(visible, splits), chunk) * chunk;
    splits = ceil_div(visible, split_len);
  }
  pl.epl = epl;
  pl.gh = gh;
  pl.head_groups = static_cast<int>(ng);
  pl.splits = static_cast<int>(splits);
  pl.split_len = split_len;
  pl.cluster = splits > 1 && splits <= kMaxAttnCluster;
  const bool global = splits > 1 && !pl.cluster;
  size_t part = global ? static_cast<size_t>(batch * tokens * q_heads) * splits * (head_dim + 2) * 4 : 0;
  size_t words = global ? static_cast<size_t>(base) : 0;
  // The streaming kernel: group * T query rows per KV head fit one 8-wide MMA
  // tile, and the per-sequence prefix fits its shared memory.
  pl.stream_smem = stream_smem_bytes(head_dim, batch);
  pl.stream = visible >= kStreamMinVisible && group * tokens <= kAsRows && batch <= kAsMaxBatch &&
              pl.stream_smem > 0 && pl.stream_smem <= kMaxDynSmem && tensor_map_encoder() != nullptr;
  pl.stream_grid = sm_count();
  if (pl.stream) {
    const int64_t pairs = batch * kv_heads;
    part = std::max(part, static_cast<size_t>(pairs + pl.stream_grid) * kAsRows * (head_dim + 2) * 4);
    words = std::max(words, static_cast<size_t>(pairs) + 1);  // counters + the error word
  }
  pl.partial_bytes = align_up(part, 256);
  pl.counter_bytes = align_up(words * 4, 256);
  return true;
}

template <int D>
cudaError_t launch_stream_t(const CUtensorMap& tk, const CUtensorMap& tv, const StreamAttnParams& p, int grid,
                            uint32_t smem, cudaStream_t s, bool pdl) {
  auto* k = attn_stream_kernel<D>;
  cudaError_t e = ensure_smem(k, smem);
  if (e != cudaSuccess) return e;
  return launch(k, dim3(static_cast<unsigned>(grid)), dim3(kAsThreads), smem, s, pdl, tk, tv, p);
}

// Run attn_stream_kernel if the call allows it (returns false, launching
// nothing, otherwise); *launch_err is set if the launch itself failed.
bool try_stream_attention(const AttnPlan& pl, const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                          uint16_t* ctx, int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads,
                          int64_t capacity, int64_t head_dim, int64_t past_length, const int64_t* past_lengths,
                          void* ws, cudaStream_t s, bool pdl, int64_t pos_offset, float* out_partial,
                          cudaError_t* launch_err) {
  *launch_err = cudaSuccess;
  if (!pl.stream || !ws) return false;
  const int64_t rows = batch * kv_heads * capacity;
  if (rows >= (int64_t(1) << 31) || !aligned(kc, 16) || !aligned(vc, 16) || !aligned(q, 4)) return false;
  CUtensorMap tk, tv;
  if (!make_map_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kc, head_dim, rows, head_dim * 2, 64, kAsTile,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, vc, head_dim, rows, head_dim * 2, 64, kAsTile,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return false;
  StreamAttnParams p{};
  p.q = q;
  p.ctx = ctx;
  p.out_partial = out_partial;
  p.batch = static_cast<int>(batch);
  p.tokens = static_cast<int>(tokens);
  p.q_heads = static_cast<int>(q_heads);
  p.kv_heads = static_cast<int>(kv_heads);
  p.group = static_cast<int>(q_heads / kv_heads);
  p.capacity = capacity;
  p.past_length = past_length;
  p.past_lengths = past_lengths;
  p.pos_offset = pos_offset;
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)));
  p.partials = static_cast<float*>(ws);
  p.counters = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + pl.partial_bytes);
  p.err = p.counters + batch * kv_heads;
  p.pdl = pdl ? 1 : 0;
  switch (head_dim) {
    case 64: *launch_err = launch_stream_t<64>(tk, tv, p, pl.stream_grid, pl.stream_smem, s, pdl); break;
    case 128: *launch_err = launch_stream_t<128>(tk, tv, p, pl.stream_grid, pl.stream_smem, s, pdl); break;
    default: *launch_err = launch_stream_t<256>(tk, tv, p, pl.stream_grid, pl.stream_smem, s, pdl); break;
  }
  return true;
}

template <int EPL, int GH>
cudaError_t launch_attn_t(const AttnParams& p, dim3 grid, cudaStream_t s, bool pdl) {
  auto* k = attn_split_kernel<EPL, GH>;
  cudaError_t ec = ensure_smem(k, 0);
  if (ec != cudaSuccess) return ec;
  const unsigned cx = p.cluster_combine ? static_cast<unsigned>(p.splits) : 1u;
  if (cx > 8) {
    cudaError_t e = ensure_big_clusters(k);
    if (e != cudaSuccess) return e;
  }
  return launch_cluster(k, grid, dim3(kAttnThreads), 0, s, pdl, cx, p);
}

cudaError_t launch_attn(const AttnParams& p, const AttnPlan& pl, cudaStream_t s, bool pdl) {
  const dim3 grid(static_cast<unsigned>(pl.splits), static_cast<unsigned>(p.kv_heads * pl.head_groups),
                  static_cast<unsigned>(p.batch * p.tokens));
#define NVFP4DA_ATTN_CASE(E, G) \
  if (pl.epl == E && pl.gh == G) return launch_attn_t<E, G>(p, grid, s, pdl);
  NVFP4DA_ATTN_CASE(1, 1)
  NVFP4DA_ATTN_CASE(1, 2)
  NVFP4DA_ATTN_CASE(1, 4)
  NVFP4DA_ATTN_CASE(1, 8)
  NVFP4DA_ATTN_CASE(2, 1)
  NVFP4DA_ATTN_CASE(2, 2)
  NVFP4DA_ATTN_CASE(2, 4)
  NVFP4DA_ATTN_CASE(2, 8)
  NVFP4DA_ATTN_CASE(4, 1)
  NVFP4DA_ATTN_CASE(4, 2)
  NVFP4DA_ATTN_CASE(4, 4)
  NVFP4DA_ATTN_CASE(4, 8)
  NVFP4DA_ATTN_CASE(8, 1)
  NVFP4DA_ATTN_CASE(8, 2)
  NVFP4DA_ATTN_CASE(8, 4)
  NVFP4DA_ATTN_CASE(8, 8)
#undef NVFP4DA_ATTN_CASE
  return cudaErrorInvalidConfiguration;
}

int check_attention_dims(int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t capacity,
                         int64_t head_dim, int64_t max_past) {
  if (batch <= 0 || tokens <= 0 || q_heads <= 0 || kv_heads <= 0 || capacity <= 0 || head_dim <= 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "attention dimensions must all be positive");
  if (q_heads % kv_heads != 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "number of query heads must be divisible by number of KV heads");
  if (max_past < 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length must be nonnegative");
  if (max_past > std::numeric_limits<int64_t>::max() - tokens)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length + current token count overflows int64");
  if (max_past + tokens > capacity)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length + current token count exceeds cache capacity (%lld > %lld)",
                static_cast<long long>(max_past + tokens), static_cast<long long>(capacity));
  if (batch * tokens > 65535 || kv_heads * q_heads > 65535)
    return fail(NVFP4DA_ERR_UNSUPPORTED, "B*T and Hq*Hkv must each be at most 65535");
  return NVFP4DA_OK;
}

int run_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* ctx, int64_t batch,
                  int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t capacity, int64_t head_dim,
                  int64_t past_length, const int64_t* past_lengths, int64_t max_past, void* ws, size_t ws_bytes,
                  cudaStream_t s, bool pdl, bool clear_counters, int64_t pos_offset = 0,
                  float* out_partial = nullptr) {
  // Prefill-sized T: tcgen05 flash attention (128 query rows per CTA, TMA
  // tiles, accumulators in tensor memory).
  if (tokens >= kPrefillAttnMinT && head_dim == kPtD && !out_partial && pos_offset == 0 && aligned(q, 16) &&
      aligned(kc, 16) && aligned(vc, 16) && aligned(ctx, 16) && batch <= 65535 && q_heads <= 65535 &&
      batch * kv_heads * capacity < (int64_t(1) << 31) && batch * tokens < (int64_t(1) << 31) &&
      tensor_map_encoder() != nullptr) {
    auto fn = tensor_map_encoder();
    CUtensorMap tq, tk, tv;
    const cuuint64_t qdims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(q_heads),
                                 static_cast<cuuint64_t>(batch * tokens)};
    const cuuint64_t qstr[2] = {static_cast<cuuint64_t>(head_dim * 2), static_cast<cuuint64_t>(q_heads * head_dim * 2)};
    const cuuint32_t qbox[3] = {64, 1, static_cast<cuuint32_t>(kPtRows)};
    const cuuint32_t ones[3] = {1, 1, 1};
    const int64_t rows = batch * kv_heads * capacity;
    if (fn(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(q), qdims, qstr, qbox, ones,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
        make_map_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kc, head_dim, rows, head_dim * 2, 64, kPtKeys,
                    CU_TENSOR_MAP_SWIZZLE_128B) &&
        make_map_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, vc, head_dim, rows, head_dim * 2, 64, kPtKeys,
                    CU_TENSOR_MAP_SWIZZLE_128B)) {
      PrefillTcParams pp{ctx, static_cast<int>(batch), static_cast<int>(tokens), static_cast<int>(q_heads),
                         static_cast<int>(kv_heads), capacity, past_length, past_lengths,
                         static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim))), nullptr};
      cudaError_t e = ensure_smem(attn_prefill_tc_kernel, kPtSmem);
      if (e != cudaSuccess) return cuda_fail(e, "prefill attention shared-memory opt-in");
      const dim3 grid(static_cast<unsigned>(ceil_div(tokens, kPtRows)), static_cast<unsigned>(q_heads),
                      static_cast<unsigned>(batch));
      attn_prefill_tc_kernel<<<grid, kPtThreads, kPtSmem, s>>>(tq, tk, tv, pp);
      NVFP4DA_CHECK_LAUNCH("prefill attention launch");
      return NVFP4DA_OK;
    }
  }
  // Otherwise the mma.sync kernel (one CTA per 64 query tokens).
  if (tokens >= kPrefillAttnMinT && head_dim == kPaD && !out_partial && pos_offset == 0 && aligned(q, 16) &&
      aligned(kc, 16) && aligned(vc, 16) && aligned(ctx, 4) && batch <= 65535 && q_heads <= 65535) {
    PrefillAttnParams pp{q, kc, vc, ctx, batch, tokens, q_heads, kv_heads, capacity, past_length, past_lengths,
                         static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)))};
    cudaError_t e = ensure_smem(attn_prefill_kernel, kPaSmem);
    if (e != cudaSuccess) return cuda_fail(e, "prefill attention shared-memory opt-in");
    const dim3 grid(static_cast<unsigned>(ceil_div(tokens, kPaRows)), static_cast<unsigned>(q_heads),
                    static_cast<unsigned>(batch));
    attn_prefill_kernel<<<grid, kPaThreads, kPaSmem, s>>>(pp);
    NVFP4DA_CHECK_LAUNCH("prefill attention launch");
    return NVFP4DA_OK;
  }
  AttnPlan pl;
  if (!plan_attention(batch, tokens, q_heads, kv_heads, head_dim, max_past, pl))
    return fail(NVFP4DA_ERR_UNSUPPORTED, "head_dim %lld is not supported (need head_dim <= 256 and divisible by "
                "its per-lane vector width)", static_cast<long long>(head_dim));
  if (pl.partial_bytes + pl.counter_bytes > ws_bytes || (pl.partial_bytes > 0 && !ws))
    return fail(NVFP4DA_ERR_WORKSPACE, "attention workspace too small (%zu < %zu bytes)", ws_bytes,
                pl.partial_bytes + pl.counter_bytes);
  if (pl.stream && clear_counters) {
    cudaError_t e = cudaMemsetAsync(static_cast<char*>(ws) + pl.partial_bytes, 0, pl.counter_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "attention counter clear");
  }
  {
    cudaError_t le;
    if (try_stream_attention(pl, q, kc, vc, ctx, batch, tokens, q_heads, kv_heads, capacity, head_dim, past_length,
                             past_lengths, ws, s, pdl, pos_offset, out_partial, &le)) {
      if (le != cudaSuccess) return cuda_fail(le, "streaming attention launch");
      return NVFP4DA_OK;
    }
  }
  AttnParams p{};
  p.q = q;
  p.k_cache = kc;
  p.v_cache = vc;
  p.ctx = ctx;
  p.batch = batch;
  p.tokens = tokens;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.capacity = capacity;
  p.head_dim = head_dim;
  p.past_length = past_length;
  p.past_lengths = past_lengths;
  p.split_len = pl.split_len;
  p.splits = pl.splits;
  p.head_groups = pl.head_groups;
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)));
  const bool global = pl.splits > 1 && !pl.cluster;
  p.partials = global ? static_cast<float*>(ws) : nullptr;
  p.counters = global ? reinterpret_cast<unsigned*>(static_cast<char*>(ws) + pl.partial_bytes) : nullptr;
  p.pdl = pdl ? 1 : 0;
  p.cluster_combine = pl.cluster ? 1 : 0;
  p.pos_offset = pos_offset;
  p.out_partial = out_partial;
  if (clear_counters && global && !pl.stream) {
    cudaError_t e = cudaMemsetAsync(p.counters, 0, pl.counter_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "attention counter clear");
  }
  cudaError_t e = launch_attn(p, pl, s, pdl);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return NVFP4DA_OK;
}

// ---------------------------------------------------------------- fused QKV plan
struct QkvPlan {
  int rows;  // D / 4
  int mg;
  uint32_t smem;
};

bool plan_qkv(int64_t m, int64_t hidden, int64_t head_dim, QkvPlan& pl) {
  if (!mma_gemv_supported(hidden)) return false;
  if (head_dim % 32 != 0 || head_dim > kMaxHeadDim) return false;
  const int rows = static_cast<int>(head_dim / 4);
  const int mg = static_cast<int>(m < kMmaMaxM ? m : kMmaMaxM);
  const uint32_t bytes = qkv_layout(rows, hidden, head_dim, mg).total();
  if (bytes > kMaxDynSmem - 16 * 1024) return false;
  pl = {rows, mg, bytes};
  return true;
}

template <int ROWS>
cudaError_t launch_qkv_t(const QkvParams& p, const QkvPlan& pl, int64_t units, cudaStream_t s, bool pdl) {
  auto* k = qkv_fused_kernel<ROWS>;
  cudaError_t e = ensure_smem(k, pl.smem);
  if (e != cudaSuccess) return e;
  return launch(k, dim3(static_cast<unsigned>(units * kQkvCluster)), dim3(kMmaThreads), pl.smem, s, pdl, p);
}

cudaError_t launch_qkv(const QkvParams& p, const QkvPlan& pl, int64_t units, cudaStream_t s, bool pdl) {
  switch (pl.rows) {
    case 8: return launch_qkv_t<8>(p, pl, units, s, pdl);
    case 16: return launch_qkv_t<16>(p, pl, units, s, pdl);
    case 32: return launch_qkv_t<32>(p, pl, units, s, pdl);
    case 64: return launch_qkv_t<64>(p, pl, units, s, pdl);
    default: return cudaErrorInvalidConfiguration;
  }
}

template <int NT>
cudaError_t launch_qkv_batched_t(const QkvParams& p, int64_t units, cudaStream_t s) {
  auto* k = qkv_batched_kernel<NT>;
  const uint32_t smem = bat_smem_bytes(p.hidden, NT * 8);
  cudaError_t e = ensure_smem(k, smem);
  if (e != cudaSuccess) return e;
  return launch(k, dim3(static_cast<unsigned>(units * kBatCluster)), dim3(kBatThreads), smem, s, true, p);
}

// The batched front half: the rows' RMSNorm and RoPE table, then the
// projections with the head epilogue; both PDL-chained.
cudaError_t launch_qkv_batched(const QkvParams& p, int64_t units, cudaStream_t s) {
  cudaError_t e = launch(bat_norm_kernel, dim3(static_cast<unsigned>(p.m)), dim3(kNormThreads), 0, s, true, p);
  if (e != cudaSuccess) return e;
  const int nt = bat_tiles(p.m);
  return nt == 1 ? launch_qkv_batched_t<1>(p, units, s)
         : nt == 2 ? launch_qkv_batched_t<2>(p, units, s)
         : nt == 4 ? launch_qkv_batched_t<4>(p, units, s)
                   : launch_qkv_batched_t<8>(p, units, s);
}

// ---------------------------------------------------------------- forward plan
struct ForwardLayout {
  bool fused;
  bool batched;  // fused path with the batched front half (bat_norm + qkv_batched)
  QkvPlan qkv;
  AttnPlan attn;
  size_t q_buf, ctx_buf, attn_ws, scratch;  // byte offsets
  size_t total;
  // modular-path buffers (offsets)
  size_t xn, qp, kp, vp, qn, kn, kr;
  // batched front half (offsets)
  size_t bxn, brope;
};

int check_forward(const nvfp4da_forward_args* a) {
  if (!a) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "args is NULL");
  if (!a->x || !a->input_norm_weight || !a->q_norm_weight || !a->k_norm_weight || !a->k_cache || !a->v_cache ||
      !a->output)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (a->batch <= 0 || a->tokens <= 0 || a->hidden <= 0 || a->kv_heads <= 0 || a->head_dim <= 0 ||
      a->capacity <= 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "dimensions must all be positive");
  if (a->hidden % a->head_dim != 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "hidden size must be divisible by head dimension");
  const int64_t hq = a->hidden / a->head_dim;
  if (hq % a->kv_heads != 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "number of query heads must be divisible by number of KV heads");
  if (a->head_dim % 2 != 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "head dimension must be even");
  if (!(a->rms_eps > 0.0f) || !std::isfinite(a->rms_eps))
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "rms_eps must be finite and positive");
  if (!(a->rope_theta > 0.0f) || !std::isfinite(a->rope_theta))
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "rope_theta must be finite and positive");
  const int64_t maxp = a->past_lengths ? a->max_past_length : a->past_length;
  int r = check_attention_dims(a->batch, a->tokens, hq, a->kv_heads, a->capacity, a->head_dim, maxp);
  if (r) return r;
  const int64_t kvw = a->kv_heads * a->head_dim;
  struct {
    const nvfp4da_weight* w;
    const char* name;
    int64_t rows, cols;
  } ws[4] = {{&a->q_weight, "q_weight", a->hidden, a->hidden},
             {&a->k_weight, "k_weight", kvw, a->hidden},
             {&a->v_weight, "v_weight", kvw, a->hidden},
             {&a->out_weight, "out_weight", a->hidden, a->hidden}};
  for (auto& w : ws) {
    if ((r = check_weight(w.w, w.name))) return r;
    if (w.w->rows != w.rows || w.w->cols != w.cols)
      return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "%s must be [%lld, %lld]", w.name, static_cast<long long>(w.rows),
                  static_cast<long long>(w.cols));
  }
  return NVFP4DA_OK;
}

bool bat_weights_aligned(const nvfp4da_forward_args* a) {
  for (const nvfp4da_weight* w : {&a->q_weight, &a->k_weight, &a->v_weight})
    if (!aligned(w->packed_values, 16) || !aligned(w->block_scales, 16)) return false;
  return true;
}

bool step_covers(const nvfp4da_forward_args* a);  // the one-kernel step plans this shape (below)

// The batched front half (bat_norm_kernel + qkv_batched_kernel) applies:
// 2..64 rows, D = 128, K a multiple of 1024 that fits its shared memory and
// the norm kernel's registers, 16-byte aligned rows, gains and weights.
bool bat_front_ok(const nvfp4da_forward_args* a) {
  const int64_t m = a->batch * a->tokens;
  return a->head_dim == kBatRows && bat_shape_ok(m, a->hidden, a->hidden) && a->hidden <= 64 * kNormThreads &&
         bat_smem_bytes(a->hidden, 64) + kBatMaxM * kBatRows * 2 <= kMaxDynSmem &&  // + the static head rows
         aligned(a->x, 16) && aligned(a->input_norm_weight, 16) &&
         !(a->stages && a->stages->input_normalized && !aligned(a->stages->input_normalized, 16)) &&
         bat_weights_aligned(a);
}

// Its scratch: the normalised rows [M, H] BF16 (256-byte padded), then the
// RoPE table [M, D/2].
size_t bat_rows_bytes(const nvfp4da_forward_args* a) {
  return align_up(static_cast<size_t>(a->batch * a->tokens * a->hidden) * 2, 256);
}
size_t bat_front_bytes(const nvfp4da_forward_args* a) {
  return bat_rows_bytes(a) + align_up(static_cast<size_t>(a->batch * a->tokens * (a->head_dim / 2)) * sizeof(float2), 256);
}

int plan_forward(const nvfp4da_forward_args* a, ForwardLayout& L) {
  const int64_t hq = a->hidden / a->head_dim, m = a->batch * a->tokens;
  const int64_t maxp = a->past_lengths ? a->max_past_length : a->past_length;
  if (!plan_attention(a->batch, a->tokens, hq, a->kv_heads, a->head_dim, maxp, L.attn))
    return fail(NVFP4DA_ERR_UNSUPPORTED, "head_dim %lld is not supported", static_cast<long long>(a->head_dim));
  // Prefill-sized M: the modular chain, whose projections run on the
  // tensor-core GEMM; the fused front half re-decodes its weights for every 8
  // activation rows.
  L.fused = m < kPrefillMinM && plan_qkv(m, a->hidden, a->head_dim, L.qkv);
  // Up to 8 rows the batched front half only where the one-kernel step does
  // not cover the shape: the step reproduces the decode kernels' Q/K/V sums
  // bit for bit, so on its shapes the chain keeps those kernels.
  L.batched = L.fused && bat_front_ok(a) && (m > kMmaMaxM || !step_covers(a));
  const size_t act = align_up(static_cast<size_t>(m * a->hidden) * 2, 256);
  const size_t kvact = align_up(static_cast<size_t>(m * a->kv_heads * a->head_dim) * 2, 256);
  size_t off = 0;
  L.q_buf = off;
  off += act;
  L.ctx_buf = off;
  off += act;
  L.attn_ws = off;
  off += L.attn.partial_bytes + L.attn.counter_bytes;
  L.scratch = off;
  if (L.batched) {
    L.bxn = off;
    L.brope = off + act;
    off += bat_front_bytes(a);
  }
  if (!L.fused) {
    L.xn = off;
    off += act;
    L.qp = off;
    off += act;
    L.kp = off;
    off += kvact;
    L.vp = off;
    off += kvact;
    L.qn = off;
    off += act;
    L.kn = off;
    off += kvact;
    L.kr = off;
    off += kvact;
  }
  L.total = off;
  return NVFP4DA_OK;
}

// theta^(2m/D) rounded to FP32 with the arithmetic of reference
// decoder_attention.py:237-257 (FP32 exponent, the power in double rounded
// once), for m < D/2.  Host work every forward needs, so each host thread
// keeps the last (D, theta) table.
const float* rope_denominators(int64_t d, float theta) {
  thread_local int64_t cached_d = -1;
  thread_local float cached_theta = 0.0f;
  thread_local float tab[kMaxHeadDim / 2];
  if (cached_d != d || cached_theta != theta) {
    for (int64_t m = 0; m < d / 2 && m < kMaxHeadDim / 2; ++m) {
      const float expo = static_cast<float>(2 * m) / static_cast<float>(d);
      tab[m] = static_cast<float>(std::pow(static_cast<double>(theta), static_cast<double>(expo)));
    }
    cached_d = d;
    cached_theta = theta;
  }
  return tab;
}

// cos / sin of RoPE at position pos for every pair m < D/2: the FP32 angle
// pos / theta^(2m/D), each transcendental evaluated in double and rounded
// once (position 0: cos 1, sin 0).  Each host thread keeps the tables of its
// last few positions (a batch of prompts, or a benchmark, repeats them).
const float2* rope_cos_sin_row(int64_t pos, int64_t d, float theta) {
  struct Row {
    int64_t pos = -1, d = -1;
    float theta = 0.0f;
    float2 cs[kMaxHeadDim / 2];
  };
  constexpr int kRows = 8;
  thread_local Row rows[kRows];
  thread_local int next = 0;
  for (const Row& r : rows)
    if (r.pos == pos && r.d == d && r.theta == theta) return r.cs;
  Row& r = rows[next];
  next = (next + 1) % kRows;
  const float* den = rope_denominators(d, theta);
  for (int64_t m = 0; m < d / 2 && m < kMaxHeadDim / 2; ++m) {
    float c = 1.0f, sn = 0.0f;
    if (pos != 0) {
      const float angle = static_cast<float>(pos) / den[m];
      c = static_cast<float>(std::cos(static_cast<double>(angle)));
      sn = static_cast<float>(std::sin(static_cast<double>(angle)));
    }
    r.cs[m] = make_float2(c, sn);
  }
  r.pos = pos;
  r.d = d;
  r.theta = theta;
  return r.cs;
}

QkvParams qkv_params(const nvfp4da_forward_args* a, uint16_t* q_out) {
  QkvParams p{};
  p.x = a->x;
  p.g_in = a->input_norm_weight;
  const nvfp4da_weight* w3[3] = {&a->q_weight, &a->k_weight, &a->v_weight};
  for (int i = 0; i < 3; ++i) {
    p.packed[i] = w3[i]->packed_values;
    p.scales[i] = w3[i]->block_scales;
    p.gamma[i] = w3[i]->global_decode_scale;
  }
  p.g_q = a->q_norm_weight;
  p.g_k = a->k_norm_weight;
  p.q_out = q_out;
  p.k_cache = a->k_cache;
  p.v_cache = a->v_cache;
  p.m = a->batch * a->tokens;
  p.tokens = a->tokens;
  p.hidden = a->hidden;
  p.q_heads = a->hidden / a->head_dim;
  p.kv_heads = a->kv_heads;
  p.head_dim = a->head_dim;
  p.capacity = a->capacity;
  p.past_length = a->past_length;
  p.past_lengths = a->past_lengths;
  p.eps = a->rms_eps;
  p.theta = a->rope_theta;
  if (const nvfp4da_forward_stages* st = a->stages) {
    p.dbg_xnorm = st->input_normalized;
    p.dbg_q = st->q_projected;
    p.dbg_k = st->k_projected;
    p.dbg_v = st->v_projected;
    p.dbg_qn = st->q_normalized;
    p.dbg_kn = st->k_normalized;
  }
  p.pdl = 1;
  // RoPE cos/sin for positions past_length + t, t < min(T, kMaxRopeRows), on the
  // host with the arithmetic of reference/decoder_attention.py:237-257: FP32
  // exponent 2m/D, FP32 theta^exponent, FP32 angle = p / denominator, FP32
  // cos / sin -- each transcendental evaluated in double and rounded once.
  p.rope_rows = 0;
  if (a->head_dim <= kMaxHeadDim) {
    const float* den = rope_denominators(a->head_dim, a->rope_theta);
    for (int64_t m = 0; m < a->head_dim / 2; ++m) p.rope_denom[m] = den[m];
  }
  if (!a->past_lengths && a->tokens <= kMaxRopeRows && a->head_dim <= kMaxHeadDim) {
    const int64_t d = a->head_dim;
    for (int64_t t = 0; t < a->tokens; ++t) {
      const float2* cs = rope_cos_sin_row(a->past_length + t, d, a->rope_theta);
      for (int64_t m = 0; m < d / 2; ++m) p.rope_host[t][m] = cs[m];
    }
    p.rope_rows = static_cast<int>(a->tokens);
  }
  return p;
}


// ---------------------------------------------------------------- one-kernel decode step
// Synchronisation slots of the step kernel: zero-initialised at load, left
// zero by every completed launch.  One slot per (device, stream): launches on
// one stream are ordered, so they never share a slot concurrently.
constexpr int kStepSlots = 64;
__device__ unsigned g_step_sync[kStepSlots][kStepSyncWords];
// The step kernel's hand-off words (tagged, see decode_step.cuh), one region
// per slot: only launches of that slot's stream ever write it, so a word can
// carry the current tag only if this launch wrote it.
__device__ unsigned long long g_step_tagged[kStepSlots][kStepTagWords];
// Scratch words of the bounded-wait probe (nvfp4da_debug_wait_timeout).
__device__ unsigned g_probe_words[4];

std::mutex g_slot_mutex;
std::map<std::pair<int, uintptr_t>, int> g_slot_of;
int g_slots_used[kMaxDevices] = {0};
unsigned* g_slot_base[kMaxDevices] = {nullptr};
unsigned long long* g_tag_base[kMaxDevices] = {nullptr};

unsigned* slot_base_for_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  if (!g_slot_base[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_step_sync) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    void* tags = nullptr;
    if (cudaGetSymbolAddress(&tags, g_step_tagged) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    g_slot_base[dev] = static_cast<unsigned*>(ptr);
    g_tag_base[dev] = static_cast<unsigned long long*>(tags);
  }
  return g_slot_base[dev];
}

// The slot of `stream` on the current device (assigned on first use), or
// nullptr when every slot is taken; *tagged (if given) = the slot's hand-off
// region.  Slots are never released, so a (device, stream) -> slot answer
// stays valid for the life of the process: each host thread keeps its last
// answer and repeats it without the lock or the map lookup.  (A device reset
// after the first call is not supported: the addresses would be stale.)
struct SlotHit {
  int dev = -1;
  uintptr_t stream = 0;
  unsigned* slot = nullptr;
  unsigned long long* tagged = nullptr;
};
thread_local SlotHit tl_slot_hit;

unsigned* step_slot(cudaStream_t stream, unsigned long long** tagged = nullptr) {
  const int dev = current_device();
  const uintptr_t key_stream = reinterpret_cast<uintptr_t>(stream);
  SlotHit& hit = tl_slot_hit;
  if (hit.slot && hit.dev == dev && hit.stream == key_stream) {
    if (tagged) *tagged = hit.tagged;
    return hit.slot;
  }
  std::lock_guard<std::mutex> lock(g_slot_mutex);
  unsigned* base = slot_base_for_device(dev);
  if (!base) return nullptr;
  const auto key = std::make_pair(dev, key_stream);
  auto it = g_slot_of.find(key);
  int slot;
  if (it != g_slot_of.end()) {
    slot = it->second;
  } else {
    if (g_slots_used[dev] >= kStepSlots) return nullptr;
    slot = g_slots_used[dev]++;
    g_slot_of[key] = slot;
  }
  hit.dev = dev;
  hit.stream = key_stream;
  hit.slot = base + static_cast<size_t>(slot) * kStepSyncWords;
  hit.tagged = g_tag_base[dev] + static_cast<size_t>(slot) * kStepTagWords;
  if (tagged) *tagged = hit.tagged;
  return hit.slot;
}

// xi: the activation rows in the parameter block (instantiated for D = 128).
const void* step_kernel_ptr(int epl, int gh, bool xi = false) {
  if (xi) {
    if (epl != 4) return nullptr;
    switch (gh) {
      case 1: return reinterpret_cast<const void*>(decode_step_kernel<4, 1, true>);
      case 2: return reinterpret_cast<const void*>(decode_step_kernel<4, 2, true>);
      case 4: return reinterpret_cast<const void*>(decode_step_kernel<4, 4, true>);
      case 8: return reinterpret_cast<const void*>(decode_step_kernel<4, 8, true>);
      default: return nullptr;
    }
  }
#define NVFP4DA_STEP_CASE(E, G) \
  if (epl == E && gh == G) return reinterpret_cast<const void*>(decode_step_kernel<E, G, false>);
  NVFP4DA_STEP_CASE(2, 1)
  NVFP4DA_STEP_CASE(2, 2)
  NVFP4DA_STEP_CASE(2, 4)
  NVFP4DA_STEP_CASE(2, 8)
  NVFP4DA_STEP_CASE(4, 1)
  NVFP4DA_STEP_CASE(4, 2)
  NVFP4DA_STEP_CASE(4, 4)
  NVFP4DA_STEP_CASE(4, 8)
  NVFP4DA_STEP_CASE(8, 1)
  NVFP4DA_STEP_CASE(8, 2)
  NVFP4DA_STEP_CASE(8, 4)
  NVFP4DA_STEP_CASE(8, 8)
#undef NVFP4DA_STEP_CASE
  return nullptr;
}

struct StepPlan {
  int epl, gh;
  int rq, n_qkv;
  int o_rows_big, o_n_big, o_rows_small, o_tile_rows;
  int splits, split_len, grid;
  uint32_t smem;
  uint32_t off_qs, off_qw, off_kv, off_q, off_os, off_ow, off_xs, off_x16, off_red;
  int o_predecode, od_ld;
  uint32_t off_od;
  size_t proj, ctx, part_o, part_ml, xin, total;
  static constexpr size_t kNoWords = ~size_t(0);  // workspace offsets / bytes
};

// Static shared memory of a step-kernel instantiation (cached per device).
std::map<std::pair<const void*, int>, size_t> g_static_smem;

size_t static_smem(const void* fn) {
  const int dev = current_device();
  thread_local const void* last_fn = nullptr;
  thread_local int last_dev = -1;
  thread_local size_t last_v = 0;
  if (fn == last_fn && dev == last_dev) return last_v;
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  auto it = g_static_smem.find({fn, dev});
  if (it != g_static_smem.end()) return it->second;
  cudaFuncAttributes fa{};
  size_t v = 16 * 1024;  // conservative if the query fails
  if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess) {
    v = fa.sharedSizeBytes;
    last_fn = fn;
    last_dev = dev;
    last_v = v;
  } else {
    cudaGetLastError();
  }
  g_static_smem[{fn, dev}] = v;
  return v;
}

// The step kernel covers decode (T == 1) of up to 8 sequences with
// hidden % 256 == 0, hidden <= 4096, head_dim in {64, 128, 256}, 1/2/4/8 query
// heads per KV head, no stage outputs, and a K/V tile per split that fits in
// shared memory.  Returns false (no error) otherwise.
bool plan_step(const nvfp4da_forward_args* a, StepPlan& s) {
  if (a->tokens != 1 || a->batch > kMmaMaxM || a->stages) return false;
  const int64_t k = a->hidden, d = a->head_dim, hkv = a->kv_heads, hq = k / d, nb = a->batch;
  if (k % 256 != 0 || k / 8 > 2 * kStepThreads) return false;
  if (d % 32 != 0 || d > kMaxHeadDim) return false;
  const int epl = static_cast<int>(d / 32);
  const int64_t group = hq / hkv;
  if (group != 1 && group != 2 && group != 4 && group != 8) return false;
  const void* fn = step_kernel_ptr(epl, static_cast<int>(group));
  if (!fn) return false;
  const std::pair<const nvfp4da_weight*, int> ws[4] = {{&a->q_weight, 0}, {&a->k_weight, 1}, {&a->v_weight, 2},
                                                       {&a->out_weight, 3}};
  for (auto& w : ws)
    if (!aligned(w.first->packed_values, 16) || !aligned(w.first->block_scales, 16)) return false;
  if (!aligned(a->x, 16) || !aligned(a->input_norm_weight, 16) || !aligned(a->k_cache, 16) ||
      !aligned(a->v_cache, 16) || !aligned(a->output, 16))
    return false;
  const int grid = sm_count();
  const int64_t nqkv = (hq + 2 * hkv) * d;
  int rq = 0;
  for (int r : {16, 32, 64, 128}) {
    if (d % r == 0 && ceil_div(nqkv, r) <= grid) {
      rq = r;
      break;
    }
  }
  if (!rq) return false;
  // O rows in units of 8, spread over every CTA: o_n_big CTAs take one unit more.
  const int64_t units8 = k / 8;
  const int64_t per = units8 / grid, n_big = units8 - per * grid;
  const int rows_big = static_cast<int>(8 * (per + (n_big > 0 ? 1 : 0)));
  int tiles = 1;
  while (16 * tiles < rows_big) tiles <<= 1;
  if (16 * tiles > kStepMaxRows) return false;
  const int64_t bh = nb * hkv;
  if (bh > grid) return false;
  const int64_t visible = (a->past_lengths ? a->max_past_length : a->past_length) + 1;
  // The hand-off words must fit the slot's region: projections and context
  // (BF16 pairs) and every split's partials (FP32 singles).
  const int64_t fixed_words = nb * nqkv / 2 + nb * k / 2 + 64;
  const int64_t per_split_words = bh * group * (d + 2);
  if (fixed_words + per_split_words > static_cast<int64_t>(kStepTagWords)) return false;
  const int64_t max_splits = (static_cast<int64_t>(kStepTagWords) - fixed_words) / per_split_words;
  int64_t splits = std::max<int64_t>(
      1, std::min<int64_t>(std::min<int64_t>(grid / bh, max_splits), ceil_div(visible, 64)));
  const int64_t split_len = ceil_div(ceil_div(visible, splits), 8) * 8;
  splits = ceil_div(visible, split_len);
  s.epl = epl;
  s.gh = static_cast<int>(group);
  s.rq = rq;
  s.n_qkv = static_cast<int>(nqkv / rq);
  s.o_rows_big = rows_big;
  s.o_n_big = static_cast<int>(n_big > 0 ? n_big : grid);
  s.o_rows_small = static_cast<int>(8 * per);
  s.o_tile_rows = 16 * tiles;
  s.splits = static_cast<int>(splits);
  s.split_len = static_cast<int>(split_len);
  s.grid = grid;
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t o = off;
    off += (bytes + 127) / 128 * 128;
    return static_cast<uint32_t>(o);
  };
  const uint64_t ks = k / 16, kb = k / 2;
  // Overlay region: QKV rows, K/V tile (later the warps' o vectors, then the
  // split weights of the combine) and q.
  const uint64_t tile = 2ull * split_len * d * 2, smo = 1ull * kStepWarps * group * d * 4,
                 comb_w = 2ull * group * splits * 4;
  const uint64_t items = nb * hq;
  s.off_os = take(rows_big * ks);
  s.off_ow = take(rows_big * kb);
  s.off_xs = take(nb * k * 2);
  s.off_x16 = take(nb * k * 2);
  s.off_red = take(kMmaWarps * 128 * 4);
  // Early-phase buffers: QKV rows, the K/V tile (later the warps' o vectors,
  // then the split weights of the combine) and q.  The O rows decoded ahead
  // overlay them once they are consumed.
  s.off_qs = take(rq * ks);
  s.off_qw = take(rq * kb);
  s.off_kv = take(std::max(tile, std::max(smo, comb_w)));
  s.off_q = take(group * d * 4);
  const uint64_t early = off - s.off_qs;
  s.od_ld = static_cast<int>(k + 8);  // f16 row stride: 16 bytes of padding keep ldmatrix conflict-free
  const uint64_t od_bytes = static_cast<uint64_t>(rows_big) * s.od_ld * 2;
  s.off_od = s.off_qs;
  s.o_predecode = 0;
  if (od_bytes <= early) {
    s.o_predecode = 1;
  } else if (off + (od_bytes - early) + static_smem(fn) <= kMaxDynSmem) {
    take(od_bytes - early);
    s.o_predecode = 1;
  }
  if (off + static_smem(fn) > kMaxDynSmem) return false;
  // The MMA tiles read up to o_tile_rows rows; the rows past the CTA's own
  // land in the buffers that follow (in bounds, their outputs discarded).
  if (s.off_ow + static_cast<uint64_t>(s.o_tile_rows) * kb > off) return false;
  s.smem = static_cast<uint32_t>(off);
  // Word offsets in the slot's hand-off region: BF16 pairs for the
  // projections and the context, single FP32 values for the partials.
  size_t w = 0;
  s.proj = w;
  w += static_cast<size_t>(nb * nqkv / 2);
  s.ctx = w;
  w += static_cast<size_t>(nb * k / 2);
  s.part_o = w;
  w += static_cast<size_t>(items) * splits * d;
  s.part_ml = w;
  w += static_cast<size_t>(items) * splits * 2;
  if (w > kStepTagWords) return false;
  // Activation rows read from host memory (host-buffer entry point), where
  // the region has room for them after the partials.
  s.xin = w + static_cast<size_t>(nb * k / 2) <= kStepTagWords ? w : StepPlan::kNoWords;
  s.total = 256;  // the step keeps nothing in the caller's workspace
  return true;
}

bool step_covers(const nvfp4da_forward_args* a) {
  StepPlan sp;
  return plan_step(a, sp);
}

// Whether the step can carry the activation rows of `a` in its parameter block.
bool step_inline_ok(const nvfp4da_forward_args* a, const StepPlan& pl) {
  return a->batch * a->tokens * a->hidden <= kStepInlineX && step_kernel_ptr(pl.epl, pl.gh, true) != nullptr;
}

// x_inline: host copy of the activation rows to send in the parameter block
// (step_inline_ok must hold), or nullptr to read a->x.
// x_mapped: the device address of activation rows in mapped page-locked host
// memory, read by the kernel itself, or nullptr.
int run_step(const nvfp4da_forward_args* a, const StepPlan& pl, void* ws, cudaStream_t stream, unsigned* slot,
             unsigned long long* tagged, const uint16_t* x_inline = nullptr, const uint16_t* x_mapped = nullptr) {
  thread_local StepLaunch<true> inl;  // the parameter block with room for inline rows
  StepParams& p = inl.p;
  p = StepParams{};
  p.x = a->x;
  p.g_in = a->input_norm_weight;
  const nvfp4da_weight* w4[4] = {&a->q_weight, &a->k_weight, &a->v_weight, &a->out_weight};
  for (int i = 0; i < 4; ++i) {
    p.packed[i] = w4[i]->packed_values;
    p.scales[i] = w4[i]->block_scales;
    p.gamma[i] = w4[i]->global_decode_scale;
  }
  p.g_q = a->q_norm_weight;
  p.g_k = a->k_norm_weight;
  p.k_cache = a->k_cache;
  p.v_cache = a->v_cache;
  p.out = a->output;
  p.batch = a->batch;
  p.hidden = a->hidden;
  p.q_heads = a->hidden / a->head_dim;
  p.kv_heads = a->kv_heads;
  p.head_dim = a->head_dim;
  p.capacity = a->capacity;
  p.past_length = a->past_length;
  p.past_lengths = a->past_lengths;
  p.eps = a->rms_eps;
  p.theta = a->rope_theta;
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(a->head_dim)));
  p.rq = pl.rq;
  p.n_qkv_blocks = pl.n_qkv;
  p.o_rows_big = pl.o_rows_big;
  p.o_n_big = pl.o_n_big;
  p.o_rows_small = pl.o_rows_small;
  p.o_tile_rows = pl.o_tile_rows;
  p.splits = pl.splits;
  p.split_len = pl.split_len;
  (void)ws;
  p.proj = tagged + pl.proj;
  p.ctx = tagged + pl.ctx;
  p.part_o = tagged + pl.part_o;
  p.part_ml = tagged + pl.part_ml;
  p.xin = x_mapped ? tagged + pl.xin : nullptr;
  p.x_mapped = x_mapped;
  p.tag_words = kStepTagWords;
  p.sync = slot;
  p.timeout_ns = 500ull * 1000 * 1000;
  p.off_qs = pl.off_qs;
  p.off_qw = pl.off_qw;
  p.off_kv = pl.off_kv;
  p.off_q = pl.off_q;
  p.off_os = pl.off_os;
  p.off_ow = pl.off_ow;
  p.off_xs = pl.off_xs;
  p.off_x16 = pl.off_x16;
  p.off_red = pl.off_red;
  p.o_predecode = pl.o_predecode;
  p.off_od = pl.off_od;
  p.od_ld = pl.od_ld;
  // RoPE cos/sin at position past_length, the host arithmetic of qkv_params.
  p.rope_host_ok = 2;
  if (!a->past_lengths) {
    const float2* cs = rope_cos_sin_row(a->past_length, a->head_dim, a->rope_theta);
    for (int64_t m = 0; m < a->head_dim / 2; ++m) p.rope_host[m] = cs[m];
    p.rope_host_ok = 1;
  } else {
    const float* den = rope_denominators(a->head_dim, a->rope_theta);
    for (int64_t m = 0; m < a->head_dim / 2; ++m) p.rope_host[m] = make_float2(den[m], 0.0f);
  }
  const void* fn = step_kernel_ptr(pl.epl, pl.gh, x_inline != nullptr);
  if (x_inline) std::memcpy(inl.x, x_inline, static_cast<size_t>(a->batch * a->tokens * a->hidden) * 2);
  cudaError_t e = ensure_smem(fn, pl.smem);
  if (e != cudaSuccess) return cuda_fail(e, "step kernel shared-memory opt-in");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: the counters are waited on
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // StepLaunch<false> is StepParams alone, so &p serves both instantiations.
  void* kargs[] = {x_inline ? static_cast<void*>(&inl) : static_cast<void*>(&p)};
  e = cudaLaunchKernelExC(&cfg, fn, kargs);
  if (e != cudaSuccess) return cuda_fail(e, "decode step launch");
  return NVFP4DA_OK;
}

// Bounded-wait probe: one CTA waits on a counter that nothing sets.
__global__ void wait_probe_kernel(unsigned* words, unsigned long long timeout_ns) {
  const int idx = 0;
  cta_wait(words, &idx, 1, 1u, words + 1, timeout_ns);
}
}  // namespace
}  // namespace nvfp4da

using namespace nvfp4da;

// Lets other translation units of this library report through
// nvfp4da_last_error(); not exported.
__attribute__((visibility("hidden"))) void nvfp4da_set_last_error(const char* msg) { g_last_error = msg; }

extern "C" {

const char* nvfp4da_last_error(void) { return g_last_error.c_str(); }

int nvfp4da_abi_version(void) { return 1; }

int nvfp4da_unpack_e2m1_codes(const uint8_t* packed, uint8_t* codes, int64_t rows, int64_t packed_cols,
                              void* stream) {
  if (!packed || !codes || rows <= 0 || packed_cols <= 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "unpack: invalid arguments");
  const int64_t n = rows * packed_cols;
  unpack_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, codes, n);
  NVFP4DA_CHECK_LAUNCH("unpack launch");
  return NVFP4DA_OK;
}

int nvfp4da_dequantize_nvfp4(const nvfp4da_weight* w, float* out, void* stream) {
  int r = check_weight(w, "weight");
  if (r) return r;
  if (!out) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "out is NULL");
  const int64_t nb = w->rows * (w->cols / 2);
  dequant_kernel<<<static_cast<unsigned>(ceil_div(nb, 256)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w->packed_values, w->block_scales, w->global_decode_scale, out, nb, w->cols / 2);
  NVFP4DA_CHECK_LAUNCH("dequantize launch");
  return NVFP4DA_OK;
}

size_t nvfp4da_quantize_workspace_size(int64_t, int64_t) { return 256; }

int nvfp4da_quantize_nvfp4(const void* src, int is_bf16, int64_t rows, int64_t cols, uint8_t* packed,
                           uint8_t* scales, float* gamma, void* ws, size_t ws_bytes, void* stream) {
  if (!src || !packed || !scales || !gamma || rows <= 0 || cols < 16 || cols % 16 != 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "quantize: invalid arguments (K must be a positive multiple of 16)");
  if (!ws || ws_bytes < 4) return fail(NVFP4DA_ERR_WORKSPACE, "quantize workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* amax = static_cast<unsigned*>(ws);
  cudaError_t e = cudaMemsetAsync(amax, 0, 4, s);
  if (e != cudaSuccess) return cuda_fail(e, "quantize clear");
  const int64_t n = rows * cols;
  const int64_t grid = std::min<int64_t>(ceil_div(n, 256), 4LL * sm_count());
  quant_amax_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(src, is_bf16, n, amax);
  NVFP4DA_CHECK_LAUNCH("quantize amax launch");
  const int64_t nblk = rows * (cols / 16);
  quant_blocks_kernel<<<static_cast<unsigned>(ceil_div(nblk, 128)), 128, 0, s>>>(src, is_bf16, rows, cols, amax,
                                                                                 packed, scales, gamma);
  NVFP4DA_CHECK_LAUNCH("quantize blocks launch");
  return NVFP4DA_OK;
}

int nvfp4da_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* out, int64_t rows, int64_t cols, float eps,
                     void* stream) {
  if (!x || !w || !out || rows <= 0 || cols <= 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "rms_norm: invalid arguments");
  if (!(eps > 0.0f) || !std::isfinite(eps)) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "eps must be finite and positive");
  if (rows > std::numeric_limits<int32_t>::max())
    return fail(NVFP4DA_ERR_UNSUPPORTED, "x has too many logical rows for a one-dimensional CUDA grid");
  rms_norm_kernel<<<static_cast<unsigned>(rows), kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, w, out,
                                                                                                     cols, eps);
  NVFP4DA_CHECK_LAUNCH("rms_norm launch");
  return NVFP4DA_OK;
}

int nvfp4da_apply_rope(const uint16_t* x, uint16_t* out, int64_t batch, int64_t tokens, int64_t heads,
                       int64_t head_dim, int64_t past_length, float theta, void* stream) {
  if (!x || !out || batch <= 0 || tokens <= 0 || heads <= 0 || head_dim < 2 || head_dim % 2)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "apply_rope: invalid arguments");
  if (past_length < 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length must be nonnegative");
  if (!(theta > 0.0f) || !std::isfinite(theta))
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "rope_theta must be finite and positive");
  const int64_t pairs = batch * tokens * heads * head_dim / 2;
  rope_kernel<<<static_cast<unsigned>(ceil_div(pairs, 256)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, out, pairs, tokens, heads, head_dim, past_length, theta);
  NVFP4DA_CHECK_LAUNCH("rope launch");
  return NVFP4DA_OK;
}

int nvfp4da_w4a16_linear(const uint16_t* x, int64_t m, const nvfp4da_weight* w, uint16_t* y, void* stream) {
  int r = check_weight(w, "weight");
  if (r) return r;
  if (!x || !y || m <= 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "w4a16_linear: invalid arguments");
  return run_gemv(x, m, *w, y, static_cast<cudaStream_t>(stream), false);
}

int nvfp4da_w4a16_gemm(const uint16_t* x, int64_t m, const nvfp4da_weight* w, uint16_t* y, void* stream) {
  int r = check_weight(w, "weight");
  if (r) return r;
  if (!x || !y || m <= 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "w4a16_gemm: invalid arguments");
  if (!gemm_tc_supported(x, m, *w, y))
    return fail(NVFP4DA_ERR_UNSUPPORTED, "the tensor-core GEMM needs K %% 256 == 0 and 16-byte aligned operands");
  return run_gemm_tc(x, m, *w, y, static_cast<cudaStream_t>(stream));
}

int nvfp4da_kv_cache_append(uint16_t* kc, uint16_t* vc, const uint16_t* nk, const uint16_t* nv, int64_t batch,
                            int64_t kv_heads, int64_t capacity, int64_t head_dim, int64_t tokens,
                            int64_t past_length, const int64_t* past_lengths, void* stream) {
  if (!kc || !vc || !nk || !nv || batch <= 0 || kv_heads <= 0 || capacity <= 0 || head_dim <= 0 || tokens <= 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "kv_cache_append: invalid arguments");
  if (!past_lengths) {
    if (past_length < 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length must be nonnegative");
    if (past_length > std::numeric_limits<int64_t>::max() - tokens)
      return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length + current token count overflows int64");
    if (past_length + tokens > capacity)
      return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "past_length + current token count exceeds cache capacity");
  }
  const int64_t total = batch * tokens * kv_heads * head_dim;
  kv_append_kernel<<<static_cast<unsigned>(ceil_div(total, 256)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      kc, vc, nk, nv, total, tokens, kv_heads, head_dim, capacity, past_length, past_lengths);
  NVFP4DA_CHECK_LAUNCH("kv append launch");
  return NVFP4DA_OK;
}

size_t nvfp4da_gqa_attention_workspace_size(int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads,
                                            int64_t head_dim, int64_t max_past) {
  AttnPlan pl;
  if (batch <= 0 || tokens <= 0 || kv_heads <= 0 || q_heads % kv_heads ||
      !plan_attention(batch, tokens, q_heads, kv_heads, head_dim, max_past, pl))
    return 0;
  return pl.partial_bytes + pl.counter_bytes;
}

int nvfp4da_gqa_attention_cached(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* ctx,
                                 int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t capacity,
                                 int64_t head_dim, int64_t past_length, const int64_t* past_lengths,
                                 int64_t max_past, void* ws, size_t ws_bytes, void* stream) {
  if (!q || !kc || !vc || !ctx) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "attention: NULL pointer");
  if (!past_lengths) max_past = past_length;
  int r = check_attention_dims(batch, tokens, q_heads, kv_heads, capacity, head_dim, max_past);
  if (r) return r;
  if (!aligned(q, 16) || !aligned(kc, 16) || !aligned(vc, 16) || !aligned(ctx, 16))
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "attention tensors must be 16-byte aligned");
  return run_attention(q, kc, vc, ctx, batch, tokens, q_heads, kv_heads, capacity, head_dim, past_length,
                       past_lengths, max_past, ws, ws_bytes, static_cast<cudaStream_t>(stream), false, true);
}

size_t nvfp4da_forward_workspace_size(const nvfp4da_forward_args* a) {
  if (check_forward(a)) return 0;
  ForwardLayout L;
  if (plan_forward(a, L)) return 0;
  StepPlan sp;
  return plan_step(a, sp) ? std::max(L.total, sp.total) : L.total;
}

int nvfp4da_forward_step_supported(const nvfp4da_forward_args* a) {
  if (check_forward(a)) return 0;
  StepPlan sp;
  return plan_step(a, sp) ? 1 : 0;
}

int nvfp4da_decoder_attention_forward(const nvfp4da_forward_args* a, void* ws, size_t ws_bytes, void* stream) {
  return nvfp4da_decoder_attention_forward_path(a, ws, ws_bytes, stream, NVFP4DA_PATH_AUTO);
}

}  // extern "C"

namespace nvfp4da {
namespace {
// The device address of page-locked host memory that the device can address
// (16-byte aligned), else nullptr.  Asked on every call (well under a
// microsecond): a cached answer could outlive the buffer's registration.
void* mapped_address(const void* host) {
  cudaPointerAttributes at{};
  void* dev = nullptr;
  if (cudaPointerGetAttributes(&at, host) == cudaSuccess && at.type == cudaMemoryTypeHost && at.devicePointer &&
      aligned(at.devicePointer, 16))
    dev = at.devicePointer;
  cudaGetLastError();
  return dev;
}

// The forward.  x_host (the host-buffer entry point): the activation rows in
// host memory, and x_host_dev their device address when they are mapped
// page-locked memory (else nullptr).  On the one-kernel step the rows travel
// in the launch's parameter block when they fit (6 KB), else the kernel reads
// them from mapped memory; every other case copies them into a->x on the
// stream first (a copy-engine transfer, ~10 us of stream time on B200).
int forward_impl(const nvfp4da_forward_args* a, void* ws, size_t ws_bytes, void* stream, int path,
                 const uint16_t* x_host, const uint16_t* x_host_dev) {
  int r = check_forward(a);
  if (r) return r;
  if (path != NVFP4DA_PATH_AUTO && path != NVFP4DA_PATH_CHAIN && path != NVFP4DA_PATH_STEP)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "unknown forward path %d", path);
  ForwardLayout L;
  if ((r = plan_forward(a, L))) return r;
  // AUTO takes the one-kernel step where it applies: on B200 it is faster
  // than the three-kernel chain on the canonical decode step and needs one
  // launch instead of three.  It needs a synchronisation slot for the
  // stream; when every slot is taken AUTO takes the chain instead.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  StepPlan sp;
  bool step_ok = (path == NVFP4DA_PATH_STEP || path == NVFP4DA_PATH_AUTO) && plan_step(a, sp);
  if (path == NVFP4DA_PATH_STEP && !step_ok)
    return fail(NVFP4DA_ERR_UNSUPPORTED, "the one-kernel decode step does not cover this configuration");
  unsigned* slot = nullptr;
  unsigned long long* tagged = nullptr;
  if (step_ok && !(slot = step_slot(s, &tagged))) {
    if (path == NVFP4DA_PATH_STEP)
      return fail(NVFP4DA_ERR_UNSUPPORTED, "no free synchronisation slot for another stream (%d streams per device)",
                  kStepSlots);
    step_ok = false;
  }
  const size_t need = step_ok ? std::max(L.total, sp.total) : L.total;
  if (!ws || ws_bytes < need)
    return fail(NVFP4DA_ERR_WORKSPACE, "forward workspace too small (%zu < %zu bytes)", ws_bytes, need);
  if (!aligned(ws, 256)) return fail(NVFP4DA_ERR_WORKSPACE, "forward workspace must be 256-byte aligned");
  const bool inline_x = x_host && step_ok && step_inline_ok(a, sp);
  const bool mapped_x = !inline_x && x_host_dev && step_ok && sp.xin != StepPlan::kNoWords;
  if (x_host && !inline_x && !mapped_x) {
    const size_t bytes = static_cast<size_t>(a->batch * a->tokens * a->hidden) * 2;
    cudaError_t e = cudaMemcpyAsync(const_cast<uint16_t*>(a->x), x_host, bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "forward_hostio: input copy");
  }
  if (step_ok)
    return run_step(a, sp, ws, s, slot, tagged, inline_x ? x_host : nullptr, mapped_x ? x_host_dev : nullptr);
  char* base = static_cast<char*>(ws);
  const nvfp4da_forward_stages* st = a->stages;
  const int64_t hq = a->hidden / a->head_dim, m = a->batch * a->tokens, d = a->head_dim;
  const int64_t maxp = a->past_lengths ? a->max_past_length : a->past_length;
  uint16_t* q_buf = (st && st->q_rope) ? st->q_rope : reinterpret_cast<uint16_t*>(base + L.q_buf);
  uint16_t* ctx_buf = (st && st->context) ? st->context : reinterpret_cast<uint16_t*>(base + L.ctx_buf);
  void* attn_ws = base + L.attn_ws;

  if (L.fused) {
    QkvParams p = qkv_params(a, q_buf);
    p.zero_words = L.attn.counter_bytes ? reinterpret_cast<unsigned*>(static_cast<char*>(attn_ws) + L.attn.partial_bytes)
                                        : nullptr;
    p.n_zero_words = static_cast<int64_t>(L.attn.counter_bytes / 4);
    cudaError_t e;
    if (L.batched) {
      p.xn = reinterpret_cast<uint16_t*>(base + L.bxn);
      p.rope_tab = reinterpret_cast<float2*>(base + L.brope);
      e = launch_qkv_batched(p, hq + 2 * a->kv_heads, s);
    } else {
      e = launch_qkv(p, L.qkv, hq + 2 * a->kv_heads, s, true);
    }
    if (e != cudaSuccess) return cuda_fail(e, "fused qkv launch");
    r = run_attention(q_buf, a->k_cache, a->v_cache, ctx_buf, a->batch, a->tokens, hq, a->kv_heads, a->capacity, d,
                      a->past_length, a->past_lengths, maxp, attn_ws, L.attn.partial_bytes + L.attn.counter_bytes, s,
                      true, false);
    if (r) return r;
  } else {
    // General shapes: the reference's modular chain on the standalone kernels.
    auto buf = [&](uint16_t* user, size_t off) { return user ? user : reinterpret_cast<uint16_t*>(base + off); };
    uint16_t* xn = buf(st ? st->input_normalized : nullptr, L.xn);
    uint16_t* qp = buf(st ? st->q_projected : nullptr, L.qp);
    uint16_t* kp = buf(st ? st->k_projected : nullptr, L.kp);
    uint16_t* vp = buf(st ? st->v_projected : nullptr, L.vp);
    uint16_t* qn = buf(st ? st->q_normalized : nullptr, L.qn);
    uint16_t* kn = buf(st ? st->k_normalized : nullptr, L.kn);
    uint16_t* kr = reinterpret_cast<uint16_t*>(base + L.kr);
    if ((r = nvfp4da_rms_norm(a->x, a->input_norm_weight, xn, m, a->hidden, a->rms_eps, s))) return r;
    if ((r = run_gemv(xn, m, a->q_weight, qp, s, false))) return r;
    if ((r = run_gemv(xn, m, a->k_weight, kp, s, false))) return r;
    if ((r = run_gemv(xn, m, a->v_weight, vp, s, false))) return r;
    if ((r = nvfp4da_rms_norm(qp, a->q_norm_weight, qn, m * hq, d, a->rms_eps, s))) return r;
    if ((r = nvfp4da_rms_norm(kp, a->k_norm_weight, kn, m * a->kv_heads, d, a->rms_eps, s))) return r;
    auto rope = [&](const uint16_t* in, uint16_t* out, int64_t heads) {
      const int64_t pairs = a->batch * a->tokens * heads * d / 2;
      rope_kernel<<<static_cast<unsigned>(ceil_div(pairs, 256)), 256, 0, s>>>(
          in, out, pairs, a->tokens, heads, d, a->past_length, a->rope_theta, a->past_lengths);
      NVFP4DA_CHECK_LAUNCH("rope launch");
      return NVFP4DA_OK;
    };
    if ((r = rope(qn, q_buf, hq))) return r;
    if ((r = rope(kn, kr, a->kv_heads))) return r;
    if ((r = nvfp4da_kv_cache_append(a->k_cache, a->v_cache, kr, vp, a->batch, a->kv_heads, a->capacity, d,
                                     a->tokens, a->past_length, a->past_lengths, s)))
      return r;
    r = run_attention(q_buf, a->k_cache, a->v_cache, ctx_buf, a->batch, a->tokens, hq, a->kv_heads, a->capacity, d,
                      a->past_length, a->past_lengths, maxp, attn_ws, L.attn.partial_bytes + L.attn.counter_bytes, s,
                      false, true);
    if (r) return r;
  }
  if ((r = run_gemv(ctx_buf, m, a->out_weight, a->output, s, L.fused))) return r;
  return NVFP4DA_OK;
}
}  // namespace
}  // namespace nvfp4da

extern "C" {

int nvfp4da_decoder_attention_forward_path(const nvfp4da_forward_args* a, void* ws, size_t ws_bytes, void* stream,
                                           int path) {
  return forward_impl(a, ws, ws_bytes, stream, path, nullptr, nullptr);
}

int nvfp4da_forward_sync_status(void* stream, unsigned* flags, int clear) {
  if (!flags) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "flags is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* slot = step_slot(s);
  if (!slot) return fail(NVFP4DA_ERR_UNSUPPORTED, "no synchronisation slot for this stream");
  cudaError_t e = cudaMemcpyAsync(flags, slot + kSyncErr, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(slot + kSyncErr, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? NVFP4DA_OK : cuda_fail(e, "sync status read");
}

int nvfp4da_debug_wait_timeout(void* stream, unsigned long long timeout_ns, unsigned* flags) {
  if (!flags) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "flags is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* words = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&words, g_probe_words);
  if (e == cudaSuccess) e = cudaMemsetAsync(words, 0, sizeof(g_probe_words), s);
  if (e != cudaSuccess) return cuda_fail(e, "probe setup");
  wait_probe_kernel<<<1, 32, 0, s>>>(static_cast<unsigned*>(words), timeout_ns);
  NVFP4DA_CHECK_LAUNCH("probe launch");
  e = cudaMemcpyAsync(flags, static_cast<unsigned*>(words) + 1, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? NVFP4DA_OK : cuda_fail(e, "probe read");
}

// ---------------------------------------------------------------- KV-length sharding
// A shard holds global positions [shard_start, shard_start + capacity) of every
// sequence; plan its attention over the keys it can see.
static int64_t shard_visible_max(int64_t max_past, int64_t tokens, int64_t shard_start, int64_t capacity) {
  int64_t v = max_past + tokens - shard_start;
  if (v > capacity) v = capacity;
  return v < 1 ? 1 : v;
}

size_t nvfp4da_qkv_rope_append_shard_workspace_size(const nvfp4da_forward_args* a) {
  if (!a || a->batch <= 0 || a->tokens <= 0 || a->hidden <= 0 || a->head_dim <= 0) return 0;
  return bat_front_ok(a) ? bat_front_bytes(a) : 0;
}

int nvfp4da_qkv_rope_append_shard(const nvfp4da_forward_args* a, int64_t shard_start, int64_t global_capacity,
                                  uint16_t* q_rope_out, void* ws, size_t ws_bytes, void* stream) {
  if (!a) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "args is NULL");
  if (shard_start < 0 || a->capacity <= 0 || global_capacity <= 0 ||
      shard_start > global_capacity - a->capacity)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "shard [%lld, %lld) is not inside the cache capacity %lld",
                static_cast<long long>(shard_start), static_cast<long long>(shard_start + a->capacity),
                static_cast<long long>(global_capacity));
  nvfp4da_forward_args g = *a;  // validate against the whole (global) cache
  g.capacity = global_capacity;
  int r = check_forward(&g);
  if (r) return r;
  if (!q_rope_out) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "q_rope_out is NULL");
  QkvPlan pl;
  if (!plan_qkv(a->batch * a->tokens, a->hidden, a->head_dim, pl))
    return fail(NVFP4DA_ERR_UNSUPPORTED, "the fused QKV kernel needs head_dim %% 32 == 0, head_dim <= 256 and hidden %% 128 == 0");
  QkvParams p = qkv_params(a, q_rope_out);
  p.slot_offset = shard_start;
  const int64_t hq = a->hidden / a->head_dim;
  cudaError_t e;
  if (ws && bat_front_ok(a)) {
    if (ws_bytes < bat_front_bytes(a) || !aligned(ws, 256))
      return fail(NVFP4DA_ERR_WORKSPACE, "shard front-half workspace too small (%zu < %zu bytes) or not 256-byte aligned",
                  ws_bytes, bat_front_bytes(a));
    p.xn = static_cast<uint16_t*>(ws);
    p.rope_tab = reinterpret_cast<float2*>(static_cast<char*>(ws) + bat_rows_bytes(a));
    e = launch_qkv_batched(p, hq + 2 * a->kv_heads, static_cast<cudaStream_t>(stream));
  } else {
    e = launch_qkv(p, pl, hq + 2 * a->kv_heads, static_cast<cudaStream_t>(stream), true);
  }
  if (e != cudaSuccess) return cuda_fail(e, "fused qkv launch");
  return NVFP4DA_OK;
}

size_t nvfp4da_gqa_attention_partials_workspace_size(int64_t batch, int64_t tokens, int64_t q_heads,
                                                     int64_t kv_heads, int64_t head_dim, int64_t shard_start,
                                                     int64_t shard_capacity, int64_t max_past_length) {
  AttnPlan pl;
  if (batch <= 0 || tokens <= 0 || kv_heads <= 0 || q_heads % kv_heads || shard_capacity <= 0 ||
      !plan_attention(batch, tokens, q_heads, kv_heads, head_dim,
                      shard_visible_max(max_past_length, tokens, shard_start, shard_capacity) - tokens, pl))
    return 0;
  return std::max<size_t>(256, pl.partial_bytes + pl.counter_bytes);
}

int nvfp4da_gqa_attention_partials(const uint16_t* q, const uint16_t* k_shard, const uint16_t* v_shard,
                                   float* partials, int64_t batch, int64_t tokens, int64_t q_heads, int64_t kv_heads,
                                   int64_t shard_capacity, int64_t head_dim, int64_t shard_start,
                                   int64_t past_length, const int64_t* past_lengths, int64_t max_past_length,
                                   void* ws, size_t ws_bytes, void* stream) {
  if (!q || !k_shard || !v_shard || !partials) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "attention partials: NULL pointer");
  if (!past_lengths) max_past_length = past_length;
  if (shard_start < 0) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "shard_start must be nonnegative");
  // Dimensions as for one cache of capacity shard_start + shard_capacity.
  int r = check_attention_dims(batch, tokens, q_heads, kv_heads,
                               std::max<int64_t>(shard_start + shard_capacity, max_past_length + tokens), head_dim,
                               max_past_length);
  if (r) return r;
  if (!aligned(q, 16) || !aligned(k_shard, 16) || !aligned(v_shard, 16) || !aligned(partials, 16))
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "attention tensors must be 16-byte aligned");
  const int64_t vis = shard_visible_max(max_past_length, tokens, shard_start, shard_capacity);
  return run_attention(q, k_shard, v_shard, nullptr, batch, tokens, q_heads, kv_heads, shard_capacity, head_dim,
                       past_length, past_lengths, vis - tokens, ws, ws_bytes, static_cast<cudaStream_t>(stream),
                       false, true, shard_start, partials);
}

int nvfp4da_attention_combine(const float* partials, int shards, int64_t rows, int64_t head_dim, uint16_t* ctx,
                              void* stream) {
  if (!partials || !ctx || shards <= 0 || rows <= 0 || head_dim <= 0)
    return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "attention combine: invalid arguments");
  if (ceil_div(rows, 8) > std::numeric_limits<int32_t>::max())
    return fail(NVFP4DA_ERR_UNSUPPORTED, "too many rows for a one-dimensional grid");
  attn_combine_kernel<<<static_cast<unsigned>(ceil_div(rows, 8)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      partials, shards, rows, head_dim, ctx);
  NVFP4DA_CHECK_LAUNCH("attention combine launch");
  return NVFP4DA_OK;
}

#ifdef NVFP4DA_PHASES
// Diagnostic build only: max co-resident clusters of the fused QKV kernel
// (ROWS = 32) and of the attention kernel (EPL 4, GH 4) for a cluster size.
int nvfp4da_debug_occupancy(int which, int cluster, int smem, int* out) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.dynamicSmemBytes = smem;
  cudaError_t e;
  if (which == 0) {
    cfg.gridDim = dim3(144);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.numAttrs = 0;  // compile-time cluster dims
    ensure_smem(qkv_fused_kernel<32>, smem);
    e = cudaOccupancyMaxActiveClusters(out, qkv_fused_kernel<32>, &cfg);
  } else {
    cfg.gridDim = dim3(cluster * 6);
    cfg.blockDim = dim3(kAttnThreads);
    if (cluster > 8) ensure_big_clusters(attn_split_kernel<4, 4>);
    e = cudaOccupancyMaxActiveClusters(out, attn_split_kernel<4, 4>, &cfg);
  }
  return e == cudaSuccess ? 0 : cuda_fail(e, "occupancy");
}

// Diagnostic build only: copy the phase table (CTA-major, 16 slots) to host.
int nvfp4da_debug_phases(unsigned long long* host, size_t n) {
  cudaError_t e = cudaMemcpyFromSymbol(host, g_phase_table, std::min(n, sizeof(g_phase_table)));
  return e == cudaSuccess ? NVFP4DA_OK : cuda_fail(e, "phase table copy");
}
#endif

int nvfp4da_decoder_attention_forward_hostio(const nvfp4da_forward_args* a, const uint16_t* x_host,
                                             uint16_t* output_host, void* workspace, size_t workspace_bytes,
                                             void* stream) {
  if (!a || !x_host || !output_host) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "forward_hostio: NULL argument");
  int r = check_forward(a);
  if (r) return r;
  const size_t bytes = static_cast<size_t>(a->batch * a->tokens * a->hidden) * 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Input: see forward_impl (parameter block, mapped read or copy).  Output:
  // into page-locked host memory that the device can address, the last
  // kernel stores it directly (visible once the stream reaches this point),
  // which saves a copy-engine round trip; other buffers are copied.
  const uint16_t* x_dev = static_cast<const uint16_t*>(mapped_address(x_host));
  uint16_t* out_dev = static_cast<uint16_t*>(mapped_address(output_host));
  if (out_dev) {
    nvfp4da_forward_args direct = *a;
    direct.output = out_dev;
    return forward_impl(&direct, workspace, workspace_bytes, stream, NVFP4DA_PATH_AUTO, x_host, x_dev);
  }
  if ((r = forward_impl(a, workspace, workspace_bytes, stream, NVFP4DA_PATH_AUTO, x_host, x_dev))) return r;
  cudaError_t e = cudaMemcpyAsync(output_host, a->output, bytes, cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e, "forward_hostio: output copy");
  return NVFP4DA_OK;
}

int nvfp4da_qkv_rope_append(const nvfp4da_forward_args* a, uint16_t* q_rope_out, void* stream) {
  int r = check_forward(a);
  if (r) return r;
  if (!q_rope_out) return fail(NVFP4DA_ERR_INVALID_ARGUMENT, "q_rope_out is NULL");
  QkvPlan pl;
  if (!plan_qkv(a->batch * a->tokens, a->hidden, a->head_dim, pl))
    return fail(NVFP4DA_ERR_UNSUPPORTED, "the fused QKV kernel needs head_dim %% 32 == 0, head_dim <= 256 and hidden %% 128 == 0");
  QkvParams p = qkv_params(a, q_rope_out);
  const int64_t hq = a->hidden / a->head_dim;
  cudaError_t e = launch_qkv(p, pl, hq + 2 * a->kv_heads, static_cast<cudaStream_t>(stream), true);
  if (e != cudaSuccess) return cuda_fail(e, "fused qkv launch");
  return NVFP4DA_OK;
}

}  // extern "C"
