// Allocation-free variant of the decoder-attention forward.
//
// Some callers cannot call cudaMalloc at all: a serving loop whose memory is
// budgeted up front (a hard HBM reservation or a pool that must not fragment),
// a plugin host that forbids allocation outside its own allocator, or code that
// runs where an allocation would synchronise the device.  They still pass the
// inputs and outputs; this entry point takes the forward's scratch memory
// (q after RoPE, the attention context and the split-KV partials and
// counters) from one file-scope device array instead of a caller workspace.
//
// The array is NVFP4DA_NOALLOC_SCRATCH_BYTES (8 MiB) per GPU that loads the
// library, held until the process exits.  Host code must not hand the array's
// name to a kernel (on the host it is only a stand-in symbol); the device
// address is looked up once per device with cudaGetSymbolAddress.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/nvfp4_decoder_attention.h"

namespace {

constexpr size_t kScratchBytes = NVFP4DA_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

}  // namespace

void nvfp4da_set_last_error(const char* msg);  // capi.cu

namespace {

int report(int code, const std::string& msg) {
  nvfp4da_set_last_error(msg.c_str());
  return code;
}

// Device address of this GPU's copy of the array; looked up on the first call
// made with the device current.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return report(NVFP4DA_ERR_CUDA, "no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return report(NVFP4DA_ERR_CUDA,
                    std::string("cudaGetSymbolAddress of the scratch array failed: ") + cudaGetErrorString(e));
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return NVFP4DA_OK;
}

}  // namespace

extern "C" int nvfp4da_decoder_attention_forward_noalloc(const nvfp4da_forward_args* args, void* stream) {
  const size_t need = nvfp4da_forward_workspace_size(args);
  if (need == 0) return NVFP4DA_ERR_INVALID_ARGUMENT;  // message set by the size query
  if (need > kScratchBytes)
    return report(NVFP4DA_ERR_WORKSPACE, "forward needs " + std::to_string(need) +
                                             " bytes of scratch, more than the " + std::to_string(kScratchBytes) +
                                             " bytes the allocation-free entry point holds; call "
                                             "nvfp4da_decoder_attention_forward with a workspace instead");
  void* scratch = nullptr;
  const int r = scratch_for_current_device(&scratch);
  if (r != NVFP4DA_OK) return r;
  // Every call shares the array; the forward clears what must start at zero
  // (the split-KV counters) itself.
  return nvfp4da_decoder_attention_forward(args, scratch, kScratchBytes, stream);
}
