// no_alloc.cu — an allocation-free variant of llmoc_moe_forward.
//
// Some callers cannot hand this library device memory for its workspace:
// a host whose device memory is owned by another allocator (for example a
// framework's caching allocator that must not grow), a serving loop that
// forbids cudaMalloc/cudaFree after start-up because they synchronize the
// device, or a foreign-function caller with no device allocator at all.
// llmoc_moe_forward_noalloc runs the same forward with its workspace in a
// fixed, file-scope device array instead of caller-provided memory.
//
// The array (kNoAllocScratchBytes, 8 MiB) exists on every GPU that loads
// this library, for the life of the process.  The first call on a device
// looks up its device address there (cudaGetSymbolAddress, with that device
// current) and caches it; that first call should therefore come before any
// stream capture on the device.  All calls on a device share the one array,
// so calls whose work overlaps on the GPU (different streams, or host
// threads) race on it and must be serialized by the caller.  Everything the
// forward reads from the scratch is written earlier in the same call (the
// device error word is cleared there too), so stale contents of a previous
// call do not matter.  The cached address belongs to the device's current
// context: after cudaDeviceReset every layer (and this address) is invalid,
// so such a caller creates new layers and must not call this entry point
// again in that process.
//
// The scratch also holds the forward's device error word, which the caller
// cannot reach through a workspace pointer of its own:
// llmoc_moe_noalloc_status reads it (after synchronizing the stream) and
// reports LLMOC_ERR_TIMEOUT when a bounded device-side wait of the forward
// gave up, i.e. when that forward's outputs are not valid.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/llmoc_b200.h"

namespace llmoc {
int layer_device(const llmoc_moe_layer* L);
void set_last_error(const std::string& msg);
}

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

// Host code must never use this name as a device address (in host code it is
// a stand-in object); the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_na_mu;
void* g_na_ptr[kMaxDevices] = {};

// The array's device address on `dev`, looked up once per device with that
// device current.
llmoc_status scratch_of(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (g_na_ptr[dev]) {
    *out = g_na_ptr[dev];
    return LLMOC_OK;
  }
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) {
    llmoc::set_last_error(std::string("llmoc_moe_forward_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    cudaGetLastError();
    return LLMOC_ERR_CUDA;
  }
  if (prev != dev && cudaSetDevice(dev) != cudaSuccess) {
    llmoc::set_last_error("llmoc_moe_forward_noalloc: cannot select the layer's device");
    cudaGetLastError();
    return LLMOC_ERR_NO_DEVICE;
  }
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (prev != dev && cudaSetDevice(prev) != cudaSuccess) {
    llmoc::set_last_error("llmoc_moe_forward_noalloc: cannot restore the caller's device");
    cudaGetLastError();
    return LLMOC_ERR_CUDA;
  }
  if (e != cudaSuccess || !ptr) {
    llmoc::set_last_error(std::string("llmoc_moe_forward_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    cudaGetLastError();
    return LLMOC_ERR_CUDA;
  }
  g_na_ptr[dev] = ptr;
  *out = ptr;
  return LLMOC_OK;
}

}  // namespace

extern "C" {

LLMOC_API size_t llmoc_moe_noalloc_capacity(void) { return kNoAllocScratchBytes; }

LLMOC_API llmoc_status llmoc_moe_forward_noalloc(const llmoc_moe_layer* layer, const uint16_t* X,
                                                 int T, uint16_t* Y, void* stream) {
  const int dev = llmoc::layer_device(layer);
  if (dev < 0 || dev >= kMaxDevices || T < 0) {
    llmoc::set_last_error("llmoc_moe_forward_noalloc: bad layer or token count");
    return LLMOC_ERR_INVALID;
  }
  const size_t need = llmoc_moe_workspace_bytes(layer, T);
  if (need > kNoAllocScratchBytes) {
    llmoc::set_last_error("llmoc_moe_forward_noalloc: " + std::to_string(T) + " tokens need " +
                          std::to_string(need) + " bytes of workspace, more than the " +
                          std::to_string(kNoAllocScratchBytes) + "-byte static scratch");
    return LLMOC_ERR_WORKSPACE;
  }
  void* ptr = nullptr;
  const llmoc_status rc = scratch_of(dev, &ptr);
  if (rc != LLMOC_OK) return rc;
  return llmoc_moe_forward(layer, X, T, Y, ptr, kNoAllocScratchBytes, stream);
}

LLMOC_API llmoc_status llmoc_moe_noalloc_status(const llmoc_moe_layer* layer, int T, void* stream) {
  const int dev = llmoc::layer_device(layer);
  if (dev < 0 || dev >= kMaxDevices || T < 0 || llmoc_moe_workspace_bytes(layer, T) > kNoAllocScratchBytes) {
    llmoc::set_last_error("llmoc_moe_noalloc_status: bad layer or token count");
    return LLMOC_ERR_INVALID;
  }
  void* ptr = nullptr;
  llmoc_status rc = scratch_of(dev, &ptr);
  if (rc != LLMOC_OK) return rc;
  llmoc_route_views v{};
  rc = llmoc_moe_route_views(layer, T, ptr, kNoAllocScratchBytes, &v);
  if (rc != LLMOC_OK) return rc;
  int word = 0;
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaMemcpy(&word, v.error_flag, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    llmoc::set_last_error(std::string("llmoc_moe_noalloc_status: ") + cudaGetErrorString(e));
    return LLMOC_ERR_CUDA;
  }
  if (word != 0) {
    llmoc::set_last_error("llmoc_moe_noalloc_status: a bounded device-side wait gave up; the outputs are not valid");
    return LLMOC_ERR_TIMEOUT;
  }
  return LLMOC_OK;
}

}  // extern "C"
