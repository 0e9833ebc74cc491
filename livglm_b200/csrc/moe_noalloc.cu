// Allocation-free forward of the MoE block.
//
// lg_moe_forward needs a caller-provided workspace.  Some callers cannot
// allocate device memory when they run the block: a host framework that owns
// every byte of device memory and hands plugins no allocator, a latency-bound
// decode loop where cudaMalloc may synchronise the whole device, or code that
// runs while holding a lock the framework's allocator also takes.  For them
// this file keeps the scratch in a fixed device array that is part of the
// library image, so the call itself allocates nothing.
#include <cstdio>
#include <mutex>

#include "livglm_moe.h"

#include <cuda_runtime.h>

int lg_internal_set_error(int code, const char* msg);

namespace {

// 4 MiB of scratch on every GPU where this library's device code is loaded,
// held until the process exits.  All calls on a device share it.
constexpr size_t kStaticScratchBytes = size_t(4) << 20;
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch, resolved once per device.  In host code
// the array's name is only a host-side stand-in, never a device address.
constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof msg, "static-scratch forward: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return lg_internal_set_error(LG_ERR_CUDA, msg);
  }
  if (dev < 0 || dev >= kMaxDevices)
    return lg_internal_set_error(LG_ERR_UNSUPPORTED, "static-scratch forward: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof msg, "static-scratch forward: cudaGetSymbolAddress failed on device %d: %s", dev,
               cudaGetErrorString(e));
      return lg_internal_set_error(LG_ERR_CUDA, msg);
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return LG_OK;
}

}  // namespace

extern "C" int lg_moe_static_scratch_status(int clear, int32_t* status_out, void* stream) {
  if (!status_out) return lg_internal_set_error(LG_ERR_INVALID_ARG, "static-scratch status: NULL status_out");
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != LG_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, scratch, sizeof word, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(scratch, 0, sizeof word, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof msg, "static-scratch status: %s", cudaGetErrorString(e));
    return lg_internal_set_error(LG_ERR_CUDA, msg);
  }
  *status_out = word;
  return LG_OK;
}

extern "C" int lg_moe_forward_static_scratch(const lg_moe_config* cfg, const lg_moe_weights* w,
                                             const uint16_t* x, int64_t M, float* out,
                                             float* weights_out, uint32_t* indices_out, void* stream) {
  const size_t need = lg_moe_workspace_size(cfg, M > 0 ? M : 1);
  if (need == 0) return LG_ERR_INVALID_ARG;  // message already set by the size query
  if (need > kStaticScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof msg,
             "static-scratch forward: %lld tokens need %zu bytes of scratch, more than the fixed %zu; "
             "call lg_moe_forward with a caller workspace or split the tokens",
             static_cast<long long>(M), need, kStaticScratchBytes);
    return lg_internal_set_error(LG_ERR_UNSUPPORTED, msg);
  }
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != LG_OK) return rc;
  return lg_moe_forward(cfg, w, x, M, out, weights_out, indices_out, scratch, kStaticScratchBytes, stream);
}
