// Route-layer forward for callers that cannot allocate device memory.
//
// Some hosts drive this library from places where cudaMalloc is off limits:
// a plugin running inside a framework that owns every device allocation, or
// an inference server whose memory pool is fixed at start-up.  They still own
// the inputs and outputs, but cannot hand over the ~27 KB-per-token workspace
// the fused layer needs.
// This entry point uses a fixed scratch area that is part of the library
// image instead: MRSA_NOALLOC_SCRATCH_BYTES (32 MiB) of device memory that
// every GPU which loads the library keeps until the process exits.  That is
// enough for about 1200 tokens of the Dream shape (28/4 heads, d=128).
//
// The scratch is shared by every call on a device and keeps whatever the last
// call left in it.  The layer writes every intermediate before reading it, so
// nothing has to start at zero; but two calls whose work overlaps on the GPU
// (different streams, no ordering between them) race on it.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_scratch[MRSA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
struct ScratchAddr {
  CUcontext ctx;      // the context the address was looked up in
  void* addr;
};
ScratchAddr g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent g_ctx_get = nullptr;
std::once_flag g_ctx_once;

// Device address of g_scratch on the current device.  In host code the
// symbol names a host-side stand-in, so the address has to come from the
// runtime, once per device, with that device current.  It is looked up again
// when the device's current context differs from the one it was found in
// (a cudaDeviceReset destroys the context and the module with the scratch).
int scratch_on_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return MRSA_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return MRSA_ERR_ARG;
  // CUDA 12 creates the device's primary context here if the runtime has not yet
  if (cudaSetDevice(dev) != cudaSuccess) return MRSA_ERR_LAUNCH;
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<CtxGetCurrent>(fn);
  });
  if (g_ctx_get == nullptr) return MRSA_ERR_LAUNCH;
  CUcontext ctx = nullptr;
  if (g_ctx_get(&ctx) != CUDA_SUCCESS || ctx == nullptr) return MRSA_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& e = g_scratch_addr[dev];
  if (e.addr == nullptr || e.ctx != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return MRSA_ERR_LAUNCH;
    e.ctx = ctx;
    e.addr = p;
  }
  *out = e.addr;
  return MRSA_OK;
}

}  // namespace

extern "C" int mrsa_route_layer_forward_noalloc(const mrsa_route_layer_args* a,
                                                mrsa_stream_t stream) {
  if (a == nullptr) return MRSA_ERR_NULL;
  // the scratch of the device that holds the inputs, whichever is current on this thread
  mrsa::DeviceScope device_scope(a->q_pre);
  const size_t need = mrsa_route_layer_workspace_size(a);
  if (need == 0) return MRSA_ERR_SHAPE;
  if (need > MRSA_NOALLOC_SCRATCH_BYTES) return MRSA_ERR_WORKSPACE;   // too large for the scratch
  void* ws = nullptr;
  const int rc = scratch_on_current_device(&ws);
  if (rc != MRSA_OK) return rc;
  return mrsa_route_layer_forward(a, ws, MRSA_NOALLOC_SCRATCH_BYTES, stream);
}
