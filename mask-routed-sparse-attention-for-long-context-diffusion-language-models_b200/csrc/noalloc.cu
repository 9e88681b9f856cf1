// Route-layer forward for callers that cannot allocate device memory.
//
// Some hosts drive this library from places where cudaMalloc is off limits:
// a plugin running inside a framework that owns every device allocation, an
// inference server whose memory pool is fixed at start-up, or code that runs
// while a stream is being recorded.  They still own the inputs and outputs,
// but cannot hand over the ~27 KB-per-token workspace the fused layer needs.
// This entry point uses a fixed scratch area that is part of the library
// image instead: MRSA_NOALLOC_SCRATCH_BYTES (32 MiB) of device memory that
// every GPU which loads the library keeps until the process exits.  That is
// enough for about 1200 tokens of the Dream shape (28/4 heads, d=128).
//
// The scratch is shared by every call on a device and keeps whatever the last
// call left in it.  The layer writes every intermediate before reading it, so
// nothing has to start at zero; but two calls whose work overlaps on the GPU
// (different streams, no ordering between them) race on it.
#include <mutex>

#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_scratch[MRSA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_scratch on the current device.  In host code the
// symbol names a host-side stand-in, so the address has to come from the
// runtime, once per device, with that device current.
int scratch_on_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return MRSA_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return MRSA_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return MRSA_ERR_LAUNCH;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return MRSA_OK;
}

}  // namespace

extern "C" int mrsa_route_layer_forward_noalloc(const mrsa_route_layer_args* a,
                                                mrsa_stream_t stream) {
  if (a == nullptr) return MRSA_ERR_NULL;
  const size_t need = mrsa_route_layer_workspace_size(a);
  if (need == 0) return MRSA_ERR_SHAPE;
  if (need > MRSA_NOALLOC_SCRATCH_BYTES) return MRSA_ERR_WORKSPACE;   // too large for the scratch
  void* ws = nullptr;
  const int rc = scratch_on_current_device(&ws);
  if (rc != MRSA_OK) return rc;
  return mrsa_route_layer_forward(a, ws, MRSA_NOALLOC_SCRATCH_BYTES, stream);
}
