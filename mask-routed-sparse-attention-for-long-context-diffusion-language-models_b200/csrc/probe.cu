// Tile-gather probe: the L2 -> shared-memory ceiling of the selected-attention
// kernel's loads, measured with the same tensor maps and boxes and nothing
// computed.  Each CTA (one per SM) runs two producer lanes, each with its own
// two stages; per work item a producer loads the 64-key K tile and V tile of
// a pseudo-random (chunk, KV head) plus `owners` 8-row query boxes, and a
// consumer warp waits for the bytes and frees the stage.  Two producers reach
// the per-SM L2 read rate that one issuing lane cannot.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int kProducers = 2, kStages = 2, kMaxOwners = 8;
constexpr int kStageBytes = 32768 + kMaxOwners * 2048;

struct ProbeArgs {
  int64_t items;
  int chunks, heads, q_boxes, owners;
  int* status;
};

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

__global__ void __launch_bounds__(128, 1) probe_gather_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                              const __grid_constant__ CUtensorMap tm_v,
                                                              const __grid_constant__ CUtensorMap tm_q, ProbeArgs a) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kProducers][kStages], empty[kProducers][kStages];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int p = 0; p < kProducers; ++p)
      for (int s = 0; s < kStages; ++s) {
        tc::mbar_init(tc::smem_addr(&full[p][s]), 1);
        tc::mbar_init(tc::smem_addr(&empty[p][s]), 1);
      }
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  volatile int* ab = &abort_flag;
  const int p = warp >> 1;                       // warps 0/1: producer 0 and its consumer; 2/3: producer 1
  const int64_t mine = (a.items - p + kProducers - 1) / kProducers;
  const uint32_t bytes = 32768u + 2048u * static_cast<uint32_t>(a.owners);
  unsigned char* stage0 = base + static_cast<size_t>(p) * kStages * kStageBytes;
  int64_t issued = 0;
  if ((warp & 1) == 0) {
    if (lane == 0) {
      for (int64_t i = 0; i < mine; ++i) {
        const int s = static_cast<int>(i % kStages);
        if (i >= kStages && !tc::wait_bounded(tc::smem_addr(&empty[p][s]), static_cast<uint32_t>(((i / kStages) - 1) & 1), ab))
          break;
        const uint32_t dst = tc::smem_addr(stage0 + s * kStageBytes);
        const uint32_t bar = tc::smem_addr(&full[p][s]);
        const uint32_t h = mix32(static_cast<uint32_t>(blockIdx.x * 2654435761u) ^ static_cast<uint32_t>(i * 2 + p));
        const int c = static_cast<int>(h % static_cast<uint32_t>(a.chunks));
        const int hd = static_cast<int>((h >> 20) % static_cast<uint32_t>(a.heads));
        tc::mbar_arrive_expect_tx(bar, bytes);
        tc::tma_load_4d(dst, &tm_k, 0, c * 64, 0, hd, bar);
        tc::tma_load_4d(dst + 16384, &tm_v, 0, c * 64, 0, hd, bar);
        for (int j = 0; j < a.owners; ++j) {
          const int row = static_cast<int>(mix32(h + 977u * static_cast<uint32_t>(j + 1)) % static_cast<uint32_t>(a.q_boxes)) * 8;
          tc::tma_load_3d(dst + 32768 + 2048 * j, &tm_q, 0, row, 0, bar);
        }
        ++issued;
      }
      // an aborted producer still waits (bounded) for the copies it issued
      for (int64_t i = issued > kStages ? issued - kStages : 0; i < issued && *ab; ++i)
        tc::mbar_wait(tc::smem_addr(&full[p][i % kStages]), static_cast<uint32_t>((i / kStages) & 1), 4000000u);
    }
  } else {
    for (int64_t i = 0; i < mine; ++i) {
      const int s = static_cast<int>(i % kStages);
      if (!tc::wait_bounded_warp(tc::smem_addr(&full[p][s]), static_cast<uint32_t>((i / kStages) & 1), ab)) break;
      if (lane == 0) tc::mbar_arrive(tc::smem_addr(&empty[p][s]));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) atomicExch(a.status, 1);
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool probe_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
               const cuuint32_t* box) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return false;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int mrsa_probe_tile_gather(const void* k, const void* v, const void* q, int64_t kv_len, int64_t kv_heads,
                                      int64_t q_rows, int owners, int64_t items_per_cta, int* status,
                                      mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(k);
  if (!k || !v || !q || !status) return MRSA_ERR_NULL;
  if (kv_len < 64 || kv_len % 64 || kv_len / 64 > 0x7fffffffLL || kv_heads < 1 || kv_heads > 4096 || q_rows < 8 ||
      q_rows > 0x7fffffffLL || owners < 0 || owners > kMaxOwners || items_per_cta < 1 || items_per_cta > (1LL << 40))
    return MRSA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(q)) & 15u)
    return MRSA_ERR_ALIGN;
  // K and V: [kv_len rows][kv_heads * 128] bf16 viewed as (dim-in-half, row, half, head), the selected
  // kernel's boxes; q: [q_rows][128] viewed as (dim-in-half, row, half), 8-row boxes
  CUtensorMap tk, tv, tq;
  const cuuint64_t kv_dims[4] = {64, static_cast<cuuint64_t>(kv_len), 2, static_cast<cuuint64_t>(kv_heads)};
  const cuuint64_t kv_str[3] = {static_cast<cuuint64_t>(kv_heads * 256), 128, 256};
  const cuuint32_t kv_box[4] = {64, 64, 2, 1};
  const cuuint64_t q_dims[3] = {64, static_cast<cuuint64_t>(q_rows), 2};
  const cuuint64_t q_str[2] = {256, 128};
  const cuuint32_t q_box[3] = {64, 8, 2};
  if (!probe_map(&tk, k, 4, kv_dims, kv_str, kv_box) || !probe_map(&tv, v, 4, kv_dims, kv_str, kv_box) ||
      !probe_map(&tq, q, 3, q_dims, q_str, q_box))
    return MRSA_ERR_LAUNCH;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return MRSA_ERR_LAUNCH;
  const size_t smem = static_cast<size_t>(kProducers) * kStages * kStageBytes + 1024;
  if (cudaFuncSetAttribute(probe_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  ProbeArgs a;
  a.items = items_per_cta;
  a.chunks = static_cast<int>(kv_len / 64);
  a.heads = static_cast<int>(kv_heads);
  a.q_boxes = static_cast<int>(q_rows / 8);
  a.owners = owners;
  a.status = status;
  probe_gather_kernel<<<sms, 128, smem, static_cast<cudaStream_t>(stream)>>>(tk, tv, tq, a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
