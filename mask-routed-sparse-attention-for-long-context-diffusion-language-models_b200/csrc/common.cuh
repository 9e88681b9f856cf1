// Shared device helpers for the MRSA sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mrsa.h"

namespace mrsa {

constexpr int kHeadDim = 128;   // Dream-7B head_dim; every kernel is specialised to it
constexpr int kChunk = 64;      // chunk_size of the canonical config
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }
__device__ __forceinline__ float round_bf16(float x) { return bf2f(f2bf(x)); }

// One 32-byte global store (a whole sector per thread); `p` 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- cp.async (16-byte, L2-only caching) -----------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool pred) {
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---- ldmatrix / mma.sync m16n8k16 (bf16 in, fp32 accumulate) ---------------
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 operands (P.V runs in fp16: P keeps 11 significant bits instead of
// bf16's 8, and bf16 V converts to fp16 exactly inside the fp16 range).
__device__ __forceinline__ void mma_f16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// bf16x2 word -> f16x2 word (saturating at +-65504)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t u) {
  const float lo = __uint_as_float(u << 16), hi = __uint_as_float(u & 0xffff0000u);
  return pack_f16x2(lo, hi);
}
// Convert a 64-row x 128-column bf16 tile in shared memory to fp16 in place,
// cooperatively over `nthreads` threads.
__device__ __forceinline__ void tile_bf16_to_f16(void* tile, int tid, int nthreads) {
  uint4* t = reinterpret_cast<uint4*>(tile);
  for (int i = tid; i < 64 * 128 / 8; i += nthreads) {
    uint4 v = t[i];
    v.x = bf16x2_to_f16x2(v.x);
    v.y = bf16x2_to_f16x2(v.y);
    v.z = bf16x2_to_f16x2(v.z);
    v.w = bf16x2_to_f16x2(v.w);
    t[i] = v;
  }
}

// 128-byte row of 8 16-byte pieces, XOR-swizzled by row to spread ldmatrix
// row reads over all banks.  `piece` indexes 16-byte units inside the row.
__device__ __forceinline__ int swz(int row, int piece) { return (piece ^ (row & 7)); }

// Float <-> order-preserving unsigned key (larger float => larger key).
__device__ __forceinline__ uint32_t f2ord(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 2^x on the special-function unit (relative error ~2^-22; -inf -> +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Device error flags of the routing and local-window kernels; -1 when unreadable.
int route_error_flags(int clear);
int local_error_flags(int clear);
int convert_error_flags(int clear);
int bwd_error_flags(int clear);
int gemm_error_flags(int clear);
int local_bwd_error_flags(int clear);

// Inverted chunk -> (query, slot) index of indices [B,Lq,Hkv,K] int32: per
// segment (b, h, c) (flattened as (b*Hkv + h)*C + c) cnt[seg] entries from
// pairs[off[seg]] on, each (l << 5) | slot, in (l, slot) order.  Built in
// `workspace` (at least chunk_index_bytes() bytes); C <= 12288.
struct ChunkIndex {
  const int32_t *cnt, *off, *pairs;
};
size_t chunk_index_bytes(int64_t batch, int64_t q_len, int64_t kv_heads, int64_t topk, int64_t chunks);
int build_chunk_index(const int32_t* indices, int64_t batch, int64_t q_len, int kv_heads, int topk, int chunks,
                      void* workspace, cudaStream_t s, ChunkIndex* out);

// ---- sm_100 paired fp32 arithmetic (one instruction for two lanes of work)
// fma/add/mul on a register pair, each half rounded as the scalar op would be.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// max of three (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mrsa

namespace mrsa {
// For the scope of an entry point: makes the primary context of the device
// that owns `p` current on the calling thread (a thread that has made no CUDA
// runtime call yet -- an autograd worker, say -- has none, and the tensor-map
// encoder needs one), and restores the thread's previous device afterwards.
class DeviceScope {
 public:
  explicit DeviceScope(const void* p) {
    cudaPointerAttributes at{};
    if (p == nullptr || cudaPointerGetAttributes(&at, p) != cudaSuccess ||
        (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)) {
      (void)cudaGetLastError();
      return;
    }
    if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
    if (cudaSetDevice(at.device) == cudaSuccess) dev_ = at.device;
  }
  ~DeviceScope() {
    if (prev_ >= 0 && dev_ >= 0 && prev_ != dev_) (void)cudaSetDevice(prev_);
  }
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;

 private:
  int prev_ = -1, dev_ = -1;
};

// Keeps, per host thread, the CUDA error behind the last MRSA_ERR_LAUNCH
// (read through mrsa_last_error()).
void note_cuda_error(cudaError_t e, const char* where);
}  // namespace mrsa

#define MRSA_CHECK_LAUNCH()                                   \
  do {                                                        \
    cudaError_t _e = cudaGetLastError();                      \
    if (_e != cudaSuccess) {                                  \
      mrsa::note_cuda_error(_e, __func__);                    \
      return MRSA_ERR_LAUNCH;                                 \
    }                                                         \
  } while (0)
