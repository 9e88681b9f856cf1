// Dense bf16 GEMM on the 5th-generation tensor cores for the projections and
// the MLP of the Dream-shaped forward: C[M, N] = A[M, K] . B[N, K]^T (B in
// nn.Linear's [out, in] layout), fp32 accumulation, with the epilogue of the
// layer that follows fused in:
//   MRSA_GEMM_PLAIN    C = bf16(acc + bias)              (q/k/v projections, lm_head)
//   MRSA_GEMM_SWIGLU   B rows interleaved in blocks of 128: [gate n0..n0+127 ;
//                      up n0..n0+127] per 256-row block; C[M, N/2] =
//                      bf16(bf16(silu(bf16(gate))) * bf16(up))   (Qwen2 MLP)
//   MRSA_GEMM_RESIDUAL C = bf16(residual + bf16(acc))     (o_proj, down_proj)
// N % 8 == 0 (the last N tile may be partial: its B rows beyond N load as
// zeros and its columns beyond N are not stored); SwiGLU needs N % 256 == 0.
// Persistent: one CTA per SM walks 128 x 256 output tiles (grouped along M so
// the B tiles of neighbouring tiles stay in L2).  Warp 0 streams A and B
// 64-wide K blocks by TMA into four stages (48 KB each, 128-byte swizzle), warp
// 1 issues UMMA M=128 N=256 K=16 (four per stage) into one of two 256-column
// TMEM accumulators, warps 4-7 drain a finished accumulator (one output row
// per thread) while the next tile accumulates into the other.  Every wait is
// bounded; an aborted CTA drains its copies and MMAs and sets bit 5 of
// mrsa_device_error_flags.
//
// RMSNorm (Qwen2RMSNorm): y = w * bf16(x * rsqrt(mean(x^2) + eps)), fp32
// statistics, one CTA per row.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int BM = 128, BN = 256, BK = 64, ST = 4;
constexpr int GEMM_THREADS = 256;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int GROUP_M = 16;               // M tiles walked per N stripe

__device__ int g_gemm_error;

struct GemmArgs {
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  __nv_bfloat16* c;
  int64_t M, N, K, ldc;
  int mode, m_tiles, n_tiles, k_blocks;
};

struct __align__(1024) GemmSmem {
  unsigned char tiles[ST][STAGE_BYTES];
  uint64_t full[ST], empty[ST], acc_full[2], acc_empty[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(GemmSmem) + 1024 <= 232448, "GEMM shared memory over budget");

__device__ __forceinline__ void tile_coords(int t, const GemmArgs& a, int& tm, int& tn) {
  // grouped order: GROUP_M consecutive M tiles share one N stripe before moving on
  const int per_group = GROUP_M * a.n_tiles;
  const int group = t / per_group;
  const int first_m = group * GROUP_M;
  const int rows = min(GROUP_M, a.m_tiles - first_m);
  const int r = t % per_group;
  tm = first_m + r % rows;
  tn = r / rows;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                                                               const __grid_constant__ CUtensorMap tm_b, GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.full[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(tc::smem_addr(&sm.acc_full[b]), 1);
      tc::mbar_init(tc::smem_addr(&sm.acc_empty[b]), 4);
    }
    tc::mbar_init(tc::smem_addr(&sm.drain), 1);
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_addr(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base;
  volatile int* ab = &sm.abort_flag;
  const int n_tiles = a.m_tiles * a.n_tiles;

  if (warp == 0) {
    // ============================ TMA producer ==============================
    if (lane == 0) {
      tc::prefetch_tensormap(&tm_a);
      tc::prefetch_tensormap(&tm_b);
      int64_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, a, tm, tn);
        for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
          const int s = static_cast<int>(it % ST);
          if (it >= ST && !tc::wait_bounded(tc::smem_addr(&sm.empty[s]), static_cast<uint32_t>(((it / ST) - 1) & 1), ab)) {
            ok = false;
            break;
          }
          const uint32_t bar = tc::smem_addr(&sm.full[s]);
          tc::mbar_arrive_expect_tx(bar, STAGE_BYTES);
          tc::tma_load_2d(tc::smem_addr(sm.tiles[s]), &tm_a, kb * BK, tm * BM, bar);
          tc::tma_load_2d(tc::smem_addr(sm.tiles[s] + A_BYTES), &tm_b, kb * BK, tn * BN, bar);
        }
      }
      // copies still in flight after an abort: the last one issued into each stage
      if (*ab)
        for (int64_t j = it > ST ? it - ST : 0; j < it; ++j)
          tc::mbar_wait(tc::smem_addr(&sm.full[j % ST]), static_cast<uint32_t>((j / ST) & 1), 4000000u);
    }
  } else if (warp == 1) {
    // ============================ MMA issue ================================
    constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN, 0, 0);
    const uint64_t da0 = tc::smem_desc_sw128(tc::smem_addr(sm.tiles[0]), 16, 1024);
    const uint64_t db0 = tc::smem_desc_sw128(tc::smem_addr(sm.tiles[0] + A_BYTES), 16, 1024);
    int64_t it = 0;
    int tl = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      if (tl >= 2 && !tc::wait_bounded_warp(tc::smem_addr(&sm.acc_empty[buf]), static_cast<uint32_t>(((tl >> 1) - 1) & 1), ab))
        break;
      tc::fence_after_sync();
      const uint32_t d = tbase + static_cast<uint32_t>(buf * BN);
      for (int kb = 0; kb < a.k_blocks; ++kb, ++it) {
        const int s = static_cast<int>(it % ST);
        if (!tc::wait_bounded_warp(tc::smem_addr(&sm.full[s]), static_cast<uint32_t>((it / ST) & 1), ab)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t so = static_cast<uint32_t>(s) * STAGE_BYTES;
        if (tc::elect_one()) {
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc::mma_bf16_ss(d, tc::desc_adv(da0, so + kk * 32), tc::desc_adv(db0, so + kk * 32), idesc,
                            kb > 0 || kk > 0);
          tc::mma_commit(tc::smem_addr(&sm.empty[s]));
          if (kb == a.k_blocks - 1) tc::mma_commit(tc::smem_addr(&sm.acc_full[buf]));
        }
        __syncwarp();
      }
    }
    if (tc::elect_one()) {
      tc::mma_commit(tc::smem_addr(&sm.drain));
      tc::mbar_wait(tc::smem_addr(&sm.drain), 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ============================ epilogue ==================================
    const int q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    int tl = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.acc_full[buf]), static_cast<uint32_t>((tl >> 1) & 1), ab)) break;
      tc::fence_after_sync();
      int tm, tn;
      tile_coords(t, a, tm, tn);
      const int64_t row = static_cast<int64_t>(tm) * BM + q * 32 + lane;
      const uint32_t tacc = tbase + lane_off + static_cast<uint32_t>(buf * BN);
      if (a.mode == MRSA_GEMM_SWIGLU) {
        // columns 0-127 gate, 128-255 up, for output columns tn*128 .. +127
        for (int j = 0; j < BN / 2; j += 32) {
          uint32_t gr[32], ur[32];
          tc::tmem_ld16(tacc + j, *reinterpret_cast<uint32_t(*)[16]>(&gr[0]));
          tc::tmem_ld16(tacc + j + 16, *reinterpret_cast<uint32_t(*)[16]>(&gr[16]));
          tc::tmem_ld16(tacc + BN / 2 + j, *reinterpret_cast<uint32_t(*)[16]>(&ur[0]));
          tc::tmem_ld16(tacc + BN / 2 + j + 16, *reinterpret_cast<uint32_t(*)[16]>(&ur[16]));
          tc::tmem_wait_ld();
          if (j + 32 >= BN / 2) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_addr(&sm.acc_empty[buf]));
          }
          uint32_t o[16];
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            float v2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float g = round_bf16(__uint_as_float(gr[2 * h + e]));
              const float u = round_bf16(__uint_as_float(ur[2 * h + e]));
              v2[e] = round_bf16(silu_f(g)) * u;
            }
            o[h] = pack_bf16x2(v2[0], v2[1]);
          }
          if (row < a.M) {
            uint4* dst = reinterpret_cast<uint4*>(a.c + row * a.ldc + static_cast<int64_t>(tn) * (BN / 2) + j);
#pragma unroll
            for (int p = 0; p < 4; ++p) dst[p] = make_uint4(o[4 * p], o[4 * p + 1], o[4 * p + 2], o[4 * p + 3]);
          }
        }
      } else {
        for (int j = 0; j < BN; j += 32) {
          uint32_t r[32];
          tc::tmem_ld16(tacc + j, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
          tc::tmem_ld16(tacc + j + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
          tc::tmem_wait_ld();
          if (j + 32 >= BN) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_addr(&sm.acc_empty[buf]));
          }
          const int64_t col = static_cast<int64_t>(tn) * BN + j;
          if (col >= a.N) continue;              // the ragged last N tile: nothing to store
          const int pieces = a.N - col >= 32 ? 4 : static_cast<int>((a.N - col) / 8);
          float add[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) add[e] = 0.f;
          if (a.mode == MRSA_GEMM_PLAIN && a.bias != nullptr) {
            const uint4* bp = reinterpret_cast<const uint4*>(a.bias + col);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              if (p >= pieces) break;
              const uint4 w = __ldg(bp + p);
              const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack_bf16x2(wd[e]);
                add[8 * p + 2 * e] = f.x;
                add[8 * p + 2 * e + 1] = f.y;
              }
            }
          }
          uint32_t o[16];
          if (a.mode == MRSA_GEMM_RESIDUAL && row < a.M) {
            const uint4* rp = reinterpret_cast<const uint4*>(a.resid + row * a.ldc + col);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              if (p >= pieces) break;
              const uint4 w = __ldg(rp + p);
              const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack_bf16x2(wd[e]);
                o[4 * p + e] = pack_bf16x2(f.x + round_bf16(__uint_as_float(r[8 * p + 2 * e])),
                                           f.y + round_bf16(__uint_as_float(r[8 * p + 2 * e + 1])));
              }
            }
          } else {
#pragma unroll
            for (int h = 0; h < 16; ++h)
              o[h] = pack_bf16x2(__uint_as_float(r[2 * h]) + add[2 * h], __uint_as_float(r[2 * h + 1]) + add[2 * h + 1]);
          }
          if (row < a.M) {
            uint4* dst = reinterpret_cast<uint4*>(a.c + row * a.ldc + col);
#pragma unroll
            for (int p = 0; p < 4; ++p)
              if (p < pieces) dst[p] = make_uint4(o[4 * p], o[4 * p + 1], o[4 * p + 2], o[4 * p + 3]);
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && sm.abort_flag) atomicOr(&g_gemm_error, 1);
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------ RMSNorm
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       __nv_bfloat16* __restrict__ y, int dim, float eps) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * dim;
  float ss = 0.f;
  for (int e = threadIdx.x * 8; e < dim; e += 256 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + e);
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 f = unpack_bf16x2(wd[p]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / static_cast<float>(dim) + eps);
  for (int e = threadIdx.x * 8; e < dim; e += 256 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + e);
    const uint4 g = *reinterpret_cast<const uint4*>(w + e);
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w}, gd[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 f = unpack_bf16x2(wd[p]), gw = unpack_bf16x2(gd[p]);
      o[p] = pack_bf16x2(gw.x * round_bf16(f.x * inv), gw.y * round_bf16(f.y * inv));
    }
    *reinterpret_cast<uint4*>(y + row * dim + e) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool make_map2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {BK, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace mrsa {
int gemm_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
}  // namespace mrsa

extern "C" int mrsa_gemm_bf16(const void* a, const void* b, const void* bias, const void* residual, void* c,
                              int64_t m, int64_t n, int64_t k, int epilogue, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(a);
  if (!a || !b || !c) return MRSA_ERR_NULL;
  if (epilogue != MRSA_GEMM_PLAIN && epilogue != MRSA_GEMM_SWIGLU && epilogue != MRSA_GEMM_RESIDUAL)
    return MRSA_ERR_ARG;
  if (epilogue == MRSA_GEMM_RESIDUAL && residual == nullptr) return MRSA_ERR_NULL;
  if (m < 1 || n < 8 || k < BK || n % 8 || k % BK || (epilogue == MRSA_GEMM_SWIGLU && n % BN) ||
      m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                       reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(bias) |
                       reinterpret_cast<uintptr_t>(residual);
  if (al & 15u) return MRSA_ERR_ALIGN;
  (void)cudaGetLastError();
  const int64_t m_tiles = (m + BM - 1) / BM, n_tiles = (n + BN - 1) / BN;
  if (m_tiles * n_tiles > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  CUtensorMap tma, tmb;
  if (!make_map2d(&tma, a, static_cast<uint64_t>(k), static_cast<uint64_t>(m), BM) ||
      !make_map2d(&tmb, b, static_cast<uint64_t>(k), static_cast<uint64_t>(n), BN)) {
    mrsa::note_cuda_error(cudaErrorInvalidValue, "mrsa_gemm_bf16: tensor map encoding");
    return MRSA_ERR_LAUNCH;
  }
  GemmArgs g;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.resid = static_cast<const __nv_bfloat16*>(residual);
  g.c = static_cast<__nv_bfloat16*>(c);
  g.M = m;
  g.N = n;
  g.K = k;
  g.ldc = epilogue == MRSA_GEMM_SWIGLU ? n / 2 : n;
  g.mode = epilogue;
  g.m_tiles = static_cast<int>(m_tiles);
  g.n_tiles = static_cast<int>(n_tiles);
  g.k_blocks = static_cast<int>(k / BK);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return MRSA_ERR_LAUNCH;
  const size_t smem = sizeof(GemmSmem) + 1024;
  if (const cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
      e != cudaSuccess) {
    mrsa::note_cuda_error(e, "mrsa_gemm_bf16: shared-memory opt-in");
    return MRSA_ERR_LAUNCH;
  }
  const int64_t tiles = m_tiles * n_tiles;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  gemm_kernel<<<grid, GEMM_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(tma, tmb, g);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" int mrsa_rms_norm(const void* x, const void* weight, void* y, int64_t rows, int64_t dim, float eps,
                             mrsa_stream_t stream) {
  if (!x || !weight || !y) return MRSA_ERR_NULL;
  if (rows < 0 || dim < 8 || dim % 8 || dim > 65536 || rows > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return MRSA_ERR_ALIGN;
  if (rows == 0) return MRSA_OK;
  (void)cudaGetLastError();
  rms_norm_kernel<<<static_cast<unsigned>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
      static_cast<__nv_bfloat16*>(y), static_cast<int>(dim), eps);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
