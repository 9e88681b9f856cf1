// Backward of the bidirectional window attention (the local branch of the
// route layer and the SWA layers) on the 5th-generation tensor cores.
//
// Semantics: the gradient of dream_dllm_hils/local_attention.py:110-144
// bidir_local_attention (flash-attn's backward in the reference): for query
// row r = (i, head) and key j with |i - j| <= W, keys that are invalid (or
// landmark slots with skip_inert) enter with K = V = 0 (logit 0), and with
//   P[r, j]  = exp(q_r . k'_j * scale - lse_r)
//   dP[r, j] = dO_r . v'_j
//   delta_r  = dO_r . O_r - dlse_r                     (delta_kernel)
//   dS[r, j] = bf16(P[r, j] * (dP[r, j] - delta_r))
//   dQ_r = scale * sum_j dS[r, j] k'_j,  dK_j = scale * sum_r dS[r, j] q_r,
//   dV_j = sum_r bf16(P[r, j]) dO_r     (dK_j = dV_j = 0 for zeroed keys)
// Two kernels, both over 128-row tiles (16 queries x the 8 head rows of a KV
// group) with S and dP as UMMA M=128 N=64 K=128 into TMEM, each with two row
// groups on alternate tiles, every group with its own MMA warp and TMEM
// accumulators (added in a fixed order at the end, so the result does not
// depend on timing):
//  * local_dkv_kernel: one CTA per 64-key block and KV head walks the query
//    tiles of its band; dV^T += dO^T . P and dK^T += Q^T . dS (MN-major
//    operands) stay in TMEM and are stored once;
//  * local_dq_kernel: one CTA per 16-query tile and KV head walks the key
//    blocks of its band; dQ += dS . K (K as an MN-major B operand) stays in
//    TMEM and is stored once.
// Every mbarrier wait is bounded; an aborted CTA unwinds, waits (bounded) for
// its copies and MMAs and sets bit 6 of mrsa_device_error_flags.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int D = kHeadDim, KB = 64, PT = 16, GMAX = 8;

__device__ int g_local_bwd_error;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ int swz_off(int row, int piece) { return row * 128 + ((piece ^ (row & 7)) << 4); }
__device__ __forceinline__ uint64_t adv(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }
__device__ __forceinline__ bool wait_ab_warp(uint64_t* bar, uint32_t parity, int* abort_flag) {
  return tc::wait_bounded_warp(su32(bar), parity, reinterpret_cast<volatile int*>(abort_flag));
}

struct LocalBwdArgs {
  const uint8_t* key_valid;
  const float* lse;            // [B, L, Hq] natural log
  const float* delta;          // [B, L, Hq]
  float *dq, *dk, *dv;
  float sm_scale;
  int64_t L;
  int Hkv, G, window, skip_inert, chunk;
};

// Zeroed keys of the 64-key block starting at global row `j0` of batch b
// (invalid, or a landmark slot with skip_inert): bit s set = key j0 + s is zeroed.
__device__ __forceinline__ unsigned long long zeroed_keys(const LocalBwdArgs& a, int64_t b, int64_t j0, int lane) {
  bool z0 = false, z1 = false;
  if (a.key_valid != nullptr) {
    z0 = a.key_valid[b * a.L + j0 + lane] == 0;
    z1 = a.key_valid[b * a.L + j0 + 32 + lane] == 0;
  }
  if (a.skip_inert) {
    z0 |= ((j0 + lane + 1) % a.chunk) == 0;
    z1 |= ((j0 + 32 + lane + 1) % a.chunk) == 0;
  }
  const uint32_t m0 = __ballot_sync(0xffffffffu, z0), m1 = __ballot_sync(0xffffffffu, z1);
  return static_cast<unsigned long long>(m0) | (static_cast<unsigned long long>(m1) << 32);
}

// delta[r] = dO_r . O_r - dlse_r; one warp per row, 4 dims per lane
__global__ void __launch_bounds__(256) delta_kernel(const __nv_bfloat16* __restrict__ out,
                                                    const __nv_bfloat16* __restrict__ dout,
                                                    const float* __restrict__ dlse, float* __restrict__ delta,
                                                    int64_t rows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (row >= rows) return;
  const uint2 o = *reinterpret_cast<const uint2*>(out + row * D + 4 * lane);
  const uint2 g = *reinterpret_cast<const uint2*>(dout + row * D + 4 * lane);
  const float2 o0 = unpack_bf16x2(o.x), o1 = unpack_bf16x2(o.y), g0 = unpack_bf16x2(g.x), g1 = unpack_bf16x2(g.y);
  float s = o0.x * g0.x + o0.y * g0.y + o1.x * g1.x + o1.y * g1.y;
  s = warp_sum(s);
  if (lane == 0) delta[row] = s - (dlse != nullptr ? dlse[row] : 0.f);
}

// ============================================================ dK / dV
// One CTA per 64-key block and KV head walks the query tiles of its band.  Two
// row groups (warps 4-7 and 8-11) take the even and the odd tiles, each with
// its own MMA warp (1 and 2), Q/dO stage, P/dS buffers and S, dP, dV^T, dK^T
// accumulators in TMEM, so the two groups' tiles overlap; the epilogue adds
// the groups' accumulators in a fixed order.
constexpr int DKV_THREADS = 384;             // warp 0 loads, warps 1-2 issue MMAs, warps 4-11 two row groups

struct __align__(1024) DkvSmem {
  unsigned char kt[16384];                   // the block's K tile (loaded once), [half][64 keys][64 dims]
  unsigned char vt[16384];                   // and V tile
  struct Stage {
    unsigned char qt[PT * 2048];             // 16 queries x [half][8 head rows][64 dims]
    unsigned char ot[PT * 2048];             // their dO rows
  } st[2];                                   // group g's tiles use stage g
  unsigned char wp[2][16384];                // bf16(P) of each group [128 rows x 64 keys], 128-byte swizzled rows
  unsigned char dsb[2][16384];               // dS, same layout
  uint64_t bar_kv, bar_full[2], bar_free[2], bar_sdone[2], bar_pready[2], bar_done[2];
  int last[2];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(DkvSmem) + 1024 <= 232448, "local dK/dV shared memory over budget");

__global__ void __launch_bounds__(DKV_THREADS, 1) local_dkv_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                                   const __grid_constant__ CUtensorMap tm_v,
                                                                   const __grid_constant__ CUtensorMap tm_q,
                                                                   const __grid_constant__ CUtensorMap tm_do,
                                                                   LocalBwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  DkvSmem& sm = *reinterpret_cast<DkvSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G, Hq = a.Hkv * a.G, W = a.window;
  const int64_t j0 = static_cast<int64_t>(c) * KB;                 // first key of the block (in the sequence)
  const int64_t q_start = j0 - W > 0 ? j0 - W : 0;
  const int64_t q_end = j0 + KB + W < a.L ? j0 + KB + W : a.L;      // exclusive
  const int n_tiles = static_cast<int>((q_end - q_start + PT - 1) / PT);
  const int64_t krow0 = static_cast<int64_t>(b) * a.L + j0;

  // query rows past the band's end stay zero (their P and dS are zero, but a
  // NaN from stale shared memory would still reach dK through Q^T . dS)
  for (int e = tid; e < 2 * static_cast<int>(sizeof(DkvSmem::Stage)) / 16; e += DKV_THREADS)
    reinterpret_cast<uint4*>(&sm.st[0])[e] = make_uint4(0u, 0u, 0u, 0u);
  for (int e = tid; e < 4 * 16384 / 16; e += DKV_THREADS) reinterpret_cast<uint4*>(&sm.wp[0][0])[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    tc::mbar_init(su32(&sm.bar_kv), 1);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(su32(&sm.bar_full[s]), 1);
      tc::mbar_init(su32(&sm.bar_free[s]), 1);
      tc::mbar_init(su32(&sm.bar_sdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_pready[s]), 4);
      tc::mbar_init(su32(&sm.bar_done[s]), 1);
      sm.last[s] = -1;
    }
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(su32(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  const unsigned long long zm = zeroed_keys(a, b, j0, lane);
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base;
  int* abf = &sm.abort_flag;
  // TMEM columns: S of group g at 64 g, dP at 128 + 64 g, dV^T_g at 256 + 128 g, dK^T_g at 320 + 128 g
  constexpr uint32_t kS = 0, kDP = 128, kDV = 256, kDK = 320;

  if (warp == 0) {
    // ============================ loader =====================================
    if (lane == 0) {
      tc::prefetch_tensormap(&tm_q);
      tc::prefetch_tensormap(&tm_do);
      tc::mbar_arrive_expect_tx(su32(&sm.bar_kv), 32768u);
      tc::tma_load_4d(su32(sm.kt), &tm_k, 0, static_cast<int>(krow0), 0, hk, su32(&sm.bar_kv));
      tc::tma_load_4d(su32(sm.vt), &tm_v, 0, static_cast<int>(krow0), 0, hk, su32(&sm.bar_kv));
    }
    __syncwarp();
    for (int t = 0; t < n_tiles; ++t) {
      const int g2 = t & 1;
      const int64_t l0 = q_start + static_cast<int64_t>(t) * PT;
      const int nq = static_cast<int>(q_end - l0 < PT ? q_end - l0 : PT);
      // group g2's stage was last read by the gradient MMAs of tile t-2
      if (t >= 2 && !wait_ab_warp(&sm.bar_free[g2], ((t >> 1) - 1) & 1, abf)) break;
      if (lane == 0) tc::mbar_arrive_expect_tx(su32(&sm.bar_full[g2]), static_cast<uint32_t>(nq) * 4096u);
      __syncwarp();
      if (lane < nq) {
        const int qy = static_cast<int>((static_cast<int64_t>(b) * a.L + l0 + lane) * Hq + hk * G);
        tc::tma_load_3d(su32(sm.st[g2].qt + lane * 2048), &tm_q, 0, qy, 0, su32(&sm.bar_full[g2]));
        tc::tma_load_3d(su32(sm.st[g2].ot + lane * 2048), &tm_do, 0, qy, 0, su32(&sm.bar_full[g2]));
      }
      if (lane == 0) sm.last[g2] = t;
    }
    __syncwarp();
    if (lane == 0) {
      tc::mbar_wait(su32(&sm.bar_kv), 0);
      for (int s2 = 0; s2 < 2; ++s2)
        if (sm.last[s2] >= 0) tc::mbar_wait(su32(&sm.bar_full[s2]), (sm.last[s2] >> 1) & 1);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ============================ MMA issue (one warp per row group) =========
    const int g2 = warp - 1;                      // tiles t with t % 2 == g2
    constexpr uint32_t id_s = tc::idesc_bf16_f32(128, 64, 0, 0);
    constexpr uint32_t id_g = tc::idesc_bf16_f32(128, 64, 1, 1);    // MN-major A and B
    const uint64_t dk = tc::smem_desc_sw128(su32(sm.kt), 16, 1024);
    const uint64_t dv = tc::smem_desc_sw128(su32(sm.vt), 16, 1024);
    const uint64_t dq = tc::smem_desc_sw128(su32(sm.st[g2].qt), 16, 2048);      // Q rows, K-major
    const uint64_t dob = tc::smem_desc_sw128(su32(sm.st[g2].ot), 16, 2048);
    const uint64_t dqm = tc::smem_desc_sw128(su32(sm.st[g2].qt), 1024, 2048);   // Q^T, MN-major
    const uint64_t dom = tc::smem_desc_sw128(su32(sm.st[g2].ot), 1024, 2048);
    // [rows x keys] as an MN-major B: N = 64 keys is one swizzle atom wide, so
    // only the 8-row stride (1024 B) matters; both offset fields carry it
    const uint64_t dwp = tc::smem_desc_sw128(su32(sm.wp[g2]), 1024, 1024);
    const uint64_t dds = tc::smem_desc_sw128(su32(sm.dsb[g2]), 1024, 1024);
    const uint32_t tS = tbase + kS + 64 * g2, tP = tbase + kDP + 64 * g2;
    const uint32_t tV = tbase + kDV + 128 * g2, tK = tbase + kDK + 128 * g2;
    bool ok = wait_ab_warp(&sm.bar_kv, 0, abf);
    tc::fence_after_sync();
    for (int t = g2; ok && t < n_tiles; t += 2) {
      if (!(ok = wait_ab_warp(&sm.bar_full[g2], (t >> 1) & 1, abf))) break;
      tc::fence_after_sync();
      // S and dP of tile t (the group's previous P, dS and S reads all precede:
      // its gradient MMAs were issued before, in order, and its rows read S, dP
      // before signalling P and dS ready)
      if (tc::elect_one()) {
        tc::mma_bf16<false>(tS, dq, dk, id_s);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          tc::mma_bf16<true>(tS, adv(dq, (kk >> 2) * 1024 + (kk & 3) * 32), adv(dk, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
        tc::mma_bf16<false>(tP, dob, dv, id_s);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          tc::mma_bf16<true>(tP, adv(dob, (kk >> 2) * 1024 + (kk & 3) * 32), adv(dv, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
        tc::mma_commit(su32(&sm.bar_sdone[g2]));
      }
      __syncwarp();
      // dV^T_g += dO^T . P and dK^T_g += Q^T . dS of tile t
      if (!(ok = wait_ab_warp(&sm.bar_pready[g2], (t >> 1) & 1, abf))) break;
      tc::fence_after_sync();
      if (tc::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const bool acc = t > g2 || kk > 0;
          tc::mma_bf16_ss(tV, adv(dom, kk * 4096), adv(dwp, kk * 2048), id_g, acc);
          tc::mma_bf16_ss(tK, adv(dqm, kk * 4096), adv(dds, kk * 2048), id_g, acc);
        }
        tc::mma_commit(su32(&sm.bar_free[g2]));
      }
      __syncwarp();
    }
    if (tc::elect_one()) tc::mma_commit(su32(&sm.bar_done[g2]));
    __syncwarp();
  } else if (warp >= 4) {
    // ============================ rows (two groups, one tile row per thread) =
    const int grp = (warp - 4) >> 2;              // tiles t with t % 2 == grp
    const int r = (warp & 3) * 32 + lane, pq = r >> 3, g = r & 7;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float sl2 = a.sm_scale * kLog2e;
    for (int t = grp; t < n_tiles; t += 2) {
      const int64_t l = q_start + static_cast<int64_t>(t) * PT + pq;
      const bool row_on = l < q_end && g < G;
      float lse_l2 = 0.f, delta = 0.f;
      if (row_on) {
        const int64_t ri = (static_cast<int64_t>(b) * a.L + l) * Hq + hk * G + g;
        lse_l2 = a.lse[ri] * kLog2e;
        delta = a.delta[ri];
      }
      if (!wait_ab_warp(&sm.bar_sdone[grp], (t >> 1) & 1, abf)) break;
      tc::fence_after_sync();
      const int64_t rel = l - j0;                   // query position - first key of the block
      // every key of the block in this row's band and none zeroed: no per-key tests
      const bool dense = row_on && zm == 0ull && rel <= W && rel - (KB - 1) >= -W;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32], y[32];
        tc::tmem_ld16(tbase + lane_off + kS + 64 * grp + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(&x[0]));
        tc::tmem_ld16(tbase + lane_off + kS + 64 * grp + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(&x[16]));
        tc::tmem_ld16(tbase + lane_off + kDP + 64 * grp + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(&y[0]));
        tc::tmem_ld16(tbase + lane_off + kDP + 64 * grp + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(&y[16]));
        tc::tmem_wait_ld();
        uint32_t pw[16], dsv[16];
        if (dense) {
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(x[2 * h]), sl2, -lse_l2));
            const float p1 = fast_exp2(fmaf(__uint_as_float(x[2 * h + 1]), sl2, -lse_l2));
            pw[h] = pack_bf16x2(p0, p1);
            dsv[h] = pack_bf16x2(p0 * (__uint_as_float(y[2 * h]) - delta), p1 * (__uint_as_float(y[2 * h + 1]) - delta));
          }
        } else {
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            float p2[2], d2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int s = 32 * half + 2 * h + e;
              const int64_t dist = rel - s;
              const bool zero = (zm >> s) & 1ull;
              const bool live = row_on && dist <= W && -dist <= W;
              const float sv = zero ? 0.f : __uint_as_float(x[2 * h + e]);
              const float p = live ? fast_exp2(fmaf(sv, sl2, -lse_l2)) : 0.f;
              const float dp = zero ? 0.f : __uint_as_float(y[2 * h + e]);
              p2[e] = p;
              d2[e] = p * (dp - delta);
            }
            pw[h] = pack_bf16x2(p2[0], p2[1]);
            dsv[h] = pack_bf16x2(d2[0], d2[1]);
          }
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          *reinterpret_cast<uint4*>(sm.wp[grp] + swz_off(r, 4 * half + p)) =
              make_uint4(pw[4 * p], pw[4 * p + 1], pw[4 * p + 2], pw[4 * p + 3]);
          *reinterpret_cast<uint4*>(sm.dsb[grp] + swz_off(r, 4 * half + p)) =
              make_uint4(dsv[4 * p], dsv[4 * p + 1], dsv[4 * p + 2], dsv[4 * p + 3]);
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_pready[grp]));
    }
    // ============================ epilogue: dK, dV (fp32) ====================
    // dV = dV_0 + dV_1, dK = dK_0 + dK_1 (a group without tiles never wrote its
    // accumulators); group grp writes keys [32 grp, 32 grp + 32)
    const bool has1 = n_tiles > 1;
    bool ok = wait_ab_warp(&sm.bar_done[0], 0, abf);
    if (ok) ok = wait_ab_warp(&sm.bar_done[1], 0, abf);
    tc::fence_after_sync();
    if (ok && !__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(abf) != 0)) {
      const int d = (warp & 3) * 32 + lane;
#pragma unroll 1
      for (int s0 = 32 * grp; s0 < 32 * grp + 32; s0 += 16) {
        uint32_t v0[16], k0[16], v1[16], k1[16];
        tc::tmem_ld16(tbase + lane_off + kDV + s0, v0);
        tc::tmem_ld16(tbase + lane_off + kDK + s0, k0);
        if (has1) {
          tc::tmem_ld16(tbase + lane_off + kDV + 128 + s0, v1);
          tc::tmem_ld16(tbase + lane_off + kDK + 128 + s0, k1);
        }
        tc::tmem_wait_ld();
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          const bool zero = (zm >> (s0 + s)) & 1ull;
          const int64_t o = ((krow0 + s0 + s) * a.Hkv + hk) * D + d;
          const float vv = has1 ? __uint_as_float(v0[s]) + __uint_as_float(v1[s]) : __uint_as_float(v0[s]);
          const float kv = has1 ? __uint_as_float(k0[s]) + __uint_as_float(k1[s]) : __uint_as_float(k0[s]);
          a.dv[o] = zero ? 0.f : vv;
          a.dk[o] = zero ? 0.f : a.sm_scale * kv;
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && sm.abort_flag) atomicOr(&g_local_bwd_error, 1);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ============================================================ dQ
// One CTA per 16-query tile and KV head walks the key blocks of its band.
// Two row groups (warps 4-7 and 8-11) take the even and the odd blocks, each
// with its own MMA warp (1 and 2), S / dP buffers and dQ accumulator in TMEM
// and dS buffer in shared memory: a group's MMA warp issues S and dP of block
// t+2 as soon as block t's have been read into registers, then dQ_g +=
// dS(t) . K(t) once its dS is stored, so neither group waits for an MMA round
// trip or for the other group.  The epilogue adds the two accumulators in a
// fixed order.  K/V blocks use three stages.
constexpr int DQ_THREADS = 384;              // warp 0 loads, warps 1-2 issue MMAs, warps 4-11 two row groups
constexpr int DQ_NST = 3;                    // K/V stages

struct __align__(1024) DqSmem {
  unsigned char qt[PT * 2048];               // the tile's 16 queries x 8 head rows (loaded once)
  unsigned char ot[PT * 2048];               // their dO rows
  struct Stage {
    unsigned char kt[16384];                 // K tile of one 64-key block, [half][64 keys][64 dims]
    unsigned char vt[16384];                 // V tile
  } st[DQ_NST];
  unsigned char ds[2][16384];                // dS of each group [128 rows x 64 keys] bf16, 128-byte swizzled rows
  unsigned long long zm[DQ_NST];             // zeroed keys of the block in each stage
  uint64_t bar_q, bar_full[DQ_NST], bar_free[DQ_NST], bar_zm[DQ_NST];
  uint64_t bar_sdone[2], bar_sfree[2], bar_pready[2], bar_pvdone[2];
  uint64_t bar_done[2];
  int last[DQ_NST];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(DqSmem) + 1024 <= 232448, "local dQ shared memory over budget");

__global__ void __launch_bounds__(DQ_THREADS, 1) local_dq_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                                 const __grid_constant__ CUtensorMap tm_v,
                                                                 const __grid_constant__ CUtensorMap tm_q,
                                                                 const __grid_constant__ CUtensorMap tm_do,
                                                                 LocalBwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  DqSmem& sm = *reinterpret_cast<DqSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G, Hq = a.Hkv * a.G, W = a.window;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * PT;
  const int nq = static_cast<int>(a.L - q0 < PT ? a.L - q0 : PT);
  const int64_t k_lo = q0 - W > 0 ? q0 - W : 0;
  const int64_t k_hi = q0 + nq - 1 + W < a.L - 1 ? q0 + nq - 1 + W : a.L - 1;   // inclusive
  const int kb0 = static_cast<int>(k_lo / KB), n_blocks = static_cast<int>(k_hi / KB) - kb0 + 1;

  for (int e = tid; e < 2 * PT * 2048 / 16; e += DQ_THREADS) reinterpret_cast<uint4*>(sm.qt)[e] = make_uint4(0u, 0u, 0u, 0u);
  for (int e = tid; e < 2 * 16384 / 16; e += DQ_THREADS) reinterpret_cast<uint4*>(&sm.ds[0][0])[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    tc::mbar_init(su32(&sm.bar_q), 1);
    for (int s = 0; s < DQ_NST; ++s) {
      tc::mbar_init(su32(&sm.bar_full[s]), 1);
      tc::mbar_init(su32(&sm.bar_free[s]), 1);
      tc::mbar_init(su32(&sm.bar_zm[s]), 1);
      sm.last[s] = -1;
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(su32(&sm.bar_sdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_sfree[s]), 4);
      tc::mbar_init(su32(&sm.bar_pready[s]), 4);
      tc::mbar_init(su32(&sm.bar_pvdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_done[s]), 1);
    }
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(su32(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base;
  int* abf = &sm.abort_flag;
  // TMEM columns: S of group g at 64 g, dP at 128 + 64 g, dQ_g at 256 + 128 g
  constexpr uint32_t kS = 0, kDP = 128, kDQ = 256;

  if (warp == 0) {
    // ============================ loader =====================================
    if (lane == 0) {
      tc::prefetch_tensormap(&tm_k);
      tc::prefetch_tensormap(&tm_v);
      tc::mbar_arrive_expect_tx(su32(&sm.bar_q), static_cast<uint32_t>(nq) * 4096u);
    }
    __syncwarp();
    if (lane < nq) {
      const int qy = static_cast<int>((static_cast<int64_t>(b) * a.L + q0 + lane) * Hq + hk * G);
      tc::tma_load_3d(su32(sm.qt + lane * 2048), &tm_q, 0, qy, 0, su32(&sm.bar_q));
      tc::tma_load_3d(su32(sm.ot + lane * 2048), &tm_do, 0, qy, 0, su32(&sm.bar_q));
    }
    // key-validity bytes of block tt (this lane's keys 32h + lane), requested one
    // block ahead so their latency is not on the copy-issue path
    auto valid_bytes = [&](int tt, uint32_t (&vb)[2]) {
      const int64_t jt = static_cast<int64_t>(kb0 + tt) * KB;
#pragma unroll
      for (int h = 0; h < 2; ++h)
        vb[h] = (a.key_valid != nullptr && tt < n_blocks) ? a.key_valid[b * a.L + jt + 32 * h + lane] : 1u;
    };
    uint32_t vb_next[2];
    valid_bytes(0, vb_next);
    for (int t = 0; t < n_blocks; ++t) {
      const int st = t % DQ_NST;
      const int64_t j0 = static_cast<int64_t>(kb0 + t) * KB;
      const uint32_t vb[2] = {vb_next[0], vb_next[1]};
      valid_bytes(t + 1, vb_next);
      // stage st was last read by the dQ MMAs of block t - DQ_NST, and its zeroed-key
      // word by that block's rows, which precede those MMAs
      if (t >= DQ_NST && !wait_ab_warp(&sm.bar_free[st], ((t / DQ_NST) - 1) & 1, abf)) break;
      bool z0 = vb[0] == 0u, z1 = vb[1] == 0u;
      if (a.skip_inert) {
        z0 |= ((j0 + lane + 1) % a.chunk) == 0;
        z1 |= ((j0 + 32 + lane + 1) % a.chunk) == 0;
      }
      const unsigned long long zm = static_cast<unsigned long long>(__ballot_sync(0xffffffffu, z0)) |
                                    (static_cast<unsigned long long>(__ballot_sync(0xffffffffu, z1)) << 32);
      if (lane == 0) {
        sm.zm[st] = zm;
        tc::mbar_arrive(su32(&sm.bar_zm[st]));
        const int krow = static_cast<int>(static_cast<int64_t>(b) * a.L + j0);
        tc::mbar_arrive_expect_tx(su32(&sm.bar_full[st]), 32768u);
        tc::tma_load_4d(su32(sm.st[st].kt), &tm_k, 0, krow, 0, hk, su32(&sm.bar_full[st]));
        tc::tma_load_4d(su32(sm.st[st].vt), &tm_v, 0, krow, 0, hk, su32(&sm.bar_full[st]));
        sm.last[st] = t;
      }
      __syncwarp();
    }
    __syncwarp();
    if (lane == 0) {
      tc::mbar_wait(su32(&sm.bar_q), 0);
      for (int s2 = 0; s2 < DQ_NST; ++s2)
        if (sm.last[s2] >= 0) tc::mbar_wait(su32(&sm.bar_full[s2]), (sm.last[s2] / DQ_NST) & 1);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ============================ MMA issue (one warp per row group) =========
    const int g2 = warp - 1;                      // this warp's group: blocks t with t % 2 == g2
    constexpr uint32_t id_s = tc::idesc_bf16_f32(128, 64, 0, 0);
    constexpr uint32_t id_q = tc::idesc_bf16_f32(128, 128, 0, 1);   // dS K-major, K as an MN-major B
    constexpr uint32_t kStageBytes = sizeof(DqSmem::Stage);
    const uint64_t dq = tc::smem_desc_sw128(su32(sm.qt), 16, 2048);
    const uint64_t dob = tc::smem_desc_sw128(su32(sm.ot), 16, 2048);
    const uint64_t dk0 = tc::smem_desc_sw128(su32(sm.st[0].kt), 16, 1024);
    const uint64_t dv0 = tc::smem_desc_sw128(su32(sm.st[0].vt), 16, 1024);
    const uint64_t dkm0 = tc::smem_desc_sw128(su32(sm.st[0].kt), 8192, 1024);   // N = dims: halves 8 KB apart
    const uint64_t dds0 = tc::smem_desc_sw128(su32(sm.ds[0]), 16, 1024);
    bool ok = wait_ab_warp(&sm.bar_q, 0, abf);
    tc::fence_after_sync();
    // S and dP of block t into its group's TMEM buffers
    auto issue_s = [&](int t) -> bool {
      const int st = t % DQ_NST;
      if (!wait_ab_warp(&sm.bar_full[st], (t / DQ_NST) & 1, abf)) return false;
      if (t >= 2 && !wait_ab_warp(&sm.bar_sfree[g2], ((t >> 1) - 1) & 1, abf)) return false;
      tc::fence_after_sync();
      const uint32_t so = st * kStageBytes;
      const uint64_t dk = adv(dk0, so), dv = adv(dv0, so);
      if (tc::elect_one()) {
        const uint32_t tS = tbase + kS + 64 * g2, tP = tbase + kDP + 64 * g2;
        tc::mma_bf16<false>(tS, dq, dk, id_s);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          tc::mma_bf16<true>(tS, adv(dq, (kk >> 2) * 1024 + (kk & 3) * 32), adv(dk, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
        tc::mma_bf16<false>(tP, dob, dv, id_s);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          tc::mma_bf16<true>(tP, adv(dob, (kk >> 2) * 1024 + (kk & 3) * 32), adv(dv, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
        tc::mma_commit(su32(&sm.bar_sdone[g2]));
      }
      __syncwarp();
      return true;
    };
    // dQ_g += dS(t) . K(t)
    auto dq_part = [&](int t) -> bool {
      const int st = t % DQ_NST;
      if (!wait_ab_warp(&sm.bar_pready[g2], (t >> 1) & 1, abf)) return false;
      tc::fence_after_sync();
      const uint64_t da = adv(dds0, g2 * 16384), dbk = adv(dkm0, st * kStageBytes);
      if (tc::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_bf16_ss(tbase + kDQ + 128 * g2, adv(da, kk * 32), adv(dbk, kk * 2048), id_q, t > g2 || kk > 0);
        tc::mma_commit(su32(&sm.bar_pvdone[g2]));
        tc::mma_commit(su32(&sm.bar_free[st]));
      }
      __syncwarp();
      return true;
    };
    if (ok && g2 < n_blocks) ok = issue_s(g2);
    for (int t = g2; ok && t < n_blocks; t += 2) {
      // S(t+2) as soon as block t's S and dP are in registers, then block t's dQ part
      if (t + 2 < n_blocks && !(ok = issue_s(t + 2))) break;
      ok = dq_part(t);
    }
    if (tc::elect_one()) tc::mma_commit(su32(&sm.bar_done[g2]));
    __syncwarp();
  } else if (warp >= 4) {
    // ============================ rows (two groups, one tile row per thread) =
    const int grp = (warp - 4) >> 2;              // blocks t with t % 2 == grp
    const int r = (warp & 3) * 32 + lane, pq = r >> 3, g = r & 7;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float sl2 = a.sm_scale * kLog2e;
    const int64_t l = q0 + pq;
    const bool row_on = pq < nq && g < G;
    float lse_l2 = 0.f, delta = 0.f;
    if (row_on) {
      const int64_t ri = (static_cast<int64_t>(b) * a.L + l) * Hq + hk * G + g;
      lse_l2 = a.lse[ri] * kLog2e;
      delta = a.delta[ri];
    }
    bool okr = true;
    for (int t = grp; t < n_blocks; t += 2) {
      const int st = t % DQ_NST;
      const int64_t j0 = static_cast<int64_t>(kb0 + t) * KB;
      if (!(okr = wait_ab_warp(&sm.bar_zm[st], (t / DQ_NST) & 1, abf))) break;
      const unsigned long long zm = sm.zm[st];
      if (!(okr = wait_ab_warp(&sm.bar_sdone[grp], (t >> 1) & 1, abf))) break;
      tc::fence_after_sync();
      const int64_t rel = l - j0;                   // query position - first key of the block
      // every column of the block in this row's band and no zeroed key: no per-key tests
      const bool dense = row_on && zm == 0ull && rel <= W && rel - (KB - 1) >= -W;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32], y[32];
        tc::tmem_ld16(tbase + lane_off + kS + 64 * grp + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(&x[0]));
        tc::tmem_ld16(tbase + lane_off + kS + 64 * grp + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(&x[16]));
        tc::tmem_ld16(tbase + lane_off + kDP + 64 * grp + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(&y[0]));
        tc::tmem_ld16(tbase + lane_off + kDP + 64 * grp + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(&y[16]));
        tc::tmem_wait_ld();
        if (half == 1) {
          // both halves of S and dP are in registers: the buffers take block t+2
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(su32(&sm.bar_sfree[grp]));
        }
        uint32_t dsv[16];
        if (dense) {
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(x[2 * h]), sl2, -lse_l2));
            const float p1 = fast_exp2(fmaf(__uint_as_float(x[2 * h + 1]), sl2, -lse_l2));
            dsv[h] = pack_bf16x2(p0 * (__uint_as_float(y[2 * h]) - delta), p1 * (__uint_as_float(y[2 * h + 1]) - delta));
          }
        } else {
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            float d2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int s = 32 * half + 2 * h + e;
              const int64_t dist = rel - s;
              const bool zero = (zm >> s) & 1ull;
              const bool live = row_on && dist <= W && -dist <= W;
              const float sv = zero ? 0.f : __uint_as_float(x[2 * h + e]);
              const float p = live ? fast_exp2(fmaf(sv, sl2, -lse_l2)) : 0.f;
              const float dp = zero ? 0.f : __uint_as_float(y[2 * h + e]);
              // zeroed keys contribute nothing to dQ (k' = 0 there)
              d2[e] = zero ? 0.f : p * (dp - delta);
            }
            dsv[h] = pack_bf16x2(d2[0], d2[1]);
          }
        }
        // dS(t) overwrites dS(t-2) once that block's dQ MMAs completed
        if (half == 0 && t >= 2 && !(okr = wait_ab_warp(&sm.bar_pvdone[grp], ((t >> 1) - 1) & 1, abf))) break;
#pragma unroll
        for (int p = 0; p < 4; ++p)
          *reinterpret_cast<uint4*>(sm.ds[grp] + swz_off(r, 4 * half + p)) =
              make_uint4(dsv[4 * p], dsv[4 * p + 1], dsv[4 * p + 2], dsv[4 * p + 3]);
      }
      if (!okr) break;
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_pready[grp]));
    }
    // ============================ epilogue: dQ (fp32) ========================
    // dQ = dQ_0 + dQ_1 (a group without blocks never wrote its accumulator);
    // group grp writes dims [64 grp, 64 grp + 64) of the tile's rows
    const bool has1 = n_blocks > 1;
    bool ok = wait_ab_warp(&sm.bar_done[0], 0, abf);
    if (ok) ok = wait_ab_warp(&sm.bar_done[1], 0, abf);
    tc::fence_after_sync();
    if (ok && !__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(abf) != 0)) {
      float* dst = row_on ? a.dq + ((static_cast<int64_t>(b) * a.L + l) * Hq + hk * G + g) * D : nullptr;
#pragma unroll 1
      for (int c0 = 64 * grp; c0 < 64 * grp + 64; c0 += 16) {
        uint32_t v0[16], v1[16];
        tc::tmem_ld16(tbase + lane_off + kDQ + c0, v0);
        if (has1) tc::tmem_ld16(tbase + lane_off + kDQ + 128 + c0, v1);
        tc::tmem_wait_ld();
        if (dst != nullptr) {
          float f[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            f[i] = a.sm_scale * (has1 ? __uint_as_float(v0[i]) + __uint_as_float(v1[i]) : __uint_as_float(v0[i]));
#pragma unroll
          for (int p = 0; p < 4; ++p)
            reinterpret_cast<float4*>(dst + c0)[p] = make_float4(f[4 * p], f[4 * p + 1], f[4 * p + 2], f[4 * p + 3]);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && sm.abort_flag) atomicOr(&g_local_bwd_error, 2);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

}  // namespace

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool make_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
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
                  strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

namespace mrsa {
int local_bwd_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_local_bwd_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_local_bwd_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
}  // namespace mrsa

extern "C" size_t mrsa_local_attention_backward_workspace(int64_t batch, int64_t seq_len, int64_t q_heads) {
  if (batch < 1 || seq_len < 0 || q_heads < 1) return 0;
  return static_cast<size_t>(batch * seq_len * q_heads) * sizeof(float);
}

extern "C" int mrsa_local_attention_backward(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                                             const void* out, const float* lse, const void* grad_out,
                                             const float* grad_lse, float* dq, float* dk, float* dv, void* workspace,
                                             size_t ws_bytes, int64_t window, int skip_inert, int64_t chunk,
                                             float sm_scale, int64_t batch, int64_t seq_len, int64_t q_heads,
                                             int64_t kv_heads, int64_t head_dim, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  if (!q || !k || !v || !out || !lse || !grad_out || !dq || !dk || !dv) return MRSA_ERR_NULL;
  if (head_dim != D || batch < 1 || seq_len < KB || seq_len % KB || kv_heads < 1 || q_heads % kv_heads ||
      q_heads / kv_heads > GMAX || chunk < 1 || batch > 65535 || kv_heads > 65535 ||
      batch * seq_len * q_heads > 0x7fffffffLL || seq_len / PT > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if (window < 0 || window > (1LL << 30) || !(sm_scale > 0.f)) return MRSA_ERR_ARG;
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out) |
                       reinterpret_cast<uintptr_t>(grad_out) | reinterpret_cast<uintptr_t>(dq) |
                       reinterpret_cast<uintptr_t>(workspace);
  if (al & 15u) return MRSA_ERR_ALIGN;
  if (workspace == nullptr || ws_bytes < mrsa_local_attention_backward_workspace(batch, seq_len, q_heads))
    return MRSA_ERR_WORKSPACE;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  CUtensorMap tm_k, tm_v, tm_q, tm_do;
  const cuuint64_t kv_dims[4] = {64, static_cast<cuuint64_t>(batch * seq_len), 2, static_cast<cuuint64_t>(kv_heads)};
  const cuuint64_t kv_str[3] = {static_cast<cuuint64_t>(kv_heads * D * 2), 128, 256};
  const cuuint32_t kv_box[4] = {64, 64, 2, 1};
  const cuuint64_t q_dims[3] = {64, static_cast<cuuint64_t>(batch * seq_len * q_heads), 2};
  const cuuint64_t q_str[2] = {256, 128};
  const cuuint32_t q_box[3] = {64, 8, 2};
  if (!make_map(&tm_k, k, 4, kv_dims, kv_str, kv_box) || !make_map(&tm_v, v, 4, kv_dims, kv_str, kv_box) ||
      !make_map(&tm_q, q, 3, q_dims, q_str, q_box) || !make_map(&tm_do, grad_out, 3, q_dims, q_str, q_box)) {
    mrsa::note_cuda_error(cudaErrorInvalidValue, "mrsa_local_attention_backward: tensor map encoding");
    return MRSA_ERR_LAUNCH;
  }
  float* delta = static_cast<float*>(workspace);
  const int64_t rows = batch * seq_len * q_heads;
  delta_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(out),
                                                                     static_cast<const __nv_bfloat16*>(grad_out),
                                                                     grad_lse, delta, rows);
  MRSA_CHECK_LAUNCH();
  LocalBwdArgs a;
  a.key_valid = key_valid;
  a.lse = lse;
  a.delta = delta;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.sm_scale = sm_scale;
  a.L = seq_len;
  a.Hkv = static_cast<int>(kv_heads);
  a.G = static_cast<int>(q_heads / kv_heads);
  a.window = static_cast<int>(window);
  a.skip_inert = skip_inert ? 1 : 0;
  a.chunk = static_cast<int>(chunk);
  const size_t smem_kv = sizeof(DkvSmem) + 1024, smem_q = sizeof(DqSmem) + 1024;
  if (const cudaError_t e = cudaFuncSetAttribute(local_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem_kv));
      e != cudaSuccess) {
    mrsa::note_cuda_error(e, "mrsa_local_attention_backward: shared-memory opt-in");
    return MRSA_ERR_LAUNCH;
  }
  if (const cudaError_t e = cudaFuncSetAttribute(local_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem_q));
      e != cudaSuccess) {
    mrsa::note_cuda_error(e, "mrsa_local_attention_backward: shared-memory opt-in");
    return MRSA_ERR_LAUNCH;
  }
  local_dkv_kernel<<<dim3(static_cast<unsigned>(seq_len / KB), static_cast<unsigned>(kv_heads),
                          static_cast<unsigned>(batch)),
                     DKV_THREADS, smem_kv, s>>>(tm_k, tm_v, tm_q, tm_do, a);
  MRSA_CHECK_LAUNCH();
  local_dq_kernel<<<dim3(static_cast<unsigned>((seq_len + PT - 1) / PT), static_cast<unsigned>(kv_heads),
                         static_cast<unsigned>(batch)),
                    DQ_THREADS, smem_q, s>>>(tm_k, tm_v, tm_q, tm_do, a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
