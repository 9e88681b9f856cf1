// Selected-chunk attention backward on the 5th-generation tensor cores.
//
// Semantics: the reference's backward of HiLS_block_M_head
// (ops/hils_fwd_bwd_head.py:573-910; autograd of the torch reference
// hils_torch_ref :21-93).  For row r = (query l, head hq) and a selected chunk
// c = indices[l, h, k] (slot k, route weight w = W[l, hq, k]), with
//   P[r, s]  = softmax_s(q_r . K[c, s] * scale) over the chunk's usable keys
//   dP[r, s] = dO_r . V[c, s]
//   di_r     = sum_s P[r, s] dP[r, s]                      -> dW[l, hq, k]
//   dS[r, s] = bf16(scale * w * P[r, s] * (dP[r, s] - di_r))
//   dQ_r    += dS_r . K[c]
//   dK[c]   += dS^T . Q,   dV[c] += bf16(w * P)^T . dO        (fp32 sums)
// Two kernels, independent of each other:
//  * dq_kernel walks the forward's items -- per CTA 32 queries of one KV head,
//    per item one chunk and up to 8 of those queries ("owners"):
//      S  [64 x 64]  = Q_own . K^T      dP [64 x 64] = dO_own . V^T   (M=64)
//      softmax warps: P, di (-> dW), dS (bf16, to shared memory)
//      dQ_part^T [128 x 8n] = K^T . dS^T                              (M=128)
//      accumulate warps: dQ^T[:, 8q..8q+7] += part (TMEM read-modify-write)
//    and writes dQ (fp32) once per CTA.
//  * dkv_kernel owns one chunk's 64 keys of one KV head and walks the
//    (query, slot) pairs that selected it (an inverted index built by
//    histogram / scan / place kernels, in query order), 16 pairs (128 rows) per tile:
//      S, dP [128 x 64] (M=128) -> rows warps: P, di, w*P and dS (bf16)
//      dV^T [128 x 64] += dO_tile^T . (w P),  dK^T += Q_tile^T . dS   (MN-major operands)
//    with two row groups on alternate tiles, each with its own MMA warp,
//    stage, buffers and accumulators (added in a fixed order at the end), and
//    stores dK, dV (fp32) for its 64 rows: no atomics on the gradients.
// A chunk listed twice by a query shares one softmax in the forward (its
// weights summed); here the first slot carries the summed weight in the dQ
// kernel, the dK/dV kernel sums the slots' contributions (linear in w), and
// dW_fixup_kernel copies di to the repeated slots and writes 0 for empty ones.
// Every mbarrier wait is bounded; an aborted CTA unwinds, waits (bounded) for
// its copies and MMAs in flight, frees its TMEM and sets bit 4 of
// mrsa_device_error_flags.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <utility>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int D = kHeadDim, S = kChunk, KMAX = 32;
constexpr int QB = 32, GMAX = 8, OWN = 8, NST = 2, RING = 16;
constexpr int NTHREADS_A = 512;
constexpr int W_SMX = 4, W_LOAD = 12, W_LOAD2 = 13, W_MMA = 14;   // MMA warps 14 (S, dP) and 15 (dQ part)
constexpr int kAccCols = QB * GMAX;          // 256
constexpr int kSCol = 256, kDPCol = 384;     // S buffers at 256/320 (later the dQ parts), dP at 384/448

__device__ int g_bwd_error;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ int swz_off(int row, int piece) { return row * 128 + ((piece ^ (row & 7)) << 4); }
__device__ __forceinline__ uint64_t adv(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 %%rx;\n\t.reg .pred %%px;\n\t"
      "elect.sync %%rx|%%px, %1;\n\t"
      "@%%px mov.s32 %0, 1;\n\t}\n"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// bounded wait taken by a whole warp that also gives up once another role of the CTA has aborted
__device__ __forceinline__ bool wait_ab_warp(uint64_t* bar, uint32_t parity, int* abort_flag) {
  return tc::wait_bounded_warp(su32(bar), parity, reinterpret_cast<volatile int*>(abort_flag));
}

struct BwdArgs {
  const __nv_bfloat16* w;
  const int32_t* indices;
  const uint8_t* key_valid;
  float *dq, *dk, *dv;
  __nv_bfloat16* dw;
  const int32_t *cnt, *off, *pairs;
  float sm_scale;
  int mask_last;
  int64_t Lq, Lk;
  int Hkv, G, K, C;
};

// ============================================================ dQ / dW kernel
struct ItemA {
  int n, u, c;
  uint8_t oq[OWN];
  uint8_t slot[OWN];
};

struct __align__(1024) SmemA {
  struct Stage {
    unsigned char kt[16384];      // K tile [half][64 keys][64 dims], 128-byte swizzled
    unsigned char vt[16384];      // V tile, same layout
    unsigned char qt[16384];      // owner query rows: 8 slots x [half][8 rows][64 dims]
    unsigned char ot[16384];      // owner dO rows, same layout
  } st[NST];
  unsigned char ds[2][8192];      // dS [64 rows x 64 keys] bf16, row 8j+g = owner j head g
  float w[QB][GMAX][KMAX];
  unsigned long long vmask[QB * KMAX];
  int2 ulist[QB * KMAX];
  ItemA ring[RING];
  uint64_t bar_full[NST], bar_free[NST];
  uint64_t bar_sdone[2], bar_pready[2], bar_pvdone[2], bar_partfree[2];
  uint64_t bar_ring[RING], bar_drain[2];
  int last[2][NST];
  uint32_t tmem_base;
  int nu, n_items, abort_flag;
};
static_assert(sizeof(SmemA) + 1024 <= 232448, "dQ kernel shared memory over budget");

__global__ void __launch_bounds__(NTHREADS_A, 1) dq_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                           const __grid_constant__ CUtensorMap tm_v,
                                                           const __grid_constant__ CUtensorMap tm_q,
                                                           const __grid_constant__ CUtensorMap tm_do, BwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SmemA& sm = *reinterpret_cast<SmemA*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * QB;
  const int G = a.G, K = a.K, C = a.C, Hq = a.Hkv * a.G;
  uint32_t* ownmask = reinterpret_cast<uint32_t*>(sm.st[0].qt);          // [C <= 2048]
  int (*idx)[KMAX + 1] = reinterpret_cast<int (*)[KMAX + 1]>(sm.st[1].qt);  // [QB][KMAX+1]

  // ---------------- set-up (the forward kernel's, plus zeroed dS buffers) ----
  if ((warp == W_LOAD || warp == W_LOAD2) && lane == 0) {
    tc::prefetch_tensormap(&tm_k);
    tc::prefetch_tensormap(&tm_v);
    tc::prefetch_tensormap(&tm_q);
    tc::prefetch_tensormap(&tm_do);
  }
  for (int e = tid; e < C; e += NTHREADS_A) ownmask[e] = 0u;
  for (int e = tid; e < 2 * 8192 / 16; e += NTHREADS_A) reinterpret_cast<uint4*>(&sm.ds[0][0])[e] = make_uint4(0u, 0u, 0u, 0u);
  for (int e = tid; e < QB * KMAX; e += NTHREADS_A) {
    const int qi = e / KMAX, kk = e % KMAX;
    int c = -1;
    if (kk < K && q0 + qi < a.Lq) {
      c = a.indices[((b * a.Lq + q0 + qi) * a.Hkv + hk) * K + kk];
      if (c >= C) c = -1;
    }
    idx[qi][kk] = c < 0 ? -1 : c;
  }
  for (int e = tid; e < QB * GMAX * KMAX; e += NTHREADS_A) {
    const int qi = e / (GMAX * KMAX), g = (e / KMAX) % GMAX, kk = e % KMAX;
    float wv = 0.f;
    if (g < G && kk < K && q0 + qi < a.Lq) wv = bf2f(a.w[((b * a.Lq + q0 + qi) * Hq + hk * G + g) * K + kk]);
    sm.w[qi][g][kk] = wv;
  }
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(su32(&sm.bar_full[s]), 1);
      tc::mbar_init(su32(&sm.bar_free[s]), 1);
      sm.last[0][s] = sm.last[1][s] = -1;
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(su32(&sm.bar_sdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_pready[s]), 4);
      tc::mbar_init(su32(&sm.bar_pvdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_partfree[s]), 4);
      tc::mbar_init(su32(&sm.bar_drain[s]), 1);
    }
    for (int r = 0; r < RING; ++r) tc::mbar_init(su32(&sm.bar_ring[r]), 1);
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(su32(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  __syncthreads();
  // repeated chunks: weights summed into the first slot (one softmax, as in the forward)
  for (int e = tid; e < QB * KMAX; e += NTHREADS_A) {
    const int qi = e / KMAX, kk = e % KMAX, c = idx[qi][kk];
    bool first = c >= 0;
    for (int k2 = 0; k2 < kk && first; ++k2) first = idx[qi][k2] != c;
    if (!first) continue;
    for (int k2 = kk + 1; k2 < KMAX; ++k2) {
      if (idx[qi][k2] != c) continue;
      for (int g = 0; g < G; ++g) sm.w[qi][g][kk] += sm.w[qi][g][k2];
    }
  }
  __syncthreads();
  for (int e = tid; e < QB * KMAX; e += NTHREADS_A) {
    const int c = idx[e / KMAX][e % KMAX];
    if (c >= 0) atomicOr(&ownmask[c], 1u << (e / KMAX));
  }
  __syncthreads();
  if (warp == W_LOAD) {
    int base = 0, items = 0;
    for (int c0 = 0; c0 < C; c0 += 32) {
      const uint32_t m = c0 + lane < C ? ownmask[c0 + lane] : 0u;
      const uint32_t nz = __ballot_sync(0xffffffffu, m != 0u);
      if (m != 0u) {
        sm.ulist[base + __popc(nz & ((1u << lane) - 1u))] = make_int2(c0 + lane, static_cast<int>(m));
        items += (__popc(m) + OWN - 1) / OWN;
      }
      base += __popc(nz);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) items += __shfl_xor_sync(0xffffffffu, items, o);
    if (lane == 0) {
      sm.nu = base;
      sm.n_items = items;
    }
  }
  __syncthreads();
  for (int e = tid; e < sm.nu; e += NTHREADS_A) {
    const int64_t j0 = static_cast<int64_t>(sm.ulist[e].x) * S;
    unsigned long long m = ~0ull;
    if (a.key_valid != nullptr) {
      m = 0ull;
      for (int s = 0; s < S; ++s) m |= static_cast<unsigned long long>(a.key_valid[b * a.Lk + j0 + s] != 0) << s;
    }
    if (a.mask_last) m &= ~(1ull << 63);
    sm.vmask[e] = m;
  }
  const uint32_t tbase = sm.tmem_base;
  if (warp < 4) {
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < kAccCols; c += 8) tc::tmem_st8(tbase + lane_off + c, z);
    tc::tmem_wait_st();
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const int n_items = sm.n_items;
  const float sl2 = a.sm_scale * kLog2e;

  if (warp == W_LOAD || warp == W_LOAD2) {
    // ============================ loaders (even / odd items) ================
    const int par = warp == W_LOAD ? 0 : 1;
    int myc[KMAX];
#pragma unroll
    for (int kk = 0; kk < KMAX; ++kk) myc[kk] = idx[lane][kk];
    tc::fence_proxy_async();
    asm volatile("bar.sync 2, 64;\n" ::: "memory");
    const uint32_t below = (1u << lane) - 1u;
    int item = 0;
    bool ok = true;
    for (int u = 0; ok && u < sm.nu; ++u) {
      const int2 ue = sm.ulist[u];
      const int c = ue.x;
      uint32_t owners = static_cast<uint32_t>(ue.y);
      while (owners) {
        const int j = __popc(owners & below);
        const bool mine = ((owners >> lane) & 1u) && j < OWN;
        const uint32_t grp = __ballot_sync(0xffffffffu, mine);
        owners &= ~grp;
        if ((item & 1) == par) {
          const int st = item % NST, r = item % RING, n = __popc(grp);
          if (mine) {
            int slot = 0;
#pragma unroll
            for (int kk = KMAX - 1; kk >= 0; --kk) slot = myc[kk] == c ? kk : slot;
            sm.ring[r].oq[j] = static_cast<uint8_t>(lane);
            sm.ring[r].slot[j] = static_cast<uint8_t>(slot);
          }
          if (lane == 0) {
            sm.ring[r].n = n;
            sm.ring[r].u = u;
            sm.ring[r].c = c;
          }
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(su32(&sm.bar_ring[r]));
          if (item >= NST && !wait_ab_warp(&sm.bar_free[st], ((item / NST) - 1) & 1, &sm.abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = su32(&sm.bar_full[st]);
          const int krow = static_cast<int>(b * a.Lk + static_cast<int64_t>(c) * S);
          if (lane == 0) {
            tc::mbar_arrive_expect_tx(bar, 32768u + static_cast<uint32_t>(n) * 4096u);
            tc::tma_load_4d(su32(sm.st[st].kt), &tm_k, 0, krow, 0, hk, bar);
            tc::tma_load_4d(su32(sm.st[st].vt), &tm_v, 0, krow, 0, hk, bar);
          }
          __syncwarp();
          if (mine) {
            const int qy = static_cast<int>((b * a.Lq + q0 + lane) * Hq + hk * G);
            tc::tma_load_3d(su32(sm.st[st].qt + j * 2048), &tm_q, 0, qy, 0, bar);
            tc::tma_load_3d(su32(sm.st[st].ot + j * 2048), &tm_do, 0, qy, 0, bar);
          }
          if (lane == 0) sm.last[par][st] = item;
        }
        ++item;
      }
    }
    asm volatile("bar.sync 2, 64;\n" ::: "memory");
    if (lane == 0) {
      for (int s2 = 0; s2 < NST; ++s2) {
        const int it = max(sm.last[0][s2], sm.last[1][s2]);
        if (it >= 0 && (it & 1) == par) tc::mbar_wait(su32(&sm.bar_full[s2]), (it / NST) & 1);
      }
    }
    __syncwarp();
  } else if (warp >= W_MMA) {
    // ============================ MMA issue =================================
    // Warp 14: S(i) -> S buffer i%2 and dP(i) -> dP buffer i%2, once the
    // accumulate warps have read the dQ part of item i-2 (written over S).
    // Warp 15: the dQ part of item i (K^T . dS^T) into S buffer i%2, once the
    // softmax has written dS(i); its completion frees the K/V/Q/dO stage.
    const bool s_role = warp == W_MMA;
    const uint64_t dq0 = tc::smem_desc_sw128(su32(sm.st[0].qt), 16, 2048);
    const uint64_t do0 = tc::smem_desc_sw128(su32(sm.st[0].ot), 16, 2048);
    const uint64_t dk0 = tc::smem_desc_sw128(su32(sm.st[0].kt), 16, 1024);
    const uint64_t dv0 = tc::smem_desc_sw128(su32(sm.st[0].vt), 16, 1024);
    const uint64_t dkt0 = tc::smem_desc_sw128(su32(sm.st[0].kt), 8192, 1024);   // K^T, MN-major
    const uint64_t dds0 = tc::smem_desc_sw128(su32(sm.ds[0]), 16, 1024);
    constexpr uint32_t kStageBytes = sizeof(SmemA::Stage);
    if (s_role) {
      constexpr uint32_t id_s = tc::idesc_bf16_f32(64, 64, 0, 0);
      for (int it = 0; it < n_items; ++it) {
        const int st = it % NST, s2 = it & 1;
        if (!wait_ab_warp(&sm.bar_full[st], (it / NST) & 1, &sm.abort_flag)) break;
        if (it >= 2 && !wait_ab_warp(&sm.bar_partfree[s2], ((it >> 1) - 1) & 1, &sm.abort_flag)) break;
        tc::fence_after_sync();
        const uint32_t so = st * kStageBytes;
        const uint64_t da = adv(dq0, so), db = adv(dk0, so), dao = adv(do0, so), dbv = adv(dv0, so);
        const uint32_t tS = tbase + kSCol + 64 * s2, tP = tbase + kDPCol + 64 * s2;
        if (elect_one()) {
          tc::mma_bf16<false>(tS, da, db, id_s);
#pragma unroll
          for (int kk = 1; kk < 8; ++kk)
            tc::mma_bf16<true>(tS, adv(da, (kk >> 2) * 1024 + (kk & 3) * 32), adv(db, (kk >> 2) * 8192 + (kk & 3) * 32),
                               id_s);
          tc::mma_bf16<false>(tP, dao, dbv, id_s);
#pragma unroll
          for (int kk = 1; kk < 8; ++kk)
            tc::mma_bf16<true>(tP, adv(dao, (kk >> 2) * 1024 + (kk & 3) * 32),
                               adv(dbv, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
          tc::mma_commit(su32(&sm.bar_sdone[s2]));
        }
        __syncwarp();
      }
    } else {
      for (int it = 0; it < n_items; ++it) {
        const int st = it % NST, p2 = it & 1;
        if (!wait_ab_warp(&sm.bar_pready[p2], (it >> 1) & 1, &sm.abort_flag)) break;
        tc::fence_after_sync();
        const int np = ((8 * min(max(sm.ring[it % RING].n, 1), OWN) + 15) / 16) * 16;
        const uint32_t id_o = tc::idesc_bf16_f32(128, np, 1, 0);
        const uint64_t dkt = adv(dkt0, st * kStageBytes), dds = adv(dds0, p2 * 8192);
        const uint32_t tD = tbase + kSCol + 64 * p2;
        if (elect_one()) {
          tc::mma_bf16<false>(tD, dkt, dds, id_o);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk) tc::mma_bf16<true>(tD, adv(dkt, kk * 2048), adv(dds, kk * 32), id_o);
          tc::mma_commit(su32(&sm.bar_pvdone[p2]));
          tc::mma_commit(su32(&sm.bar_free[st]));
        }
        __syncwarp();
      }
    }
    if (elect_one()) {
      tc::mma_commit(su32(&sm.bar_drain[s_role ? 0 : 1]));
      tc::mbar_wait(su32(&sm.bar_drain[s_role ? 0 : 1]), 0);
    }
    __syncwarp();
  } else if (warp >= W_SMX) {
    // ============================ softmax (warps 4-7, 8-11) ==================
    // Quadrant q of the M=64 tiles holds owners 2q and 2q+1 (16 rows); two
    // threads per row, 32 keys each.
    const int grp = (warp - W_SMX) >> 2, q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int t = lane & 15, hf = lane >> 4, g = t & 7;
    const float scale = a.sm_scale;
    for (int it = grp; it < n_items; it += 2) {
      const int p2 = it & 1, r = it % RING;
      if (!wait_ab_warp(&sm.bar_ring[r], (it / RING) & 1, &sm.abort_flag)) break;
      const int n = sm.ring[r].n;
      const int jrow = 2 * q + (t >> 3);
      const bool row_on = jrow < n;
      const bool quad_on = 2 * q < n;
      float w = 0.f;
      uint32_t km = 0xFFFFFFFFu;
      int oqj = 0, slot = 0;
      if (row_on) {
        oqj = sm.ring[r].oq[jrow];
        slot = sm.ring[r].slot[jrow];
        if (g < G) w = sm.w[oqj][g][slot];
        const unsigned long long vm = sm.vmask[sm.ring[r].u];
        km = static_cast<uint32_t>(hf ? (vm >> 32) : vm);
      }
      if (!wait_ab_warp(&sm.bar_sdone[p2], (it >> 1) & 1, &sm.abort_flag)) break;
      tc::fence_after_sync();
      uint32_t x[32], y[32];
      if (quad_on) {
        tc::tmem_ld_16x32bx2_x32(tbase + lane_off + kSCol + 64 * p2, x);
        tc::tmem_ld_16x32bx2_x32(tbase + lane_off + kDPCol + 64 * p2, y);
        tc::tmem_wait_ld();
      }
      uint32_t ds[16];
      float di = 0.f;
      if (quad_on) {
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (!((km >> c) & 1u)) x[c] = __float_as_uint(-INFINITY);
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; ++c) mx = fmaxf(mx, __uint_as_float(x[c]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float nb = mx == -INFINITY ? 0.f : -mx * sl2;
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float e = fast_exp2(fmaf(__uint_as_float(x[c]), sl2, nb));
          x[c] = __float_as_uint(e);
          sum += e;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        const float inv = sum > 0.f ? 1.f / sum : 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p = __uint_as_float(x[c]) * inv;
          x[c] = __float_as_uint(p);
          di = fmaf(p, __uint_as_float(y[c]), di);
        }
        di += __shfl_xor_sync(0xffffffffu, di, 16);
        const float f = scale * w;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float d0 = f * __uint_as_float(x[2 * h]) * (__uint_as_float(y[2 * h]) - di);
          const float d1 = f * __uint_as_float(x[2 * h + 1]) * (__uint_as_float(y[2 * h + 1]) - di);
          ds[h] = pack_bf16x2(d0, d1);
        }
      }
      if (row_on && hf == 0 && g < G)
        a.dw[((b * a.Lq + q0 + oqj) * Hq + hk * G + g) * K + slot] = f2bf(di);
      // the dS buffer is free once the dQ part of item it-2 has completed
      if (it >= 2 && !wait_ab_warp(&sm.bar_pvdone[p2], ((it - 2) >> 1) & 1, &sm.abort_flag)) break;
      if (row_on) {
        const int row = 8 * jrow + g;
#pragma unroll
        for (int p = 0; p < 4; ++p)
          *reinterpret_cast<uint4*>(sm.ds[p2] + swz_off(row, 4 * hf + p)) =
              make_uint4(ds[4 * p], ds[4 * p + 1], ds[4 * p + 2], ds[4 * p + 3]);
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_pready[p2]));
    }
  } else {
    // ============================ accumulate (warps 0-3) =====================
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    for (int it = 0; it < n_items; ++it) {
      const int p2 = it & 1, r = it % RING;
      if (!wait_ab_warp(&sm.bar_ring[r], (it / RING) & 1, &sm.abort_flag)) break;
      const int n = sm.ring[r].n;
      int oq[OWN];
#pragma unroll
      for (int j = 0; j < OWN; ++j) oq[j] = sm.ring[r].oq[j];
      if (!wait_ab_warp(&sm.bar_pvdone[p2], (it >> 1) & 1, &sm.abort_flag)) break;
      tc::fence_after_sync();
      tc::tmem_wait_st();
#pragma unroll
      for (int j0 = 0; j0 < OWN; j0 += 4) {
        if (j0 >= n) break;
        uint32_t pv[4][8], acc[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j0 + j < n) {
            tc::tmem_ld8(tbase + lane_off + kSCol + 64 * p2 + 8 * (j0 + j), pv[j]);
            tc::tmem_ld8(tbase + lane_off + 8 * oq[j0 + j], acc[j]);
          }
        }
        tc::tmem_wait_ld();
        if (j0 + 4 >= n) {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(su32(&sm.bar_partfree[p2]));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j0 + j < n) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
              acc[j][c] = __float_as_uint(__uint_as_float(acc[j][c]) + __uint_as_float(pv[j][c]));
            tc::tmem_st8(tbase + lane_off + 8 * oq[j0 + j], acc[j]);
          }
        }
      }
    }
    tc::tmem_wait_st();
  }

  if (warp < W_LOAD) {
    // ============================ epilogue: dQ (fp32) ========================
    tc::fence_before_sync();
    asm volatile("bar.sync 1, 384;\n" ::: "memory");
    tc::fence_after_sync();
    if (!__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0)) {
      const int qd = warp & 3, part = warp >> 2;
      const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
      const int d = qd * 32 + lane;
      for (int q1 = part * 4; q1 < QB; q1 += 12) {
        uint32_t acc[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) tc::tmem_ld8(tbase + lane_off + 8 * (q1 + j), acc[j]);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t rowq = q0 + q1 + j;
          if (q1 + j >= QB || rowq >= a.Lq) continue;
#pragma unroll
          for (int gg = 0; gg < GMAX; ++gg)
            if (gg < G) a.dq[((b * a.Lq + rowq) * Hq + hk * G + gg) * static_cast<int64_t>(D) + d] = __uint_as_float(acc[j][gg]);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && sm.abort_flag) atomicOr(&g_bwd_error, 1);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ============================================================ dK / dV kernel
constexpr int NTHREADS_B = 384;              // warp 0 loads, warps 1-2 issue MMAs, warps 4-11 two row groups
constexpr int PT = 16;                       // (query, slot) pairs per tile: 128 rows

// Two row groups (warps 4-7 and 8-11) take the even and the odd tiles, each
// with its own MMA warp, stage, w*P / dS buffers and S, dP, dV^T, dK^T in
// TMEM; the epilogue adds the groups' accumulators in a fixed order.
struct __align__(1024) SmemB {
  unsigned char kt[16384];                   // this chunk's K tile (loaded once)
  unsigned char vt[16384];                   // and V tile
  struct Stage {
    unsigned char qt[PT * 2048];             // 16 pairs x [half][8 rows][64 dims]
    unsigned char ot[PT * 2048];             // their dO rows
  } st[2];                                   // group g's tiles use stage g
  unsigned char wp[2][16384];                // w * P of each group [128 rows x 64 keys] bf16, 128-byte swizzled rows
  unsigned char dsb[2][16384];               // dS, same layout
  int pl[2][PT], pslot[2][PT], pn[2];
  uint64_t bar_kv, bar_full[2], bar_free[2], bar_ring[2], bar_sdone[2], bar_pready[2], bar_done[2];
  int last[2];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SmemB) + 1024 <= 232448, "dK/dV kernel shared memory over budget");

__global__ void __launch_bounds__(NTHREADS_B, 1) dkv_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                            const __grid_constant__ CUtensorMap tm_v,
                                                            const __grid_constant__ CUtensorMap tm_q,
                                                            const __grid_constant__ CUtensorMap tm_do, BwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SmemB& sm = *reinterpret_cast<SmemB*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G, K = a.K, Hq = a.Hkv * a.G;
  const int seg = (b * a.Hkv + hk) * a.C + c;
  const int n_pairs = a.cnt[seg], p_off = a.off[seg];
  const int n_tiles = (n_pairs + PT - 1) / PT;
  const int64_t krow0 = b * a.Lk + static_cast<int64_t>(c) * S;

  if (n_pairs == 0) {                        // no query selected this chunk: zero gradients
    for (int e = tid; e < S * D; e += NTHREADS_B) {
      const int64_t o = ((krow0 + e / D) * a.Hkv + hk) * D + e % D;
      a.dk[o] = 0.f;
      a.dv[o] = 0.f;
    }
    return;
  }
  for (int e = tid; e < 2 * static_cast<int>(sizeof(SmemB::Stage)) / 16; e += NTHREADS_B)
    reinterpret_cast<uint4*>(&sm.st[0])[e] = make_uint4(0u, 0u, 0u, 0u);
  for (int e = tid; e < 4 * 16384 / 16; e += NTHREADS_B) reinterpret_cast<uint4*>(&sm.wp[0][0])[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    tc::mbar_init(su32(&sm.bar_kv), 1);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(su32(&sm.bar_full[s]), 1);
      tc::mbar_init(su32(&sm.bar_free[s]), 1);
      tc::mbar_init(su32(&sm.bar_ring[s]), 1);
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
  // usable keys of this chunk
  unsigned long long vm = ~0ull;
  if (a.key_valid != nullptr) {
    const uint32_t bit = __ballot_sync(0xffffffffu, a.key_valid[krow0 + lane] != 0);
    const uint32_t bit2 = __ballot_sync(0xffffffffu, a.key_valid[krow0 + 32 + lane] != 0);
    vm = static_cast<unsigned long long>(bit) | (static_cast<unsigned long long>(bit2) << 32);
  }
  if (a.mask_last) vm &= ~(1ull << 63);
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
      const int np = min(PT, n_pairs - t * PT);
      // group g2's stage (and its pair list) was last read for tile t-2, whose
      // gradient MMAs have completed
      if (t >= 2 && !wait_ab_warp(&sm.bar_free[g2], ((t >> 1) - 1) & 1, abf)) break;
      int l = 0, slot = 0;
      if (lane < np) {
        const int pr = a.pairs[p_off + t * PT + lane];
        l = pr >> 5;
        slot = pr & 31;
        sm.pl[g2][lane] = l;
        sm.pslot[g2][lane] = slot;
      }
      if (lane == 0) sm.pn[g2] = np;
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(su32(&sm.bar_ring[g2]));
        tc::mbar_arrive_expect_tx(su32(&sm.bar_full[g2]), static_cast<uint32_t>(np) * 4096u);
      }
      __syncwarp();
      if (lane < np) {
        const int qy = static_cast<int>((b * a.Lq + l) * Hq + hk * G);
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
    // [rows x keys], MN-major B: N = 64 keys is one swizzle atom wide, so only
    // the 8-row stride (1024 B) matters; both offset fields carry it
    const uint64_t dwp = tc::smem_desc_sw128(su32(sm.wp[g2]), 1024, 1024);
    const uint64_t dds = tc::smem_desc_sw128(su32(sm.dsb[g2]), 1024, 1024);
    const uint32_t tS = tbase + kS + 64 * g2, tP = tbase + kDP + 64 * g2;
    const uint32_t tV = tbase + kDV + 128 * g2, tK = tbase + kDK + 128 * g2;
    bool ok = wait_ab_warp(&sm.bar_kv, 0, abf);
    tc::fence_after_sync();
    for (int t = g2; ok && t < n_tiles; t += 2) {
      if (!(ok = wait_ab_warp(&sm.bar_full[g2], (t >> 1) & 1, abf))) break;
      tc::fence_after_sync();
      // S and dP of tile t (the group's previous gradient MMAs, issued before,
      // and its rows' reads of S and dP precede)
      if (elect_one()) {
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
      // dV^T_g += dO^T . (w P) and dK^T_g += Q^T . dS of tile t
      if (!(ok = wait_ab_warp(&sm.bar_pready[g2], (t >> 1) & 1, abf))) break;
      tc::fence_after_sync();
      if (elect_one()) {
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
    if (elect_one()) tc::mma_commit(su32(&sm.bar_done[g2]));
    __syncwarp();
  } else if (warp >= 4) {
    // ============================ rows (two groups, one tile row per thread) =
    const int grp = (warp - 4) >> 2;              // tiles t with t % 2 == grp
    const int r = (warp & 3) * 32 + lane, pr = r >> 3, g = r & 7;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float scale = a.sm_scale, sl2 = scale * kLog2e;
    const uint32_t tS = tbase + lane_off + kS + 64 * grp, tP = tbase + lane_off + kDP + 64 * grp;
    for (int t = grp; t < n_tiles; t += 2) {
      if (!wait_ab_warp(&sm.bar_ring[grp], (t >> 1) & 1, abf)) break;
      const int np = sm.pn[grp];
      const bool row_on = pr < np && g < G;
      float w = 0.f;
      if (row_on) w = bf2f(a.w[((b * a.Lq + sm.pl[grp][pr]) * Hq + hk * G + g) * K + sm.pslot[grp][pr]]);
      if (!wait_ab_warp(&sm.bar_sdone[grp], (t >> 1) & 1, abf)) break;
      tc::fence_after_sync();
      // P of the chunk's softmax stays in registers; dP is read twice in halves
      // (for di, then for dS) to keep the register count down
      uint32_t x[64];
#pragma unroll
      for (int h = 0; h < 4; ++h) tc::tmem_ld16(tS + 16 * h, *reinterpret_cast<uint32_t(*)[16]>(&x[16 * h]));
      tc::tmem_wait_ld();
      float mx = -INFINITY;
#pragma unroll
      for (int s = 0; s < 64; ++s) {
        if (!((vm >> s) & 1ull)) x[s] = __float_as_uint(-INFINITY);
        mx = fmaxf(mx, __uint_as_float(x[s]));
      }
      const float nb = mx == -INFINITY ? 0.f : -mx * sl2;
      float sum = 0.f;
#pragma unroll
      for (int s = 0; s < 64; ++s) {
        const float e = fast_exp2(fmaf(__uint_as_float(x[s]), sl2, nb));
        x[s] = __float_as_uint(e);
        sum += e;
      }
      const float inv = sum > 0.f ? 1.f / sum : 0.f;
      float di = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t y[32];
        tc::tmem_ld16(tP + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(&y[0]));
        tc::tmem_ld16(tP + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(&y[16]));
        tc::tmem_wait_ld();
#pragma unroll
        for (int s = 0; s < 32; ++s) {
          const float p = __uint_as_float(x[32 * half + s]) * inv;
          x[32 * half + s] = __float_as_uint(p);
          di = fmaf(p, __uint_as_float(y[s]), di);
        }
      }
      const float f = row_on ? scale * w : 0.f, wr = row_on ? w : 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t y[32];
        tc::tmem_ld16(tP + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(&y[0]));
        tc::tmem_ld16(tP + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(&y[16]));
        tc::tmem_wait_ld();
        uint32_t pw[16], dsv[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float p0 = __uint_as_float(x[32 * half + 2 * h]), p1 = __uint_as_float(x[32 * half + 2 * h + 1]);
          pw[h] = pack_bf16x2(wr * p0, wr * p1);
          dsv[h] = pack_bf16x2(f * p0 * (__uint_as_float(y[2 * h]) - di), f * p1 * (__uint_as_float(y[2 * h + 1]) - di));
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
          const int64_t o = ((krow0 + s0 + s) * a.Hkv + hk) * D + d;
          a.dv[o] = has1 ? __uint_as_float(v0[s]) + __uint_as_float(v1[s]) : __uint_as_float(v0[s]);
          a.dk[o] = has1 ? __uint_as_float(k0[s]) + __uint_as_float(k1[s]) : __uint_as_float(k0[s]);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && sm.abort_flag) atomicOr(&g_bwd_error, 2);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ============================================================ inverted index
// Pairs of segment (b, h, c): (l << 5) | slot for every slot whose index is c,
// in (l, slot) order -- built without order-dependent atomics, so the dK / dV
// sums (and every other walk of a segment) are the same on every run:
//   hist_kernel   per block of QT queries: how many of its slots pick each chunk
//   colscan_kernel per segment: prefix over the query blocks, and its count
//   scan_kernel   segment offsets
//   place_kernel  per block of QT queries, in query order: each slot's position
constexpr int QT = 256;

__global__ void __launch_bounds__(256) hist_kernel(const int32_t* __restrict__ idx, int32_t* __restrict__ hist,
                                                   int64_t Lq, int Hkv, int K, int C) {
  extern __shared__ int ctr[];
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z, nqb = gridDim.x;
  for (int c = threadIdx.x; c < C; c += blockDim.x) ctr[c] = 0;
  __syncthreads();
  const int64_t l0 = static_cast<int64_t>(qb) * QT;
  const int nq = static_cast<int>(Lq - l0 < QT ? Lq - l0 : QT);
  for (int e = threadIdx.x; e < nq * K; e += blockDim.x) {
    const int c = idx[((b * Lq + l0 + e / K) * Hkv + h) * K + e % K];
    if (c >= 0 && c < C) atomicAdd(&ctr[c], 1);
  }
  __syncthreads();
  int32_t* out = hist + ((static_cast<int64_t>(b) * Hkv + h) * nqb + qb) * C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) out[c] = ctr[c];
}

// hist[b,h,qb,c] -> its exclusive prefix over qb; cnt[(b*Hkv + h)*C + c] = the total
__global__ void colscan_kernel(int32_t* __restrict__ hist, int32_t* __restrict__ cnt, int64_t segs, int nqb, int C) {
  const int64_t seg = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (seg >= segs) return;
  const int64_t bh = seg / C;
  const int c = static_cast<int>(seg % C);
  int32_t* col = hist + bh * nqb * C + c;
  int run = 0;
  for (int qb = 0; qb < nqb; ++qb) {
    const int v = col[static_cast<int64_t>(qb) * C];
    col[static_cast<int64_t>(qb) * C] = run;
    run += v;
  }
  cnt[seg] = run;
}

// exclusive scan of n counts into off[0..n] (one CTA)
__global__ void __launch_bounds__(1024) scan_kernel(const int32_t* __restrict__ cnt, int32_t* __restrict__ off, int n) {
  __shared__ int part[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < n; base += 1024) {
    const int i = base + static_cast<int>(threadIdx.x);
    const int v = i < n ? cnt[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) part[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int p = part[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, p, o);
        if (lane >= o) p += y;
      }
      part[lane] = p;
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? part[warp - 1] : 0) + x - v;
    if (i < n) off[i] = excl;
    __syncthreads();
    if (threadIdx.x == 1023) carry = excl + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) off[n] = carry;
}

// The block's chunk lists are staged in shared memory by all threads; then one
// warp walks the queries in order, lane k placing slot k.  A chunk listed twice
// by one query takes consecutive positions in slot order.
__global__ void __launch_bounds__(128) place_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ hist,
                                                    const int32_t* __restrict__ off, int32_t* __restrict__ pairs,
                                                    int64_t Lq, int Hkv, int K, int C) {
  extern __shared__ int place_smem[];
  int* ctr = place_smem;                     // [C]
  int* lists = place_smem + C;               // [QT][K]
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z, nqb = gridDim.x;
  const int64_t seg0 = (static_cast<int64_t>(b) * Hkv + h) * C;
  const int32_t* pre = hist + ((static_cast<int64_t>(b) * Hkv + h) * nqb + qb) * C;
  const int64_t l0 = static_cast<int64_t>(qb) * QT;
  const int nq = static_cast<int>(Lq - l0 < QT ? Lq - l0 : QT);
  for (int c = threadIdx.x; c < C; c += blockDim.x) ctr[c] = off[seg0 + c] + pre[c];
  for (int e = threadIdx.x; e < nq * K; e += blockDim.x) lists[e] = idx[((b * Lq + l0 + e / K) * Hkv + h) * K + e % K];
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  for (int i = 0; i < nq; ++i) {
    const int64_t l = l0 + i;
    const int c = lane < K ? lists[i * K + lane] : -1;
    const bool ok = c >= 0 && c < C;
    const uint32_t act = __ballot_sync(0xffffffffu, ok);
    if (ok) {
      const uint32_t peers = __match_any_sync(act, c);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      pairs[ctr[c] + rank] = static_cast<int32_t>((l << 5) | lane);
      __syncwarp(act);
      if (rank == 0) ctr[c] += __popc(peers);
    }
    __syncwarp();
  }
}

// dW of empty slots is 0; a repeated chunk's slots all get the first slot's di
__global__ void dw_fixup_kernel(const int32_t* __restrict__ idx, __nv_bfloat16* __restrict__ dw, int64_t rows, int Hkv,
                                int G, int K, int C) {
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;   // (b, l, h)
  if (row >= rows) return;
  const int32_t* ix = idx + row * K;
  __nv_bfloat16* out = dw + row * static_cast<int64_t>(G) * K;   // [G][K] of this (b, l, h)
  for (int k = 0; k < K; ++k) {
    const int c = ix[k];
    int first = k;
    if (c >= 0 && c < C)
      for (int k2 = 0; k2 < k; ++k2)
        if (ix[k2] == c) {
          first = k2;
          break;
        }
    if (c < 0 || c >= C) {
      for (int g = 0; g < G; ++g) out[g * K + k] = f2bf(0.f);
    } else if (first != k) {
      for (int g = 0; g < G; ++g) out[g * K + k] = out[g * K + first];
    }
  }
}

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

size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

namespace mrsa {
size_t chunk_index_bytes(int64_t batch, int64_t q_len, int64_t kv_heads, int64_t topk, int64_t chunks) {
  const int64_t segs = batch * kv_heads * chunks, nqb = (q_len + QT - 1) / QT;
  return al256(segs * 4) + al256((segs + 1) * 4) + al256(batch * kv_heads * nqb * chunks * 4) +
         al256(batch * q_len * kv_heads * topk * 4);
}

int build_chunk_index(const int32_t* indices, int64_t batch, int64_t q_len, int kv_heads, int topk, int chunks,
                      void* workspace, cudaStream_t s, ChunkIndex* out) {
  const int64_t segs = batch * kv_heads * static_cast<int64_t>(chunks), nqb = (q_len + QT - 1) / QT;
  if (segs + 1 > 0x7fffffffLL || batch * q_len * kv_heads * topk > 0x7fffffffLL || q_len >= (1LL << 26) ||
      nqb > 0x7fffffffLL || chunks > 12288)
    return MRSA_ERR_SHAPE;
  char* ws = static_cast<char*>(workspace);
  int32_t* cnt = reinterpret_cast<int32_t*>(ws);
  int32_t* off = reinterpret_cast<int32_t*>(ws + al256(segs * 4));
  int32_t* hist = reinterpret_cast<int32_t*>(ws + al256(segs * 4) + al256((segs + 1) * 4));
  int32_t* pairs = reinterpret_cast<int32_t*>(ws + al256(segs * 4) + al256((segs + 1) * 4) +
                                              al256(batch * kv_heads * nqb * chunks * 4));
  out->cnt = cnt;
  out->off = off;
  out->pairs = pairs;
  const size_t ctr_bytes = static_cast<size_t>(chunks) * sizeof(int);
  const size_t place_bytes = ctr_bytes + static_cast<size_t>(QT) * topk * sizeof(int);
  if (const cudaError_t e = cudaFuncSetAttribute(place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(place_bytes));
      e != cudaSuccess) {
    note_cuda_error(e, "build_chunk_index: shared-memory opt-in");
    return MRSA_ERR_LAUNCH;
  }
  if (const cudaError_t e = cudaFuncSetAttribute(hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(ctr_bytes));
      e != cudaSuccess) {
    note_cuda_error(e, "build_chunk_index: shared-memory opt-in");
    return MRSA_ERR_LAUNCH;
  }
  if (nqb > 0) {
    const dim3 grid(static_cast<unsigned>(nqb), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
    hist_kernel<<<grid, 256, ctr_bytes, s>>>(indices, hist, q_len, kv_heads, topk, chunks);
    colscan_kernel<<<static_cast<unsigned>((segs + 255) / 256), 256, 0, s>>>(hist, cnt, segs, static_cast<int>(nqb),
                                                                            chunks);
    scan_kernel<<<1, 1024, 0, s>>>(cnt, off, static_cast<int>(segs));
    place_kernel<<<grid, 128, place_bytes, s>>>(indices, hist, off, pairs, q_len, kv_heads, topk, chunks);
  } else {
    if (const cudaError_t e = cudaMemsetAsync(cnt, 0, segs * 4, s); e != cudaSuccess) {
      note_cuda_error(e, "build_chunk_index: clearing the chunk counts");
      return MRSA_ERR_LAUNCH;
    }
    scan_kernel<<<1, 1024, 0, s>>>(cnt, off, static_cast<int>(segs));
  }
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

int bwd_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bwd_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_bwd_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
}  // namespace mrsa

extern "C" size_t mrsa_selected_attention_backward_workspace(int64_t batch, int64_t q_len, int64_t kv_len,
                                                             int64_t kv_heads, int64_t topk) {
  if (batch < 1 || q_len < 0 || kv_len < S || kv_heads < 1 || topk < 1) return 0;
  return mrsa::chunk_index_bytes(batch, q_len, kv_heads, topk, kv_len / S);
}

extern "C" int mrsa_selected_attention_backward(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                                                const void* weights, const int32_t* indices, const void* grad_out,
                                                float* dq, float* dk, float* dv, void* dw, float sm_scale,
                                                int mask_last_token, int64_t batch, int64_t q_len, int64_t kv_len,
                                                int64_t kv_heads, int64_t groups, int64_t head_dim, int64_t topk,
                                                int64_t chunk, void* workspace, size_t ws_bytes,
                                                mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  if (!q || !k || !v || !weights || !indices || !grad_out || !dq || !dk || !dv || !dw) return MRSA_ERR_NULL;
  if (head_dim != D || chunk != S || groups < 1 || groups > GMAX || kv_heads < 1 || batch < 1 || q_len < 0 ||
      kv_len < S || kv_len % S || kv_len / S > 64 * 32 || topk < 1 || topk > KMAX || kv_heads > 65535 ||
      batch > 65535 || q_len >= (1LL << 26) || batch * q_len * kv_heads * groups > 0x7fffffffLL ||
      batch * kv_len > 0x7fffffffLL || batch * q_len * kv_heads * topk > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(grad_out) |
                       reinterpret_cast<uintptr_t>(workspace);
  if (al & 15u) return MRSA_ERR_ALIGN;
  const size_t need = mrsa_selected_attention_backward_workspace(batch, q_len, kv_len, kv_heads, topk);
  if (workspace == nullptr || ws_bytes < need) return MRSA_ERR_WORKSPACE;
  const int C = static_cast<int>(kv_len / S);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();                  // a stale error of this thread is not this call's
  if (q_len == 0) {                          // no queries: dK = dV = 0
    if (cudaMemsetAsync(dk, 0, batch * kv_len * kv_heads * D * sizeof(float), s) != cudaSuccess ||
        cudaMemsetAsync(dv, 0, batch * kv_len * kv_heads * D * sizeof(float), s) != cudaSuccess)
      return MRSA_ERR_LAUNCH;
    return MRSA_OK;
  }
  CUtensorMap tm_k, tm_v, tm_q, tm_do;
  const cuuint64_t kv_dims[4] = {64, static_cast<cuuint64_t>(batch * kv_len), 2, static_cast<cuuint64_t>(kv_heads)};
  const cuuint64_t kv_str[3] = {static_cast<cuuint64_t>(kv_heads * D * 2), 128, 256};
  const cuuint32_t kv_box[4] = {64, 64, 2, 1};
  const cuuint64_t q_dims[3] = {64, static_cast<cuuint64_t>(batch * q_len * kv_heads * groups), 2};
  const cuuint64_t q_str[2] = {256, 128};
  const cuuint32_t q_box[3] = {64, 8, 2};
  if (!make_map(&tm_k, k, 4, kv_dims, kv_str, kv_box) || !make_map(&tm_v, v, 4, kv_dims, kv_str, kv_box) ||
      !make_map(&tm_q, q, 3, q_dims, q_str, q_box) || !make_map(&tm_do, grad_out, 3, q_dims, q_str, q_box)) {
    mrsa::note_cuda_error(cudaErrorInvalidValue, "mrsa_selected_attention_backward: tensor map encoding");
    return MRSA_ERR_LAUNCH;
  }
  BwdArgs a;
  a.w = static_cast<const __nv_bfloat16*>(weights);
  a.indices = indices;
  a.key_valid = key_valid;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.dw = static_cast<__nv_bfloat16*>(dw);
  a.sm_scale = sm_scale;
  a.mask_last = mask_last_token;
  a.Lq = q_len;
  a.Lk = kv_len;
  a.Hkv = static_cast<int>(kv_heads);
  a.G = static_cast<int>(groups);
  a.K = static_cast<int>(topk);
  a.C = C;
  // inverted index
  mrsa::ChunkIndex ix;
  if (const int rc = mrsa::build_chunk_index(indices, batch, q_len, a.Hkv, a.K, C, workspace, s, &ix); rc != MRSA_OK)
    return rc;
  a.cnt = ix.cnt;
  a.off = ix.off;
  a.pairs = ix.pairs;
  // dQ and dW
  const size_t smem_a = sizeof(SmemA) + 1024, smem_b = sizeof(SmemB) + 1024;
  for (const auto& fa : {std::make_pair(reinterpret_cast<const void*>(dq_kernel), smem_a),
                         std::make_pair(reinterpret_cast<const void*>(dkv_kernel), smem_b)}) {
    if (const cudaError_t e = cudaFuncSetAttribute(fa.first, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(fa.second));
        e != cudaSuccess) {
      mrsa::note_cuda_error(e, "mrsa_selected_attention_backward: shared-memory opt-in");
      return MRSA_ERR_LAUNCH;
    }
  }
  const int64_t blocks = (q_len + QB - 1) / QB;
  dq_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch)),
              NTHREADS_A, smem_a, s>>>(tm_k, tm_v, tm_q, tm_do, a);
  MRSA_CHECK_LAUNCH();
  const int64_t rows = batch * q_len * kv_heads;
  dw_fixup_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, s>>>(indices, a.dw, rows, a.Hkv, a.G, a.K, C);
  MRSA_CHECK_LAUNCH();
  // dK and dV
  dkv_kernel<<<dim3(static_cast<unsigned>(C), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch)),
               NTHREADS_B, smem_b, s>>>(tm_k, tm_v, tm_q, tm_do, a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
