// Selected-chunk attention on the 5th-generation tensor cores (tcgen05/TMEM).
//
// Semantics (ops/hils_fwd_bwd_head.py:21-93 torch reference, kernel :423-559;
// fusion ops/hils_bidir_output_fusion_tilelang.py:15-37):
//   out[q,g] = bf16( bf16( sum_k w[q,g,k] * softmax_s(q.K_{c_k,s}/sqrt(D))_{valid s != 63} V_{c_k,s} )
//                    + w_local[q,g] * local[q,g] )
// Every chunk is normalised on its own; the chunk probabilities times the route
// weight are split into bf16 hi + lo parts, so P.V keeps ~16 significant bits.
//
// One CTA owns QB = 32 queries of one KV head.  Their outputs accumulate as
// O^T in tensor memory: TMEM lane = output dim (128 lanes), column 8*q + g =
// (query, head).  The CTA walks the union of its queries' chunk lists; per
// chunk the queries that selected it ("owners", up to 8 per work item) are
// compacted into the rows of one MMA tile:
//   S[64 x 64]        = Q_own[64 x 128] . K_c^T         (UMMA M=64,  N=64)
//   P                 = per-row softmax of S times the route weight (hi + lo)
//   O_part^T[128 x N] = V_c^T[128 x 64] . P^T           (UMMA M=128, N=8*owners)
//   O^T[:, 8q..8q+7] += O_part^T[:, 8j..8j+7]           (TMEM read-modify-write)
// Warp roles: 0-3 and 4-7 are two groups that take alternate work items
// (softmax with TMEM lane = S row, then the read-modify-write with TMEM lane
// = dim; the read-modify-writes are chained item by item); warp 8 is the
// loader (owner compaction + TMA of K, V and the owners' Q rows into
// 128-byte-swizzled tiles, three stages); warp 9 issues the MMAs.  Every
// mbarrier wait is bounded and a shared abort flag unwinds all roles.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int QB = 32;            // queries per CTA (== warp size: one loader lane per query)
constexpr int GMAX = 8;           // head rows per query in the MMA tile
constexpr int OWN = 8;            // owners per work item (64 S rows)
constexpr int NST = 3;            // load stages
constexpr int D = kHeadDim, S = kChunk, KMAX = 32;
constexpr int NTHREADS = 320;
constexpr int kAccCols = QB * GMAX;          // 256
constexpr int kSCol = 256, kPCol = 384;      // S[2] at 256/320, partial[2] at 384/448

struct __align__(1024) TcSmem {
  unsigned char kt[NST][16384];   // K tile: 2 sub-tiles [64 keys x 64 dims] (K-major SW128)
  unsigned char vt[NST][16384];   // V tile, same layout, read as V^T (MN-major)
  unsigned char at[NST][16384];   // owner Q rows: 2 sub-tiles [64 rows x 64 dims]
  unsigned char ph[2][8192];      // P hi: [64 rows x 64 keys]
  unsigned char pl[2][8192];      // P lo
  __nv_bfloat16 w[QB][GMAX][KMAX];
  int idx[QB][KMAX + 1];          // padded: lane-per-query reads are bank-conflict free
  int ulist[QB * KMAX];
  unsigned long long vmask[QB * KMAX];   // per union chunk: bit s = key s usable
  unsigned long long kvmask[NST];
  int item_own_q[NST][OWN];       // owner query (CTA-local) per compact group
  int item_own_slot[NST][OWN];
  int item_n[NST];
  uint64_t bar_full[NST], bar_kvfree[NST], bar_sdone[2], bar_pready[2], bar_pvdone[2], bar_rmw[2];
  uint32_t tmem_base;
  int nu, n_items, abort_flag;
  uint32_t bitmap[64];            // C <= 2048 chunks
};

struct TcArgs {
  const __nv_bfloat16* w;
  const int32_t* indices;
  const uint8_t* key_valid;
  const __nv_bfloat16 *local_out, *local_w;
  __nv_bfloat16* out;
  float sm_scale;
  int mask_last;
  int64_t Lq, Lk;
  int Hkv, G, K, C;
};

// Set (bit 0) when a selected-attention CTA gave up on a wait; read and
// cleared by mrsa_device_error_flags().
__device__ int g_tc_error;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ int swz_off(int row, int piece) { return row * 128 + ((piece ^ (row & 7)) << 4); }

__device__ __forceinline__ bool wait_bar(TcSmem& sm, uint64_t* bar, uint32_t parity) {
  // bounded wait that also gives up when another role has aborted
  for (int round = 0; round < 4000; ++round) {
    if (tc::mbar_wait(su32(bar), parity, 1000u)) return true;
    if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) return false;
  }
  *reinterpret_cast<volatile int*>(&sm.abort_flag) = 1;
  return false;
}

__global__ void __launch_bounds__(NTHREADS, 1) selected_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const __grid_constant__ CUtensorMap tm_q, TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * QB;
  const int G = a.G, K = a.K, C = a.C, Hq = a.Hkv * a.G;
  const int nwords = (C + 31) >> 5;

  // ---------------- set-up: chunk lists, weights, union of chunks ----------
  for (int e = tid; e < 64; e += NTHREADS) sm.bitmap[e] = 0u;
  for (int e = tid; e < QB * KMAX; e += NTHREADS) {
    const int qi = e / KMAX, kk = e % KMAX;
    int c = -1;
    if (kk < K && q0 + qi < a.Lq) {
      c = a.indices[((b * a.Lq + q0 + qi) * a.Hkv + hk) * K + kk];
      if (c >= C) c = -1;
    }
    sm.idx[qi][kk] = c < 0 ? -1 : c;
  }
  for (int e = tid; e < QB * GMAX * KMAX; e += NTHREADS) {
    const int qi = e / (GMAX * KMAX), g = (e / KMAX) % GMAX, kk = e % KMAX;
    __nv_bfloat16 wv = f2bf(0.f);
    if (g < G && kk < K && q0 + qi < a.Lq) wv = a.w[((b * a.Lq + q0 + qi) * Hq + hk * G + g) * K + kk];
    sm.w[qi][g][kk] = wv;
  }
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(su32(&sm.bar_full[s]), 1);
      tc::mbar_init(su32(&sm.bar_kvfree[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(su32(&sm.bar_sdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_pready[s]), 4);
      tc::mbar_init(su32(&sm.bar_pvdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_rmw[s]), 4);
    }
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(su32(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  __syncthreads();
  for (int e = tid; e < QB * KMAX; e += NTHREADS) {
    const int c = sm.idx[e / KMAX][e % KMAX];
    if (c >= 0) atomicOr(&sm.bitmap[c >> 5], 1u << (c & 31));
  }
  __syncthreads();
  if (warp == 8) {
    // compact the union bitmap into an ascending chunk list, then count work items
    int base = 0;
    for (int wb = 0; wb < nwords; wb += 32) {
      const uint32_t word = (wb + lane < nwords) ? sm.bitmap[wb + lane] : 0u;
      const int cnt = __popc(word);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int pos = base + incl - cnt;
      uint32_t bits = word;
      while (bits) {
        sm.ulist[pos++] = ((wb + lane) << 5) + (__ffs(bits) - 1);
        bits &= bits - 1;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    __syncwarp();
    int items = 0;
    for (int u = 0; u < base; ++u) {
      const int c = sm.ulist[u];
      bool own = false;
      for (int kk = 0; kk < K; ++kk) own |= sm.idx[lane][kk] == c;   // K <= 32
      items += (__popc(__ballot_sync(0xffffffffu, own)) + OWN - 1) / OWN;
    }
    if (lane == 0) {
      sm.nu = base;
      sm.n_items = items;
    }
  }
  __syncthreads();
  // per union chunk: 64-bit mask of usable keys (valid, and not the landmark slot)
  for (int e = tid; e < sm.nu; e += NTHREADS) sm.vmask[e] = 0ull;
  __syncthreads();
  for (int e = tid; e < sm.nu * 4; e += NTHREADS) {
    const int u = e >> 2, qt = e & 3;
    const int64_t j0 = static_cast<int64_t>(sm.ulist[u]) * S + qt * 16;
    unsigned long long m = 0xFFFFull;
    if (a.key_valid != nullptr) {
      const uint4 raw = *reinterpret_cast<const uint4*>(a.key_valid + b * a.Lk + j0);
      const uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
      m = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) m |= static_cast<unsigned long long>(((wds[i >> 2] >> (8 * (i & 3))) & 0xFF) != 0) << i;
    }
    if (a.mask_last && qt == 3) m &= 0x7FFFull;
    atomicOr(&sm.vmask[u], m << (16 * qt));
  }
  const uint32_t tbase = sm.tmem_base;
  if (warp < 4) {
    // zero the accumulators (this warp's 32 lanes, all accumulator columns)
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < kAccCols; c += 8) tc::tmem_st8(tbase + lane_off + c, z);
    tc::tmem_wait_st();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const int n_items = sm.n_items;
  const float sl2 = a.sm_scale * kLog2e;

  if (warp == 8) {
    // ============================ loader =====================================
    int item = 0;
    for (int u = 0; u < sm.nu && item < n_items; ++u) {
      const int c = sm.ulist[u];
      int my_slot = -1;
      for (int kk = 0; kk < K; ++kk)
        if (my_slot < 0 && sm.idx[lane][kk] == c) my_slot = kk;
      uint32_t owners = __ballot_sync(0xffffffffu, my_slot >= 0);
      while (owners) {
        const int ls = item % NST;
        if (item >= NST && !wait_bar(sm, &sm.bar_kvfree[ls], ((item - NST) / NST) & 1)) {
          u = sm.nu;
          break;
        }
        int n = 0;
        uint32_t grp = 0;
        for (uint32_t m = owners; m && n < OWN; m &= m - 1, ++n) grp |= m & (~m + 1);
        owners &= ~grp;
        const bool mine = (grp >> lane) & 1u;
        const int pos = __popc(grp & ((1u << lane) - 1u));
        if (mine) {
          sm.item_own_q[ls][pos] = lane;
          sm.item_own_slot[ls][pos] = my_slot;
        }
        const int64_t j0 = static_cast<int64_t>(c) * S;
        if (lane == 0) {
          sm.item_n[ls] = n;
          sm.kvmask[ls] = sm.vmask[u];
        }
        __syncwarp();
        if (lane == 0) {
          const uint32_t bar = su32(&sm.bar_full[ls]);
          tc::mbar_arrive_expect_tx(bar, 2u * 16384u + static_cast<uint32_t>(n) * 2048u);
          const int ky = static_cast<int>(b * a.Lk + j0);
          for (int h = 0; h < 2; ++h) {
            tc::tma_load_2d(su32(sm.kt[ls] + h * 8192), &tm_k, hk * D + 64 * h, ky, bar);
            tc::tma_load_2d(su32(sm.vt[ls] + h * 8192), &tm_v, hk * D + 64 * h, ky, bar);
          }
          for (int j = 0; j < n; ++j) {
            const int qy = static_cast<int>((b * a.Lq + q0 + sm.item_own_q[ls][j]) * Hq + hk * G);
            for (int h = 0; h < 2; ++h)
              tc::tma_load_2d(su32(sm.at[ls] + h * 8192 + j * 1024), &tm_q, 64 * h, qy, bar);
          }
        }
        ++item;
      }
    }
  } else if (warp == 9) {
    // ============================ MMA issue ==================================
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16_f32(64, 64, 0, 0);
      auto issue_s = [&](int it) -> bool {
        const int ls = it % NST, s2 = it & 1;
        if (!wait_bar(sm, &sm.bar_full[ls], (it / NST) & 1)) return false;
        tc::fence_after_sync();
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = tc::smem_desc_sw128(su32(sm.at[ls] + (kk >> 2) * 8192 + (kk & 3) * 32), 16, 1024);
          const uint64_t bd = tc::smem_desc_sw128(su32(sm.kt[ls] + (kk >> 2) * 8192 + (kk & 3) * 32), 16, 1024);
          tc::mma_bf16_ss(tbase + kSCol + 64 * s2, ad, bd, id_s, kk > 0);
        }
        tc::mma_commit(su32(&sm.bar_sdone[s2]));
        return true;
      };
      bool ok = true;
      for (int it = 0; ok && it < n_items && it < 2; ++it) ok = issue_s(it);
      for (int it = 0; ok && it < n_items; ++it) {
        const int ls = it % NST, s2 = it & 1;
        if (!wait_bar(sm, &sm.bar_pready[s2], (it >> 1) & 1)) break;
        tc::fence_after_sync();
        const int np = ((8 * sm.item_n[ls] + 15) / 16) * 16;
        const uint32_t id_o = tc::idesc_bf16_f32(128, np, 1, 0);
        for (int part = 0; part < 2; ++part) {
          const unsigned char* pt = part ? sm.pl[s2] : sm.ph[s2];
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = tc::smem_desc_sw128(su32(sm.vt[ls] + kk * 2048), 8192, 1024);
            const uint64_t bd = tc::smem_desc_sw128(su32(pt + kk * 32), 16, 1024);
            tc::mma_bf16_ss(tbase + kPCol + 64 * s2, ad, bd, id_o, part > 0 || kk > 0);
          }
        }
        tc::mma_commit(su32(&sm.bar_pvdone[s2]));
        tc::mma_commit(su32(&sm.bar_kvfree[ls]));
        if (it + 2 < n_items) ok = issue_s(it + 2);
      }
    }
    __syncwarp();
  } else {
    // ============================ item groups (warps 0-3, 4-7) ===============
    const int grp = warp >> 2, wq = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const int row = wq * 16 + lane;          // S row of this thread's TMEM lane (M=64 layout)
    for (int it = grp; it < n_items; it += 2) {
      const int ls = it % NST, s2 = it & 1;
      if (!wait_bar(sm, &sm.bar_sdone[s2], (it >> 1) & 1)) break;
      tc::fence_after_sync();
      const int n = sm.item_n[ls];
      int oq[OWN];
#pragma unroll
      for (int j = 0; j < OWN; ++j) oq[j] = j < n ? sm.item_own_q[ls][j] : 0;
      // ---- softmax: one S row per thread (lanes 0-15 of each warp) ----
      if (wq * 16 < 8 * n) {
        uint32_t r[64];
#pragma unroll
        for (int c = 0; c < 64; c += 16)
          tc::tmem_ld16(tbase + lane_off + kSCol + 64 * s2 + c, *reinterpret_cast<uint32_t(*)[16]>(&r[c]));
        tc::tmem_wait_ld();
        const int j = row >> 3, g = row & 7;
        if (lane < 16 && j < n && g < G) {
          const float w = bf2f(sm.w[sm.item_own_q[ls][j]][g][sm.item_own_slot[ls][j]]);
          const unsigned long long km = sm.kvmask[ls];
          const uint32_t km_lo = static_cast<uint32_t>(km), km_hi = static_cast<uint32_t>(km >> 32);
          float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int t = 0; t < 64; ++t) {
            const uint32_t bit = t < 32 ? (km_lo >> t) & 1u : (km_hi >> (t - 32)) & 1u;
            const float x = bit ? __uint_as_float(r[t]) * sl2 : -INFINITY;
            r[t] = __float_as_uint(x);
            mx4[t & 3] = fmaxf(mx4[t & 3], x);
          }
          const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
          const float base = mx == -INFINITY ? 0.f : mx;
          float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int t = 0; t < 64; ++t) {
            const float e = fast_exp2(__uint_as_float(r[t]) - base);   // masked keys: 2^-inf = 0
            r[t] = __float_as_uint(e);
            sum4[t & 3] += e;
          }
          const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
          const float f = sum > 0.f ? w / sum : 0.f;
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int h = 0; h < 32; ++h) {
            const float p0 = __uint_as_float(r[2 * h]) * f;
            const float p1 = __uint_as_float(r[2 * h + 1]) * f;
            hi[h] = pack_bf16x2(p0, p1);
            lo[h] = pack_bf16x2(p0 - __uint_as_float(hi[h] << 16), p1 - __uint_as_float(hi[h] & 0xffff0000u));
          }
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            *reinterpret_cast<uint4*>(sm.ph[s2] + swz_off(row, p)) =
                make_uint4(hi[4 * p], hi[4 * p + 1], hi[4 * p + 2], hi[4 * p + 3]);
            *reinterpret_cast<uint4*>(sm.pl[s2] + swz_off(row, p)) =
                make_uint4(lo[4 * p], lo[4 * p + 1], lo[4 * p + 2], lo[4 * p + 3]);
          }
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_pready[s2]));
      // ---- read-modify-write of the owners' accumulator columns ----
      if (!wait_bar(sm, &sm.bar_pvdone[s2], (it >> 1) & 1)) break;
      if (it >= 1 && !wait_bar(sm, &sm.bar_rmw[(it - 1) & 1], ((it - 1) >> 1) & 1)) break;
      tc::fence_after_sync();
#pragma unroll
      for (int j0 = 0; j0 < OWN; j0 += 4) {      // owners in batches of 4: loads, one wait, stores
        if (j0 >= n) break;
        uint32_t pv[4][8], acc[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j0 + j < n) {
            tc::tmem_ld8(tbase + lane_off + kPCol + 64 * s2 + 8 * (j0 + j), pv[j]);
            tc::tmem_ld8(tbase + lane_off + 8 * oq[j0 + j], acc[j]);
          }
        }
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j0 + j < n) {
#pragma unroll
            for (int t = 0; t < 8; ++t)
              acc[j][t] = __float_as_uint(__uint_as_float(acc[j][t]) + __uint_as_float(pv[j][t]));
            tc::tmem_st8(tbase + lane_off + 8 * oq[j0 + j], acc[j]);
          }
        }
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_rmw[s2]));
    }
    // ---- epilogue: after every item's accumulate, each group writes 16 queries
    asm volatile("bar.sync 1, 256;\n" ::: "memory");
    tc::fence_after_sync();
    if (!*reinterpret_cast<volatile int*>(&sm.abort_flag)) {
      const int d = wq * 32 + lane;
      for (int qi = grp * 16; qi < grp * 16 + 16; ++qi) {
        const int64_t rowq = q0 + qi;
        uint32_t acc[8];
        tc::tmem_ld8(tbase + lane_off + 8 * qi, acc);
        tc::tmem_wait_ld();
        if (rowq >= a.Lq) continue;
        for (int g = 0; g < G; ++g) {
          const int64_t o = ((b * a.Lq + rowq) * Hq + hk * G + g) * (int64_t)D + d;
          float r = round_bf16(__uint_as_float(acc[g]));
          if (a.local_out) r += bf2f(a.local_w[(b * a.Lq + rowq) * Hq + hk * G + g]) * bf2f(a.local_out[o]);
          a.out[o] = f2bf(r);
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && sm.abort_flag) atomicOr(&g_tc_error, 1);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

// 2-D bf16 tensor map over a row-major [rows x cols] matrix with row stride
// `stride` elements, box [box_cols x box_rows], 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t stride,
              uint32_t box_cols, uint32_t box_rows) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int mrsa_selected_attention(const void* q, const void* k, const void* v,
                                       const uint8_t* key_valid, const void* weights,
                                       const int32_t* indices, const void* local_out,
                                       const void* local_w, void* out, float sm_scale,
                                       int mask_last_token, int64_t batch, int64_t q_len,
                                       int64_t kv_len, int64_t kv_heads, int64_t groups,
                                       int64_t head_dim, int64_t topk, int64_t chunk,
                                       mrsa_stream_t stream) {
  if (!q || !k || !v || !weights || !indices || !out) return MRSA_ERR_NULL;
  if ((local_out == nullptr) != (local_w == nullptr)) return MRSA_ERR_NULL;
  if (head_dim != D || chunk != S || groups < 1 || groups > GMAX || kv_heads < 1 || batch < 1 ||
      q_len < 0 || kv_len < S || kv_len % S || kv_len / S > 64 * 32 || topk < 1 || topk > KMAX ||
      kv_heads > 65535 || batch > 65535 || batch * q_len * kv_heads * groups > 0x7fffffffLL ||
      batch * kv_len > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (local_out && !aligned16(local_out)) || (key_valid && !aligned16(key_valid)))
    return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  CUtensorMap tm_k, tm_v, tm_q;
  const uint64_t hq = static_cast<uint64_t>(kv_heads * groups);
  if (!make_map(&tm_k, k, kv_heads * D, batch * kv_len, kv_heads * D, 64, 64) ||
      !make_map(&tm_v, v, kv_heads * D, batch * kv_len, kv_heads * D, 64, 64) ||
      !make_map(&tm_q, q, D, batch * q_len * hq, D, 64, 8))
    return MRSA_ERR_LAUNCH;
  TcArgs a;
  a.w = static_cast<const __nv_bfloat16*>(weights);
  a.indices = indices;
  a.key_valid = key_valid;
  a.local_out = static_cast<const __nv_bfloat16*>(local_out);
  a.local_w = static_cast<const __nv_bfloat16*>(local_w);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.sm_scale = sm_scale;
  a.mask_last = mask_last_token;
  a.Lq = q_len;
  a.Lk = kv_len;
  a.Hkv = static_cast<int>(kv_heads);
  a.G = static_cast<int>(groups);
  a.K = static_cast<int>(topk);
  a.C = static_cast<int>(kv_len / S);
  const size_t smem = sizeof(TcSmem) + 1024;
  if (cudaFuncSetAttribute(selected_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const int64_t blocks = (q_len + QB - 1) / QB;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(kv_heads),
            static_cast<unsigned>(batch));
  selected_tc_kernel<<<grid, NTHREADS, smem, static_cast<cudaStream_t>(stream)>>>(tm_k, tm_v, tm_q, a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" int mrsa_device_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return MRSA_ERR_LAUNCH;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int)) != cudaSuccess) return MRSA_ERR_LAUNCH;
  }
  return v;
}
