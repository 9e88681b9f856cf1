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
// gathered into the rows of one MMA tile:
//   S[64 x 64]        = Q_own[64 x 128] . K_c^T         (UMMA M=64,  N=64)
//   P                 = per-row softmax of S times the route weight (hi + lo)
//   O_part^T[128 x N] = V_c^T[128 x 64] . P^T           (UMMA M=128, N=8*owners)
//   O^T[:, 8q..8q+7] += O_part^T[:, 8j..8j+7]           (TMEM read-modify-write)
// For these small shapes the tensor pipe retires about one MMA instruction per
// 44 cycles (its shared-memory operand reads), so an item costs 16 MMAs and the
// rest of the work runs beside them:
//   warps 0-3   accumulate: the read-modify-write of every item, in order,
//               one quadrant of output dims each.  Warps 1-3 also request the
//               V tiles, warp w for stage w-1: once it has accumulated item i
//               (so P.V(i) has completed and freed stage i % 3) it asks for
//               item i+3's tile.  One request per warp every third item keeps
//               them off every other role's per-item path;
//   warps 4-11  softmax, two groups of four taking alternate items; each S row
//               is read by two threads (32 columns each) with 16x32bx2 loads;
//   warps 12-13 K/Q loaders, taking alternate items: owner lists into an item
//               ring, TMA of the K tile (one 4-D box) and each owner's 8 query
//               rows (3-D box); stages are released when the item's S MMAs
//               complete.  One warp issuing every item's 1 + n copies set
//               the item rate (about 1700 cycles an item), so two share it;
//   warps 14-15 MMA issue, S and P.V respectively: each warp stays converged
//               and one elected lane issues (about a third cheaper than
//               issuing from a lone lane);
//   warps 0-11  finally, the epilogue: bf16 rounding, the fused local-branch
//               merge and the stores, three warps per TMEM quadrant.
// TMEM: accumulators in columns 0-255, two 64-column S buffers and two 64-column
// partial buffers.  An S buffer is released as soon as the item's softmax has
// loaded it and a partial buffer as soon as the accumulate warps have read it,
// so neither cycle waits on the other.
// Owners fill TMEM quadrants two at a time: owner j of an item goes to S row
// slot 2*((base + j/2) % 4) + j%2, and each softmax group's items take the
// quadrants in turn (base advances by ceil(owners/2) per item of the group),
// so an item with n owners keeps ceil(n/2) softmax warps busy with full rows
// and the group's next item runs on the other warps beside it.  Every mbarrier
// wait is bounded and a shared abort flag unwinds all roles; an aborted CTA
// waits (bounded) for its own copies and MMAs in flight.
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
constexpr int NKQ = 3;            // K/Q load stages (released after S)
constexpr int NVMAX = 4;          // V load stages: 3 with bf16 hi + lo P, 4 with fp16 P (stage 3 in the lo area)
constexpr int RING = 16;          // item-ring entries
constexpr int D = kHeadDim, S = kChunk, KMAX = 32;
constexpr int NTHREADS = 512;
constexpr int W_SMX = 4, W_LOADKQ = 12, W_LOADKQ2 = 13, W_MMA = 14;   // MMA warps 14 (S) and 15 (P.V)
constexpr int kAccCols = QB * GMAX;          // 256
constexpr int kSCol = 256, kPCol = 384;      // S buffers at 256 / 320, partial buffers at 384 / 448

struct Item {
  int n;                          // owners
  int u;                          // union index (key mask)
  int c;                          // chunk
  uint8_t oq[OWN];                // owner query (CTA-local), compact order
  uint8_t slot[OWN];              // owner's slot in its chunk list (route weight)
  int base;                       // TMEM quadrant of owners 0 and 1 (see the S row placement)
};

struct __align__(1024) TcSmem {
  unsigned char kt[NKQ][16384];   // K tile: [half][64 keys][64 dims], 128-byte swizzled
  unsigned char at[NKQ][16384];   // owner Q rows: 8 slots x [half][8 rows][64 dims]
  unsigned char vt[3][16384];     // V tiles, K's layout, read as V^T (MN-major)
  union {                         // directly after the V tiles, so stage 3 continues them
    unsigned char pl[2][8192];    // bf16 P: the lo part
    unsigned char vt3[16384];     // fp16 P: V stage 3
  };
  unsigned char ph[2][8192];      // P (bf16 hi, or fp16): [64 rows x 64 keys], row 8j+g = owner j head g
  float w[QB][GMAX][KMAX];        // route weights; a chunk's repeats summed into its first slot
  unsigned long long vmask[QB * KMAX];   // per union chunk: bit s = key s usable
  int2 ulist[QB * KMAX];          // per union chunk: (chunk, owner-query mask)
  Item ring[RING];
  uint64_t bar_kqfull[NKQ], bar_kqfree[NKQ], bar_vfull[NVMAX];
  uint64_t bar_sdone[2], bar_sfree[2], bar_pready[2], bar_pvdone[2], bar_partfree[2];
  uint64_t bar_ring[RING], bar_mma_drain[2];
  int kq_last[2][NKQ];            // per K/Q loader: last item it issued into each stage
  uint32_t tmem_base;
  int nu, n_items, abort_flag;
};
// one CTA per SM: the tile set plus 1 KB of alignment slack fits the 227 KB opt-in limit
static_assert(sizeof(TcSmem) + 1024 <= 232448, "selected-attention shared memory over budget");
static_assert(offsetof(TcSmem, vt3) == offsetof(TcSmem, vt) + 3 * 16384, "V stage 3 must follow stages 0-2");

struct TcArgs {
  const __nv_bfloat16* w;
  const int32_t* indices;
  const uint8_t* key_valid;
  const int8_t* token_keep;       // [B, Lq, Hkv, K, 64] (token refinement), or NULL
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

__device__ __forceinline__ bool aborted(TcSmem& sm) { return *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0; }

__device__ __forceinline__ bool wait_bar(TcSmem& sm, uint64_t* bar, uint32_t parity) {
  // bounded wait that also gives up when another role has aborted; a phase
  // that has already completed is seen by the cheap non-blocking test
  if (tc::mbar_test(su32(bar), parity)) return true;
  for (int round = 0; round < 4000; ++round) {
    if (tc::mbar_wait(su32(bar), parity, 1000u)) return true;
    if (aborted(sm)) return false;
  }
  *reinterpret_cast<volatile int*>(&sm.abort_flag) = 1;
  return false;
}

// The same wait taken by a whole warp: every lane gets the same answer, so the
// warp stays converged for the collective operations that follow.
__device__ __forceinline__ bool wait_bar_warp(TcSmem& sm, uint64_t* bar, uint32_t parity) {
  const bool ok = wait_bar(sm, bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// One lane of a converged warp (elect.sync).
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

// UMMA descriptor start-address field advance for a byte offset.
__device__ __forceinline__ uint64_t adv(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }

// kF16: V arrives in fp16 and P is one fp16 tile, one P.V MMA per k-step and
// four V stages; otherwise V is bf16 and P is split into bf16 hi + lo.
// kKeep: token refinement's keep rows (a.token_keep) mask each owner row.
template <bool kF16, bool kKeep>
__global__ void __launch_bounds__(NTHREADS, 1) selected_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    const __grid_constant__ CUtensorMap tm_q, TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * QB;
  const int G = a.G, K = a.K, C = a.C, Hq = a.Hkv * a.G;
  constexpr int NV = kF16 ? 4 : 3;
  unsigned char* const vbase = &sm.vt[0][0];           // V stage st at vbase + st * 16384
  // set-up tables live in the Q staging area, which is idle until the loader starts:
  // per-chunk owner masks, and the chunk lists (read once more by the loader)
  uint32_t* ownmask = reinterpret_cast<uint32_t*>(&sm.at[0][0]);
  int (*idx)[KMAX + 1] = reinterpret_cast<int (*)[KMAX + 1]>(&sm.at[1][0]);

  // ---------------- set-up: chunk lists, weights, union of chunks ----------
  if ((warp == W_LOADKQ || warp == W_LOADKQ2) && lane == 0) {
    tc::prefetch_tensormap(&tm_k);
    tc::prefetch_tensormap(&tm_q);
  }
  if (warp >= (kF16 ? 0 : 1) && warp < 4 && lane == 0) tc::prefetch_tensormap(&tm_v);
  for (int e = tid; e < C; e += NTHREADS) ownmask[e] = 0u;
  // Chunk lists and route weights.  Each query's list (K ints) and weights
  // (G x K bf16) are contiguous, so where K allows it they are read as 16-byte
  // pieces, every load issued before any is used; the scalar loops serve the
  // other cases.  Slots kk >= K, heads g >= G and queries past Lq read as
  // "no chunk" / weight 0.
  const bool vec_i = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(a.indices) & 15u) == 0;
  const bool vec_w = (K & 7) == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15u) == 0;
  if (vec_i) {
    const int per_q = K >> 2, qi = tid / per_q, piece = tid % per_q;
    int4 v = make_int4(-1, -1, -1, -1);
    if (tid < QB * per_q && q0 + qi < a.Lq)
      v = __ldg(reinterpret_cast<const int4*>(a.indices + ((b * a.Lq + q0 + qi) * a.Hkv + hk) * K) + piece);
    for (int e = tid; e < QB * KMAX; e += NTHREADS)
      if (e % KMAX >= K) idx[e / KMAX][e % KMAX] = -1;
    if (tid < QB * per_q) {
      const int cv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) idx[qi][4 * piece + i] = (cv[i] < 0 || cv[i] >= C) ? -1 : cv[i];
    }
  } else {
    for (int e = tid; e < QB * KMAX; e += NTHREADS) {
      const int qi = e / KMAX, kk = e % KMAX;
      int c = -1;
      if (kk < K && q0 + qi < a.Lq) {
        c = a.indices[((b * a.Lq + q0 + qi) * a.Hkv + hk) * K + kk];
        if (c >= C) c = -1;
      }
      idx[qi][kk] = c < 0 ? -1 : c;
    }
  }
  if (vec_w) {
    constexpr int WP = (QB * GMAX * KMAX / 8 + NTHREADS - 1) / NTHREADS;
    const int per_q = G * K / 8;
    uint4 wv[WP];
#pragma unroll
    for (int i = 0; i < WP; ++i) {
      const int k = tid + NTHREADS * i, qi = k / per_q;
      wv[i] = make_uint4(0u, 0u, 0u, 0u);
      if (qi < QB && q0 + qi < a.Lq)
        wv[i] = __ldg(reinterpret_cast<const uint4*>(a.w + ((b * a.Lq + q0 + qi) * Hq + hk * G) * K) + k % per_q);
    }
    for (int e = tid; e < QB * GMAX * KMAX; e += NTHREADS) {
      const int g = (e / KMAX) % GMAX, kk = e % KMAX;
      if (g >= G || kk >= K) sm.w[e / (GMAX * KMAX)][g][kk] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < WP; ++i) {
      const int k = tid + NTHREADS * i, qi = k / per_q;
      if (qi >= QB) continue;
      const uint32_t wd[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int e = (k % per_q) * 8 + t, g = e / K, kk = e % K;
        sm.w[qi][g][kk] = __uint_as_float((t & 1) ? (wd[t >> 1] & 0xffff0000u) : (wd[t >> 1] << 16));
      }
    }
  } else {
    for (int e = tid; e < QB * GMAX * KMAX; e += NTHREADS) {
      const int qi = e / (GMAX * KMAX), g = (e / KMAX) % GMAX, kk = e % KMAX;
      float wv = 0.f;
      if (g < G && kk < K && q0 + qi < a.Lq) wv = bf2f(a.w[((b * a.Lq + q0 + qi) * Hq + hk * G + g) * K + kk]);
      sm.w[qi][g][kk] = wv;
    }
  }
  if (tid == 0) {
    for (int s = 0; s < NKQ; ++s) {
      tc::mbar_init(su32(&sm.bar_kqfull[s]), 1);
      tc::mbar_init(su32(&sm.bar_kqfree[s]), 1);
    }
    for (int s = 0; s < NV; ++s) tc::mbar_init(su32(&sm.bar_vfull[s]), 1);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(su32(&sm.bar_sdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_sfree[s]), 4);
      tc::mbar_init(su32(&sm.bar_pvdone[s]), 1);
      tc::mbar_init(su32(&sm.bar_partfree[s]), 4);
    }
    for (int s = 0; s < 2; ++s) tc::mbar_init(su32(&sm.bar_pready[s]), 4);
    for (int r = 0; r < RING; ++r) tc::mbar_init(su32(&sm.bar_ring[r]), 1);
    for (int s = 0; s < 2; ++s) tc::mbar_init(su32(&sm.bar_mma_drain[s]), 1);
    sm.abort_flag = 0;
    for (int s = 0; s < NKQ; ++s) sm.kq_last[0][s] = sm.kq_last[1][s] = -1;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(su32(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  __syncthreads();
  // A chunk listed more than once by a query: the slots share one softmax, so
  // their weights are summed (in slot order) into the first slot.
  for (int e = tid; e < QB * KMAX; e += NTHREADS) {
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
  // owner mask per chunk (the loader picks each query's first slot of a chunk)
  for (int e = tid; e < QB * KMAX; e += NTHREADS) {
    const int c = idx[e / KMAX][e % KMAX];
    if (c >= 0) atomicOr(&ownmask[c], 1u << (e / KMAX));
  }
  __syncthreads();
  if (warp == W_LOADKQ) {
    // compact into an ascending (chunk, owners) list and count work items
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
  // per union chunk: 64-bit mask of usable keys (valid, and not the landmark slot)
  for (int e = tid; e < sm.nu; e += NTHREADS) sm.vmask[e] = 0ull;
  __syncthreads();
  for (int e = tid; e < sm.nu * 4; e += NTHREADS) {
    const int u = e >> 2, qt = e & 3;
    const int64_t j0 = static_cast<int64_t>(sm.ulist[u].x) * S + qt * 16;
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
  tc::fence_proxy_async();                   // set-up writes to the staging area precede TMA writes
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const int n_items = sm.n_items;
  const float sl2 = a.sm_scale * kLog2e;

  if (warp == W_LOADKQ || warp == W_LOADKQ2) {
    // ============================ K/Q loaders ================================
    // Both warps walk the same item sequence; warp 12 issues the even items,
    // warp 13 the odd ones.
    const int par = warp == W_LOADKQ ? 0 : 1;
    int myc[KMAX];                           // this lane's (query's) chunk list
#pragma unroll
    for (int kk = 0; kk < KMAX; ++kk) myc[kk] = idx[lane][kk];
    tc::fence_proxy_async();                 // these reads precede TMA writes to the same area
    // the chunk lists live in a K/Q stage that the first items overwrite: both
    // loaders have read them before either issues a copy
    asm volatile("bar.sync 2, 64;\n" ::: "memory");
    const uint32_t below = (1u << lane) - 1u;
    // A list of distinct chunks in ascending order, -1 only after them (as the
    // routing produces it): the union walk visits this lane's chunks in slot
    // order, so the slot of its k-th chunk is k.  Other lists search for it.
    bool sorted_list = true;
#pragma unroll
    for (int kk = 0; kk + 1 < KMAX; ++kk)
      sorted_list &= myc[kk + 1] < 0 || (myc[kk] >= 0 && myc[kk] < myc[kk + 1]);
    int visited = 0;                         // this lane's chunks walked so far
    int item = 0;
    int qcur = 0;                            // next S-tile quadrant of this warp's (softmax group's) items
    bool ok = true;
    for (int u = 0; ok && u < sm.nu; ++u) {
      const int2 ue = sm.ulist[u];
      const int c = ue.x;
      uint32_t owners = static_cast<uint32_t>(ue.y);
      int my_slot = sorted_list ? visited : -1;   // -1: found on first use
      visited += (owners >> lane) & 1u;
      while (owners) {
        // the next (up to) OWN owners, in query order
        const int j = __popc(owners & below);
        const bool mine = ((owners >> lane) & 1u) && j < OWN;
        const uint32_t grp = __ballot_sync(0xffffffffu, mine);
        owners &= ~grp;
        if ((item & 1) == par) {
          const int st = item % NKQ, r = item % RING, n = __popc(grp);
          if (my_slot < 0) {                 // only for chunks that carry one of this warp's items
            my_slot = 0;
#pragma unroll
            for (int kk = KMAX - 1; kk >= 0; --kk) my_slot = myc[kk] == c ? kk : my_slot;
          }
          // the item's owner list goes into the ring before the stage is free
          if (mine) {
            sm.ring[r].oq[j] = static_cast<uint8_t>(lane);
            sm.ring[r].slot[j] = static_cast<uint8_t>(my_slot);
          }
          const int base = qcur;
          qcur = (qcur + (n + 1) / 2) & 3;
          if (lane == 0) {
            sm.ring[r].n = n;
            sm.ring[r].u = u;
            sm.ring[r].c = c;
            sm.ring[r].base = base;
          }
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(su32(&sm.bar_ring[r]));
          if (item >= NKQ && !wait_bar_warp(sm, &sm.bar_kqfree[st], ((item / NKQ) - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t bar = su32(&sm.bar_kqfull[st]);
          if (lane == 0) {
            tc::mbar_arrive_expect_tx(bar, 16384u + static_cast<uint32_t>(n) * 2048u);
            tc::tma_load_4d(su32(sm.kt[st]), &tm_k, 0, static_cast<int>(b * a.Lk + static_cast<int64_t>(c) * S), 0,
                            hk, bar);
          }
          __syncwarp();
          if (mine) {
            const int slot = 2 * ((base + (j >> 1)) & 3) + (j & 1);
            const int qy = static_cast<int>((b * a.Lq + q0 + lane) * Hq + hk * G);
            tc::tma_load_3d(su32(sm.at[st] + slot * 2048), &tm_q, 0, qy, 0, bar);
          }
          if (lane == 0) sm.kq_last[par][st] = item;
        }
        ++item;
      }
    }
    // Wait (bounded, even after an abort) for this CTA's copies in flight.  A
    // stage is reused only after the S MMAs of its previous item completed, so
    // only the last item issued into each stage (by either warp) can be in flight.
    asm volatile("bar.sync 2, 64;\n" ::: "memory");
    if (lane == 0) {
      for (int s2 = 0; s2 < NKQ; ++s2) {
        const int it = max(sm.kq_last[0][s2], sm.kq_last[1][s2]);
        if (it >= 0 && (it & 1) == par) tc::mbar_wait(su32(&sm.bar_kqfull[s2]), (it / NKQ) & 1);
      }
    }
    __syncwarp();
  } else if (warp >= W_MMA) {
    // ============================ MMA issue (two converged warps) ============
    // Warp 14 issues the S MMAs, warp 15 the P.V MMAs.  S(i) lands in S buffer
    // i%2, free once the softmax of item i-2 has loaded it; P.V(i) lands in
    // partial buffer i%2, free once the accumulate warps have read item i-2's.
    // Each warp waits only for its own operands; every hand-off between them
    // goes through an mbarrier.
    const bool s_role = warp == W_MMA;
    const uint64_t dq0 = tc::smem_desc_sw128(su32(sm.at[0]), 16, 2048);
    const uint64_t dk0 = tc::smem_desc_sw128(su32(sm.kt[0]), 16, 1024);
    const uint64_t dv0 = tc::smem_desc_sw128(su32(vbase), 8192, 1024);
    const uint64_t dh0 = tc::smem_desc_sw128(su32(sm.ph[0]), 16, 1024);
    const uint64_t dl0 = tc::smem_desc_sw128(su32(sm.pl[0]), 16, 1024);
    if (s_role) {
      constexpr uint32_t id_s = tc::idesc_bf16_f32(64, 64, 0, 0);
      for (int it = 0; it < n_items; ++it) {
        const int st = it % NKQ, s2 = it & 1;
        bool rdy = tc::mbar_test(su32(&sm.bar_kqfull[st]), (it / NKQ) & 1);
        if (it >= 2) rdy &= tc::mbar_test(su32(&sm.bar_sfree[s2]), ((it >> 1) - 1) & 1);
        if (!__all_sync(0xffffffffu, rdy)) {
          if (!wait_bar_warp(sm, &sm.bar_kqfull[st], (it / NKQ) & 1)) break;
          if (it >= 2 && !wait_bar_warp(sm, &sm.bar_sfree[s2], ((it >> 1) - 1) & 1)) break;
        }
        tc::fence_after_sync();
        const uint64_t da = adv(dq0, st * 16384), db = adv(dk0, st * 16384);
        const uint32_t dS = tbase + kSCol + 64 * s2;
        if (elect_one()) {
          tc::mma_bf16<false>(dS, da, db, id_s);
#pragma unroll
          for (int kk = 1; kk < 8; ++kk)
            tc::mma_bf16<true>(dS, adv(da, (kk >> 2) * 1024 + (kk & 3) * 32),
                               adv(db, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
          tc::mma_commit(su32(&sm.bar_sdone[s2]));
          tc::mma_commit(su32(&sm.bar_kqfree[st]));
        }
        __syncwarp();
      }
    } else {
      for (int it = 0; it < n_items; ++it) {
        const int sv = it % NV, p2 = it & 1;
        bool rdy = tc::mbar_test(su32(&sm.bar_pready[p2]), (it >> 1) & 1) &
                   tc::mbar_test(su32(&sm.bar_vfull[sv]), (it / NV) & 1);
        if (it >= 2) rdy &= tc::mbar_test(su32(&sm.bar_partfree[p2]), ((it >> 1) - 1) & 1);
        if (!__all_sync(0xffffffffu, rdy)) {
          if (!wait_bar_warp(sm, &sm.bar_pready[p2], (it >> 1) & 1)) break;
          if (!wait_bar_warp(sm, &sm.bar_vfull[sv], (it / NV) & 1)) break;
          if (it >= 2 && !wait_bar_warp(sm, &sm.bar_partfree[p2], ((it >> 1) - 1) & 1)) break;
        }
        tc::fence_after_sync();
        // the owner count is read only now: the item's softmax has consumed its ring
        // entry (pready), so it is written; clamped so the MMA shape is always valid
        const int np = ((8 * min(max(sm.ring[it % RING].n, 1), OWN) + 15) / 16) * 16;
        // kind::f16 with fp16 A and B: the bf16 format bits cleared
        const uint32_t id_o = tc::idesc_bf16_f32(128, np, 1, 0) & (kF16 ? ~((1u << 7) | (1u << 10)) : ~0u);
        const uint64_t dv = adv(dv0, sv * 16384), dh = adv(dh0, p2 * 8192), dl = adv(dl0, p2 * 8192);
        const uint32_t dP = tbase + kPCol + 64 * p2;
        if (elect_one()) {
          tc::mma_bf16<false>(dP, dv, dh, id_o);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk) tc::mma_bf16<true>(dP, adv(dv, kk * 2048), adv(dh, kk * 32), id_o);
          if constexpr (!kF16) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) tc::mma_bf16<true>(dP, adv(dv, kk * 2048), adv(dl, kk * 32), id_o);
          }
          tc::mma_commit(su32(&sm.bar_pvdone[p2]));
        }
        __syncwarp();
      }
    }
    // every MMA issued by this warp has completed once this phase lands
    if (elect_one()) {
      tc::mma_commit(su32(&sm.bar_mma_drain[s_role ? 0 : 1]));
      tc::mbar_wait(su32(&sm.bar_mma_drain[s_role ? 0 : 1]), 0);
    }
    __syncwarp();
  } else if (warp >= W_SMX) {
    // ============================ softmax (warps 4-7, 8-11) ==================
    const int grp = (warp - W_SMX) >> 2, q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int t = lane & 15, hf = lane >> 4;

    const int g = t & 7;
    for (int it = grp; it < n_items; it += 2) {
      const int p2 = it & 1, r = it % RING;
      if (!wait_bar_warp(sm, &sm.bar_ring[r], (it / RING) & 1)) break;
      const int n = sm.ring[r].n;
      const int qo = 2 * ((q - sm.ring[r].base) & 3);   // this quadrant holds owners qo and qo + 1
      const int jrow = qo + (t >> 3);        // owner (compact index) of this thread's row
      const bool row_on = jrow < n;
      float w = 0.f;
      uint32_t km = 0xFFFFFFFFu;             // rows without an owner are computed and dropped
      uint4 keep[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};   // token refinement: this row's 32 keep bytes
      if (row_on) {
        const int oqj = sm.ring[r].oq[jrow], slot = sm.ring[r].slot[jrow];
        if (g < G) w = sm.w[oqj][g][slot];
        const unsigned long long vm = sm.vmask[sm.ring[r].u];
        km = static_cast<uint32_t>(hf ? (vm >> 32) : vm);
        if constexpr (kKeep) {               // issued before the S wait, used after it
          const uint4* kp = reinterpret_cast<const uint4*>(
              a.token_keep + (((b * a.Lq + q0 + oqj) * a.Hkv + hk) * K + slot) * S + 32 * hf);
          keep[0] = __ldg(kp);
          keep[1] = __ldg(kp + 1);
        }
      }
      if (!wait_bar_warp(sm, &sm.bar_sdone[p2], (it >> 1) & 1)) break;
      if constexpr (kKeep) {
        if (row_on) {
          const uint32_t wd[8] = {keep[0].x, keep[0].y, keep[0].z, keep[0].w,
                                  keep[1].x, keep[1].y, keep[1].z, keep[1].w};
          uint32_t kb = 0u;
#pragma unroll
          for (int i = 0; i < 32; ++i) kb |= static_cast<uint32_t>(((wd[i >> 2] >> (8 * (i & 3))) & 0xFFu) != 0u) << i;
          km &= kb;
        }
      }
      tc::fence_after_sync();
      // Quadrant q holds the rows of owners qo and qo+1: with fewer than qo+1
      // owners the warp has no row to compute and keeps only its hand-offs,
      // which frees issue slots for the other roles.
      const bool quad_on = qo < n;           // warp-uniform
      uint32_t x[32];
      if (quad_on) {
        tc::tmem_ld_16x32bx2_x32(tbase + lane_off + kSCol + 64 * p2, x);
        tc::tmem_wait_ld();
      }
      // the S buffer is free once every warp of the group has loaded its rows
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_sfree[p2]));
      uint32_t hi[16], lo[16];
      if (quad_on) {
        // masked keys -> -inf; the common case (every key usable but possibly the
        // last of the chunk) takes one select instead of 32
        if (__all_sync(0xffffffffu, (km | 0x80000000u) == 0xFFFFFFFFu)) {
          if (!(km >> 31)) x[31] = __float_as_uint(-INFINITY);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (!((km >> c) & 1u)) x[c] = __float_as_uint(-INFINITY);
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(x[c]));
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float nb = mx == -INFINITY ? 0.f : -mx * sl2;
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float e = fast_exp2(fmaf(__uint_as_float(x[c]), sl2, nb));   // masked keys: 2^-inf = 0
          x[c] = __float_as_uint(e);
          sum4[c & 3] += e;
        }
        float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        // P = route weight x softmax: as bf16 hi + lo, or as one fp16 tile (11
        // significant bits; values small enough to be fp16 subnormals carry an
        // absolute error below 2^-25, far under the bf16 output's resolution)
        const float f = sum > 0.f ? __fdividef(w, sum) : 0.f;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float p0 = __uint_as_float(x[2 * h]) * f;
          const float p1 = __uint_as_float(x[2 * h + 1]) * f;
          if constexpr (kF16) {
            hi[h] = pack_f16x2(p0, p1);
          } else {
            hi[h] = pack_bf16x2(p0, p1);
            lo[h] = pack_bf16x2(p0 - __uint_as_float(hi[h] << 16), p1 - __uint_as_float(hi[h] & 0xffff0000u));
          }
        }
      }
      // the P buffer is free once the P.V of item it-2 has completed
      if (it >= 2 && !wait_bar_warp(sm, &sm.bar_pvdone[p2], ((it - 2) >> 1) & 1)) break;
      if (row_on) {
        const int row = 8 * jrow + g;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          *reinterpret_cast<uint4*>(sm.ph[p2] + swz_off(row, 4 * hf + p)) =
              make_uint4(hi[4 * p], hi[4 * p + 1], hi[4 * p + 2], hi[4 * p + 3]);
          if constexpr (!kF16)
            *reinterpret_cast<uint4*>(sm.pl[p2] + swz_off(row, 4 * hf + p)) =
                make_uint4(lo[4 * p], lo[4 * p + 1], lo[4 * p + 2], lo[4 * p + 3]);
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(su32(&sm.bar_pready[p2]));
    }
  } else {
    // ============================ accumulate (warps 0-3) =====================
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    // V tile of item `v` into stage v % NV (warp v % NV, +1 with three stages); the ring entry names the chunk
    auto load_v = [&](int v) -> bool {
      const int r = v % RING;
      if (!wait_bar_warp(sm, &sm.bar_ring[r], (v / RING) & 1)) return false;
      if (elect_one()) {
        const uint32_t bar = su32(&sm.bar_vfull[v % NV]);
        tc::mbar_arrive_expect_tx(bar, 16384u);
        tc::tma_load_4d(su32(vbase + (v % NV) * 16384), &tm_v, 0, static_cast<int>(b * a.Lk + static_cast<int64_t>(sm.ring[r].c) * S),
                        0, hk, bar);
      }
      __syncwarp();
      return true;
    };
    const int vst = kF16 ? warp : warp - 1;  // this warp's V stage (warps 0-3, or 1-3 with three stages)
    int vlast = -1;                          // last item whose V tile this warp requested
    bool ok = true;
    if (vst >= 0 && vst < n_items) {
      ok = load_v(vst);
      if (ok) vlast = vst;
    }
    for (int it = 0; ok && it < n_items; ++it) {
      const int p2 = it & 1, r = it % RING;
      if (!wait_bar_warp(sm, &sm.bar_ring[r], (it / RING) & 1)) break;
      const int n = sm.ring[r].n;
      int oq[OWN];
#pragma unroll
      for (int j = 0; j < OWN; ++j) oq[j] = sm.ring[r].oq[j];
      if (!wait_bar_warp(sm, &sm.bar_pvdone[p2], (it >> 1) & 1)) break;
      tc::fence_after_sync();
      tc::tmem_wait_st();                    // previous item's accumulator stores have landed
#pragma unroll
      for (int j0 = 0; j0 < OWN; j0 += 4) {  // owners in batches of 4: loads, one wait, stores
        if (j0 >= n) break;
        uint32_t pv[4][8], acc[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j0 + j < n) {
            tc::tmem_ld8(tbase + lane_off + kPCol + 64 * p2 + 8 * (j0 + j), pv[j]);
            tc::tmem_ld8(tbase + lane_off + 8 * oq[j0 + j], acc[j]);
          }
        }
        tc::tmem_wait_ld();
        if (j0 + 4 >= n) {                   // last partial columns read: release the buffer
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
      // P.V(it) has completed: stage it % NV takes item it+NV's tile
      if (vst == it % NV && it + NV < n_items) {
        if (!load_v(it + NV)) break;
        vlast = it + NV;
      }
    }
    tc::tmem_wait_st();
    // (bounded) wait for this warp's last V copy, in flight after an abort; only
    // this warp loads its stage, so the phase it waits for is unambiguous
    if (vlast >= 0 && lane == 0) tc::mbar_wait(su32(&sm.bar_vfull[vst]), (vlast / NV) & 1);
    __syncwarp();
  }

  if (warp < W_LOADKQ) {
    // ============================ epilogue (warps 0-11) ======================
    // The softmax warps join the accumulate warps once the last item has been
    // accumulated: three warps per TMEM quadrant, each taking batches of four
    // queries whose local-branch inputs are loaded before the accumulators.
    tc::fence_before_sync();
    asm volatile("bar.sync 1, 384;\n" ::: "memory");
    tc::fence_after_sync();
    // The local branch of this CTA's rows (G contiguous rows of D values per
    // query) is staged in the idle K/Q staging area first: every K/Q copy and
    // S MMA has completed once the last item is accumulated.  Sixteen-byte
    // loads, all issued before any is used, instead of one two-byte load per
    // (query, head, dim) that each waited out its own memory latency.
    __nv_bfloat16* lsm = reinterpret_cast<__nv_bfloat16*>(&sm.kt[0][0]);   // [QB][G][D]
    __nv_bfloat16* lwsm = lsm + QB * GMAX * D;                              // [QB][G]
    static_assert(QB * GMAX * (D + 1) * 2 <= 2 * NKQ * 16384, "local-branch staging over the K/Q area");
    const bool fused = a.local_out != nullptr;
    if (fused && !__any_sync(0xffffffffu, aborted(sm))) {
      constexpr int kEpiThreads = 384;
      constexpr int LMAX = (QB * GMAX * D * 2 / 16 + kEpiThreads - 1) / kEpiThreads;
      const int per_q = G * (D * 2 / 16);    // 16-byte pieces of one query's rows
      uint4 v[LMAX];
#pragma unroll
      for (int i = 0; i < LMAX; ++i) {
        const int k = tid + kEpiThreads * i, q = k / per_q;
        v[i] = make_uint4(0u, 0u, 0u, 0u);
        if (q < QB && q0 + q < a.Lq)
          v[i] = __ldg(reinterpret_cast<const uint4*>(a.local_out + ((b * a.Lq + q0 + q) * Hq + hk * G) * D) + k % per_q);
      }
      __nv_bfloat16 wv = f2bf(0.f);
      if (tid < QB * G && q0 + tid / G < a.Lq) wv = a.local_w[(b * a.Lq + q0 + tid / G) * Hq + hk * G + tid % G];
#pragma unroll
      for (int i = 0; i < LMAX; ++i) {
        const int k = tid + kEpiThreads * i;
        if (k < QB * per_q) reinterpret_cast<uint4*>(lsm)[k] = v[i];
      }
      if (tid < QB * G) lwsm[tid] = wv;
    }
    asm volatile("bar.sync 1, 384;\n" ::: "memory");
    if (!__any_sync(0xffffffffu, aborted(sm))) {
      constexpr int EB = 4;
      const int qd = warp & 3, part = warp >> 2;
      const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
      const int d = qd * 32 + lane;
      for (int q1 = part * EB; q1 < QB; q1 += 3 * EB) {
        uint32_t acc[EB][8];
        float lw[EB][GMAX], lo[EB][GMAX];
#pragma unroll
        for (int j = 0; j < EB; ++j) {
#pragma unroll
          for (int gg = 0; gg < GMAX; ++gg) {
            lw[j][gg] = 0.f;
            lo[j][gg] = 0.f;
            if (fused && gg < G) {
              lw[j][gg] = bf2f(lwsm[(q1 + j) * G + gg]);
              lo[j][gg] = bf2f(lsm[((q1 + j) * G + gg) * D + d]);
            }
          }
          tc::tmem_ld8(tbase + lane_off + 8 * (q1 + j), acc[j]);
        }
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < EB; ++j) {
          const int64_t rowq = q0 + q1 + j;
          if (rowq >= a.Lq) continue;
#pragma unroll
          for (int gg = 0; gg < GMAX; ++gg) {
            if (gg >= G) continue;
            const int64_t o = ((b * a.Lq + rowq) * Hq + hk * G + gg) * (int64_t)D + d;
            a.out[o] = f2bf(round_bf16(__uint_as_float(acc[j][gg])) + lw[j][gg] * lo[j][gg]);
          }
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

// bf16 tensor map with 128-byte swizzle over `rank` dims (innermost first).
bool make_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
              const cuuint32_t* box, CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return false;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return g_encode(m, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims,
                  strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace {

template <bool kF16, bool kKeep>
int selected_launch(const void* q, const void* k, const void* v, const uint8_t* key_valid, const void* weights,
                    const int32_t* indices, const void* local_out, const void* local_w, void* out, float sm_scale,
                    int mask_last_token, int64_t batch, int64_t q_len, int64_t kv_len, int64_t kv_heads,
                    int64_t groups, int64_t head_dim, int64_t topk, int64_t chunk, mrsa_stream_t stream,
                    const int8_t* token_keep = nullptr) {
  if (!q || !k || !v || !weights || !indices || !out) return MRSA_ERR_NULL;
  if ((local_out == nullptr) != (local_w == nullptr)) return MRSA_ERR_NULL;
  if (head_dim != D || chunk != S || groups < 1 || groups > GMAX || kv_heads < 1 || batch < 1 ||
      q_len < 0 || kv_len < S || kv_len % S || kv_len / S > 64 * 32 || topk < 1 || topk > KMAX ||
      kv_heads > 65535 || batch > 65535 || batch * q_len * kv_heads * groups > 0x7fffffffLL ||
      batch * kv_len > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (local_out && !aligned16(local_out)) || (key_valid && !aligned16(key_valid)) ||
      (token_keep && !aligned16(token_keep)))
    return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  // K, V: [B*Lk rows][Hkv*128] viewed as (dim-in-half, row, half, head): one box = one chunk tile.
  // Q: [B*Lq*Hq rows][128] viewed as (dim-in-half, row, half): one box = 8 rows of one query.
  CUtensorMap tm_k, tm_v, tm_q;
  const cuuint64_t kv_dims[4] = {64, static_cast<cuuint64_t>(batch * kv_len), 2, static_cast<cuuint64_t>(kv_heads)};
  const cuuint64_t kv_str[3] = {static_cast<cuuint64_t>(kv_heads * D * 2), 128, 256};
  const cuuint32_t kv_box[4] = {64, 64, 2, 1};
  const cuuint64_t q_dims[3] = {64, static_cast<cuuint64_t>(batch * q_len * kv_heads * groups), 2};
  const cuuint64_t q_str[2] = {256, 128};
  const cuuint32_t q_box[3] = {64, 8, 2};
  if (!make_map(&tm_k, k, 4, kv_dims, kv_str, kv_box) ||
      !make_map(&tm_v, v, 4, kv_dims, kv_str, kv_box,
                kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) ||
      !make_map(&tm_q, q, 3, q_dims, q_str, q_box))
    return MRSA_ERR_LAUNCH;
  TcArgs a;
  a.w = static_cast<const __nv_bfloat16*>(weights);
  a.indices = indices;
  a.key_valid = key_valid;
  a.token_keep = token_keep;
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
  if (kKeep != (token_keep != nullptr)) return MRSA_ERR_NULL;
  if (cudaFuncSetAttribute(selected_tc_kernel<kF16, kKeep>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const int64_t blocks = (q_len + QB - 1) / QB;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(kv_heads),
            static_cast<unsigned>(batch));
  selected_tc_kernel<kF16, kKeep><<<grid, NTHREADS, smem, static_cast<cudaStream_t>(stream)>>>(tm_k, tm_v, tm_q, a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
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
  mrsa::DeviceScope device_scope(q);
  return selected_launch<false, false>(q, k, v, key_valid, weights, indices, local_out, local_w, out, sm_scale,
                                mask_last_token, batch, q_len, kv_len, kv_heads, groups, head_dim, topk, chunk,
                                stream);
}

extern "C" int mrsa_selected_attention_f16v(const void* q, const void* k, const void* v_f16,
                                            const uint8_t* key_valid, const void* weights,
                                            const int32_t* indices, const void* local_out,
                                            const void* local_w, void* out, float sm_scale,
                                            int mask_last_token, int64_t batch, int64_t q_len,
                                            int64_t kv_len, int64_t kv_heads, int64_t groups,
                                            int64_t head_dim, int64_t topk, int64_t chunk,
                                            mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  return selected_launch<true, false>(q, k, v_f16, key_valid, weights, indices, local_out, local_w, out, sm_scale,
                               mask_last_token, batch, q_len, kv_len, kv_heads, groups, head_dim, topk, chunk,
                               stream);
}

extern "C" int mrsa_selected_attention_keep(const void* q, const void* k, const void* v,
                                            const uint8_t* key_valid, const void* weights,
                                            const int32_t* indices, const int8_t* token_keep,
                                            const void* local_out, const void* local_w, void* out,
                                            float sm_scale, int mask_last_token, int v_f16, int64_t batch,
                                            int64_t q_len, int64_t kv_len, int64_t kv_heads, int64_t groups,
                                            int64_t head_dim, int64_t topk, int64_t chunk,
                                            mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  if (token_keep == nullptr) return MRSA_ERR_NULL;
  if (v_f16)
    return selected_launch<true, true>(q, k, v, key_valid, weights, indices, local_out, local_w, out, sm_scale,
                                       mask_last_token, batch, q_len, kv_len, kv_heads, groups, head_dim, topk,
                                       chunk, stream, token_keep);
  return selected_launch<false, true>(q, k, v, key_valid, weights, indices, local_out, local_w, out, sm_scale,
                                      mask_last_token, batch, q_len, kv_len, kv_heads, groups, head_dim, topk,
                                      chunk, stream, token_keep);
}

extern "C" int mrsa_device_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return MRSA_ERR_LAUNCH;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int)) != cudaSuccess) return MRSA_ERR_LAUNCH;
  }
  const int r = mrsa::route_error_flags(clear), l = mrsa::local_error_flags(clear),
            cv = mrsa::convert_error_flags(clear), bw = mrsa::bwd_error_flags(clear),
            gm = mrsa::gemm_error_flags(clear), lb = mrsa::local_bwd_error_flags(clear);
  if (r < 0 || l < 0 || cv < 0 || bw < 0 || gm < 0 || lb < 0) return MRSA_ERR_LAUNCH;
  return (v ? 1 : 0) | (r ? 2 : 0) | (l ? 4 : 0) | (cv ? 8 : 0) | (bw ? 16 : 0) | (gm ? 32 : 0) | (lb ? 64 : 0);
}
