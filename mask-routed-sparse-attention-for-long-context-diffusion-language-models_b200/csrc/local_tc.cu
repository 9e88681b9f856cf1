// Bidirectional banded GQA attention with natural-log LSE on the tcgen05
// tensor cores (local branch of the route layer, window W+63 with
// landmark/invalid K,V zeroed; SWA layers, window 1280).  Semantics of
// dream_dllm_hils/local_attention.py:35-107: zeroed keys keep logit 0 in the
// softmax and add no value; keys with |i-j| > window are out.
//
// One CTA owns two query tiles of LQ = floor(128 / G) queries each (18 for
// GQA 7:1) of one KV head.  A tile's MMA rows are G*qi + g = (query qi, head
// g of the group; rows >= LQ*G are zero padding), so each 64-key K/V tile is
// read once for all heads of the group and both query tiles.  Per query tile
// and key tile t:
//   S[128 x 64]  = Q . K_t^T               (UMMA M=128, N=64,  K=128, TMEM)
//   P            = exp2(S*scale*log2e - m)  (one thread per row, online max)
//   O[128 x 128] += P . V_t                (UMMA M=128, N=128, K=64, A = P in TMEM)
// P (fp16 when V is fp16, else bf16 hi + lo parts, ~16 significant bits) is
// written back over its own S buffer and read by P.V from there.  Each row keeps a
// reference max that moves (rescaling O in TMEM) only when a tile max exceeds
// it by more than 2^8.
// Warps 0-3 and 4-7: the softmax and epilogue of query tiles 0 and 1 (warp w
// = TMEM lanes 32(w%4)..+31 = rows); group g walks the key tiles of its own
// band in order with two S buffers, so the S of its next tile is computed
// while it works on the current one.  Warp 8: TMA of Q and of the K tiles (4
// stages) and the per-tile key validity masks; warp 11: TMA of the V tiles
// (4 stages); warps 9 and 10: MMA issue for groups 0 and 1 (converged,
// elect.sync): S(first), S(first+1), then per tile P.V(t) and, once that P.V
// has read the buffer, S(t+2) into it.  A K or V stage is released by both
// groups (an MMA commit, or a plain arrive for a tile outside the group's
// band).  Every mbarrier wait is bounded and unwinds through a shared abort
// flag.  A row's tiles are its own group's, in order, whichever rows share its
// CTA (tiles outside its band add exact zeros), so a row's result does not
// depend on how rows are cut into CTAs.
//
// The same kernel also runs the causal chunk-expanded window of
// ops/flex_attn_tilelang.py:26-276 (flex_attn_tl): a row at absolute position
// p sees keys j in [start, p] with start = p - W + 1, rounded down to a chunk
// boundary when expanding, and masked keys (landmark slots, mask_lmk) are
// excluded from the softmax instead of zeroed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int LN = 64;            // keys per tile
constexpr int NKS = 4;            // K stages
constexpr int NVS = 4;            // V stages
constexpr int NMS = 8;            // key-mask slots
constexpr int D = kHeadDim;
constexpr int L_THREADS = 384;    // warps 0-7 softmax (two groups), 8 Q/K TMA + masks, 9-10 MMA, 11 V TMA
constexpr int L_W_KLOAD = 8, L_W_MMA = 9, L_W_VLOAD = 11;
constexpr uint32_t kOCol = 256;   // O of groups 0 / 1 at [256, 384) / [384, 512); S buffer i at [64 i, 64 i + 64)

struct __align__(1024) LocalSmem {
  unsigned char q[2][2][16384];       // [query tile][half][128 rows = (query, head)][64 dims], 128-byte swizzled
  unsigned char k[NKS][16384];        // [half][64 keys][64 dims]
  unsigned char v[NVS][16384];        // same, read as the MN-major B operand of P.V
  unsigned long long kmask[NMS];      // bit j: key j of the tile is usable (not zeroed); slot t % NMS
  uint64_t qfull, kfull[NKS], kfree[NKS], vfull[NVS], vfree[NVS], mfull[NMS];
  uint64_t sfull[4], pready[4], pfree[4], drain[2];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(LocalSmem) + 1024 <= 232448, "local attention shared memory over budget");

struct LocalArgs {
  const uint8_t* key_valid;
  const int64_t* qpos;  // per query row position (NULL: q_offset + row)
  __nv_bfloat16* out;
  float* lse;
  int64_t window, Lq, Lk, q_offset;
  int64_t shift;        // absolute position of key 0 (landmark test, chunk rounding)
  int skip_inert, chunk, Hq, Hkv, G;
  int causal;           // 0: |i-j| <= window;  1: flex_attn_tl's causal window
  int expand;           // causal: round the left edge down to a chunk boundary
  int exclude;          // masked keys leave the softmax (-inf) instead of keeping logit 0
  float sm_scale;
};

__device__ __host__ __forceinline__ int64_t floor_div(int64_t x, int64_t d) {
  return x >= 0 ? x / d : -((-x + d - 1) / d);
}

// Key range [lo, hi] (key indices, before clipping to the sequence) of the row
// at key-index position pos.
__device__ __forceinline__ void row_band(const LocalArgs& a, int64_t pos, int64_t& lo, int64_t& hi) {
  if (a.causal) {
    int64_t start = pos + a.shift - a.window + 1;
    if (a.expand) start = floor_div(start, a.chunk) * a.chunk;
    lo = start - a.shift;
    hi = pos;
  } else {
    lo = pos - a.window;
    hi = pos + a.window;
  }
}

__device__ int g_local_error;

// 2^y for a pair on the FMA pipe, taking load off the special-function unit:
// Cody-Waite reduction y = n + f (n = round(y) through the 1.5 * 2^23 shift,
// |f| <= 1/2), 2^f by a degree-4 polynomial whose coefficients were fitted
// for this kernel by Remez exchange on [-1/2, 1/2] (relative error 2.7e-6
// evaluated in fp32, below fp16 P's rounding), and 2^n added to the exponent
// field.  y is clamped to >= -126, so -inf gives 2^-126 rather than 0: only
// for tiles without masked columns, where every row's sum is >= 1.
__device__ __forceinline__ float2 exp2_poly2(float2 y) {
  constexpr float kShift = 12582912.0f;   // 1.5 * 2^23
  y.x = fmaxf(y.x, -126.0f);
  y.y = fmaxf(y.y, -126.0f);
  const float2 r = fadd2(y, make_float2(kShift, kShift));
  const float2 n = fadd2(r, make_float2(-kShift, -kShift));
  const float2 f = ffma2(n, make_float2(-1.0f, -1.0f), y);
  float2 p = ffma2(make_float2(0.009570102f, 0.009570102f), f, make_float2(0.05591786f, 0.05591786f));
  p = ffma2(p, f, make_float2(0.24024744f, 0.24024744f));
  p = ffma2(p, f, make_float2(0.69312179f, 0.69312179f));
  p = ffma2(p, f, make_float2(0.99999928f, 0.99999928f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(r.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(r.y) << 23)));
}

// kF16: V arrives in fp16 and P (values up to 2^8 under the lazy rescale) is
// one fp16 tile, one P.V MMA per k-step; otherwise P is bf16 hi + lo.
template <bool kF16>
__global__ void __launch_bounds__(L_THREADS, 1) local_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, LocalArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  LocalSmem& sm = *reinterpret_cast<LocalSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int G = a.G, LQ = 128 / G, nrows = LQ * G;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 2 * LQ;   // query tile g starts at q0 + g LQ
  // key tiles of each query tile's band (absolute tile indices; empty: lo > hi)
  int64_t tile_lo[2], tile_hi[2];
#pragma unroll
  for (int qt = 0; qt < 2; ++qt) {
    const int64_t r0 = q0 + qt * LQ;
    const int64_t nr = (a.Lq - r0) < LQ ? (a.Lq - r0) : LQ;
    tile_lo[qt] = 1;
    tile_hi[qt] = 0;
    if (nr <= 0) continue;
    // positions of the tile's first and last rows (the band is monotone in the
    // position); with explicit row positions, their minimum and maximum
    int64_t p_min = a.q_offset + r0, p_max = a.q_offset + r0 + nr - 1;
    if (a.qpos != nullptr) {
      p_min = a.qpos[r0];
      p_max = p_min;
      for (int i = 1; i < nr; ++i) {
        const int64_t p = a.qpos[r0 + i];
        p_min = p < p_min ? p : p_min;
        p_max = p > p_max ? p : p_max;
      }
    }
    int64_t j_lo, j_hi, unused;
    row_band(a, p_min, j_lo, unused);
    row_band(a, p_max, unused, j_hi);
    if (j_lo < 0) j_lo = 0;
    if (j_hi > a.Lk - 1) j_hi = a.Lk - 1;
    if (j_hi < j_lo) continue;
    tile_lo[qt] = j_lo / LN;
    tile_hi[qt] = j_hi / LN;
  }
  // the CTA's key tiles: the union of the two ranges, local index t in [0, NTL)
  const bool has0 = tile_lo[0] <= tile_hi[0], has1 = tile_lo[1] <= tile_hi[1];
  int64_t u_lo = 0, u_hi = -1;
  if (has0 || has1) {
    u_lo = has0 ? tile_lo[0] : tile_lo[1];
    u_hi = has1 ? tile_hi[1] : tile_hi[0];
    if (has0 && has1) {
      u_lo = tile_lo[0] < tile_lo[1] ? tile_lo[0] : tile_lo[1];
      u_hi = tile_hi[0] > tile_hi[1] ? tile_hi[0] : tile_hi[1];
    }
  }
  const int t_lo = static_cast<int>(u_lo);
  const int NTL = static_cast<int>(u_hi - u_lo + 1);
  // group g's local tiles [ga[g], gb[g]] (empty: ga > gb); its k-th tile uses S
  // buffer 2g + (k & 1) for the (k >> 1)-th time
  int ga[2], gb[2];
#pragma unroll
  for (int qt = 0; qt < 2; ++qt) {
    const bool h = qt ? has1 : has0;
    ga[qt] = h ? static_cast<int>(tile_lo[qt] - u_lo) : 1;
    gb[qt] = h ? static_cast<int>(tile_hi[qt] - u_lo) : 0;
  }

  if (tid == 0) {
    tc::mbar_init(tc::smem_addr(&sm.qfull), 1);
    for (int s = 0; s < NKS; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.kfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.kfree[s]), 2);
    }
    for (int s = 0; s < NVS; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.vfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.vfree[s]), 2);
    }
    for (int s = 0; s < NMS; ++s) tc::mbar_init(tc::smem_addr(&sm.mfull[s]), 1);
    for (int s = 0; s < 4; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.sfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.pready[s]), 4);
      tc::mbar_init(tc::smem_addr(&sm.pfree[s]), 1);
    }
    for (int s = 0; s < 2; ++s) tc::mbar_init(tc::smem_addr(&sm.drain[s]), 1);
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  // zero the padding rows of the Q tiles (the TMA boxes fill rows [0, nrows)),
  // visible to the tensor core's async proxy
  for (int i = tid; i < 4 * (128 - nrows) * 8; i += L_THREADS) {
    const int h = i / ((128 - nrows) * 8), rem = i % ((128 - nrows) * 8);
    *reinterpret_cast<uint4*>(sm.q[h >> 1][h & 1] + (nrows + rem / 8) * 128 + (rem % 8) * 16) =
        make_uint4(0u, 0u, 0u, 0u);
  }
  tc::fence_proxy_async();
  if (warp == 0) {
    tc::tmem_alloc(tc::smem_addr(&sm.tmem_base), 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base;

  if (warp == L_W_KLOAD) {
    // ============================ Q, K tiles + key masks ======================
    const uint32_t qb = tc::smem_addr(&sm.qfull);
    if (lane == 0) {
      tc::prefetch_tensormap(&tm_q);
      tc::prefetch_tensormap(&tm_k);
      tc::mbar_arrive_expect_tx(qb, static_cast<uint32_t>(nrows) * 512u);
#pragma unroll
      for (int qt = 0; qt < 2; ++qt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tc::tma_load_4d(tc::smem_addr(sm.q[qt][h]), &tm_q, 0, hk * G, h, static_cast<int>(b * a.Lq + q0 + qt * LQ), qb);
    }
    // key-validity bytes of tile tt (this lane's keys 32h + lane), requested one
    // tile ahead so their latency is not on the copy-issue path
    auto valid_bytes = [&](int tt, uint32_t (&vb)[2]) {
      const int64_t jt = static_cast<int64_t>(t_lo + tt) * LN;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t j = jt + 32 * h + lane;
        vb[h] = (a.key_valid != nullptr && tt < NTL && j < a.Lk) ? a.key_valid[b * a.Lk + j] : 1u;
      }
    };
    uint32_t vb_next[2];
    valid_bytes(0, vb_next);
    int t = 0;
    for (; t < NTL; ++t) {
      const int st = t % NKS;
      const uint32_t vb[2] = {vb_next[0], vb_next[1]};
      valid_bytes(t + 1, vb_next);
      // stage st was released by both groups for tile t - NKS; mask slot t % NMS
      // was last read by the softmax of tile t - NMS, which precedes that release
      if (t >= NKS && !tc::wait_bounded_warp(tc::smem_addr(&sm.kfree[st]), ((t / NKS) - 1) & 1, abort_flag)) break;
      const int64_t j0 = static_cast<int64_t>(t_lo + t) * LN;
      // usable keys of the tile: inside the sequence, valid, and not a landmark slot when skip_inert
      uint32_t mk[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t j = j0 + 32 * h + lane;
        bool ok = j < a.Lk && vb[h] != 0u;
        if (ok && a.skip_inert) ok = ((j + a.shift + 1) % a.chunk) != 0;
        mk[h] = __ballot_sync(0xffffffffu, ok);
      }
      if (lane == 0) {
        sm.kmask[t % NMS] = static_cast<unsigned long long>(mk[0]) | (static_cast<unsigned long long>(mk[1]) << 32);
        tc::mbar_arrive(tc::smem_addr(&sm.mfull[t % NMS]));
        const uint32_t kb = tc::smem_addr(&sm.kfull[st]);
        tc::mbar_arrive_expect_tx(kb, 16384u);
        tc::tma_load_4d(tc::smem_addr(sm.k[st]), &tm_k, 0, static_cast<int>(b * a.Lk + j0), 0, hk, kb);
      }
      __syncwarp();
    }
    // wait (bounded, even after an abort) for the copies in flight
    if (lane == 0) {
      tc::mbar_wait(qb, 0);
      for (int tt = t - NKS < 0 ? 0 : t - NKS; tt < t; ++tt)
        tc::mbar_wait(tc::smem_addr(&sm.kfull[tt % NKS]), (tt / NKS) & 1);
    }
    __syncwarp();
  } else if (warp == L_W_VLOAD) {
    // ============================ V tiles =====================================
    if (lane == 0) tc::prefetch_tensormap(&tm_v);
    int t = 0;
    for (; t < NTL; ++t) {
      const int st = t % NVS;
      if (t >= NVS && !tc::wait_bounded_warp(tc::smem_addr(&sm.vfree[st]), ((t / NVS) - 1) & 1, abort_flag)) break;
      if (lane == 0) {
        const uint32_t vb = tc::smem_addr(&sm.vfull[st]);
        tc::mbar_arrive_expect_tx(vb, 16384u);
        tc::tma_load_4d(tc::smem_addr(sm.v[st]), &tm_v, 0, static_cast<int>(b * a.Lk + static_cast<int64_t>(t_lo + t) * LN),
                        0, hk, vb);
      }
      __syncwarp();
    }
    if (lane == 0)
      for (int tt = t - NVS < 0 ? 0 : t - NVS; tt < t; ++tt)
        tc::mbar_wait(tc::smem_addr(&sm.vfull[tt % NVS]), (tt / NVS) & 1);
    __syncwarp();
  } else if (warp >= L_W_MMA) {
    // ============================ MMA issue (one warp per query tile) =========
    const int g = warp - L_W_MMA;
    constexpr uint32_t id_s = tc::idesc_bf16_f32(128, LN, 0, 0);
    // kind::f16 with fp16 A and B: the bf16 format bits cleared
    constexpr uint32_t id_o = tc::idesc_bf16_f32(128, D, 0, 1) & (kF16 ? ~((1u << 7) | (1u << 10)) : ~0u);
    const uint64_t dq = tc::smem_desc_sw128(tc::smem_addr(sm.q[g][0]), 16, 1024);
    const uint64_t dk0 = tc::smem_desc_sw128(tc::smem_addr(sm.k[0]), 16, 1024);
    const uint64_t dv0 = tc::smem_desc_sw128(tc::smem_addr(sm.v[0]), 8192, 1024);
    const int t0 = g ? ga[1] : ga[0], t1 = g ? gb[1] : gb[0];
    // the K and V stages of a tile outside this group's band, released unused (in tile order)
    auto release = [&](int t) -> bool {
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.kfull[t % NKS]), (t / NKS) & 1, abort_flag)) return false;
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.vfull[t % NVS]), (t / NVS) & 1, abort_flag)) return false;
      if (lane == 0) {
        tc::mbar_arrive(tc::smem_addr(&sm.kfree[t % NKS]));
        tc::mbar_arrive(tc::smem_addr(&sm.vfree[t % NVS]));
      }
      __syncwarp();
      return true;
    };
    // S(t) into buffer 2g + ((t - t0) & 1)
    auto issue_s = [&](int t) -> bool {
      const int k = t - t0, sb = 2 * g + (k & 1), st = t % NKS;
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.kfull[st]), (t / NKS) & 1, abort_flag)) return false;
      tc::fence_after_sync();
      const uint64_t db = tc::desc_adv(dk0, st * 16384);
      const uint32_t dS = tbase + LN * sb;
      if (tc::elect_one()) {
        tc::mma_bf16<false>(dS, dq, db, id_s);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          tc::mma_bf16<true>(dS, tc::desc_adv(dq, (kk >> 2) * 16384 + (kk & 3) * 32),
                             tc::desc_adv(db, (kk >> 2) * 8192 + (kk & 3) * 32), id_s);
        tc::mma_commit(tc::smem_addr(&sm.sfull[sb]));
        tc::mma_commit(tc::smem_addr(&sm.kfree[st]));
      }
      __syncwarp();
      return true;
    };
    const int pre_end = t0 < NTL ? t0 : NTL;           // tiles [0, pre_end) lie before the band
    bool ok = tc::wait_bounded_warp(tc::smem_addr(&sm.qfull), 0, abort_flag);
    for (int t = 0; ok && t < pre_end; ++t) ok = release(t);
    if (ok && t0 <= t1) ok = issue_s(t0);
    if (ok && t0 + 1 <= t1) ok = issue_s(t0 + 1);
    for (int t = t0; ok && t <= t1; ++t) {
      const int k = t - t0, sb = 2 * g + (k & 1), sv = t % NVS;
      if (!(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pready[sb]), (k >> 1) & 1, abort_flag))) break;
      if (!(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.vfull[sv]), (t / NVS) & 1, abort_flag))) break;
      tc::fence_after_sync();
      const uint64_t dv = tc::desc_adv(dv0, sv * 16384);
      const uint32_t dO = tbase + kOCol + D * g, aP = tbase + LN * sb;
      if (tc::elect_one()) {
        // the group's first tile overwrites its O (TMEM is not zeroed); P from
        // TMEM, 16 keys (8 columns of 16-bit pairs) per k-step
        if (k == 0) tc::mma_f16_ts<false>(dO, aP, dv, id_o);
        else tc::mma_f16_ts<true>(dO, aP, dv, id_o);
#pragma unroll
        for (int kk = 1; kk < 4; ++kk) tc::mma_f16_ts<true>(dO, aP + 8 * kk, tc::desc_adv(dv, kk * 2048), id_o);
        if constexpr (!kF16) {
          // bf16 P's lo part, columns 32-63 of the buffer
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) tc::mma_f16_ts<true>(dO, aP + 32 + 8 * kk, tc::desc_adv(dv, kk * 2048), id_o);
        }
        tc::mma_commit(tc::smem_addr(&sm.pfree[sb]));
        tc::mma_commit(tc::smem_addr(&sm.vfree[sv]));
      }
      __syncwarp();
      if (t + 2 <= t1) {
        // P(t) lives in the S buffer that S(t + 2) overwrites: wait for this P.V
        if (!(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[sb]), (k >> 1) & 1, abort_flag))) break;
        ok = issue_s(t + 2);
      }
    }
    const int post_begin = (t1 + 1) > pre_end ? (t1 + 1) : pre_end;   // tiles after the band
    for (int t = post_begin; ok && t < NTL; ++t) ok = release(t);
    if (tc::elect_one()) {
      tc::mma_commit(tc::smem_addr(&sm.drain[g]));
      tc::mbar_wait(tc::smem_addr(&sm.drain[g]), 0);
    }
    __syncwarp();
  } else {
    // ============================ softmax + epilogue (warps 0-7) ==============
    const int grp = warp >> 2;                       // this group's query tile
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t o_col = kOCol + D * grp;          // this group's O accumulator
    const int r = (warp & 3) * 32 + lane;            // MMA row = TMEM lane
    const int qi = r / G, g = r - qi * G;
    const int64_t r0 = q0 + grp * LQ;                // the tile's first query
    const int64_t nr = (a.Lq - r0) < LQ ? ((a.Lq - r0) > 0 ? (a.Lq - r0) : 0) : LQ;
    const int64_t pos = a.qpos != nullptr ? (nr > 0 ? a.qpos[r0 + (qi < nr ? qi : nr - 1)] : 0) : a.q_offset + r0 + qi;
    const float sl2 = a.sm_scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f, o_scale = 1.f;
    int64_t band_lo, band_hi;
    row_band(a, pos, band_lo, band_hi);
    if (band_hi > a.Lk - 1) band_hi = a.Lk - 1;
    const uint32_t fill = a.exclude ? __float_as_uint(-INFINITY) : 0u;
    const int t0 = grp ? ga[1] : ga[0], t1 = grp ? gb[1] : gb[0];
    bool ok = true;
    uint32_t x[64];
    auto load_s = [&](int tt) -> bool {
      const int k = tt - t0, sb = 2 * grp + (k & 1);
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.sfull[sb]), (k >> 1) & 1, abort_flag)) return false;
      tc::fence_after_sync();
      const uint32_t sa = tbase + lane_off + LN * sb;
      tc::tmem_ld16(sa + 0, *reinterpret_cast<uint32_t(*)[16]>(&x[0]));
      tc::tmem_ld16(sa + 16, *reinterpret_cast<uint32_t(*)[16]>(&x[16]));
      tc::tmem_ld16(sa + 32, *reinterpret_cast<uint32_t(*)[16]>(&x[32]));
      tc::tmem_ld16(sa + 48, *reinterpret_cast<uint32_t(*)[16]>(&x[48]));
      return true;
    };
    if (t0 <= t1) ok = load_s(t0);
    for (int t = t0; ok && t <= t1; ++t) {
      const int k = t - t0, sb = 2 * grp + (k & 1);
      const int64_t j0 = static_cast<int64_t>(t_lo + t) * LN;
      tc::tmem_wait_ld();
      if (!(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.mfull[t % NMS]), (t / NMS) & 1, abort_flag))) break;
      const unsigned long long km = sm.kmask[t % NMS];
      // Zeroed keys (invalid, or landmark slots) keep logit 0: their raw score is
      // replaced by 0 (excluded keys: -inf).  The mask is per tile, so this branch
      // is warp-uniform; with landmark skipping on 64-aligned tiles only the last
      // column is masked.
      if (km != ~0ull) {
        if (km == (~0ull >> 1)) {
          x[LN - 1] = fill;
        } else {
#pragma unroll
          for (int c = 0; c < LN; ++c)
            if (!((km >> c) & 1ull)) x[c] = fill;
        }
      }
      // the row's band [band_lo, band_hi] (clipped to j < Lk): in-band columns
      // [dlo, dhi] of this tile; columns outside are -inf (only the first and
      // last tiles of a row have any)
      const int64_t dlo = band_lo - j0;
      const int64_t dhi = band_hi - j0;
      if (dlo > 0 || dhi < LN - 1) {
        const int lo32 = dlo < 0 ? 0 : (dlo > LN ? LN : static_cast<int>(dlo));
        const int hi32 = dhi < -1 ? -1 : (dhi > LN - 1 ? LN - 1 : static_cast<int>(dhi));
#pragma unroll
        for (int c = 0; c < LN; ++c)
          if (c < lo32 || c > hi32) x[c] = __float_as_uint(-INFINITY);
      }
      // tile max of the raw scores (sl2 > 0, so it is the max of the scaled
      // ones): four chains of three-input maxima
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < LN; c += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          m4[k] = fmax3(m4[k], __uint_as_float(x[c + 2 * k]), __uint_as_float(x[c + 2 * k + 1]));
      }
      const float tmax = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * sl2;
      // Lazy rescaling: the row keeps a reference max m_run and moves it (scaling
      // O and l) only when a tile max exceeds it by more than 2^8.  Until then
      // p = 2^(s - m_run) may exceed 1, which the fp32 accumulators and the hi/lo
      // split absorb; O / l and the LSE are the same in exact arithmetic.
      bool rescale = false;
      if (tmax > m_run + 8.f) {
        const float corr = m_run == -INFINITY ? 0.f : fast_exp2(m_run - tmax);
        rescale = m_run != -INFINITY;
        l_run *= corr;
        o_scale = corr;
        m_run = tmax;
      }
      const float nbase = m_run == -INFINITY ? 0.f : -m_run;
      // exponents and their sum on column pairs (paired fp32 fma and add)
      const float2 sl2x2 = make_float2(sl2, sl2), nbx2 = make_float2(nbase, nbase);
      float2 s2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      // fp16 P on a tile with no -inf column in this row (zeroed keys hold logit
      // 0): a quarter of the exponentials on the FMA pipe, the rest on the
      // special-function unit.  The choice is the row's own (lanes differ only on
      // the band's edge tiles), so a row's bits do not depend on which rows
      // share its warp.
      if (kF16 && (km == ~0ull || !a.exclude) && dlo <= 0 && dhi >= LN - 1) {
#pragma unroll
        for (int h = 0; h < LN / 2; ++h) {
          const float2 t2 = ffma2(make_float2(__uint_as_float(x[2 * h]), __uint_as_float(x[2 * h + 1])), sl2x2, nbx2);
          const float2 e = (h % 4 == 3) ? exp2_poly2(t2) : make_float2(fast_exp2(t2.x), fast_exp2(t2.y));
          s2[h & 1] = fadd2(s2[h & 1], e);
          x[2 * h] = __float_as_uint(e.x);
          x[2 * h + 1] = __float_as_uint(e.y);
        }
      } else {
#pragma unroll
        for (int h = 0; h < LN / 2; ++h) {
          const float2 t2 = ffma2(make_float2(__uint_as_float(x[2 * h]), __uint_as_float(x[2 * h + 1])), sl2x2, nbx2);
          const float2 e = make_float2(fast_exp2(t2.x), fast_exp2(t2.y));   // -inf -> 0
          s2[h & 1] = fadd2(s2[h & 1], e);
          x[2 * h] = __float_as_uint(e.x);
          x[2 * h + 1] = __float_as_uint(e.y);
        }
      }
      l_run += (s2[0].x + s2[1].x) + (s2[0].y + s2[1].y);
      // zeroed keys are counted in l but add no value
      if (km != ~0ull) {
        if (km == (~0ull >> 1)) {
          x[LN - 1] = 0u;
        } else {
#pragma unroll
          for (int c = 0; c < LN; ++c)
            if (!((km >> c) & 1ull)) x[c] = 0u;
        }
      }
      // P as fp16, or as bf16 hi + lo parts (~16 significant bits) with bf16 V
      uint32_t pk[32], pl[kF16 ? 1 : 32];
#pragma unroll
      for (int h = 0; h < 32; ++h) {
        const float p0 = __uint_as_float(x[2 * h]), p1 = __uint_as_float(x[2 * h + 1]);
        if constexpr (kF16) {
          pk[h] = pack_f16x2(p0, p1);
        } else {
          pk[h] = pack_bf16x2(p0, p1);
          pl[h] = pack_bf16x2(p0 - __uint_as_float(pk[h] << 16), p1 - __uint_as_float(pk[h] & 0xffff0000u));
        }
      }
      // P over the first 32 columns of its own S buffer (bf16: lo over the other
      // 32), the A operand of P.V straight from TMEM (the buffer's next S is
      // issued only after this P.V has completed)
      tc::tmem_st16(tbase + lane_off + LN * sb, &pk[0]);
      tc::tmem_st16(tbase + lane_off + LN * sb + 16, &pk[16]);
      if constexpr (!kF16) {
        tc::tmem_st16(tbase + lane_off + LN * sb + 32, &pl[0]);
        tc::tmem_st16(tbase + lane_off + LN * sb + 48, &pl[16]);
      }
      tc::tmem_wait_st();
      if (__any_sync(0xffffffffu, rescale)) {
        // O must hold every earlier tile of this group before it is scaled: the
        // P.V of the previous tile (a rescale needs an earlier tile, so k >= 1)
        if (!(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[2 * grp + ((k - 1) & 1)]), ((k - 1) >> 1) & 1,
                                         abort_flag)))
          break;
        tc::fence_after_sync();
        const float c = rescale ? o_scale : 1.f;
#pragma unroll
        for (int cc = 0; cc < D; cc += 16) {
          uint32_t o[16];
          tc::tmem_ld16(tbase + lane_off + o_col + cc, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * c);
          tc::tmem_st8(tbase + lane_off + o_col + cc, *reinterpret_cast<uint32_t(*)[8]>(&o[0]));
          tc::tmem_st8(tbase + lane_off + o_col + cc + 8, *reinterpret_cast<uint32_t(*)[8]>(&o[8]));
        }
        tc::tmem_wait_st();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(tc::smem_addr(&sm.pready[sb]));
      if (t + 1 <= t1 && !(ok = load_s(t + 1))) break;
    }
    tc::tmem_wait_ld();   // an S load still in flight after an abort
    // ---- epilogue: bf16 rows and the LSE (natural log) of this query tile.
    // A group without tiles never wrote its O: its rows get zeros and -inf.
    const bool has = t0 <= t1;
    if (ok && has) {
      const int kl = t1 - t0;                        // the group's last P.V
      ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[2 * grp + (kl & 1)]), (kl >> 1) & 1, abort_flag);
    }
    tc::fence_after_sync();
    if (nr > 0 && __all_sync(0xffffffffu, ok) && !__any_sync(0xffffffffu, *abort_flag != 0)) {
      const float l = l_run;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = r < nrows && qi < nr;
      const int64_t orow = ((b * a.Lq + r0 + qi) * a.Hq + hk * G + g);
#pragma unroll
      for (int cc = 0; cc < D; cc += 32) {
        uint32_t o[32];
        if (has) {
          tc::tmem_ld16(tbase + lane_off + o_col + cc, *reinterpret_cast<uint32_t(*)[16]>(&o[0]));
          tc::tmem_ld16(tbase + lane_off + o_col + cc + 16, *reinterpret_cast<uint32_t(*)[16]>(&o[16]));
          tc::tmem_wait_ld();
        }
        if (row_ok) {
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = has ? __uint_as_float(o[i]) * inv : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(a.out + orow * D + cc);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pack_bf16x2(f[8 * i], f[8 * i + 1]), pack_bf16x2(f[8 * i + 2], f[8 * i + 3]),
                                pack_bf16x2(f[8 * i + 4], f[8 * i + 5]), pack_bf16x2(f[8 * i + 6], f[8 * i + 7]));
        }
      }
      if (row_ok && a.lse != nullptr) a.lse[orow] = l > 0.f ? (m_run + log2f(l)) * kLn2 : -INFINITY;
    }

  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && sm.abort_flag) atomicOr(&g_local_error, 1);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

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

struct Band {
  int causal = 0, expand = 0, exclude = 0;
  int64_t shift = 0;
  const int64_t* qpos = nullptr;
};

template <bool kF16>
int local_launch(const void* q, const void* k, const void* v, const uint8_t* key_valid, void* out, float* lse,
                 int64_t window, int skip_inert, int64_t chunk, float sm_scale, int64_t batch, int64_t q_len,
                 int64_t kv_len, int64_t q_offset, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                 mrsa_stream_t stream, Band band = Band()) {
  if (!q || !k || !v || !out) return MRSA_ERR_NULL;
  if (head_dim != D || kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads || q_heads / kv_heads > 8 ||
      batch < 1 || q_len < 0 || kv_len < 1 || q_offset < 0 || q_heads > 65535 || batch > 65535 ||
      batch * q_len * q_heads > 0x7fffffffLL || batch * kv_len > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if (window < 0 || ((skip_inert || band.expand) && chunk <= 0) || band.shift < 0 ||
      !(sm_scale > 0.f) || window > (int64_t(1) << 40) || band.shift > (int64_t(1) << 40))
    return MRSA_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  // Q [B*Lq][Hq][128] as (dim-in-half, head row, half, query): one box = one half of
  // the G head rows of LQ = 128 / G queries, rows (query, head) back to back
  // K, V [B*Lk][Hkv][128] as (dim-in-half, key, half, kv head): one box = 64 keys
  const int64_t G = q_heads / kv_heads, LQ = 128 / G;
  CUtensorMap tm_q, tm_k, tm_v;
  const cuuint64_t q_dims[4] = {64, static_cast<cuuint64_t>(q_heads), 2, static_cast<cuuint64_t>(batch * q_len)};
  const cuuint64_t q_str[3] = {256, 128, static_cast<cuuint64_t>(q_heads * D * 2)};
  const cuuint32_t q_box[4] = {64, static_cast<cuuint32_t>(G), 1, static_cast<cuuint32_t>(LQ)};
  const cuuint64_t kv_dims[4] = {64, static_cast<cuuint64_t>(batch * kv_len), 2, static_cast<cuuint64_t>(kv_heads)};
  const cuuint64_t kv_str[3] = {static_cast<cuuint64_t>(kv_heads * D * 2), 128, 256};
  const cuuint32_t kv_box[4] = {64, LN, 2, 1};
  if (!make_map(&tm_q, q, 4, q_dims, q_str, q_box) || !make_map(&tm_k, k, 4, kv_dims, kv_str, kv_box) ||
      !make_map(&tm_v, v, 4, kv_dims, kv_str, kv_box,
                kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))
    return MRSA_ERR_LAUNCH;
  LocalArgs a;
  a.key_valid = key_valid;
  a.qpos = band.qpos;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  a.window = window;
  a.Lq = q_len;
  a.Lk = kv_len;
  a.q_offset = q_offset;
  a.skip_inert = skip_inert;
  a.chunk = static_cast<int>(chunk > 0 ? chunk : 1);
  a.shift = band.shift;
  a.causal = band.causal;
  a.expand = band.expand;
  a.exclude = band.exclude;
  a.Hq = static_cast<int>(q_heads);
  a.Hkv = static_cast<int>(kv_heads);
  a.G = static_cast<int>(G);
  a.sm_scale = sm_scale;
  const size_t smem = sizeof(LocalSmem) + 1024;
  if (cudaFuncSetAttribute(local_tc_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const int64_t blocks = (q_len + 2 * LQ - 1) / (2 * LQ);   // two query tiles per CTA
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
  local_tc_kernel<kF16><<<grid, L_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(tm_q, tm_k, tm_v, a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

}  // namespace

extern "C" int mrsa_local_attention(const void* q, const void* k, const void* v,
                                    const uint8_t* key_valid, void* out, float* lse,
                                    int64_t window, int skip_inert, int64_t chunk, float sm_scale,
                                    int64_t batch, int64_t q_len, int64_t kv_len, int64_t q_offset,
                                    int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                    mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  return local_launch<false>(q, k, v, key_valid, out, lse, window, skip_inert, chunk, sm_scale, batch, q_len,
                             kv_len, q_offset, q_heads, kv_heads, head_dim, stream);
}

extern "C" int mrsa_local_attention_f16v(const void* q, const void* k, const void* v_f16,
                                         const uint8_t* key_valid, void* out, float* lse,
                                         int64_t window, int skip_inert, int64_t chunk, float sm_scale,
                                         int64_t batch, int64_t q_len, int64_t kv_len, int64_t q_offset,
                                         int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                         mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  return local_launch<true>(q, k, v_f16, key_valid, out, lse, window, skip_inert, chunk, sm_scale, batch, q_len,
                            kv_len, q_offset, q_heads, kv_heads, head_dim, stream);
}

extern "C" int mrsa_local_attention_positions(const void* q, const void* k, const void* v,
                                              const uint8_t* key_valid, const int64_t* query_positions,
                                              void* out, float* lse, int64_t window, int skip_inert,
                                              int64_t chunk, float sm_scale, int64_t batch, int64_t q_len,
                                              int64_t kv_len, int64_t q_heads, int64_t kv_heads,
                                              int64_t head_dim, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  if (query_positions == nullptr && q_len > 0) return MRSA_ERR_NULL;
  Band band;
  band.qpos = query_positions;
  return local_launch<false>(q, k, v, key_valid, out, lse, window, skip_inert, chunk, sm_scale, batch, q_len,
                             kv_len, 0, q_heads, kv_heads, head_dim, stream, band);
}

extern "C" int mrsa_flex_attention(const void* q, const void* k, const void* v, void* out, float* lse,
                                   int64_t window, int64_t chunk, int mask_lmk, int expand_to_chunk,
                                   int64_t kv_start, float sm_scale, int64_t batch, int64_t q_len,
                                   int64_t kv_len, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                   mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  if (q_len > kv_len) return MRSA_ERR_SHAPE;
  if (chunk <= 0 || chunk > 0x7fffffffLL) return MRSA_ERR_ARG;
  Band band;
  band.causal = 1;
  band.expand = expand_to_chunk != 0;
  band.exclude = 1;
  band.shift = kv_start;
  return local_launch<false>(q, k, v, nullptr, out, lse, window, mask_lmk != 0, chunk, sm_scale, batch, q_len,
                             kv_len, kv_len - q_len, q_heads, kv_heads, head_dim, stream, band);
}

namespace mrsa {
int local_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_local_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_local_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
}  // namespace mrsa
