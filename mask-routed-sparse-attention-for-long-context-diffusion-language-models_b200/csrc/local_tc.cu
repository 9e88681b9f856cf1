// Bidirectional banded GQA attention with natural-log LSE on the tcgen05
// tensor cores (local branch of the route layer, window W+63 with
// landmark/invalid K,V zeroed; SWA layers, window 1280).  Semantics of
// dream_dllm_hils/local_attention.py:35-107: zeroed keys keep logit 0 in the
// softmax and add no value; keys with |i-j| > window are out.
//
// One CTA owns LQ = floor(128 / G) queries of one KV head (18 for GQA 7:1).
// Its MMA tile has 128 rows, row G*qi + g = (query qi, head g of the group;
// rows >= LQ*G are zero padding), so each 64-key K/V tile is read once for all
// heads of the group.  Per key tile t:
//   S[128 x 64]  = Q . K_t^T               (UMMA M=128, N=64,  K=128, TMEM)
//   P            = exp2(S*scale*log2e - m)  (one thread per row, online max)
//   O[128 x 128] += P . V_t                (UMMA M=128, N=128, K=64, TMEM)
// P goes through shared memory: fp16 when V is fp16, else bf16 hi + lo parts
// (two MMAs per k-step, ~16 significant bits).  Each row keeps a reference
// max that moves (rescaling O in TMEM) only when a tile max exceeds it by more
// than 2^8.
// Warps 0-7: softmax and epilogue in two groups of four (warp w = TMEM lanes
// 32(w%4)..+31 = rows); group g takes every other key tile (by the tile's
// parity counted from query row 0's tile) and keeps
// its own running max, sum and O accumulator, merged in the epilogue.  Each
// group has two S buffers in TMEM, so the S of its next tile is computed while
// it works on the current one and the softmax never waits for an MMA round
// trip; with fp16 P it also has two P buffers.  Warp 8: TMA of Q and of the K
// tiles (4 stages) and the per-tile key validity masks; warp 11: TMA of the V
// tiles (4 stages, released by P.V); warps 9 and 10: MMA issue for the even
// and the odd tiles (converged, elect.sync), in the order S(t), S(t+2), then
// per tile P.V(t), S(t+4).  Every mbarrier wait is bounded and unwinds through
// a shared abort flag.
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
constexpr int NKS = 4;            // K stages (even: a stage's tiles share one parity, hence one MMA warp)
constexpr int NVS = 4;            // V stages (even, likewise)
constexpr int NMS = 8;            // key-mask slots
constexpr int D = kHeadDim;
constexpr int L_THREADS = 384;    // warps 0-7 softmax (two groups), 8 Q/K TMA + masks, 9-10 MMA, 11 V TMA
constexpr int L_W_KLOAD = 8, L_W_MMA = 9, L_W_VLOAD = 11;
constexpr uint32_t kOCol = 256;   // O of groups 0 / 1 at [256, 384) / [384, 512); S buffer i at [64 i, 64 i + 64)

struct __align__(1024) LocalSmem {
  unsigned char q[2][16384];          // [half][128 rows = (query, head)][64 dims], 128-byte swizzled
  unsigned char k[NKS][16384];        // [half][64 keys][64 dims]
  unsigned char v[NVS][16384];        // same, read as the MN-major B operand of P.V
  unsigned char p[4][16384];          // fp16 P: group g's buffers 2g, 2g+1; bf16 P: group g's hi 2g, lo 2g+1
  unsigned long long kmask[NMS];      // bit j: key j of the tile is usable (not zeroed); slot t % NMS
  uint64_t qfull, kfull[NKS], kfree[NKS], vfull[NVS], vfree[NVS], mfull[NMS];
  uint64_t sfull[4], sfree[4], pready[4], pfree[4], drain[2];
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

__device__ __forceinline__ int swz_off(int row, int piece) { return row * 128 + ((piece ^ (row & 7)) << 4); }

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
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * LQ;
  const int64_t rows_q = (a.Lq - q0) < LQ ? (a.Lq - q0) : LQ;
  // positions of the CTA's first and last rows (the band is monotone in the
  // position); with explicit row positions, their minimum and maximum
  int64_t p_min = a.q_offset + q0, p_max = a.q_offset + q0 + rows_q - 1;
  if (a.qpos != nullptr) {
    p_min = a.qpos[q0];
    p_max = p_min;
    for (int i = 1; i < rows_q; ++i) {
      const int64_t p = a.qpos[q0 + i];
      p_min = p < p_min ? p : p_min;
      p_max = p > p_max ? p : p_max;
    }
  }
  int64_t j_lo, j_hi, unused;
  row_band(a, p_min, j_lo, unused);
  row_band(a, p_max, unused, j_hi);
  if (j_lo < 0) j_lo = 0;
  if (j_hi > a.Lk - 1) j_hi = a.Lk - 1;
  const int t_lo = static_cast<int>(j_lo / LN);
  const int NTL = j_hi >= j_lo ? static_cast<int>(j_hi / LN) - t_lo + 1 : 0;
  // Tile t (key tile t_lo + t) belongs to softmax group (t + e) % 2, the parity
  // of its key tile counted from the tile of query row 0: a row's tiles then go
  // to the same groups, in the same order, whichever rows share its CTA, so a
  // row's result does not depend on how the rows are cut into CTAs (a query
  // shard with a tile-aligned halo gets the bits of the whole sequence).
  const int e = static_cast<int>((static_cast<int64_t>(t_lo) - floor_div(a.q_offset, LN)) & 1);
  auto grp_of = [e](int t) { return (t + e) & 1; };
  // P buffer of tile t and how many times that buffer was used before: fp16 P
  // alternates two buffers per group, bf16 hi + lo P has one pair per group
  auto p_idx = [grp_of](int t) { return kF16 ? 2 * grp_of(t) + ((t >> 1) & 1) : 2 * grp_of(t); };
  auto p_use = [](int t) { return kF16 ? (t >> 2) : (t >> 1); };
  // S buffer of tile t: each group alternates its two buffers
  auto s_idx = [grp_of](int t) { return 2 * grp_of(t) + ((t >> 1) & 1); };

  if (tid == 0) {
    tc::mbar_init(tc::smem_addr(&sm.qfull), 1);
    for (int s = 0; s < NKS; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.kfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.kfree[s]), 1);
    }
    for (int s = 0; s < NVS; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.vfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.vfree[s]), 1);
    }
    for (int s = 0; s < NMS; ++s) tc::mbar_init(tc::smem_addr(&sm.mfull[s]), 1);
    for (int s = 0; s < 4; ++s) {
      tc::mbar_init(tc::smem_addr(&sm.sfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&sm.sfree[s]), 4);
      tc::mbar_init(tc::smem_addr(&sm.pready[s]), 4);
      tc::mbar_init(tc::smem_addr(&sm.pfree[s]), 1);
    }
    for (int s = 0; s < 2; ++s) tc::mbar_init(tc::smem_addr(&sm.drain[s]), 1);
    sm.abort_flag = 0;
    tc::fence_mbar_init();
  }
  // zero the padding rows of the Q tile (the TMA box fills rows [0, nrows)),
  // visible to the tensor core's async proxy
  for (int i = tid; i < 2 * (128 - nrows) * 8; i += L_THREADS) {
    const int h = i / ((128 - nrows) * 8), rem = i % ((128 - nrows) * 8);
    *reinterpret_cast<uint4*>(sm.q[h] + (nrows + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0u, 0u, 0u, 0u);
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
      tc::mbar_arrive_expect_tx(qb, static_cast<uint32_t>(nrows) * 256u);
      tc::tma_load_4d(tc::smem_addr(sm.q[0]), &tm_q, 0, hk * G, 0, static_cast<int>(b * a.Lq + q0), qb);
      tc::tma_load_4d(tc::smem_addr(sm.q[1]), &tm_q, 0, hk * G, 1, static_cast<int>(b * a.Lq + q0), qb);
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
      // stage st was last read by S(t - NKS); mask slot t % NMS by the softmax of
      // tile t - NMS, which precedes the P.V(t - NMS) that S(t - NKS) is issued after
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
    // ============================ MMA issue (two converged warps) =============
    // Warp 9 issues the MMAs of the even tiles, warp 10 those of the odd tiles
    // (one issuing thread needs about twice the tensor pipe's time per MMA):
    // S(t) and S(t+2) first, then per tile P.V(t) into its group's O and S(t+4)
    // into the S buffer that tile t's softmax has released.
    const int par = warp - L_W_MMA;
    constexpr uint32_t id_s = tc::idesc_bf16_f32(128, LN, 0, 0);
    // kind::f16 with fp16 A and B: the bf16 format bits cleared
    constexpr uint32_t id_o = tc::idesc_bf16_f32(128, D, 0, 1) & (kF16 ? ~((1u << 7) | (1u << 10)) : ~0u);
    const uint64_t dq = tc::smem_desc_sw128(tc::smem_addr(sm.q[0]), 16, 1024);
    const uint64_t dk0 = tc::smem_desc_sw128(tc::smem_addr(sm.k[0]), 16, 1024);
    const uint64_t dv0 = tc::smem_desc_sw128(tc::smem_addr(sm.v[0]), 8192, 1024);
    const uint64_t dp0 = tc::smem_desc_sw128(tc::smem_addr(sm.p[0]), 16, 1024);
    auto issue_s = [&](int t) -> bool {
      const int st = t % NKS, sb = s_idx(t), use = t >> 2;
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.kfull[st]), (t / NKS) & 1, abort_flag)) return false;
      if (use >= 1 && !tc::wait_bounded_warp(tc::smem_addr(&sm.sfree[sb]), (use - 1) & 1, abort_flag)) return false;
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
    bool ok = tc::wait_bounded_warp(tc::smem_addr(&sm.qfull), 0, abort_flag);
    const int t0 = par ^ e;                           // this group's first tile
    if (ok && t0 < NTL) ok = issue_s(t0);
    if (ok && t0 + 2 < NTL) ok = issue_s(t0 + 2);
    for (int t = t0; ok && t < NTL; t += 2) {
      const int sv = t % NVS, pb = p_idx(t);
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.pready[pb]), p_use(t) & 1, abort_flag)) break;
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.vfull[sv]), (t / NVS) & 1, abort_flag)) break;
      tc::fence_after_sync();
      const uint64_t dv = tc::desc_adv(dv0, sv * 16384), dh = tc::desc_adv(dp0, pb * 16384),
                     dl = tc::desc_adv(dp0, (pb + 1) * 16384);
      const uint32_t dO = tbase + kOCol + D * par;      // group par's accumulator
      if (tc::elect_one()) {
        // each group's first tile overwrites its O (TMEM is not zeroed)
        if constexpr (kF16) {
          // P from TMEM: 16 keys (8 columns of fp16 pairs) per k-step
          const uint32_t aP = tbase + LN * s_idx(t);
          if (t < 2) tc::mma_f16_ts<false>(dO, aP, dv, id_o);
          else tc::mma_f16_ts<true>(dO, aP, dv, id_o);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk) tc::mma_f16_ts<true>(dO, aP + 8 * kk, tc::desc_adv(dv, kk * 2048), id_o);
        } else {
          if (t < 2) tc::mma_bf16<false>(dO, dh, dv, id_o);
          else tc::mma_bf16<true>(dO, dh, dv, id_o);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk) tc::mma_bf16<true>(dO, tc::desc_adv(dh, kk * 32), tc::desc_adv(dv, kk * 2048), id_o);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_bf16<true>(dO, tc::desc_adv(dl, kk * 32), tc::desc_adv(dv, kk * 2048), id_o);
        }
        tc::mma_commit(tc::smem_addr(&sm.pfree[pb]));
        tc::mma_commit(tc::smem_addr(&sm.vfree[sv]));
      }
      __syncwarp();
      // fp16 P lives in the S buffer that S(t + 4) overwrites: wait for its P.V
      if (kF16 && t + 4 < NTL && !tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[pb]), p_use(t) & 1, abort_flag)) break;
      if (t + 4 < NTL) ok = issue_s(t + 4);
    }
    if (tc::elect_one()) {
      tc::mma_commit(tc::smem_addr(&sm.drain[par]));
      tc::mbar_wait(tc::smem_addr(&sm.drain[par]), 0);
    }
    __syncwarp();
  } else {
    // ============================ softmax + epilogue (warps 0-7) ==============
    const int grp = warp >> 2;                       // tiles t with (t + e) % 2 == grp
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t o_col = kOCol + D * grp;          // this group's O accumulator
    const int r = (warp & 3) * 32 + lane;            // MMA row = TMEM lane
    const int qi = r / G, g = r - qi * G;
    const int64_t pos = a.qpos != nullptr ? a.qpos[q0 + (qi < rows_q ? qi : rows_q - 1)] : a.q_offset + q0 + qi;
    const float sl2 = a.sm_scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f, o_scale = 1.f;
    int64_t band_lo, band_hi;
    row_band(a, pos, band_lo, band_hi);
    if (band_hi > a.Lk - 1) band_hi = a.Lk - 1;
    const uint32_t fill = a.exclude ? __float_as_uint(-INFINITY) : 0u;
    bool ok = true;
    uint32_t x[64];
    auto load_s = [&](int tt) -> bool {
      if (!tc::wait_bounded_warp(tc::smem_addr(&sm.sfull[s_idx(tt)]), (tt >> 2) & 1, abort_flag)) return false;
      tc::fence_after_sync();
      const uint32_t sa = tbase + lane_off + LN * s_idx(tt);
      tc::tmem_ld16(sa + 0, *reinterpret_cast<uint32_t(*)[16]>(&x[0]));
      tc::tmem_ld16(sa + 16, *reinterpret_cast<uint32_t(*)[16]>(&x[16]));
      tc::tmem_ld16(sa + 32, *reinterpret_cast<uint32_t(*)[16]>(&x[32]));
      tc::tmem_ld16(sa + 48, *reinterpret_cast<uint32_t(*)[16]>(&x[48]));
      return true;
    };
    if ((grp ^ e) < NTL) ok = load_s(grp ^ e);
    for (int t = grp ^ e; ok && t < NTL; t += 2) {
      const int sb = s_idx(t), pb = p_idx(t), pu = p_use(t);
      const int64_t j0 = static_cast<int64_t>(t_lo + t) * LN;
      tc::tmem_wait_ld();
      // the S buffer is free for S(t + 4) as soon as it is in registers
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(tc::smem_addr(&sm.sfree[sb]));
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
      // 0): a third of the exponentials on the FMA pipe, the rest on the
      // special-function unit.  The choice is the row's own (lanes differ only on
      // the band's edge tiles), so a row's bits do not depend on which rows
      // share its warp.
      if (kF16 && (km == ~0ull || !a.exclude) && dlo <= 0 && dhi >= LN - 1) {
#pragma unroll
        for (int h = 0; h < LN / 2; ++h) {
          const float2 t2 = ffma2(make_float2(__uint_as_float(x[2 * h]), __uint_as_float(x[2 * h + 1])), sl2x2, nbx2);
          const float2 e = (h % 3 == 2) ? exp2_poly2(t2) : make_float2(fast_exp2(t2.x), fast_exp2(t2.y));
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
      uint32_t hi[32], lo[32];
#pragma unroll
      for (int h = 0; h < 32; ++h) {
        const float p0 = __uint_as_float(x[2 * h]), p1 = __uint_as_float(x[2 * h + 1]);
        if constexpr (kF16) {
          hi[h] = pack_f16x2(p0, p1);
        } else {
          hi[h] = pack_bf16x2(p0, p1);
          lo[h] = pack_bf16x2(p0 - __uint_as_float(hi[h] << 16), p1 - __uint_as_float(hi[h] & 0xffff0000u));
        }
      }
      if constexpr (kF16) {
        // fp16 P over the first 32 columns of its own S buffer, the A operand of
        // P.V straight from TMEM (the buffer's next S is issued only after this
        // P.V has completed)
        tc::tmem_st16(tbase + lane_off + LN * sb, &hi[0]);
        tc::tmem_st16(tbase + lane_off + LN * sb + 16, &hi[16]);
        tc::tmem_wait_st();
      } else {
        // the P buffer's previous tile must have been read by its P.V
        if (pu >= 1 && !(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[pb]), (pu - 1) & 1, abort_flag))) break;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          *reinterpret_cast<uint4*>(sm.p[pb] + swz_off(r, p)) = make_uint4(hi[4 * p], hi[4 * p + 1], hi[4 * p + 2], hi[4 * p + 3]);
          *reinterpret_cast<uint4*>(sm.p[pb + 1] + swz_off(r, p)) = make_uint4(lo[4 * p], lo[4 * p + 1], lo[4 * p + 2], lo[4 * p + 3]);
        }
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // O must hold every earlier tile of this group before it is scaled: the
        // P.V of tile t-2 (a rescale needs an earlier tile, so t >= 2 here); with
        // one P buffer per group that was the wait above
        if (kF16 && !(ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[p_idx(t - 2)]), p_use(t - 2) & 1, abort_flag)))
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
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(tc::smem_addr(&sm.pready[pb]));
      // the group's next S: requested here, after this tile's P is handed over
      // (waiting for it before the P store held the P.V back)
      if (t + 2 < NTL && !(ok = load_s(t + 2))) break;
    }
    tc::tmem_wait_ld();   // an S load still in flight after an abort
    // ---- epilogue: merge the two groups' partial softmaxes, bf16 rows, LSE
    // (natural log).  A group without tiles never wrote its O, which is then
    // left out.  The per-row partials go to the K stages, idle once every S is
    // done: both groups have read all their S tiles when they pass the first
    // barrier (before it, the other group's last S may still read them).
    const bool has0 = (0 ^ e) < NTL, has1 = (1 ^ e) < NTL;
    float* part_m = reinterpret_cast<float*>(sm.k[0]);          // [group][row]
    float* part_l = part_m + 2 * 128;
    asm volatile("bar.sync 1, 256;\n" ::: "memory");
    part_m[grp * 128 + r] = m_run;
    part_l[grp * 128 + r] = l_run;
    asm volatile("bar.sync 1, 256;\n" ::: "memory");
    // each group's last P.V (group g's tiles are t = g ^ e mod 2)
    if (ok && has0) {
      const int tl = (NTL - 1) - (((NTL - 1) ^ e) & 1);
      ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[p_idx(tl)]), p_use(tl) & 1, abort_flag);
    }
    if (ok && has1) {
      const int tl = (NTL - 1) - (((NTL - 1) ^ e ^ 1) & 1);
      ok = tc::wait_bounded_warp(tc::smem_addr(&sm.pfree[p_idx(tl)]), p_use(tl) & 1, abort_flag);
    }
    tc::fence_after_sync();
    if (__all_sync(0xffffffffu, ok) && !__any_sync(0xffffffffu, *abort_flag != 0)) {
      const float m0 = part_m[r], m1 = part_m[128 + r];
      const float m = fmaxf(m0, m1);
      const float f0 = m0 == -INFINITY ? 0.f : fast_exp2(m0 - m);
      const float f1 = m1 == -INFINITY ? 0.f : fast_exp2(m1 - m);
      const float l = part_l[r] * f0 + part_l[128 + r] * f1;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const float c0 = f0 * inv, c1 = f1 * inv;
      const bool row_ok = r < nrows && qi < rows_q;
      const int64_t orow = ((b * a.Lq + q0 + qi) * a.Hq + hk * G + g);
      // group 0 writes dims 0-63, group 1 dims 64-127
#pragma unroll
      for (int cc = grp * (D / 2); cc < (grp + 1) * (D / 2); cc += 32) {
        uint32_t o0[32], o1[32];
        if (has0) {
          tc::tmem_ld16(tbase + lane_off + kOCol + cc, *reinterpret_cast<uint32_t(*)[16]>(&o0[0]));
          tc::tmem_ld16(tbase + lane_off + kOCol + cc + 16, *reinterpret_cast<uint32_t(*)[16]>(&o0[16]));
        }
        if (has1) {
          tc::tmem_ld16(tbase + lane_off + kOCol + D + cc, *reinterpret_cast<uint32_t(*)[16]>(&o1[0]));
          tc::tmem_ld16(tbase + lane_off + kOCol + D + cc + 16, *reinterpret_cast<uint32_t(*)[16]>(&o1[16]));
        }
        tc::tmem_wait_ld();
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          o[i] = (has0 ? __uint_as_float(o0[i]) * c0 : 0.f) + (has1 ? __uint_as_float(o1[i]) * c1 : 0.f);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(a.out + orow * D + cc);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pack_bf16x2(o[8 * i], o[8 * i + 1]), pack_bf16x2(o[8 * i + 2], o[8 * i + 3]),
                                pack_bf16x2(o[8 * i + 4], o[8 * i + 5]), pack_bf16x2(o[8 * i + 6], o[8 * i + 7]));
        }
      }
      if (grp == 0 && row_ok && a.lse != nullptr)
        a.lse[orow] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
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
  const int64_t blocks = (q_len + LQ - 1) / LQ;
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
