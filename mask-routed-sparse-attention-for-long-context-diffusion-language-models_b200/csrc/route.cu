// Query -> chunk routing: post-softmax max-pooled top-K selection with the
// route weights fused in.  Semantics of ref_softmax_topk_max_pooling
// (ops/topk_head_softmax.py:15-156, post_softmax, non-causal, no Gumbel):
//   x[g,c]  = q_g . lmk[c,g] / sqrt(D) + bias[c,g]
//   T[g]    = logaddexp(local_lse[g], logsumexp_c x[g,c])   (all chunks)
//   key[c]  = max_g (x[g,c] - T[g]);  dropped chunks -> -inf
//   indices = the K largest finite keys, ascending, -1 padded
//   scores  = raw q_g . lmk[c,g] / sqrt(D) at the selected chunks
// and of _route_weights_torch (dream_dllm_hils/attention.py:126-227) /
// route_weights (ops/hils_bidir_route_weights_tilelang.py:15-95).
// The drop rule of remote_drop_mask (dream_dllm_hils/kernel_utils.py:75-161) is
// evaluated inline from chunk validity instead of a dense [L, C] mask.
//
// Two launches.
// route_keys_kernel (tcgen05/TMEM): one CTA per 64 queries x one KV head keeps
//   the G query tiles of its block in shared memory and streams 128-chunk
//   landmark tiles by TMA.  S_g = Q_g . LMK_g^T runs as UMMA M=64, N=128, K=128
//   into one of four 128-column TMEM buffers.  Pass 1 walks heads then tiles and
//   folds each S tile into an online log-sum-exp per (query, head), giving T;
//   pass 2 walks tiles then heads and keeps max_g (x - T_g) in registers, applies
//   the drop rule and writes the fp32 keys [B, Lq, Hkv, C] to the workspace.
//   Warps 0-15 read TMEM (four threads per S row, 16 columns each, via
//   tcgen05.ld.16x32bx2), warp 16 issues the TMA copies and fills the bias
//   ring, warp 17 the MMAs.  Every role runs at a few cycles per instruction,
//   so each keeps its per-tile instruction count small: the job order is a
//   table built once, the bias of a tile is fetched two tiles ahead from a
//   per-lane base pointer, and the readers split each row four ways.
// route_select_kernel: one warp per (query, KV head) holds that row's keys in
//   registers, finds the K-th largest with a radix search over order-preserving
//   integer keys (above 256 chunks, over the few keys a per-lane-maximum
//   filter keeps), emits the indices in ascending chunk order (ties at the
//   threshold: lowest chunk ids first), then gathers the raw scores of its
//   selection (lane = slot) and computes the route weights.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

constexpr int D = kHeadDim;
constexpr int kMaxChunks = 2048;
constexpr int RQ = 64;            // queries per key CTA (UMMA M)
constexpr int RN = 128;           // chunks per landmark tile (UMMA N)
constexpr int RBUF = 4;           // TMEM S buffers of RN columns
constexpr int RMAXST = 4;         // landmark stages (chosen at launch from the shared-memory budget)
constexpr int RGMAX = 8;
constexpr int R_THREADS = 576;    // warps 0-15 TMEM readers, 16 TMA, 17 MMA
constexpr int R_W_LOAD = 16, R_W_MMA = 17;
constexpr int RC = 16;            // tile columns per reader thread
constexpr int RMAXJ = 2 * RGMAX * (kMaxChunks / RN);   // jobs of one CTA at most
constexpr int kSmemLimit = 232448;

struct RouteArgs {
  const __nv_bfloat16* rq;
  const __nv_bfloat16* lmk;
  int lmk_per_qhead;
  const float* local_lse;
  const float* bias;
  const int32_t* drop;
  const uint8_t* chunk_ok;
  int64_t window, q_offset;
  float* keys;              // workspace: keys [B, Lq, Hkv, C] fp32
  void* raw;                // workspace: raw scaled scores [B, Lq, Hq, C] (scores dtype)
  int32_t* indices;
  void* scores;
  int scores_f32;
  __nv_bfloat16* remote_w;
  __nv_bfloat16* local_w;
  int weight_mode;
  float temperature, gate_scale, gate_offset;
  int64_t Lq;
  int C, Hkv, G, K;
  int nst;                  // landmark stages
  float sm_scale;
};

// Set (bit 0) when a key CTA gave up on a wait; read and cleared through
// mrsa_device_error_flags().
__device__ int g_route_error;

// Misc shared state of the key kernel, after the query tiles and landmark stages.
constexpr int RBR = 4;            // bias ring slots (one job's 128 bias values each)

struct RouteMisc {
  uint64_t lfull[RMAXST], lfree[RMAXST], sdone[RBUF], sfree[RBUF], qfull, mma_drain;
  uint64_t bfull[RBR], bfree[RBR];
  float bias[RBR][RN];             // bias of job j's head and tile in slot j % RBR
  uint32_t tmem_base;
  int abort_flag;
  float T[RQ][RGMAX];              // T per (query, head), natural log
  float part[2][4][RQ][2];         // pass-1 partials (max, sum) per column quarter, log2 domain; two heads
  uint16_t job[RMAXJ];             // job j -> (tile << 8) | head
  uint8_t chunk_ok[kMaxChunks];
};

__host__ __device__ constexpr size_t key_smem_bytes(int G, int nst) {
  return static_cast<size_t>(G) * 16384 + static_cast<size_t>(nst) * 32768 + sizeof(RouteMisc) + 1024;
}

// Job j of the key kernel: pass 1 visits (head, tile) head-major, pass 2 tile-major.
__device__ __forceinline__ void job_coords(int j, int G, int NT, int& g, int& t) {
  if (j < G * NT) {
    g = j / NT;
    t = j % NT;
  } else {
    const int jj = j - G * NT;
    t = jj / G;
    g = jj % G;
  }
}

__global__ void __launch_bounds__(R_THREADS, 1) route_keys_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_l, RouteArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = a.G, C = a.C, NST = a.nst, Hq = a.Hkv * a.G;
  unsigned char* qt = base;                                  // G x [half][64 rows][64 dims]
  unsigned char* lt = base + G * 16384;                      // NST x [half][128 chunks][64 dims]
  RouteMisc& ms = *reinterpret_cast<RouteMisc*>(lt + NST * 32768);
  volatile int* abort_flag = &ms.abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * RQ;
  const int NT = (C + RN - 1) / RN;
  const int J = 2 * G * NT;

  for (int c = tid; c < C; c += R_THREADS) ms.chunk_ok[c] = a.chunk_ok ? a.chunk_ok[(int64_t)b * C + c] : 1;
  for (int jj = tid; jj < J; jj += R_THREADS) {
    int g, t;
    job_coords(jj, G, NT, g, t);
    ms.job[jj] = static_cast<uint16_t>((t << 8) | g);
  }
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(tc::smem_addr(&ms.lfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&ms.lfree[s]), 1);
    }
    for (int s = 0; s < RBUF; ++s) {
      tc::mbar_init(tc::smem_addr(&ms.sdone[s]), 1);
      tc::mbar_init(tc::smem_addr(&ms.sfree[s]), 16);
    }
    for (int s = 0; s < RBR; ++s) {
      tc::mbar_init(tc::smem_addr(&ms.bfull[s]), 1);
      tc::mbar_init(tc::smem_addr(&ms.bfree[s]), 16);
    }
    tc::mbar_init(tc::smem_addr(&ms.qfull), 1);
    tc::mbar_init(tc::smem_addr(&ms.mma_drain), 1);
    ms.abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tc::smem_addr(&ms.tmem_base), 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = ms.tmem_base;

  if (warp == R_W_LOAD) {
    // ============================ TMA + bias ring =============================
    const uint32_t qb = tc::smem_addr(&ms.qfull);
    if (lane == 0) {
      tc::prefetch_tensormap(&tm_q);
      tc::prefetch_tensormap(&tm_l);
      tc::mbar_arrive_expect_tx(qb, static_cast<uint32_t>(G) * 16384u);
      for (int g = 0; g < G; ++g)
        tc::tma_load_4d(tc::smem_addr(qt + g * 16384), &tm_q, 0, static_cast<int>(b * a.Lq + q0), 0, hk * G + g, qb);
    }
    __syncwarp();
    // this lane's share of a tile's bias: chunks t*RN + 32k + lane of head g
    const float* bias_lane = a.bias != nullptr ? a.bias + ((int64_t)b * C + lane) * Hq + hk * G : nullptr;
    auto load_bias = [&](int jj, float (&bv)[RN / 32]) {
      const int jc = jj < J ? ms.job[jj] : 0, g = jc & 0xff, t = jc >> 8;
#pragma unroll
      for (int k = 0; k < RN / 32; ++k) {
        const int c = t * RN + 32 * k + lane;
        bv[k] = (jj < J && bias_lane != nullptr && c < C) ? bias_lane[(t * RN + 32 * k) * Hq + g] : 0.f;
      }
    };
    float b0[RN / 32], b1[RN / 32];
    load_bias(0, b0);
    load_bias(1, b1);
    int j = 0;
    for (; j < J; ++j) {
      const int st = j % NST, bs = j % RBR;
      if (j >= NST && !tc::wait_bounded_warp(tc::smem_addr(&ms.lfree[st]), ((j / NST) - 1) & 1, abort_flag)) break;
      const int jc = ms.job[j], g = jc & 0xff, t = jc >> 8;
      if (lane == 0) {
        const uint32_t lb = tc::smem_addr(&ms.lfull[st]);
        tc::mbar_arrive_expect_tx(lb, 32768u);
        tc::tma_load_5d(tc::smem_addr(lt + st * 32768), &tm_l, 0, b * C + t * RN, 0, a.lmk_per_qhead ? g : 0, hk, lb);
      }
      float b2[RN / 32];
      load_bias(j + 2, b2);
      if (j >= RBR && !tc::wait_bounded_warp(tc::smem_addr(&ms.bfree[bs]), ((j / RBR) - 1) & 1, abort_flag)) break;
#pragma unroll
      for (int k = 0; k < RN / 32; ++k) ms.bias[bs][32 * k + lane] = b0[k];
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(tc::smem_addr(&ms.bfull[bs]));
#pragma unroll
      for (int k = 0; k < RN / 32; ++k) {
        b0[k] = b1[k];
        b1[k] = b2[k];
      }
    }
    // wait (bounded, even after an abort) for the copies in flight
    if (lane == 0) {
      tc::mbar_wait(qb, 0);
      for (int jj = j - NST < 0 ? 0 : j - NST; jj < j; ++jj) tc::mbar_wait(tc::smem_addr(&ms.lfull[jj % NST]), (jj / NST) & 1);
    }
    __syncwarp();
  } else if (warp == R_W_MMA) {
    // ============================ MMA (converged warp) ========================
    constexpr uint32_t idesc = tc::idesc_bf16_f32(64, RN, 0, 0);
    const uint64_t dq0 = tc::smem_desc_sw128(tc::smem_addr(qt), 16, 1024);
    const uint64_t dl0 = tc::smem_desc_sw128(tc::smem_addr(lt), 16, 1024);
    bool ok = tc::wait_bounded_warp(tc::smem_addr(&ms.qfull), 0, abort_flag);
    for (int j = 0; ok && j < J; ++j) {
      const int st = j % NST, bf = j % RBUF;
      if (!tc::wait_bounded_warp(tc::smem_addr(&ms.lfull[st]), (j / NST) & 1, abort_flag)) break;
      if (j >= RBUF && !tc::wait_bounded_warp(tc::smem_addr(&ms.sfree[bf]), ((j / RBUF) - 1) & 1, abort_flag)) break;
      tc::fence_after_sync();
      const int g = ms.job[j] & 0xff;
      const uint64_t da = tc::desc_adv(dq0, g * 16384), db = tc::desc_adv(dl0, st * 32768);
      const uint32_t dS = tbase + RN * bf;
      if (tc::elect_one()) {
        tc::mma_bf16<false>(dS, da, db, idesc);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          tc::mma_bf16<true>(dS, tc::desc_adv(da, (kk >> 2) * 8192 + (kk & 3) * 32),
                             tc::desc_adv(db, (kk >> 2) * 16384 + (kk & 3) * 32), idesc);
        tc::mma_commit(tc::smem_addr(&ms.sdone[bf]));
        tc::mma_commit(tc::smem_addr(&ms.lfree[st]));
      }
      __syncwarp();
    }
    if (tc::elect_one()) {
      tc::mma_commit(tc::smem_addr(&ms.mma_drain));
      tc::mbar_wait(tc::smem_addr(&ms.mma_drain), 0);
    }
    __syncwarp();
  } else {
    // ============================ TMEM readers (warps 0-15) ===================
    // M=64 layout: S row r sits in lane (r % 16) of TMEM quadrant r / 16.  Warp
    // w reads quadrant w % 4, tile columns [32 (w / 4), +32): lanes 0-15 the
    // first 16 of those, lanes 16-31 the next 16 (tcgen05.ld.16x32bx2.x16).
    const int qd = warp & 3, cq = warp >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const int r = 16 * qd + (lane & 15);
    const int cb = 32 * cq + 16 * (lane >> 4);              // first tile column of this thread
    const int64_t rowq = q0 + r;
    const bool row_ok = rowq < a.Lq;
    const float scale = a.sm_scale;
    bool ok = true;
    int j = 0;
    // S tile of job jj into s, this thread's bias values into bias; both slots released
    auto read_tile = [&](int jj, uint32_t (&s)[RC], float (&bias)[RC]) -> bool {
      const int bf = jj % RBUF, bs = jj % RBR;
      if (!tc::wait_bounded_warp(tc::smem_addr(&ms.bfull[bs]), (jj / RBR) & 1, abort_flag)) return false;
      if (!tc::wait_bounded_warp(tc::smem_addr(&ms.sdone[bf]), (jj / RBUF) & 1, abort_flag)) return false;
      tc::fence_after_sync();
      tc::tmem_ld_16x32bx2_x16(tbase + lane_off + RN * bf + 32 * cq, s);
#pragma unroll
      for (int i = 0; i < RC; i += 4) {
        const float4 v = *reinterpret_cast<const float4*>(&ms.bias[bs][cb + i]);
        bias[i] = v.x;
        bias[i + 1] = v.y;
        bias[i + 2] = v.z;
        bias[i + 3] = v.w;
      }
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(tc::smem_addr(&ms.sfree[bf]));
        tc::mbar_arrive(tc::smem_addr(&ms.bfree[bs]));
      }
      return true;
    };
    // ---- pass 1: online log-sum-exp (log2 domain) per (query, head)
    for (int g = 0; g < G; ++g) {
      float m = -INFINITY, l = 0.f;
      for (int t = 0; ok && t < NT; ++t, ++j) {
        float bias[RC];
        uint32_t s[RC];
        if (!(ok = read_tile(j, s, bias))) break;
        float y[RC], mb = -INFINITY;
        if ((t + 1) * RN <= C) {
          // whole tile: the same roundings as the scalar form, two columns per
          // instruction (paired fp32 fma / mul, three-input max)
#pragma unroll
          for (int i = 0; i < RC; i += 2) {
            const float2 x2 = ffma2(make_float2(__uint_as_float(s[i]), __uint_as_float(s[i + 1])),
                                    make_float2(scale, scale), make_float2(bias[i], bias[i + 1]));
            const float2 y2 = fmul2(x2, make_float2(kLog2e, kLog2e));
            y[i] = y2.x;
            y[i + 1] = y2.y;
            mb = fmax3(mb, y2.x, y2.y);
          }
        } else {
#pragma unroll
          for (int i = 0; i < RC; ++i) {
            const int c = t * RN + cb + i;
            const float x = fmaf(__uint_as_float(s[i]), scale, bias[i]);
            y[i] = c < C ? x * kLog2e : -INFINITY;
            mb = fmaxf(mb, y[i]);
          }
        }
        if (mb > m) {
          l = (m == -INFINITY) ? 0.f : l * fast_exp2(m - mb);
          m = mb;
        }
        if (m != -INFINITY) {
          float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < RC; i += 4) {
            const float2 d01 = fadd2(make_float2(y[i], y[i + 1]), make_float2(-m, -m));
            const float2 d23 = fadd2(make_float2(y[i + 2], y[i + 3]), make_float2(-m, -m));
            s01 = fadd2(s01, make_float2(fast_exp2(d01.x), fast_exp2(d01.y)));
            s23 = fadd2(s23, make_float2(fast_exp2(d23.x), fast_exp2(d23.y)));
          }
          l += (s01.x + s01.y) + (s23.x + s23.y);
        }
      }
      // combine the two column halves held by this warp (lanes t, t+16); the
      // four column quarters of a row meet in shared memory (two buffers: head
      // g+2 rewrites one only after the barrier of head g+1)
      const float mo = __shfl_xor_sync(0xffffffffu, m, 16), lo = __shfl_xor_sync(0xffffffffu, l, 16);
      const float mn = fmaxf(m, mo);
      l = (mn == -INFINITY) ? 0.f : l * fast_exp2(m - mn) + lo * fast_exp2(mo - mn);
      m = mn;
      if (lane < 16) {
        ms.part[g & 1][cq][r][0] = m;
        ms.part[g & 1][cq][r][1] = l;
      }
      // every reader reaches this barrier once per head, aborted or not
      asm volatile("bar.sync 1, 512;\n" ::: "memory");
      if (ok && cq == 0 && lane < 16) {
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < 4; ++k) mx = fmaxf(mx, ms.part[g & 1][k][r][0]);
        float lsum = 0.f;
        if (mx != -INFINITY) {
#pragma unroll
          for (int k = 0; k < 4; ++k) lsum += ms.part[g & 1][k][r][1] * fast_exp2(ms.part[g & 1][k][r][0] - mx);
        }
        const float lse = lsum > 0.f ? (mx + __log2f(lsum)) * kLn2 : -INFINITY;
        const float loc = row_ok ? a.local_lse[((int64_t)b * a.Lq + rowq) * Hq + hk * G + g] : 0.f;
        const float hi = fmaxf(loc, lse), lo2 = fminf(loc, lse);
        ms.T[r][g] = (hi == -INFINITY) ? -INFINITY : hi + log1pf(expf(lo2 - hi));
      }
    }
    asm volatile("bar.sync 1, 512;\n" ::: "memory");
    // ---- pass 2: keys = max_g (x - T_g), the drop rule, fp32 keys to the workspace
    int64_t clo = 1, chi = 0;                 // dropped chunk window [clo, chi] of this row
    if (a.drop == nullptr && a.window >= 0) {
      const int64_t pos = a.q_offset + rowq, L = static_cast<int64_t>(C) * kChunk;
      int64_t lo = pos - a.window, hi = pos + a.window;
      if (lo < 0) lo = 0;
      if (hi > L - 1) hi = L - 1;
      clo = lo / kChunk;
      chi = hi / kChunk;
    }
    float* krow = a.keys + (((int64_t)b * a.Lq + rowq) * a.Hkv + hk) * C;
    for (int t = 0; ok && t < NT; ++t) {
      float key[RC];
#pragma unroll
      for (int i = 0; i < RC; ++i) key[i] = -INFINITY;
      for (int g = 0; g < G; ++g, ++j) {
        const float Tg = ms.T[r][g];
        float bias[RC];
        uint32_t s[RC];
        if (!(ok = read_tile(j, s, bias))) break;
        // raw = s * scale, key = max(key, (raw + bias) - T_g): two columns per instruction
#pragma unroll
        for (int i = 0; i < RC; i += 2) {
          const float2 raw2 = fmul2(make_float2(__uint_as_float(s[i]), __uint_as_float(s[i + 1])),
                                    make_float2(scale, scale));
          s[i] = __float_as_uint(raw2.x);
          s[i + 1] = __float_as_uint(raw2.y);
          const float2 k2 = fadd2(fadd2(raw2, make_float2(bias[i], bias[i + 1])), make_float2(-Tg, -Tg));
          key[i] = fmaxf(key[i], k2.x);
          key[i + 1] = fmaxf(key[i + 1], k2.y);
        }
        // the raw scaled scores of every (head, chunk): the selection kernel gathers its slots from here
        if (row_ok) {
          const int c0 = t * RN + cb;
          const int64_t o = (((int64_t)b * a.Lq + rowq) * Hq + hk * G + g) * C + c0;
          // whole 32-byte sectors per store where C allows (each thread's 16
          // columns start on a multiple of 16): half-sector stores from 16 rows
          // per instruction kept the L1 busy
          if (a.scores_f32) {
            float* dst = static_cast<float*>(a.raw) + o;
            if (c0 + RC <= C && (C & 15) == 0) {
#pragma unroll
              for (int i = 0; i < RC; i += 8) {
                const uint32_t v8[8] = {s[i], s[i + 1], s[i + 2], s[i + 3], s[i + 4], s[i + 5], s[i + 6], s[i + 7]};
                st_global_v8(dst + i, v8);
              }
            } else {
#pragma unroll
              for (int i = 0; i < RC; ++i)
                if (c0 + i < C) dst[i] = __uint_as_float(s[i]);
            }
          } else {
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.raw) + o;
            if (c0 + RC <= C && (C & 15) == 0) {
              uint32_t v8[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) v8[i] = pack_bf16x2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1]));
              st_global_v8(dst, v8);
            } else {
#pragma unroll
              for (int i = 0; i < RC; ++i)
                if (c0 + i < C) dst[i] = f2bf(__uint_as_float(s[i]));
            }
          }
        }
      }
      if (!ok || !row_ok) continue;
      // dropped columns as a bit mask (bit i = column cb + i of this tile)
      uint32_t dm = 0u;
      if (a.drop != nullptr) {
        const int32_t* dr = a.drop + ((int64_t)b * a.Lq + rowq) * C;
#pragma unroll 8
        for (int i = 0; i < RC; ++i) {
          const int c = t * RN + cb + i;
          if (c < C && dr[c] != 0) dm |= 1u << i;
        }
      } else {
#pragma unroll
        for (int i = 0; i < RC; ++i) {
          const int c = t * RN + cb + i;
          if (c < C && (ms.chunk_ok[c] == 0 || (c >= clo && c <= chi))) dm |= 1u << i;
        }
      }
#pragma unroll
      for (int i = 0; i < RC; ++i)
        if ((dm >> i) & 1u) key[i] = -INFINITY;
      const int c0 = t * RN + cb;
      if (c0 + RC <= C && (C & 15) == 0) {
#pragma unroll
        for (int i = 0; i < RC; i += 8) {
          const uint32_t v8[8] = {__float_as_uint(key[i]), __float_as_uint(key[i + 1]), __float_as_uint(key[i + 2]),
                                  __float_as_uint(key[i + 3]), __float_as_uint(key[i + 4]), __float_as_uint(key[i + 5]),
                                  __float_as_uint(key[i + 6]), __float_as_uint(key[i + 7])};
          st_global_v8(krow + c0 + i, v8);
        }
      } else {
#pragma unroll
        for (int i = 0; i < RC; ++i)
          if (c0 + i < C) krow[c0 + i] = key[i];
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && ms.abort_flag) atomicOr(&g_route_error, 1);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

// Route weights of one (query, head) row; lane k holds selected slot k.
// r = raw score (already bf16-rounded) + bias, -inf for empty slots.
__device__ __forceinline__ void route_weights_row(float r, bool valid, float local, int K,
                                                  int mode, float temp, float gscale, float goff,
                                                  float& w_remote, float& w_local) {
  const int lane = threadIdx.x & 31;
  const bool live = lane < K;
  const float inv_t = 1.0f / temp;
  float rl = (live && valid) ? r : -INFINITY;
  if (mode == MRSA_WEIGHTS_SOFTMAX) {
    const float lt = (local - goff) * inv_t;
    const float rt = rl * inv_t;
    const float m = fmaxf(warp_max(rt), lt);
    if (m == -INFINITY) {   // every logit masked -> zeros
      w_remote = 0.f;
      w_local = 0.f;
      return;
    }
    const float e = (rt == -INFINITY) ? 0.f : expf(rt - m);
    const float el = (lt == -INFINITY) ? 0.f : expf(lt - m);
    const float sum = warp_sum(e) + el;
    w_remote = e / sum;
    w_local = el / sum;
    return;
  }
  // affine gate (live path: fusion_gate_scale exists)
  const float rt = rl * inv_t, lt = local * inv_t;
  const float mr = warp_max(rt);
  if (mr == -INFINITY && lt == -INFINITY) {
    w_remote = 0.f;
    w_local = 0.f;
    return;
  }
  float inner = 0.f, remote_lse = -INFINITY;
  if (mr != -INFINITY) {
    const float e = (rt == -INFINITY) ? 0.f : expf(rt - mr);
    const float sum = warp_sum(e);
    inner = e / sum;
    remote_lse = mr + logf(sum);
  }
  const float gate = gscale * (remote_lse - lt) + goff;
  const float msig = 1.0f / (1.0f + expf(-gate));
  w_remote = inner * msig;
  w_local = 1.0f - msig;
}

constexpr int SEL_WARPS = 8;
constexpr int SEL_CAND = 256;     // filtered candidates one warp keeps (8 per lane)

// Largest threshold t (order-preserving key) with at least keff of the finite
// keys in u[] >= t; the search may stop early once exactly keff keys are >= t,
// since those keys are then the top keff and the selection takes all of them.
// The threshold is one of the finite keys, so the high bits every finite key
// shares are its bits from the start.  Padding slots hold 0 (below every key).
template <int N>
__device__ __forceinline__ uint32_t radix_threshold(const uint32_t (&u)[N], int keff) {
  const uint32_t neg_inf_ord = f2ord(-INFINITY);
  uint32_t orv = 0u, andv = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (u[i] > neg_inf_ord) {
      orv |= u[i];
      andv &= u[i];
    }
  orv = __reduce_or_sync(0xffffffffu, orv);
  andv = __reduce_and_sync(0xffffffffu, andv);
  const uint32_t diff = orv ^ andv;
  if (diff == 0u) return andv;           // every finite key is the same value
  const int top = 31 - __clz(diff);
  uint32_t thr = top == 31 ? 0u : (andv & ~((2u << top) - 1u));
  for (int bit = top; bit >= 0; --bit) {
    const uint32_t cand = thr | (1u << bit);
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) cnt += u[i] >= cand;
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (cnt >= keff) {
      thr = cand;
      if (cnt == keff) break;
    }
  }
  return thr;
}

// One warp per (query, KV head): top-K of the row's keys, raw scores, weights.
// CPL = keys per lane (C <= 32 * CPL), a compile-time bound so the keys stay in
// registers.  With 16 or more keys per lane the search runs on a filtered
// candidate list: the smallest of the 32 lanes' maxima, t0, has at least 32
// keys >= it (each lane's maximum), so when K <= 32 every selected key is >= t0
// and only those keys (about 125 of 2048 when each key is the maximum of seven
// Gaussian scores) are compacted into shared memory and searched.  Rows whose filter keeps fewer than K or
// more than SEL_CAND keys take the full search.  The selection is the same set
// either way: the K largest finite keys, ties at the threshold broken towards
// the lowest chunk ids, emitted in ascending chunk order.
template <int CPL>
__global__ void __launch_bounds__(SEL_WARPS * 32, 3) route_select_kernel(RouteArgs a) {
  constexpr bool kFilter = CPL >= 16;
  constexpr int NCW = kFilter ? SEL_WARPS : 1;
  __shared__ int sel_s[SEL_WARPS][32];
  __shared__ uint32_t cand_k[NCW][kFilter ? SEL_CAND : 1];
  __shared__ uint16_t cand_c[NCW][kFilter ? SEL_CAND : 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * SEL_WARPS + warp;
  if (row >= a.Lq) return;
  const int C = a.C, G = a.G, K = a.K, Hq = a.Hkv * a.G;
  const float* krow = a.keys + (((int64_t)b * a.Lq + row) * a.Hkv + hk) * C;
  uint32_t u[CPL];
  const uint32_t neg_inf_ord = f2ord(-INFINITY);
  int nf = 0;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = i * 32 + lane;
    u[i] = c < C ? f2ord(krow[c]) : 0u;
    nf += u[i] > neg_inf_ord;
  }
  nf = __reduce_add_sync(0xffffffffu, nf);
  const int keff = nf < K ? nf : K;
  uint32_t thr = 0;
  int csel = -1;
  bool sorted = false;       // csel already holds the selection in ascending order
  bool have_thr = false;
  if (kFilter && keff > 0 && nf > K && K <= 32) {
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < CPL; ++i) m = u[i] > m ? u[i] : m;
    const uint32_t t0 = __reduce_min_sync(0xffffffffu, m > neg_inf_ord ? m : 0xffffffffu);
    int cl = 0;
#pragma unroll
    for (int i = 0; i < CPL; ++i) cl += u[i] >= t0;
    const int n = __reduce_add_sync(0xffffffffu, cl);
    if (n >= keff && n <= SEL_CAND) {
      int off = cl;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, off, d);
        if (lane >= d) off += v;
      }
      off -= cl;
#pragma unroll
      for (int i = 0; i < CPL; ++i)
        if (u[i] >= t0) {
          cand_k[kFilter ? warp : 0][off] = u[i];
          cand_c[kFilter ? warp : 0][off] = static_cast<uint16_t>(i * 32 + lane);
          ++off;
        }
      __syncwarp();
      constexpr int R = SEL_CAND / 32;
      uint32_t v[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int j = r * 32 + lane;
        v[r] = j < n ? cand_k[kFilter ? warp : 0][j] : 0u;
      }
      thr = radix_threshold<R>(v, keff);
      // an early stop below t0 (only when exactly keff candidates exist) means t0 itself
      thr = thr > t0 ? thr : t0;
      have_thr = true;
      int ngt = 0, neq = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        ngt += v[r] > thr;
        neq += v[r] == thr;
      }
      ngt = __reduce_add_sync(0xffffffffu, ngt);
      neq = __reduce_add_sync(0xffffffffu, neq);
      if (ngt + neq == keff) {
        // every key at the threshold is taken: gather the picks, sort by chunk id
        int taken = 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int j = r * 32 + lane;
          const bool pick = j < n && v[r] >= thr;
          const uint32_t pm = __ballot_sync(0xffffffffu, pick);
          if (pick) sel_s[warp][taken + __popc(pm & ((1u << lane) - 1u))] = cand_c[kFilter ? warp : 0][j];
          taken += __popc(pm);
        }
        __syncwarp();
        int x = lane < keff ? sel_s[warp][lane] : 0x7fffffff;
#pragma unroll
        for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
          for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
            const int o = __shfl_xor_sync(0xffffffffu, x, j2);
            const bool up = (lane & k2) == 0, lower = (lane & j2) == 0;
            x = (lower == up) ? min(x, o) : max(x, o);
          }
        }
        csel = lane < keff ? x : -1;
        sorted = true;
      }
    }
  }
  if (!sorted) {
    if (kFilter) {
      // rare rows (ties at the threshold, or a filter that kept too few or too
      // many keys): the keys are read again from L1/L2 rather than kept live
      // in registers across the filtered search
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int c = i * 32 + lane;
        u[i] = c < C ? f2ord(krow[c]) : 0u;
      }
    }
    if (keff > 0 && !have_thr) thr = radix_threshold<CPL>(u, keff);
    int ngt = 0;
#pragma unroll
    for (int i = 0; i < CPL; ++i) ngt += u[i] > thr;
    ngt = keff > 0 ? __reduce_add_sync(0xffffffffu, ngt) : 0;
    int need_eq = keff - ngt, taken = 0;
    // ascending chunk order; ties at the threshold: lowest chunk ids first
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      if (keff == 0) break;
      const int c = i * 32 + lane;
      const bool in = c < C;
      const bool gt = in && u[i] > thr;
      const bool eq = in && u[i] == thr;
      const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
      const int eq_before = __popc(eq_mask & ((1u << lane) - 1u));
      const bool pick = gt || (eq && eq_before < need_eq);
      need_eq -= __popc(eq_mask) < need_eq ? __popc(eq_mask) : need_eq;
      const uint32_t pm = __ballot_sync(0xffffffffu, pick);
      if (pick) sel_s[warp][taken + __popc(pm & ((1u << lane) - 1u))] = c;
      taken += __popc(pm);
    }
    __syncwarp();
    csel = lane < keff ? sel_s[warp][lane] : -1;
  }
  if (lane < K) a.indices[(((int64_t)b * a.Lq + row) * a.Hkv + hk) * K + lane] = csel;
  // Raw scores of the selection, gathered from the key kernel's full score
  // rows, and the route weights of all heads at once: lane (g, sg) = (lane / 4,
  // lane % 4) takes head g's slots 8*sg .. 8*sg+7, so a head's reductions run
  // over a group of four lanes (each lane's eight values first, then two
  // shuffles) instead of a full-warp butterfly per head.  The slot sums are
  // added in the tree of a 32-lane butterfly with xor 16, 8, 4, 2, 1 (slot s =
  // 8*sg + k: s^16 and s^8 are the lanes xor 2 and xor 1, s^4, s^2, s^1 are k's
  // bits), which is the order route_weights_row() uses.
  __syncwarp();
  sel_s[warp][lane] = csel;
  __syncwarp();
  {
    const int g = lane >> 2, sg = lane & 3;
    const bool gon = g < G;
    const int hq = hk * G + (gon ? g : 0);
    const int64_t rowhq = ((int64_t)b * a.Lq + row) * Hq + hq;
    float rr[8];
    bool live[8], valid[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int slot = 8 * sg + k;
      live[k] = slot < K;
      const int c = live[k] ? sel_s[warp][slot] : -1;
      valid[k] = gon && c >= 0;
      float raw = -INFINITY, bias = 0.f;
      if (valid[k]) {
        raw = a.scores_f32 ? static_cast<const float*>(a.raw)[rowhq * C + c]
                           : bf2f(static_cast<const __nv_bfloat16*>(a.raw)[rowhq * C + c]);
        if (a.bias != nullptr) bias = a.bias[((int64_t)b * C + c) * Hq + hq];
      }
      if (gon && live[k]) {
        if (a.scores_f32) static_cast<float*>(a.scores)[rowhq * K + slot] = raw;
        else static_cast<__nv_bfloat16*>(a.scores)[rowhq * K + slot] = f2bf(raw);
      }
      // the weights see the scores as the reference stores them (bf16)
      const float sc = a.scores_f32 ? raw : round_bf16(raw);
      rr[k] = valid[k] ? sc + bias : -INFINITY;
    }
    if (a.remote_w != nullptr) {
      const float local = gon ? a.local_lse[rowhq] : 0.f;
      const float inv_t = 1.0f / a.temperature;
      float rt[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) rt[k] = rr[k] * inv_t;     // -inf stays -inf (dead and empty slots)
      float mx = rt[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) mx = fmaxf(mx, rt[k]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      const bool softmax = a.weight_mode == MRSA_WEIGHTS_SOFTMAX;
      const float lt = softmax ? (local - a.gate_offset) * inv_t : local * inv_t;
      const float m = softmax ? fmaxf(mx, lt) : mx;
      float e[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = (rt[k] == -INFINITY || m == -INFINITY) ? 0.f : expf(rt[k] - m);
      float t[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = e[k] + __shfl_xor_sync(0xffffffffu, e[k], 2);
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = t[k] + __shfl_xor_sync(0xffffffffu, t[k], 1);
#pragma unroll
      for (int k = 0; k < 4; ++k) t[k] = t[k] + t[k + 4];
      t[0] = t[0] + t[2];
      t[1] = t[1] + t[3];
      const float sum = t[0] + t[1];
      float wr[8], wl;
      if (softmax) {
        if (m == -INFINITY) {                // every logit masked -> zeros
#pragma unroll
          for (int k = 0; k < 8; ++k) wr[k] = 0.f;
          wl = 0.f;
        } else {
          const float el = (lt == -INFINITY) ? 0.f : expf(lt - m);
          const float tot = sum + el;
#pragma unroll
          for (int k = 0; k < 8; ++k) wr[k] = e[k] / tot;
          wl = el / tot;
        }
      } else if (mx == -INFINITY && lt == -INFINITY) {
#pragma unroll
        for (int k = 0; k < 8; ++k) wr[k] = 0.f;
        wl = 0.f;
      } else {
        // affine gate (live path: fusion_gate_scale exists)
        float inner[8], remote_lse = -INFINITY;
#pragma unroll
        for (int k = 0; k < 8; ++k) inner[k] = 0.f;
        if (mx != -INFINITY) {
#pragma unroll
          for (int k = 0; k < 8; ++k) inner[k] = e[k] / sum;
          remote_lse = mx + logf(sum);
        }
        const float gate = a.gate_scale * (remote_lse - lt) + a.gate_offset;
        const float msig = 1.0f / (1.0f + expf(-gate));
#pragma unroll
        for (int k = 0; k < 8; ++k) wr[k] = inner[k] * msig;
        wl = 1.0f - msig;
      }
      if (gon) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (live[k]) a.remote_w[rowhq * K + 8 * sg + k] = f2bf(wr[k]);
        if (sg == 0) a.local_w[rowhq] = f2bf(wl);
      }
    }
  }
}

__global__ void route_weights_kernel(const __nv_bfloat16* __restrict__ scores,
                                     const int32_t* __restrict__ indices,
                                     const float* __restrict__ prior,
                                     const float* __restrict__ local_lse,
                                     __nv_bfloat16* __restrict__ remote_w,
                                     __nv_bfloat16* __restrict__ local_w, int64_t rows, int Hkv,
                                     int G, int C, int K, int64_t L, int mode, float temp,
                                     float gs, float go) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  const int Hq = Hkv * G;
  const int hq = static_cast<int>(r % Hq);
  const int64_t bl = r / Hq;
  const int64_t b = bl / L;
  const int hk = hq / G;
  const int c = lane < K ? indices[(bl * Hkv + hk) * K + lane] : -1;
  const bool valid = c >= 0 && c < C;
  const float s = lane < K ? bf2f(scores[r * K + lane]) : -INFINITY;
  const float rr = valid ? s + prior[(b * C + c) * Hq + hq] : -INFINITY;
  float wr, wl;
  route_weights_row(rr, valid, local_lse[r], K, mode, temp, gs, go, wr, wl);
  if (lane < K) remote_w[r * K + lane] = f2bf(wr);
  if (lane == 0) local_w[r] = f2bf(wl);
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

}  // namespace

namespace {
size_t keys_bytes(int64_t batch, int64_t q_len, int64_t chunks, int64_t kv_heads) {
  return (static_cast<size_t>(batch * q_len * kv_heads * chunks) * sizeof(float) + 255) / 256 * 256;
}
}  // namespace

extern "C" size_t mrsa_route_topk_workspace_size(int64_t batch, int64_t q_len, int64_t chunks,
                                                 int64_t kv_heads, int64_t groups, int scores_dtype) {
  if (batch < 1 || q_len < 0 || chunks < 1 || kv_heads < 1 || groups < 1) return 0;
  if (scores_dtype != MRSA_BF16 && scores_dtype != MRSA_F32) return 0;
  const size_t raw = static_cast<size_t>(batch * q_len * kv_heads * groups * chunks) *
                     (scores_dtype == MRSA_F32 ? 4 : 2);
  return keys_bytes(batch, q_len, chunks, kv_heads) + raw;
}

extern "C" int mrsa_route_topk(const void* route_q, const void* landmarks, int lmk_per_qhead,
                               const float* local_lse, const float* bias, const int32_t* drop_mask,
                               const uint8_t* chunk_ok, int64_t window, int64_t q_offset,
                               int32_t* indices, void* scores_out, int scores_dtype,
                               void* remote_w, void* local_w, int weight_mode, float temperature,
                               float gate_scale, float gate_offset, int64_t batch, int64_t q_len,
                               int64_t chunks, int64_t kv_heads, int64_t groups, int64_t head_dim,
                               int64_t topk, void* workspace, size_t workspace_bytes,
                               mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(route_q);
  if (!route_q || !landmarks || !local_lse || !indices || !scores_out) return MRSA_ERR_NULL;
  if ((remote_w == nullptr) != (local_w == nullptr)) return MRSA_ERR_NULL;
  if (head_dim != D || groups < 1 || groups > RGMAX || kv_heads < 1 || batch < 1 || q_len < 0 ||
      chunks < 1 || chunks > kMaxChunks || topk < 1 || topk > 32 || kv_heads > 65535 ||
      batch > 65535 || q_offset < 0 || batch * q_len * kv_heads * groups > 0x7fffffffLL ||
      batch * chunks > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if (scores_dtype != MRSA_BF16 && scores_dtype != MRSA_F32) return MRSA_ERR_ARG;
  if (weight_mode != MRSA_WEIGHTS_AFFINE && weight_mode != MRSA_WEIGHTS_SOFTMAX) return MRSA_ERR_ARG;
  if (!(temperature > 0.f)) return MRSA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(route_q) & 15u) || (reinterpret_cast<uintptr_t>(landmarks) & 15u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15u))
    return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  if (workspace == nullptr ||
      workspace_bytes < mrsa_route_topk_workspace_size(batch, q_len, chunks, kv_heads, groups, scores_dtype))
    return MRSA_ERR_WORKSPACE;
  RouteArgs a;
  a.rq = static_cast<const __nv_bfloat16*>(route_q);
  a.lmk = static_cast<const __nv_bfloat16*>(landmarks);
  a.lmk_per_qhead = lmk_per_qhead ? 1 : 0;
  a.local_lse = local_lse;
  a.bias = bias;
  a.drop = drop_mask;
  a.chunk_ok = chunk_ok;
  a.window = window;
  a.q_offset = q_offset;
  a.keys = static_cast<float*>(workspace);
  a.raw = static_cast<char*>(workspace) + keys_bytes(batch, q_len, chunks, kv_heads);
  a.indices = indices;
  a.scores = scores_out;
  a.scores_f32 = scores_dtype == MRSA_F32;
  a.remote_w = static_cast<__nv_bfloat16*>(remote_w);
  a.local_w = static_cast<__nv_bfloat16*>(local_w);
  a.weight_mode = weight_mode;
  a.temperature = temperature;
  a.gate_scale = gate_scale;
  a.gate_offset = gate_offset;
  a.Lq = q_len;
  a.C = static_cast<int>(chunks);
  a.Hkv = static_cast<int>(kv_heads);
  a.G = static_cast<int>(groups);
  a.K = static_cast<int>(topk);
  a.sm_scale = 1.0f / sqrtf(static_cast<float>(D));
  int nst = RMAXST;
  while (nst > 2 && key_smem_bytes(a.G, nst) > static_cast<size_t>(kSmemLimit)) --nst;
  a.nst = nst;
  // route_q [B*Lq rows][Hq][128] as (dim-in-half, row, half, head): one box = 64 query rows of one head
  // landmarks [B*C rows][Hkv][G'][128] as (dim-in-half, row, half, head-in-group, kv head): 128 chunks
  const int64_t Hq = kv_heads * groups, Gl = lmk_per_qhead ? groups : 1;
  CUtensorMap tm_q, tm_l;
  const cuuint64_t q_dims[4] = {64, static_cast<cuuint64_t>(batch * q_len), 2, static_cast<cuuint64_t>(Hq)};
  const cuuint64_t q_str[3] = {static_cast<cuuint64_t>(Hq * D * 2), 128, 256};
  const cuuint32_t q_box[4] = {64, RQ, 2, 1};
  const cuuint64_t l_dims[5] = {64, static_cast<cuuint64_t>(batch * chunks), 2, static_cast<cuuint64_t>(Gl),
                                static_cast<cuuint64_t>(kv_heads)};
  const cuuint64_t l_str[4] = {static_cast<cuuint64_t>(kv_heads * Gl * D * 2), 128, 256, static_cast<cuuint64_t>(Gl * D * 2)};
  const cuuint32_t l_box[5] = {64, RN, 2, 1, 1};
  if (!make_map(&tm_q, route_q, 4, q_dims, q_str, q_box) || !make_map(&tm_l, landmarks, 5, l_dims, l_str, l_box))
    return MRSA_ERR_LAUNCH;
  const size_t smem = key_smem_bytes(a.G, nst);
  if (cudaFuncSetAttribute(route_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t kblocks = (q_len + RQ - 1) / RQ;
  dim3 kgrid(static_cast<unsigned>(kblocks), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
  route_keys_kernel<<<kgrid, R_THREADS, smem, st>>>(tm_q, tm_l, a);
  MRSA_CHECK_LAUNCH();
  const int64_t sblocks = (q_len + SEL_WARPS - 1) / SEL_WARPS;
  dim3 sgrid(static_cast<unsigned>(sblocks), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
  if (chunks <= 256) route_select_kernel<8><<<sgrid, SEL_WARPS * 32, 0, st>>>(a);
  else if (chunks <= 512) route_select_kernel<16><<<sgrid, SEL_WARPS * 32, 0, st>>>(a);
  else if (chunks <= 1024) route_select_kernel<32><<<sgrid, SEL_WARPS * 32, 0, st>>>(a);
  else route_select_kernel<64><<<sgrid, SEL_WARPS * 32, 0, st>>>(a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" int mrsa_route_weights(const void* scores, const int32_t* indices, const float* prior,
                                  const float* local_lse, void* remote_w, void* local_w,
                                  int weight_mode, float temperature, float gate_scale,
                                  float gate_offset, int64_t batch, int64_t seq_len,
                                  int64_t chunks, int64_t kv_heads, int64_t groups, int64_t topk,
                                  mrsa_stream_t stream) {
  if (!scores || !indices || !prior || !local_lse || !remote_w || !local_w) return MRSA_ERR_NULL;
  if (batch < 1 || seq_len < 0 || chunks < 1 || kv_heads < 1 || groups < 1 || topk < 1 || topk > 32)
    return MRSA_ERR_SHAPE;
  if (weight_mode != MRSA_WEIGHTS_AFFINE && weight_mode != MRSA_WEIGHTS_SOFTMAX) return MRSA_ERR_ARG;
  if (!(temperature > 0.f)) return MRSA_ERR_ARG;
  const int64_t rows = batch * seq_len * kv_heads * groups;
  if (rows == 0) return MRSA_OK;
  const int64_t blocks = (rows * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  route_weights_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(scores), indices, prior, local_lse,
      static_cast<__nv_bfloat16*>(remote_w), static_cast<__nv_bfloat16*>(local_w), rows,
      static_cast<int>(kv_heads), static_cast<int>(groups), static_cast<int>(chunks),
      static_cast<int>(topk), seq_len, weight_mode, temperature, gate_scale, gate_offset);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

namespace mrsa {
// Read (and optionally clear) the routing kernels' device error flag.
int route_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_route_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_route_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
}  // namespace mrsa
