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
// CTA = 16 queries x one KV head.  Warp g owns query head g of the group for
// the two GEMM passes (mma.sync m16n8k16, landmarks read through L2); the
// max-pooled keys of all chunks stay in shared memory; each warp then selects
// the top-K of two queries with a 32-step radix search over order-preserving
// integer keys, gathers raw scores for its selection and emits weights.
#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int QB = 16;      // queries per CTA
constexpr int NW = 8;       // warps per CTA
constexpr int CT = 64;      // chunks per key tile in pass 2
constexpr int D = kHeadDim;
constexpr int kMaxChunks = 2048;

struct RouteArgs {
  const __nv_bfloat16* rq;
  const __nv_bfloat16* lmk;
  int lmk_g_stride;         // elements between query heads of one chunk/kv head (D or 0)
  const float* local_lse;
  const float* bias;
  const int32_t* drop;
  const uint8_t* chunk_ok;
  int64_t window, q_offset;
  int32_t* indices;
  void* scores;
  int scores_f32;
  __nv_bfloat16* remote_w;
  __nv_bfloat16* local_w;
  int weight_mode;
  float temperature, gate_scale, gate_offset;
  int64_t Lq;
  int C, Hkv, G, K;
  float sm_scale;
};

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

__device__ __forceinline__ bool dropped(const RouteArgs& a, int b, int64_t pos, int c,
                                        const uint8_t* chunk_ok_s) {
  if (a.drop != nullptr) return a.drop[((int64_t)b * a.Lq + (pos - a.q_offset)) * a.C + c] != 0;
  if (chunk_ok_s[c] == 0) return true;
  if (a.window < 0) return false;
  const int64_t L = static_cast<int64_t>(a.C) * kChunk;
  int64_t lo = pos - a.window, hi = pos + a.window;
  if (lo < 0) lo = 0;
  if (hi > L - 1) hi = L - 1;
  return c >= lo / kChunk && c <= hi / kChunk;
}

__global__ void __launch_bounds__(NW * 32) route_kernel(RouteArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* keys = reinterpret_cast<float*>(smem_raw);                 // [QB][C]
  float* xg = keys + QB * a.C;                                      // [NW][QB][CT]
  float* Tsm = xg + NW * QB * CT;                                   // [QB][NW]
  int* sel = reinterpret_cast<int*>(Tsm + QB * NW);                 // [QB][32]
  uint8_t* chunk_ok_s = reinterpret_cast<uint8_t*>(sel + QB * 32);  // [C]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, tq = lane & 3;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * QB;
  const int C = a.C, G = a.G, Hq = a.Hkv * a.G;

  for (int c = tid; c < C; c += NW * 32)
    chunk_ok_s[c] = a.chunk_ok ? a.chunk_ok[(int64_t)b * C + c] : 1;

  const bool gemm_warp = warp < G;
  const int hq = hk * G + warp;
  const int64_t row0 = q0 + g4, row1 = q0 + g4 + 8;
  const bool ok0 = row0 < a.Lq, ok1 = row1 < a.Lq;

  uint32_t qa[D / 16][4];
  if (gemm_warp) {
    const __nv_bfloat16* r0p = a.rq + (((int64_t)b * a.Lq + (ok0 ? row0 : 0)) * Hq + hq) * D;
    const __nv_bfloat16* r1p = a.rq + (((int64_t)b * a.Lq + (ok1 ? row1 : 0)) * Hq + hq) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int c0 = ks * 16 + tq * 2;
      qa[ks][0] = ok0 ? *reinterpret_cast<const uint32_t*>(r0p + c0) : 0u;
      qa[ks][1] = ok1 ? *reinterpret_cast<const uint32_t*>(r1p + c0) : 0u;
      qa[ks][2] = ok0 ? *reinterpret_cast<const uint32_t*>(r0p + c0 + 8) : 0u;
      qa[ks][3] = ok1 ? *reinterpret_cast<const uint32_t*>(r1p + c0 + 8) : 0u;
    }
  }
  // landmark row pointer for chunk c of this warp's head
  auto lmk_row = [&](int c) {
    return a.lmk + (((int64_t)b * C + c) * a.Hkv + hk) * (int64_t)(a.lmk_g_stride ? G * D : D) +
           (int64_t)warp * a.lmk_g_stride;
  };
  // S tile (16 queries x 8 chunks starting at c0), scaled; invalid chunk cols -> -inf
  auto s_tile = [&](int c0, float* s) {
    s[0] = s[1] = s[2] = s[3] = 0.f;
    const int cc = c0 + g4;
    const __nv_bfloat16* lp = lmk_row(cc < C ? cc : 0);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(lp + ks * 16 + tq * 2);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(lp + ks * 16 + tq * 2 + 8);
      mma_bf16(s, qa[ks], b0, b1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i] *= a.sm_scale;
  };
  auto bias_of = [&](int c) -> float {
    return a.bias ? a.bias[((int64_t)b * C + c) * Hq + hq] : 0.f;
  };

  // ---- pass 1: T = logaddexp(local_lse, logsumexp_c x) ----------------------
  if (gemm_warp) {
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    for (int c0 = 0; c0 < C; c0 += 8) {
      float s[4];
      s_tile(c0, s);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = c0 + tq * 2 + (i & 1);
        const float x = c < C ? s[i] + bias_of(c) : -INFINITY;
        const int hr = i >> 1;
        if (x > m[hr]) {
          l[hr] = l[hr] * expf(m[hr] - x) + 1.f;
          m[hr] = x;
        } else if (x != -INFINITY) {
          l[hr] += expf(x - m[hr]);
        }
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[hr], o);
        const float lo = __shfl_xor_sync(0xffffffffu, l[hr], o);
        const float mn = fmaxf(m[hr], mo);
        l[hr] = (mn == -INFINITY) ? 0.f : l[hr] * expf(m[hr] - mn) + lo * expf(mo - mn);
        m[hr] = mn;
      }
      const float lse = (l[hr] > 0.f) ? m[hr] + logf(l[hr]) : -INFINITY;
      const int64_t row = hr ? row1 : row0;
      const bool ok = hr ? ok1 : ok0;
      const float loc = ok ? a.local_lse[((int64_t)b * a.Lq + row) * Hq + hq] : 0.f;
      const float mx = fmaxf(loc, lse), mnv = fminf(loc, lse);
      const float T = (mx == -INFINITY) ? -INFINITY : mx + log1pf(expf(mnv - mx));
      if (tq == 0) Tsm[(g4 + hr * 8) * NW + warp] = T;
    }
  }
  __syncthreads();

  // ---- pass 2: keys = max_g (x - T), dropped -> -inf -------------------------
  for (int ct = 0; ct < C; ct += CT) {
    if (gemm_warp) {
      const float T0 = Tsm[g4 * NW + warp], T1 = Tsm[(g4 + 8) * NW + warp];
#pragma unroll 2
      for (int n = 0; n < CT / 8; ++n) {
        const int c0 = ct + n * 8;
        if (c0 >= C) break;
        float s[4];
        s_tile(c0, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int cl = n * 8 + tq * 2 + (i & 1);
          const int c = ct + cl;
          const float x = c < C ? s[i] + bias_of(c) : -INFINITY;
          xg[(warp * QB + g4 + (i >> 1) * 8) * CT + cl] = x - ((i >> 1) ? T1 : T0);
        }
      }
    }
    __syncthreads();
    for (int e = tid; e < QB * CT; e += NW * 32) {
      const int qi = e / CT, cl = e % CT, c = ct + cl;
      if (c >= C) continue;
      float kmax = -INFINITY;
      for (int gg = 0; gg < G; ++gg) kmax = fmaxf(kmax, xg[(gg * QB + qi) * CT + cl]);
      const int64_t pos = a.q_offset + q0 + qi;
      if (q0 + qi < a.Lq && dropped(a, b, pos, c, chunk_ok_s)) kmax = -INFINITY;
      keys[qi * C + c] = kmax;
    }
    __syncthreads();
  }

  // ---- top-K per query: warp w -> queries w, w+8 ------------------------------
  for (int qi = warp; qi < QB; qi += NW) {
    const int64_t row = q0 + qi;
    if (row >= a.Lq) continue;
    const float* kr = keys + qi * C;
    const uint32_t neg_inf_ord = f2ord(-INFINITY);
    int nf = 0;
    for (int c = lane; c < C; c += 32) nf += f2ord(kr[c]) > neg_inf_ord;
    nf = __reduce_add_sync(0xffffffffu, nf);
    const int keff = nf < a.K ? nf : a.K;
    uint32_t thr = 0;
    if (keff > 0) {
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = thr | (1u << bit);
        int cnt = 0;
        for (int c = lane; c < C; c += 32) cnt += f2ord(kr[c]) >= cand;
        cnt = __reduce_add_sync(0xffffffffu, cnt);
        if (cnt >= keff) thr = cand;
      }
    }
    int ngt = 0;
    for (int c = lane; c < C; c += 32) ngt += f2ord(kr[c]) > thr;
    ngt = keff > 0 ? __reduce_add_sync(0xffffffffu, ngt) : 0;
    int need_eq = keff - ngt, taken = 0;
    // ascending chunk order; ties at the threshold: lowest chunk ids first
    for (int cb = 0; cb < C && keff > 0; cb += 32) {
      const int c = cb + lane;
      const uint32_t u = c < C ? f2ord(kr[c]) : 0u;
      const bool gt = c < C && u > thr;
      const bool eq = c < C && u == thr;
      const uint32_t eq_mask = __ballot_sync(0xffffffffu, eq);
      const int eq_before = __popc(eq_mask & ((1u << lane) - 1u));
      const bool pick = gt || (eq && eq_before < need_eq);
      need_eq -= __popc(eq_mask) < need_eq ? __popc(eq_mask) : need_eq;
      const uint32_t pm = __ballot_sync(0xffffffffu, pick);
      if (pick) sel[qi * 32 + taken + __popc(pm & ((1u << lane) - 1u))] = c;
      taken += __popc(pm);
    }
    __syncwarp();
    for (int k = lane; k < a.K; k += 32) {
      const int c = k < keff ? sel[qi * 32 + k] : -1;
      if (k >= keff) sel[qi * 32 + k] = -1;
      a.indices[(((int64_t)b * a.Lq + row) * a.Hkv + hk) * a.K + k] = c;
    }
  }
  __syncthreads();

  // ---- raw scores + route weights: warp g, lane = slot ------------------------
  if (gemm_warp) {
    for (int qi = 0; qi < QB; ++qi) {
      const int64_t row = q0 + qi;
      if (row >= a.Lq) break;
      const int c = lane < a.K ? sel[qi * 32 + lane] : -1;
      float raw = -INFINITY;
      if (c >= 0) {
        const __nv_bfloat16* qp = a.rq + (((int64_t)b * a.Lq + row) * Hq + hq) * D;
        const __nv_bfloat16* lp = lmk_row(c);
        float acc = 0.f;
#pragma unroll 4
        for (int p = 0; p < D / 8; ++p) {
          const uint4 qv = *reinterpret_cast<const uint4*>(qp + p * 8);
          const uint4 lv = *reinterpret_cast<const uint4*>(lp + p * 8);
          const uint32_t* qw = reinterpret_cast<const uint32_t*>(&qv);
          const uint32_t* lw = reinterpret_cast<const uint32_t*>(&lv);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float2 x = unpack_bf16x2(qw[w]), y = unpack_bf16x2(lw[w]);
            acc = fmaf(x.x, y.x, acc);
            acc = fmaf(x.y, y.y, acc);
          }
        }
        raw = acc * a.sm_scale;
      }
      const int64_t o = (((int64_t)b * a.Lq + row) * Hq + hq) * a.K + lane;
      if (lane < a.K) {
        if (a.scores_f32) static_cast<float*>(a.scores)[o] = raw;
        else static_cast<__nv_bfloat16*>(a.scores)[o] = f2bf(raw);
      }
      if (a.remote_w != nullptr) {
        // the weights see the scores as the reference stores them (bf16)
        const float sc = a.scores_f32 ? raw : round_bf16(raw);
        const float r = c >= 0 ? sc + bias_of(c) : -INFINITY;
        const float loc = a.local_lse[((int64_t)b * a.Lq + row) * Hq + hq];
        float wr, wl;
        route_weights_row(r, c >= 0, loc, a.K, a.weight_mode, a.temperature, a.gate_scale,
                          a.gate_offset, wr, wl);
        if (lane < a.K) a.remote_w[o] = f2bf(wr);
        if (lane == 0) a.local_w[((int64_t)b * a.Lq + row) * Hq + hq] = f2bf(wl);
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

size_t route_smem_bytes(int C) {
  return sizeof(float) * (QB * C + NW * QB * CT + QB * NW) + sizeof(int) * QB * 32 + C;
}

}  // namespace

extern "C" int mrsa_route_topk(const void* route_q, const void* landmarks, int lmk_per_qhead,
                               const float* local_lse, const float* bias, const int32_t* drop_mask,
                               const uint8_t* chunk_ok, int64_t window, int64_t q_offset,
                               int32_t* indices, void* scores_out, int scores_dtype,
                               void* remote_w, void* local_w, int weight_mode, float temperature,
                               float gate_scale, float gate_offset, int64_t batch, int64_t q_len,
                               int64_t chunks, int64_t kv_heads, int64_t groups, int64_t head_dim,
                               int64_t topk, mrsa_stream_t stream) {
  if (!route_q || !landmarks || !local_lse || !indices || !scores_out) return MRSA_ERR_NULL;
  if ((remote_w == nullptr) != (local_w == nullptr)) return MRSA_ERR_NULL;
  if (head_dim != D || groups < 1 || groups > NW || kv_heads < 1 || batch < 1 || q_len < 0 ||
      chunks < 1 || chunks > kMaxChunks || topk < 1 || topk > 32 || kv_heads > 65535 ||
      batch > 65535 || q_offset < 0)
    return MRSA_ERR_SHAPE;
  if (scores_dtype != MRSA_BF16 && scores_dtype != MRSA_F32) return MRSA_ERR_ARG;
  if (weight_mode != MRSA_WEIGHTS_AFFINE && weight_mode != MRSA_WEIGHTS_SOFTMAX) return MRSA_ERR_ARG;
  if (!(temperature > 0.f)) return MRSA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(route_q) & 15u) || (reinterpret_cast<uintptr_t>(landmarks) & 15u))
    return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  RouteArgs a;
  a.rq = static_cast<const __nv_bfloat16*>(route_q);
  a.lmk = static_cast<const __nv_bfloat16*>(landmarks);
  a.lmk_g_stride = lmk_per_qhead ? D : 0;
  a.local_lse = local_lse;
  a.bias = bias;
  a.drop = drop_mask;
  a.chunk_ok = chunk_ok;
  a.window = window;
  a.q_offset = q_offset;
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
  const size_t smem = route_smem_bytes(a.C);
  if (cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const int64_t blocks = (q_len + QB - 1) / QB;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(kv_heads),
            static_cast<unsigned>(batch));
  route_kernel<<<grid, NW * 32, smem, static_cast<cudaStream_t>(stream)>>>(a);
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
