// Backward of the routing-side ops of the route layer: the landmark pool, the
// route weights, the gathered routing scores and the output fusion.  These are
// small, memory-bound steps next to the selected-attention backward; they run
// on CUDA cores with fp32 math.
//
//  * pool_bwd_kernel -- ops/chunk_attn_pool_gqa_tilelang.py:183-325
//    (_pool_gqa_bwd): one CTA per (chunk, KV head) recomputes the pool
//    probabilities p (softmax over the chunk's valid non-landmark keys of
//    mu_q . k * scale) and the entropy H, then with pb = bf16(p),
//      dP    = grad_lmk . K^T,   delta = sum_s pb dP
//      dL    = bf16(scale * pb * ((dP - delta) - grad_H * (ln pb + H)))   (0 where pb = 0)
//      d_mu  = bf16(dL . K),     d_k = bf16(dL^T . mu + pb^T . grad_lmk)
//  * route_weights_bwd_kernel -- the softmax kernel's backward
//    (ops/hils_bidir_route_weights_tilelang.py:97-166) and the autograd of the
//    affine-gate branch of dream_dllm_hils/attention.py:126-227, one warp per
//    (query, head) row with lane k on slot k; prior-bias gradients are summed
//    with atomics (as the reference's kernel does), the gate's scale and offset
//    gradients per CTA and then with one atomic each.
//  * scores_dq_kernel / scores_dlmk_kernel -- the backward of the gathered raw
//    scores s[l,hq,k] = q[l,hq] . lmk[c_k,hq] * scale
//    (ops/topk_head_softmax.py:1071-1122): dq gathers the selected landmarks,
//    d_lmk walks the inverted chunk -> (query, slot) index.
//  * fuse_bwd_kernel -- ops/hils_bidir_output_fusion_tilelang.py:38-99.
#include <cstdio>

#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int PS = kChunk;       // keys per chunk
constexpr int PD = kHeadDim;
constexpr int PG = 16;           // most query heads per KV head in the pool

struct PoolSmem {
  float k[PS][PD + 1];
  float mu[PG][PD];
  float gk[PG][PD];
  float p[PG][PS];               // probabilities, then bf16-rounded
  float dp[PG][PS];              // dP, then dL
  float gb[PG];
  uint64_t ok;
};

__global__ void __launch_bounds__(256) pool_bwd_kernel(const __nv_bfloat16* __restrict__ mu_q,
                                                       const __nv_bfloat16* __restrict__ k,
                                                       const uint8_t* __restrict__ key_valid,
                                                       const __nv_bfloat16* __restrict__ grad_lmk,
                                                       const float* __restrict__ grad_ent, __nv_bfloat16* __restrict__ d_mu,
                                                       __nv_bfloat16* __restrict__ d_k, float scale, int C, int Hkv,
                                                       int G) {
  extern __shared__ __align__(16) unsigned char raw[];
  PoolSmem& sm = *reinterpret_cast<PoolSmem*>(raw);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row0 = static_cast<int64_t>(b) * C * PS + static_cast<int64_t>(c) * PS;   // first key row
  const int64_t grp = ((static_cast<int64_t>(b) * C + c) * Hkv + h) * G;                     // (b,c,h,0)
  for (int e = tid; e < PS * PD; e += 256) {
    const int s = e / PD, d = e % PD;
    sm.k[s][d] = bf2f(k[((row0 + s) * Hkv + h) * PD + d]);
  }
  for (int e = tid; e < G * PD; e += 256) {
    const int g = e / PD, d = e % PD;
    sm.mu[g][d] = bf2f(mu_q[(grp + g) * PD + d]);
    sm.gk[g][d] = grad_lmk ? bf2f(grad_lmk[(grp + g) * PD + d]) : 0.f;
  }
  if (tid < G) sm.gb[tid] = grad_ent ? grad_ent[grp + tid] : 0.f;
  if (warp == 0) {
    const bool v0 = lane < PS - 1 && (key_valid == nullptr || key_valid[row0 + lane] != 0);
    const bool v1 = lane + 32 < PS - 1 && (key_valid == nullptr || key_valid[row0 + 32 + lane] != 0);
    const uint32_t m0 = __ballot_sync(0xffffffffu, v0), m1 = __ballot_sync(0xffffffffu, v1);
    if (lane == 0) sm.ok = static_cast<uint64_t>(m0) | (static_cast<uint64_t>(m1) << 32);
  }
  __syncthreads();
  const uint64_t ok = sm.ok;
  // logits and dP (one (g, s) pair per thread and step)
  for (int e = tid; e < G * PS; e += 256) {
    const int g = e / PS, s = e % PS;
    float x = 0.f, y = 0.f;
#pragma unroll 8
    for (int d = 0; d < PD; ++d) {
      x = fmaf(sm.mu[g][d], sm.k[s][d], x);
      y = fmaf(sm.gk[g][d], sm.k[s][d], y);
    }
    sm.p[g][s] = ((ok >> s) & 1ull) ? x * scale : -INFINITY;
    sm.dp[g][s] = y;
  }
  __syncthreads();
  // softmax, entropy, delta: one warp per head, keys s = lane and lane + 32
  for (int g = warp; g < G; g += 8) {
    const float x0 = sm.p[g][lane], x1 = sm.p[g][lane + 32];
    const float mx = warp_max(fmaxf(x0, x1));
    float p0 = 0.f, p1 = 0.f;
    if (mx != -INFINITY) {
      const float e0 = x0 == -INFINITY ? 0.f : expf(x0 - mx), e1 = x1 == -INFINITY ? 0.f : expf(x1 - mx);
      const float inv = 1.f / warp_sum(e0 + e1);
      p0 = e0 * inv;
      p1 = e1 * inv;
    }
    const float ent = -warp_sum((p0 > 0.f ? p0 * logf(p0) : 0.f) + (p1 > 0.f ? p1 * logf(p1) : 0.f));
    const float b0 = round_bf16(p0), b1 = round_bf16(p1);
    const float dl = warp_sum(b0 * sm.dp[g][lane] + b1 * sm.dp[g][lane + 32]);
    const float gbv = sm.gb[g];
    const float l0 = b0 > 0.f ? b0 * ((sm.dp[g][lane] - dl) - gbv * (logf(b0) + ent)) : 0.f;
    const float l1 = b1 > 0.f ? b1 * ((sm.dp[g][lane + 32] - dl) - gbv * (logf(b1) + ent)) : 0.f;
    __syncwarp();
    sm.p[g][lane] = b0;
    sm.p[g][lane + 32] = b1;
    sm.dp[g][lane] = round_bf16(l0 * scale);
    sm.dp[g][lane + 32] = round_bf16(l1 * scale);
  }
  __syncthreads();
  // d_mu[g, d] = bf16(sum_s dL[g, s] K[s, d])
  for (int e = tid; e < G * PD; e += 256) {
    const int g = e / PD, d = e % PD;
    float acc = 0.f;
#pragma unroll 8
    for (int s = 0; s < PS; ++s) acc = fmaf(sm.dp[g][s], sm.k[s][d], acc);
    d_mu[(grp + g) * PD + d] = f2bf(acc);
  }
  // d_k[s, d] = bf16(sum_g dL[g, s] mu[g, d] + pb[g, s] grad_lmk[g, d])
  for (int e = tid; e < PS * PD; e += 256) {
    const int s = e / PD, d = e % PD;
    float acc = 0.f;
    for (int g = 0; g < G; ++g) acc = fmaf(sm.dp[g][s], sm.mu[g][d], fmaf(sm.p[g][s], sm.gk[g][d], acc));
    d_k[((row0 + s) * Hkv + h) * PD + d] = f2bf(acc);
  }
}

// ------------------------------------------------------------ route weights
// One warp per row (b, l, hq), lane k on slot k (K <= 32).
__global__ void __launch_bounds__(256) route_weights_bwd_kernel(
    const __nv_bfloat16* __restrict__ scores, const int32_t* __restrict__ idx, const float* __restrict__ prior,
    const float* __restrict__ local_lse, const __nv_bfloat16* __restrict__ g_remote,
    const __nv_bfloat16* __restrict__ g_local, float* __restrict__ d_scores, float* __restrict__ d_prior,
    float* __restrict__ d_local, float* __restrict__ d_gate, int64_t rows, int64_t seq_len, int Hkv, int G, int C,
    int K, int mode, float temp, float gscale, float goff) {
  __shared__ float red[2][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  const int Hq = Hkv * G;
  float dsc = 0.f, doff = 0.f;
  if (row < rows) {
    const int hq = static_cast<int>(row % Hq);
    const int64_t bl = row / Hq, b = bl / seq_len;
    const int h = hq / G, g = hq % G;
    const bool live = lane < K;
    const int c = live ? idx[(bl * Hkv + h) * K + lane] : -1;
    const bool valid = live && c >= 0 && c < C;
    const float inv_t = 1.f / temp;
    const float gr = live ? bf2f(g_remote[row * K + lane]) : 0.f;
    const float gl = bf2f(g_local[row]);
    const float loc = local_lse[row];
    const float rt = valid ? (bf2f(scores[row * K + lane]) + prior[((b * C + c) * Hkv + h) * G + g]) * inv_t : -INFINITY;
    float dz = 0.f, dlt = 0.f;
    if (mode == MRSA_WEIGHTS_SOFTMAX) {
      // probs over [r / T, (local - offset) / T]
      const float lt = (loc - goff) * inv_t;
      const float m = fmaxf(warp_max(rt), lt);
      if (m != -INFINITY) {
        const float e = rt == -INFINITY ? 0.f : expf(rt - m), el = lt == -INFINITY ? 0.f : expf(lt - m);
        const float inv = 1.f / (warp_sum(e) + el);
        const float p = e * inv, pl = el * inv;
        const float delta = warp_sum(p * gr) + pl * gl;
        dz = p * (gr - delta);
        dlt = pl * (gl - delta);
        doff = -dlt * inv_t;
      }
    } else {
      // affine gate: m = sigmoid(scale * (lse(r / T) - local / T) + offset)
      const float lt = loc * inv_t;
      const float mr = warp_max(rt);
      if (!(mr == -INFINITY && lt == -INFINITY)) {
        float ri = 0.f, lse = -INFINITY;
        if (mr != -INFINITY) {
          const float e = rt == -INFINITY ? 0.f : expf(rt - mr);
          const float sum = warp_sum(e);
          ri = e / sum;
          lse = mr + logf(sum);
        }
        const float gate = gscale * (lse - lt) + goff;
        const float msig = 1.f / (1.f + expf(-gate));
        const float dm = warp_sum(gr * ri) - gl;
        const float dri = gr * msig;
        const float dot = warp_sum(ri * dri);
        const float dgate = dm * msig * (1.f - msig);
        dz = ri * (dri - dot) + ri * dgate * gscale;
        dlt = -dgate * gscale;
        if (lse != -INFINITY && lt != -INFINITY) dsc = dgate * (lse - lt);
        doff = dgate;
      }
    }
    const float ds = valid ? dz * inv_t : 0.f;
    if (live) d_scores[row * K + lane] = ds;
    if (valid && ds != 0.f) atomicAdd(&d_prior[((b * C + c) * Hkv + h) * G + g], ds);
    if (lane == 0) d_local[row] = dlt * inv_t;
  }
  if (lane == 0) {
    red[0][warp] = dsc;
    red[1][warp] = doff;
  }
  __syncthreads();
  if (threadIdx.x < 2) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[threadIdx.x][w];
    if (t != 0.f) atomicAdd(&d_gate[threadIdx.x], t);
  }
}

// ------------------------------------------------------------ routing scores
// d_q[l, hq, :] = scale * sum_k g[l, hq, k] * lmk[c_k, hq, :]; one warp per row, 4 dims per lane.
__global__ void __launch_bounds__(256) scores_dq_kernel(const __nv_bfloat16* __restrict__ lmk,
                                                        const int32_t* __restrict__ idx,
                                                        const __nv_bfloat16* __restrict__ grad, float* __restrict__ dq,
                                                        int64_t rows, int64_t seq_len, int Hkv, int G, int C, int K,
                                                        float scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (row >= rows) return;
  const int Hq = Hkv * G;
  const int hq = static_cast<int>(row % Hq);
  const int64_t bl = row / Hq, b = bl / seq_len;
  const int h = hq / G, g = hq % G;
  const int c_l = lane < K ? idx[(bl * Hkv + h) * K + lane] : -1;
  const float g_l = lane < K ? bf2f(grad[row * K + lane]) * scale : 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < K; ++k) {
    const int c = __shfl_sync(0xffffffffu, c_l, k);
    const float gk = __shfl_sync(0xffffffffu, g_l, k);
    if (c < 0 || c >= C || gk == 0.f) continue;
    const uint2 raw = *reinterpret_cast<const uint2*>(lmk + (((b * C + c) * Hkv + h) * G + g) * PD + 4 * lane);
    const float2 a0 = unpack_bf16x2(raw.x), a1 = unpack_bf16x2(raw.y);
    acc[0] = fmaf(gk, a0.x, acc[0]);
    acc[1] = fmaf(gk, a0.y, acc[1]);
    acc[2] = fmaf(gk, a1.x, acc[2]);
    acc[3] = fmaf(gk, a1.y, acc[3]);
  }
  *reinterpret_cast<float4*>(dq + row * PD + 4 * lane) = make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// d_lmk[c, hq, :] = scale * sum over the (l, k) that selected c of g[l, hq, k] * q[l, hq, :];
// one CTA per (chunk, KV head, batch): its 8 warps take every 8th pair, lane =
// 4 dims, the G <= 8 heads in registers; the warps' sums meet in shared memory.
constexpr int SG = 8;

__global__ void __launch_bounds__(256) scores_dlmk_kernel(const __nv_bfloat16* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ grad,
                                                          const int32_t* __restrict__ cnt,
                                                          const int32_t* __restrict__ off,
                                                          const int32_t* __restrict__ pairs, float* __restrict__ dlmk,
                                                          int64_t seq_len, int Hkv, int G, int C, int K, float scale) {
  __shared__ float red[8][SG][PD];
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hq = Hkv * G;
  const int seg = (b * Hkv + h) * C + c;
  const int n = cnt[seg], o = off[seg];
  float acc[SG][4];
#pragma unroll
  for (int g = 0; g < SG; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  for (int i = warp; i < n; i += 8) {
    const int pr = pairs[o + i];
    const int64_t l = pr >> 5;
    const int slot = pr & 31;
    const int64_t base = (static_cast<int64_t>(b) * seq_len + l) * Hq + h * G;
    const float gl = lane < G ? bf2f(grad[(base + lane) * K + slot]) : 0.f;
    uint2 raw[SG];
#pragma unroll
    for (int g = 0; g < SG; ++g)
      raw[g] = g < G ? *reinterpret_cast<const uint2*>(q + (base + g) * PD + 4 * lane) : make_uint2(0u, 0u);
#pragma unroll
    for (int g = 0; g < SG; ++g) {
      const float gg = __shfl_sync(0xffffffffu, gl, g);
      const float2 a0 = unpack_bf16x2(raw[g].x), a1 = unpack_bf16x2(raw[g].y);
      acc[g][0] = fmaf(gg, a0.x, acc[g][0]);
      acc[g][1] = fmaf(gg, a0.y, acc[g][1]);
      acc[g][2] = fmaf(gg, a1.x, acc[g][2]);
      acc[g][3] = fmaf(gg, a1.y, acc[g][3]);
    }
  }
#pragma unroll
  for (int g = 0; g < SG; ++g)
    *reinterpret_cast<float4*>(&red[warp][g][4 * lane]) = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  __syncthreads();
  const int64_t out0 = ((static_cast<int64_t>(b) * C + c) * Hkv + h) * G;
  for (int e = threadIdx.x; e < G * PD; e += 256) {
    const int g = e / PD, d = e % PD;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][g][d];
    dlmk[(out0 + g) * PD + d] = t * scale;
  }
}

// ------------------------------------------------------------ output fusion
__global__ void __launch_bounds__(256) fuse_bwd_kernel(const __nv_bfloat16* __restrict__ local,
                                                       const __nv_bfloat16* __restrict__ local_w,
                                                       const __nv_bfloat16* __restrict__ grad,
                                                       __nv_bfloat16* __restrict__ d_remote,
                                                       __nv_bfloat16* __restrict__ d_local,
                                                       __nv_bfloat16* __restrict__ d_w, int64_t rows, int dim) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (row >= rows) return;
  const float w = bf2f(local_w[row]);
  float dot = 0.f;
  for (int d = lane; d < dim; d += 32) {
    const int64_t e = row * dim + d;
    const float gv = bf2f(grad[e]);
    d_remote[e] = f2bf(gv);
    d_local[e] = f2bf(gv * w);
    dot = fmaf(gv, bf2f(local[e]), dot);
  }
  dot = warp_sum(dot);
  if (lane == 0) d_w[row] = f2bf(dot);
}

}  // namespace

extern "C" int mrsa_chunk_pool_backward(const void* mu_q, const void* k, const uint8_t* key_valid,
                                        const void* grad_landmarks, const float* grad_entropy, void* d_mu, void* d_k,
                                        float sm_scale, int64_t batch, int64_t chunks, int64_t kv_heads,
                                        int64_t groups, int64_t head_dim, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(mu_q);
  if (!mu_q || !k || !d_mu || !d_k) return MRSA_ERR_NULL;
  if (head_dim != PD || batch < 1 || chunks < 0 || kv_heads < 1 || groups < 1 || groups > PG ||
      batch > 65535 || kv_heads > 65535 || chunks > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if (chunks == 0) return MRSA_OK;
  const size_t smem = sizeof(PoolSmem);
  (void)cudaGetLastError();
  if (const cudaError_t e = cudaFuncSetAttribute(pool_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
      e != cudaSuccess) {
    note_cuda_error(e, "mrsa_chunk_pool_backward: shared-memory opt-in");
    return MRSA_ERR_LAUNCH;
  }
  pool_bwd_kernel<<<dim3(static_cast<unsigned>(chunks), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch)),
                    256, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(mu_q), static_cast<const __nv_bfloat16*>(k), key_valid,
      static_cast<const __nv_bfloat16*>(grad_landmarks), grad_entropy, static_cast<__nv_bfloat16*>(d_mu),
      static_cast<__nv_bfloat16*>(d_k), sm_scale, static_cast<int>(chunks), static_cast<int>(kv_heads),
      static_cast<int>(groups));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" int mrsa_route_weights_backward(const void* scores, const int32_t* indices, const float* prior,
                                           const float* local_lse, const void* grad_remote, const void* grad_local,
                                           float* d_scores, float* d_prior, float* d_local_lse, float* d_gate,
                                           int weight_mode, float temperature, float gate_scale, float gate_offset,
                                           int64_t batch, int64_t seq_len, int64_t chunks, int64_t kv_heads,
                                           int64_t groups, int64_t topk, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(scores);
  if (!scores || !indices || !prior || !local_lse || !grad_remote || !grad_local || !d_scores || !d_prior ||
      !d_local_lse || !d_gate)
    return MRSA_ERR_NULL;
  if (batch < 1 || seq_len < 0 || chunks < 1 || kv_heads < 1 || groups < 1 || topk < 1 || topk > 32)
    return MRSA_ERR_SHAPE;
  if (weight_mode != MRSA_WEIGHTS_AFFINE && weight_mode != MRSA_WEIGHTS_SOFTMAX) return MRSA_ERR_ARG;
  if (!(temperature > 0.f)) return MRSA_ERR_ARG;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  if (cudaMemsetAsync(d_prior, 0, batch * chunks * kv_heads * groups * sizeof(float), s) != cudaSuccess ||
      cudaMemsetAsync(d_gate, 0, 2 * sizeof(float), s) != cudaSuccess) {
    note_cuda_error(cudaGetLastError(), "mrsa_route_weights_backward: clearing the sums");
    return MRSA_ERR_LAUNCH;
  }
  const int64_t rows = batch * seq_len * kv_heads * groups;
  if (rows == 0) return MRSA_OK;
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  route_weights_bwd_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(scores), indices, prior, local_lse,
      static_cast<const __nv_bfloat16*>(grad_remote), static_cast<const __nv_bfloat16*>(grad_local), d_scores, d_prior,
      d_local_lse, d_gate, rows, seq_len, static_cast<int>(kv_heads), static_cast<int>(groups),
      static_cast<int>(chunks), static_cast<int>(topk), weight_mode, temperature, gate_scale, gate_offset);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" size_t mrsa_route_scores_backward_workspace(int64_t batch, int64_t q_len, int64_t chunks,
                                                       int64_t kv_heads, int64_t topk) {
  if (batch < 1 || q_len < 0 || chunks < 1 || kv_heads < 1 || topk < 1) return 0;
  return chunk_index_bytes(batch, q_len, kv_heads, topk, chunks);
}

extern "C" int mrsa_route_scores_backward(const void* q, const void* landmarks, const int32_t* indices,
                                          const void* grad_scores, float* d_q, float* d_landmarks, float sm_scale,
                                          int64_t batch, int64_t q_len, int64_t chunks, int64_t kv_heads,
                                          int64_t groups, int64_t head_dim, int64_t topk, void* workspace,
                                          size_t ws_bytes, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(q);
  if (!q || !landmarks || !indices || !grad_scores || !d_q || !d_landmarks) return MRSA_ERR_NULL;
  if (head_dim != PD || batch < 1 || q_len < 0 || chunks < 1 || kv_heads < 1 || groups < 1 || groups > SG ||
      topk < 1 || topk > 32 || batch > 65535 || kv_heads > 65535 || chunks > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(landmarks) | reinterpret_cast<uintptr_t>(d_q) |
       reinterpret_cast<uintptr_t>(workspace)) & 15u)
    return MRSA_ERR_ALIGN;
  const size_t need = mrsa_route_scores_backward_workspace(batch, q_len, chunks, kv_heads, topk);
  if (workspace == nullptr || ws_bytes < need) return MRSA_ERR_WORKSPACE;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  (void)cudaGetLastError();
  const int hkv = static_cast<int>(kv_heads), g = static_cast<int>(groups), c = static_cast<int>(chunks),
            kk = static_cast<int>(topk);
  ChunkIndex ix;
  if (const int rc = build_chunk_index(indices, batch, q_len, hkv, kk, c, workspace, s, &ix); rc != MRSA_OK) return rc;
  const int64_t rows = batch * q_len * kv_heads * groups;
  if (rows > 0) {
    scores_dq_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(landmarks), indices, static_cast<const __nv_bfloat16*>(grad_scores), d_q,
        rows, q_len, hkv, g, c, kk, sm_scale);
    MRSA_CHECK_LAUNCH();
  }
  scores_dlmk_kernel<<<dim3(static_cast<unsigned>(chunks), static_cast<unsigned>(kv_heads),
                            static_cast<unsigned>(batch)),
                       256, 0, s>>>(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(grad_scores),
                                   ix.cnt, ix.off, ix.pairs, d_landmarks, q_len, hkv, g, c, kk, sm_scale);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" int mrsa_fuse_outputs_backward(const void* local, const void* local_w, const void* grad_out,
                                          void* d_remote, void* d_local, void* d_local_w, int64_t rows,
                                          int64_t head_dim, mrsa_stream_t stream) {
  mrsa::DeviceScope device_scope(grad_out);
  if (!local || !local_w || !grad_out || !d_remote || !d_local || !d_local_w) return MRSA_ERR_NULL;
  if (rows < 0 || head_dim < 1 || head_dim > 256) return MRSA_ERR_SHAPE;
  if (rows == 0) return MRSA_OK;
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  (void)cudaGetLastError();
  fuse_bwd_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(local), static_cast<const __nv_bfloat16*>(local_w),
      static_cast<const __nv_bfloat16*>(grad_out), static_cast<__nv_bfloat16*>(d_remote),
      static_cast<__nv_bfloat16*>(d_local), static_cast<__nv_bfloat16*>(d_local_w), rows, static_cast<int>(head_dim));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
