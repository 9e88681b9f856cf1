// Token-granular ops off the route layer's live path:
//
//  * candidate token scores (ops/hils_token_score_gqa_tilelang.py:18-116,174):
//    for each query row, KV head and selected chunk c, every slot s of the
//    chunk gets max_g(q_g . k_{c*S+s}) * scale over the G query heads of the
//    group, or -inf when the chunk index is negative, s is the chunk's last
//    (landmark) slot or the key is invalid;
//  * exact selected-token GQA attention (ops/dsa_selected_attention_tilelang.py:
//    33-250,593; torch semantics dream_dllm_hils/dsa_attention.py:498-540):
//    every query row attends its own list of token indices (clamped to the
//    sequence), invalid entries are -inf, the fp32 softmax probabilities are
//    rounded to bf16 before P.V, rows without a valid entry give 0.
//
// Neither reuses a key tile across query rows (each row has its own chunk or
// token list), so both are gathers: one CTA per (query row, KV head), the K
// (and V) rows read straight from global memory / L2, fp32 FMAs against the
// group's query rows held in shared memory.  Their bound is the gather (L2
// bandwidth) and the FMA issue rate, not the tensor cores.
#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int D = kHeadDim;
constexpr int TS_THREADS = 128;
constexpr int MAXG = 16;

// 8 bf16 (one 16-byte load) -> fp32
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// acc[g] += q_g[8p .. 8p+7] . kf, g < G (query rows fp32 in shared memory)
__device__ __forceinline__ void dot8(float (&acc)[MAXG], const float (*qs)[D], int G, int p, const float (&kf)[8]) {
#pragma unroll
  for (int g = 0; g < MAXG; ++g) {
    if (g < G) {
      const float4 q0 = *reinterpret_cast<const float4*>(&qs[g][8 * p]);
      const float4 q1 = *reinterpret_cast<const float4*>(&qs[g][8 * p + 4]);
      float a = acc[g];
      a = fmaf(q0.x, kf[0], a); a = fmaf(q0.y, kf[1], a); a = fmaf(q0.z, kf[2], a); a = fmaf(q0.w, kf[3], a);
      a = fmaf(q1.x, kf[4], a); a = fmaf(q1.y, kf[5], a); a = fmaf(q1.z, kf[6], a); a = fmaf(q1.w, kf[7], a);
      acc[g] = a;
    }
  }
}

__device__ __forceinline__ void load_group_q(float (*qs)[D], const __nv_bfloat16* q, int G, int tid) {
  for (int e = tid; e < G * D / 2; e += TS_THREADS) {
    const float2 v = unpack_bf16x2(reinterpret_cast<const uint32_t*>(q)[e]);
    qs[(2 * e) / D][(2 * e) % D] = v.x;
    qs[(2 * e) / D][(2 * e) % D + 1] = v.y;
  }
}

// grid (Lq, Hkv, B); warp w takes selected chunks w, w+4, ...; lane takes
// slots s0+lane and s0+32+lane of each 64-slot step.
__global__ void __launch_bounds__(TS_THREADS) token_score_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const int32_t* __restrict__ indices, const uint8_t* __restrict__ key_valid, float* __restrict__ scores,
    float sm_scale, int64_t Lq, int64_t Lk, int Hkv, int G, int K, int S) {
  __shared__ __align__(16) float qs[MAXG][D];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t l = blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t C = Lk / S;
  const int64_t row = (static_cast<int64_t>(b) * Lq + l) * Hkv + h;   // (b, l, h)
  load_group_q(qs, q + (row * G) * D, G, tid);
  __syncthreads();

  for (int i = warp; i < K; i += TS_THREADS / 32) {
    const int64_t c = indices[row * K + i];
    float* out = scores + (row * K + i) * S;
    const bool chunk_ok = c >= 0 && c < C;
    for (int s0 = 0; s0 < S; s0 += 64) {
      const int sa = s0 + lane, sb = s0 + 32 + lane;
      const int64_t ja = c * S + sa, jb = c * S + sb;
      const bool oka = chunk_ok && sa < S - 1 && (key_valid == nullptr || key_valid[b * Lk + ja] != 0);
      const bool okb = chunk_ok && sb < S - 1 && (key_valid == nullptr || key_valid[b * Lk + jb] != 0);
      float acca[MAXG], accb[MAXG];
#pragma unroll
      for (int g = 0; g < MAXG; ++g) acca[g] = accb[g] = 0.f;
      if (__any_sync(0xffffffffu, oka || okb)) {
        const uint4* ka = reinterpret_cast<const uint4*>(k + ((b * Lk + (oka ? ja : 0)) * Hkv + h) * D);
        const uint4* kb = reinterpret_cast<const uint4*>(k + ((b * Lk + (okb ? jb : 0)) * Hkv + h) * D);
#pragma unroll 2
        for (int p = 0; p < D / 8; ++p) {
          float fa[8], fb[8];
          const uint4 ua = oka ? __ldg(ka + p) : make_uint4(0, 0, 0, 0);
          const uint4 ub = okb ? __ldg(kb + p) : make_uint4(0, 0, 0, 0);
          unpack8(ua, fa);
          unpack8(ub, fb);
          dot8(acca, qs, G, p, fa);
          dot8(accb, qs, G, p, fb);
        }
      }
      float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
      for (int g = 0; g < MAXG; ++g)
        if (g < G) {
          ma = fmaxf(ma, acca[g]);
          mb = fmaxf(mb, accb[g]);
        }
      if (sa < S) out[sa] = oka ? ma * sm_scale : -INFINITY;
      if (sb < S) out[sb] = okb ? mb * sm_scale : -INFINITY;
    }
  }
}

// Shared memory of the selected-token kernel (dynamic; tp = topk rounded up
// to a multiple of 4 so every region starts on 16 bytes):
//   qs[G][D] f32 | prob[G][tp] f32 | tok[tp] int32 | red[4][G][D] f32
__host__ __device__ inline int sta_pad(int topk) { return (topk + 3) & ~3; }
__host__ __device__ inline size_t sta_smem_bytes(int G, int topk) {
  const size_t tp = static_cast<size_t>(sta_pad(topk));
  return static_cast<size_t>(G) * D * 4 + static_cast<size_t>(G) * tp * 4 + tp * 4 +
         static_cast<size_t>(TS_THREADS / 32) * G * D * 4;
}

// grid (Lq, Hkv, B).  Pass 1: thread per token, raw scores of the G heads.
// Softmax: warp per head.  Pass 2: warp per token residue class, lane per 4
// dims, fp32 accumulation of bf16(P) x V; the four warps' partial rows are
// summed through shared memory.
__global__ void __launch_bounds__(TS_THREADS) selected_token_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const int32_t* __restrict__ indices, const uint8_t* __restrict__ valid, __nv_bfloat16* __restrict__ out,
    float sm_scale, int64_t Lq, int64_t Lk, int Hkv, int G, int topk) {
  extern __shared__ __align__(16) float dyn[];
  float (*qs)[D] = reinterpret_cast<float (*)[D]>(dyn);
  const int tp = sta_pad(topk);
  float* prob = dyn + G * D;                     // prob[g * tp + t]
  int32_t* tok = reinterpret_cast<int32_t*>(prob + static_cast<size_t>(G) * tp);
  float* red = reinterpret_cast<float*>(tok + tp);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t l = blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t qrow = static_cast<int64_t>(b) * Lq + l;                 // (b, l)
  load_group_q(qs, q + ((qrow * Hkv + h) * G) * D, G, tid);
  __syncthreads();

  // pass 1: scores
  for (int t = tid; t < topk; t += TS_THREADS) {
    int64_t j = indices[qrow * topk + t];
    j = j < 0 ? 0 : (j > Lk - 1 ? Lk - 1 : j);
    const bool ok = valid[qrow * topk + t] != 0;
    tok[t] = ok ? static_cast<int32_t>(j) : -1;
    float acc[MAXG];
#pragma unroll
    for (int g = 0; g < MAXG; ++g) acc[g] = 0.f;
    if (ok) {
      const uint4* kr = reinterpret_cast<const uint4*>(k + ((b * Lk + j) * Hkv + h) * D);
#pragma unroll 2
      for (int p = 0; p < D / 8; ++p) {
        float f[8];
        unpack8(__ldg(kr + p), f);
        dot8(acc, qs, G, p, f);
      }
    }
#pragma unroll
    for (int g = 0; g < MAXG; ++g)
      if (g < G) prob[static_cast<size_t>(g) * tp + t] = ok ? acc[g] * sm_scale : -INFINITY;
  }
  __syncthreads();

  // softmax per head; probabilities rounded to bf16 (the P.V operand type)
  for (int g = warp; g < G; g += TS_THREADS / 32) {
    float* pr = prob + static_cast<size_t>(g) * tp;
    float m = -INFINITY;
    for (int t = lane; t < topk; t += 32) m = fmaxf(m, pr[t]);
    m = warp_max(m);
    float sum = 0.f;
    if (m != -INFINITY)
      for (int t = lane; t < topk; t += 32) sum += exp2f((pr[t] - m) * kLog2e);
    sum = warp_sum(sum);
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    for (int t = lane; t < topk; t += 32)
      pr[t] = m == -INFINITY ? 0.f : round_bf16(exp2f((pr[t] - m) * kLog2e) * inv);
  }
  __syncthreads();

  // pass 2: out_g = sum_t P[g][t] V[tok t], lane owns dims 4*lane .. 4*lane+3
  float acc[MAXG][4];
#pragma unroll
  for (int g = 0; g < MAXG; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  for (int t = warp; t < topk; t += TS_THREADS / 32) {
    const int32_t j = tok[t];
    if (j < 0) continue;   // warp-uniform
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(v + ((b * Lk + j) * Hkv + h) * D) + lane);
    const float2 v01 = unpack_bf16x2(u.x), v23 = unpack_bf16x2(u.y);
#pragma unroll
    for (int g = 0; g < MAXG; ++g)
      if (g < G) {
        const float p = prob[static_cast<size_t>(g) * tp + t];
        acc[g][0] = fmaf(p, v01.x, acc[g][0]);
        acc[g][1] = fmaf(p, v01.y, acc[g][1]);
        acc[g][2] = fmaf(p, v23.x, acc[g][2]);
        acc[g][3] = fmaf(p, v23.y, acc[g][3]);
      }
  }
#pragma unroll
  for (int g = 0; g < MAXG; ++g)
    if (g < G)
      *reinterpret_cast<float4*>(&red[(static_cast<size_t>(warp) * G + g) * D + 4 * lane]) =
          make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  __syncthreads();
  __nv_bfloat16* orow = out + ((qrow * Hkv + h) * G) * D;
  for (int e = tid; e < G * D / 2; e += TS_THREADS) {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int w = 0; w < TS_THREADS / 32; ++w) {
      s0 += red[static_cast<size_t>(w) * G * D + 2 * e];
      s1 += red[static_cast<size_t>(w) * G * D + 2 * e + 1];
    }
    reinterpret_cast<uint32_t*>(orow)[e] = pack_bf16x2(s0, s1);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int mrsa_candidate_token_scores(const void* q, const void* k, const int32_t* indices,
                                           const uint8_t* key_valid, float* scores, float sm_scale,
                                           int64_t batch, int64_t q_len, int64_t kv_len, int64_t q_heads,
                                           int64_t kv_heads, int64_t head_dim, int64_t selected, int64_t chunk,
                                           mrsa_stream_t stream) {
  if (!q || !k || !indices || !scores) return MRSA_ERR_NULL;
  if (head_dim != D || kv_heads < 1 || q_heads % kv_heads || q_heads / kv_heads > MAXG || q_heads < kv_heads ||
      batch < 1 || batch > 65535 || kv_heads > 65535 || q_len < 0 || q_len > 0x7fffffffLL || kv_len < 1 ||
      selected < 0 || selected > 0x7fffffffLL || chunk < 16 || chunk > 0x7fffffffLL || kv_len % chunk)
    return MRSA_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k)) return MRSA_ERR_ALIGN;
  if (q_len == 0 || selected == 0) return MRSA_OK;
  dim3 grid(static_cast<unsigned>(q_len), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
  token_score_kernel<<<grid, TS_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), indices, key_valid, scores,
      sm_scale, q_len, kv_len, static_cast<int>(kv_heads), static_cast<int>(q_heads / kv_heads),
      static_cast<int>(selected), static_cast<int>(chunk));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

extern "C" size_t mrsa_selected_token_attention_smem(int64_t groups, int64_t topk) {
  if (groups < 1 || groups > MAXG || topk < 1 || topk > (1 << 20)) return 0;
  return sta_smem_bytes(static_cast<int>(groups), static_cast<int>(topk));
}

extern "C" int mrsa_selected_token_attention(const void* q, const void* k, const void* v, const int32_t* indices,
                                             const uint8_t* valid, void* out, float sm_scale, int64_t batch,
                                             int64_t q_len, int64_t kv_len, int64_t q_heads, int64_t kv_heads,
                                             int64_t head_dim, int64_t topk, mrsa_stream_t stream) {
  if (!q || !k || !v || !indices || !valid || !out) return MRSA_ERR_NULL;
  if (head_dim != D || kv_heads < 1 || q_heads % kv_heads || q_heads / kv_heads > MAXG || q_heads < kv_heads ||
      batch < 1 || batch > 65535 || kv_heads > 65535 || q_len < 0 || q_len > 0x7fffffffLL || kv_len < 1 ||
      kv_len > 0x7fffffffLL || topk < 0 || topk > (1 << 20))
    return MRSA_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  const int G = static_cast<int>(q_heads / kv_heads);
  if (topk == 0) {
    // no selected token: every row is 0 (the reference's nan_to_num of an empty softmax)
    if (cudaMemsetAsync(out, 0, static_cast<size_t>(batch * q_len * q_heads * D) * 2,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
      return MRSA_ERR_LAUNCH;
    return MRSA_OK;
  }
  const size_t smem = sta_smem_bytes(G, static_cast<int>(topk));
  if (smem > 232448) return MRSA_ERR_SHAPE;
  if (cudaFuncSetAttribute(selected_token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  dim3 grid(static_cast<unsigned>(q_len), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
  selected_token_kernel<<<grid, TS_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), indices, valid, static_cast<__nv_bfloat16*>(out), sm_scale, q_len,
      kv_len, static_cast<int>(kv_heads), G, static_cast<int>(topk));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
