// Landmark attention pool + entropy prior, one CTA per (chunk, kv head).
// Semantics of _compact_pool_torch (ops/chunk_attn_pool_gqa_tilelang.py:17-37):
// per query head g of the group, p = softmax_s(mu_g . k_s * scale) over the
// valid non-landmark slots s < 63, lmk = sum_s p_s k_s (fp32 -> bf16),
// entropy = -sum p ln p; a chunk without such a slot yields zeros.
// The work is tiny (G x 64 x 128 MACs twice per CTA) and bound by reading K,
// so it is plain FMA code over a bank-conflict-free shared tile.
#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int NT = 256;
constexpr int KSTRIDE = kHeadDim / 2 + 1;   // bf16x2 words per padded K row

__global__ void __launch_bounds__(NT) pool_kernel(
    const __nv_bfloat16* __restrict__ mu, int64_t mu_sb, int64_t mu_sc,
    const __nv_bfloat16* __restrict__ k, const uint8_t* __restrict__ key_valid, float sm_scale,
    const float* __restrict__ bias_scale, __nv_bfloat16* __restrict__ lmk,
    float* __restrict__ entropy, float* __restrict__ prior, uint8_t* __restrict__ chunk_ok,
    int C, int Hkv, int G) {
  constexpr int D = kHeadDim, S = kChunk;
  __shared__ uint32_t ks[S * KSTRIDE];       // K chunk, bf16x2 words, padded rows
  __shared__ float mus[8][D];
  __shared__ float logit[8][S];
  __shared__ int valid_s[S];
  __shared__ int any_valid;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t L = static_cast<int64_t>(C) * S;

  if (tid == 0) any_valid = 0;
  __syncthreads();
  if (tid < S) {
    const int ok = (tid < S - 1) && (key_valid == nullptr || key_valid[b * L + c * S + tid] != 0);
    valid_s[tid] = ok;
    if (ok) atomicOr(&any_valid, 1);
  }
  // K rows of this chunk/head: 64 x 128 bf16 -> padded smem
  const __nv_bfloat16* kbase = k + ((static_cast<int64_t>(b) * L + c * S) * Hkv + h) * D;
  for (int e = tid; e < S * (D / 8); e += NT) {
    const int s = e >> 4, p = e & 15;
    uint4 v = *reinterpret_cast<const uint4*>(kbase + static_cast<int64_t>(s) * Hkv * D + p * 8);
    uint32_t* dst = ks + s * KSTRIDE + p * 4;
    dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
  }
  const __nv_bfloat16* mbase = mu + b * mu_sb + c * mu_sc + static_cast<int64_t>(h) * G * D;
  for (int e = tid; e < G * D; e += NT) mus[e / D][e % D] = bf2f(mbase[e]);
  __syncthreads();

  const bool chunk_valid = any_valid != 0;
  if (chunk_ok != nullptr && h == 0 && tid == 0) chunk_ok[static_cast<int64_t>(b) * C + c] = chunk_valid;

  // logits: thread -> slot s = tid & 63, heads g = tid>>6, +4
  {
    const int s = tid & 63;
    for (int g = tid >> 6; g < G; g += NT / S) {
      float acc = 0.f;
      const uint32_t* kr = ks + s * KSTRIDE;
#pragma unroll 8
      for (int w = 0; w < D / 2; ++w) {
        const float2 kv = unpack_bf16x2(kr[w]);
        acc = fmaf(mus[g][2 * w], kv.x, acc);
        acc = fmaf(mus[g][2 * w + 1], kv.y, acc);
      }
      logit[g][s] = valid_s[s] ? acc * sm_scale : -INFINITY;
    }
  }
  __syncthreads();

  // softmax + entropy per head: one warp per head, two slots per lane
  for (int g = warp; g < G; g += NT / 32) {
    float l0 = logit[g][lane], l1 = logit[g][lane + 32];
    float m = warp_max(fmaxf(l0, l1));
    float e0 = valid_s[lane] ? expf(l0 - m) : 0.f;
    float e1 = valid_s[lane + 32] ? expf(l1 - m) : 0.f;
    float sum = warp_sum(e0 + e1);
    float p0 = chunk_valid ? e0 / sum : 0.f, p1 = chunk_valid ? e1 / sum : 0.f;
    float ent = 0.f;
    if (p0 > 0.f) ent -= p0 * logf(fmaxf(p0, 1e-30f));
    if (p1 > 0.f) ent -= p1 * logf(fmaxf(p1, 1e-30f));
    ent = warp_sum(ent);
    logit[g][lane] = p0;
    logit[g][lane + 32] = p1;
    if (lane == 0) {
      const int64_t o = ((static_cast<int64_t>(b) * C + c) * Hkv + h) * G + g;
      entropy[o] = ent;
      if (prior != nullptr) prior[o] = ent * (bias_scale ? bias_scale[h * G + g] : 1.0f);
    }
  }
  __syncthreads();

  // pooled keys: thread -> (g, dim pair)
  __nv_bfloat16* obase = lmk + ((static_cast<int64_t>(b) * C + c) * Hkv + h) * G * D;
  for (int e = tid; e < G * (D / 2); e += NT) {
    const int g = e / (D / 2), w = e % (D / 2);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
    for (int s = 0; s < S; ++s) {
      const float p = logit[g][s];
      const float2 kv = unpack_bf16x2(ks[s * KSTRIDE + w]);
      a0 = fmaf(p, kv.x, a0);
      a1 = fmaf(p, kv.y, a1);
    }
    reinterpret_cast<uint32_t*>(obase + g * D)[w] = pack_bf16x2(a0, a1);
  }
}

}  // namespace

extern "C" int mrsa_chunk_pool(const void* mu_q, int64_t mu_stride_b, int64_t mu_stride_c,
                               const void* k, const uint8_t* key_valid, float sm_scale,
                               const float* bias_scale, void* landmarks, float* entropy,
                               float* prior, uint8_t* chunk_ok, int64_t batch, int64_t chunks,
                               int64_t kv_heads, int64_t groups, int64_t head_dim,
                               mrsa_stream_t stream) {
  if (!mu_q || !k || !landmarks || !entropy) return MRSA_ERR_NULL;
  if (head_dim != kHeadDim || groups < 1 || groups > 8 || kv_heads < 1 || batch < 1 ||
      chunks < 0 || kv_heads > 65535 || batch > 65535 || chunks > 0x7fffffffLL)
    return MRSA_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(k) & 15u) || (reinterpret_cast<uintptr_t>(landmarks) & 3u))
    return MRSA_ERR_ALIGN;
  if (chunks == 0) return MRSA_OK;
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(kv_heads),
            static_cast<unsigned>(batch));
  pool_kernel<<<grid, NT, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(mu_q), mu_stride_b, mu_stride_c,
      static_cast<const __nv_bfloat16*>(k), key_valid, sm_scale, bias_scale,
      static_cast<__nv_bfloat16*>(landmarks), entropy, prior, chunk_ok, static_cast<int>(chunks),
      static_cast<int>(kv_heads), static_cast<int>(groups));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
