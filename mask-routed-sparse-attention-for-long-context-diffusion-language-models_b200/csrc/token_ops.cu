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
// (and V) rows read straight from global memory / L2.  The scores run as
// mma.sync m16n8k16 tiles (16 rows = the group's <= 16 heads, 8 gathered keys
// per tile): tcgen05's smallest tile has 64 rows, of which a single query's
// group fills 7, so the warp-level MMA is the better fit for these shapes.
// The selected-token P.V stays on fp32 FMAs.
#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int D = kHeadDim;
constexpr int TS_THREADS = 128;
constexpr int MAXG = 16;

// ---- m16n8k16 fragments over gathered key rows ------------------------------
// S[heads x keys] = Q[heads x 128] . K[keys x 128]^T as mma.sync m16n8k16
// (bf16 in, fp32 accumulate): 16 A rows = the group's heads (G <= 16, the rest
// zero), 8 keys per n-tile.  The dot product does not depend on the order of
// the 128 dims, so dims are assigned to fragment slots such that lane (r, j)
// = (lane / 4, lane % 4) needs dims [32j, 32j + 32) of its rows in every
// k-step: logical k-index kk of step s is dim 32*((kk % 8) / 2) + 4*s +
// (kk % 2) + 2*(kk / 8).  Each lane then reads one contiguous 64-byte quarter
// of its key row (four 16-byte loads) and one of each of its query rows, and
// the words of those quarters are the b0/b1 (a0/a2, a1/a3) registers of the
// eight k-steps in order.
struct QFrag {
  uint32_t a[8][4];
};

__device__ __forceinline__ void load_qfrag(QFrag& f, const __nv_bfloat16* q_group, int G, int lane) {
  const int r = lane >> 2, j = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = r + 8 * half;
    uint32_t w[16];
    if (row < G) {
      const uint4* p = reinterpret_cast<const uint4*>(q_group + row * D + 32 * j);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 u = __ldg(p + i);
        w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = 0u;
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      f.a[s][half] = w[2 * s];          // a0 (rows 0-7) / a1 (rows 8-15)
      f.a[s][2 + half] = w[2 * s + 1];  // a2 / a3
    }
  }
}

// C[16 heads x 8 keys] of one n-tile whose key row (this lane's key r) is `krow`
// (NULL: a masked key, read as zeros).
__device__ __forceinline__ void mma_keys(float (&c)[4], const QFrag& f, const __nv_bfloat16* krow, int lane) {
  uint32_t w[16];
  if (krow != nullptr) {
    const uint4* p = reinterpret_cast<const uint4*>(krow + 32 * (lane & 3));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = __ldg(p + i);
      w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0u;
  }
  c[0] = c[1] = c[2] = c[3] = 0.f;
#pragma unroll
  for (int s = 0; s < 8; ++s) mma_bf16(c, f.a[s], w[2 * s], w[2 * s + 1]);
}

// grid (Lq, Hkv, B), 4 warps; warp w takes selected chunks w, w+4, ...  Per
// chunk, n-tile nt covers slots 8nt .. 8nt+7; the max over the G head rows is
// reduced across the eight lanes that share a column pair, and lane (r, j)
// keeps the result of n-tile r (mod 8): slots 8r + 2j, 8r + 2j + 1 of each
// 64-slot group, which the warp then writes as 64 contiguous floats.
__global__ void __launch_bounds__(TS_THREADS) token_score_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const int32_t* __restrict__ indices, const uint8_t* __restrict__ key_valid, float* __restrict__ scores,
    float sm_scale, int64_t Lq, int64_t Lk, int Hkv, int G, int K, int S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, j = lane & 3;
  const int64_t l = blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t C = Lk / S;
  const int64_t row = (static_cast<int64_t>(b) * Lq + l) * Hkv + h;   // (b, l, h)
  QFrag f;
  load_qfrag(f, q + (row * G) * D, G, lane);
  const int ntiles = (S + 7) / 8;

  for (int i = warp; i < K; i += TS_THREADS / 32) {
    const int64_t c = indices[row * K + i];
    float* out = scores + (row * K + i) * S;
    const bool chunk_ok = c >= 0 && c < C;
    for (int g0 = 0; g0 < ntiles; g0 += 8) {         // 64-slot groups
      float keep0 = -INFINITY, keep1 = -INFINITY;
#pragma unroll 2
      for (int t = 0; t < 8; ++t) {
        const int nt = g0 + t;
        if (nt >= ntiles) break;                      // warp-uniform
        const int s_key = 8 * nt + r;                 // this lane's key (B column)
        const __nv_bfloat16* krow = nullptr;
        if (chunk_ok && s_key < S) krow = k + ((b * Lk + c * S + s_key) * Hkv + h) * D;
        float acc[4];
        mma_keys(acc, f, krow, lane);
        // max over the head rows r (< G) and r + 8 (< G) of columns 2j, 2j+1
        float m0 = r < G ? acc[0] : -INFINITY, m1 = r < G ? acc[1] : -INFINITY;
        if (r + 8 < G) {
          m0 = fmaxf(m0, acc[2]);
          m1 = fmaxf(m1, acc[3]);
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
          m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
        }
        if (r == t) {
          keep0 = m0;
          keep1 = m1;
        }
      }
      // slots 8*(g0 + r) + 2j, +1; -inf for masked slots
      const int sa = 8 * (g0 + r) + 2 * j;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int sl = sa + e;
        if (sl < S) {
          const bool ok = chunk_ok && sl < S - 1 && (key_valid == nullptr || key_valid[b * Lk + c * S + sl] != 0);
          out[sl] = ok ? (e ? keep1 : keep0) * sm_scale : -INFINITY;
        }
      }
    }
  }
}

// Shared memory of the selected-token kernel (dynamic; tp = topk rounded up
// to a multiple of 4 so every region starts on 16 bytes):
//   prob[G][tp] f32 | tok[tp] int32 | red[4][G][D] f32
__host__ __device__ inline int sta_pad(int topk) { return (topk + 3) & ~3; }
__host__ __device__ inline size_t sta_smem_bytes(int G, int topk) {
  const size_t tp = static_cast<size_t>(sta_pad(topk));
  return static_cast<size_t>(G) * tp * 4 + tp * 4 + static_cast<size_t>(TS_THREADS / 32) * G * D * 4;
}

// grid (Lq, Hkv, B).  Pass 1: the raw scores of the G heads as m16n8k16
// tiles of 8 gathered tokens (warp w takes tiles w, w+4, ...).  Softmax: warp
// per head.  Pass 2: warp per group of eight tokens, lane per 4 dims, fp32
// accumulation of bf16(P) x V; the four warps' partial rows are summed
// through shared memory.
__global__ void __launch_bounds__(TS_THREADS) selected_token_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const int32_t* __restrict__ indices, const uint8_t* __restrict__ valid, __nv_bfloat16* __restrict__ out,
    float sm_scale, int64_t Lq, int64_t Lk, int Hkv, int G, int topk) {
  extern __shared__ __align__(16) float dyn[];
  const int tp = sta_pad(topk);
  float* prob = dyn;                             // prob[g * tp + t]
  int32_t* tok = reinterpret_cast<int32_t*>(prob + static_cast<size_t>(G) * tp);
  float* red = reinterpret_cast<float*>(tok + tp);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t l = blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t qrow = static_cast<int64_t>(b) * Lq + l;                 // (b, l)
  // token list: clamped indices, -1 where not valid
  for (int t = tid; t < topk; t += TS_THREADS) {
    int64_t j = indices[qrow * topk + t];
    j = j < 0 ? 0 : (j > Lk - 1 ? Lk - 1 : j);
    tok[t] = valid[qrow * topk + t] != 0 ? static_cast<int32_t>(j) : -1;
  }
  QFrag f;
  load_qfrag(f, q + ((qrow * Hkv + h) * G) * D, G, lane);
  __syncthreads();

  // pass 1: scores, 8 tokens per n-tile; lane (r, j) gathers token 8nt + r
  // and gets columns 2j, 2j+1 of head rows r and r + 8
  {
    const int r = lane >> 2, j = lane & 3;
    for (int nt = warp; nt * 8 < topk; nt += TS_THREADS / 32) {
      const int tk = 8 * nt + r;
      const int jt = tk < topk ? tok[tk] : -1;
      const __nv_bfloat16* krow = jt >= 0 ? k + ((b * Lk + jt) * Hkv + h) * D : nullptr;
      float acc[4];
      mma_keys(acc, f, krow, lane);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tc = 8 * nt + 2 * j + e;
        if (tc < topk) {
          const bool ok = tok[tc] >= 0;
          if (r < G) prob[static_cast<size_t>(r) * tp + tc] = ok ? acc[e] * sm_scale : -INFINITY;
          if (r + 8 < G) prob[static_cast<size_t>(r + 8) * tp + tc] = ok ? acc[2 + e] * sm_scale : -INFINITY;
        }
      }
    }
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
  // eight tokens per round: their V rows are all requested before any is used
  constexpr int TB = 8;
  for (int t0 = warp * TB; t0 < topk; t0 += TB * (TS_THREADS / 32)) {
    uint2 u[TB];
#pragma unroll
    for (int e = 0; e < TB; ++e) {
      const int t = t0 + e;
      const int32_t j = t < topk ? tok[t] : -1;
      u[e] = j >= 0 ? __ldg(reinterpret_cast<const uint2*>(v + ((b * Lk + j) * Hkv + h) * D) + lane)
                    : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int e = 0; e < TB; ++e) {
      const int t = t0 + e;
      if (t >= topk) break;                   // warp-uniform
      const float2 v01 = unpack_bf16x2(u[e].x), v23 = unpack_bf16x2(u[e].y);
#pragma unroll
      for (int g = 0; g < MAXG; ++g)
        if (g < G) {
          const float p = prob[static_cast<size_t>(g) * tp + t];   // 0 for invalid tokens
          acc[g][0] = fmaf(p, v01.x, acc[g][0]);
          acc[g][1] = fmaf(p, v01.y, acc[g][1]);
          acc[g][2] = fmaf(p, v23.x, acc[g][2]);
          acc[g][3] = fmaf(p, v23.y, acc[g][3]);
        }
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
