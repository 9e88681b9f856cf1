// Bidirectional banded GQA attention with natural-log LSE (local branch of the
// route layer, window W+63 with landmark/invalid K,V zeroed; SWA layers,
// window 1280).  Semantics of dream_dllm_hils/local_attention.py:35-107:
// zeroed keys keep logit 0 in the softmax, keys with |i-j| > window are out.
// Tile: 64 query rows of one query head per CTA (4 warps x 16 rows), 64-key
// tiles streamed by cp.async (double buffered); online softmax in registers.
// P.V runs on fp16 operands (V converted in shared memory; exact for |v| <
// 65504, saturating beyond) so P keeps 11 significant bits.
#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int BM = 64, BN = 64, NT = 128;
constexpr int D = kHeadDim;

__device__ __forceinline__ int off128(int r, int p) {
  return r * 128 + (((p & 8) | swz(r, p & 7)) << 3);
}

struct LocalSmem {
  __nv_bfloat16 q[BM * D];
  __nv_bfloat16 k[2][BN * D];
  __nv_bfloat16 v[2][BN * D];
};

__global__ void __launch_bounds__(NT) local_attn_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, const uint8_t* __restrict__ key_valid,
    __nv_bfloat16* __restrict__ out, float* __restrict__ lse, int64_t window, int skip_inert,
    int chunk, float sm_scale, int64_t Lq, int64_t Lk, int64_t q_offset, int Hq, int Hkv) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  LocalSmem& sm = *reinterpret_cast<LocalSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int hq = blockIdx.y, b = blockIdx.z, hk = hq / (Hq / Hkv);
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * BM;
  const int64_t rows_here = (Lq - q0) < BM ? (Lq - q0) : BM;
  const int64_t p_first = q_offset + q0, p_last = q_offset + q0 + rows_here - 1;
  int64_t j_lo = p_first - window, j_hi = p_last + window;
  if (j_lo < 0) j_lo = 0;
  if (j_hi > Lk - 1) j_hi = Lk - 1;
  const int t_lo = static_cast<int>(j_lo / BN), t_hi = static_cast<int>(j_hi / BN);

  // Q tile
  for (int e = tid; e < BM * 16; e += NT) {
    const int r = e >> 4, p = e & 15;
    const bool ok = r < rows_here;
    cp_async16_zfill(&sm.q[off128(r, p)],
                     q + (((b * Lq) + q0 + (ok ? r : 0)) * Hq + hq) * static_cast<int64_t>(D) + p * 8, ok);
  }
  cp_async_commit();

  auto load_kv = [&](int stage, int t) {
    const int64_t j0 = static_cast<int64_t>(t) * BN;
    for (int e = tid; e < BN * 16; e += NT) {
      const int r = e >> 4, p = e & 15;
      const int64_t j = j0 + r;
      bool ok = j < Lk;
      if (ok && key_valid != nullptr) ok = key_valid[b * Lk + j] != 0;
      if (ok && skip_inert) ok = ((j + 1) % chunk) != 0;
      const int64_t src = ((b * Lk + (ok ? j : 0)) * Hkv + hk) * static_cast<int64_t>(D) + p * 8;
      cp_async16_zfill(&sm.k[stage][off128(r, p)], k + src, ok);   // zeroed K,V slots
      cp_async16_zfill(&sm.v[stage][off128(r, p)], v + src, ok);
    }
    cp_async_commit();
  };

  load_kv(0, t_lo);
  cp_async_wait<1>();
  __syncthreads();
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int r = warp * 16 + (lane & 15), p = ks * 2 + (lane >> 4);
    ldsm_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], sm.q + off128(r, p));
  }

  const float sl2 = sm_scale * kLog2e;
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int64_t pos_r[2] = {p_first + warp * 16 + g, p_first + warp * 16 + g + 8};

  for (int t = t_lo; t <= t_hi; ++t) {
    const int st = (t - t_lo) & 1;
    if (t + 1 <= t_hi) {
      load_kv(st ^ 1, t + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    tile_bf16_to_f16(sm.v[st], tid, NT);
    __syncthreads();
    float s[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[n][i] = 0.f;
    const __nv_bfloat16* ks_ = sm.k[st];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), p = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, ks_ + off128(r, p));
        mma_bf16(s[2 * np], qa[kk], b0, b1);
        mma_bf16(s[2 * np + 1], qa[kk], b2, b3);
      }
    }
    // band mask + online softmax (log2 domain)
    const int64_t j0 = static_cast<int64_t>(t) * BN;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int hr = i >> 1;
        const int64_t j = j0 + n * 8 + tq * 2 + (i & 1);
        const int64_t dist = pos_r[hr] - j;
        const bool in = j < Lk && dist <= window && dist >= -window;
        s[n][i] = in ? s[n][i] * sl2 : -INFINITY;
        mx[hr] = fmaxf(mx[hr], s[n][i]);
      }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
    }
    float corr[2], base[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      base[hr] = mx[hr] == -INFINITY ? 0.f : mx[hr];
      corr[hr] = exp2f(m_r[hr] - base[hr]);
      m_r[hr] = mx[hr];
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s[n][i] = exp2f(s[n][i] - base[i >> 1]);
        rs[i >> 1] += s[n][i];
      }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) l_r[hr] = l_r[hr] * corr[hr] + rs[hr];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // O += P V
    const __nv_bfloat16* vs = sm.v[st];
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_f16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_f16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_f16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_f16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), p = np * 2 + (lane >> 4);
        ldsm_x4_t(b0, b1, b2, b3, vs + off128(r, p));
        mma_f16(o[2 * np], pa, b0, b1);
        mma_f16(o[2 * np + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }

  // normalise, stage through smem (the Q tile), coalesced store
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
    l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
  }
  float inv[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) inv[hr] = l_r[hr] > 0.f ? 1.f / l_r[hr] : 0.f;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int d = n * 8 + tq * 2;
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    *reinterpret_cast<uint32_t*>(&sm.q[off128(r0, d >> 3) + (d & 7)]) =
        pack_bf16x2(o[n][0] * inv[0], o[n][1] * inv[0]);
    *reinterpret_cast<uint32_t*>(&sm.q[off128(r1, d >> 3) + (d & 7)]) =
        pack_bf16x2(o[n][2] * inv[1], o[n][3] * inv[1]);
  }
  if (lse != nullptr && tq == 0) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = warp * 16 + g + hr * 8;
      if (r < rows_here)
        lse[((b * Lq) + q0 + r) * Hq + hq] =
            l_r[hr] > 0.f ? (m_r[hr] + log2f(l_r[hr])) * kLn2 : -INFINITY;
    }
  }
  __syncthreads();
  for (int e = tid; e < BM * 16; e += NT) {
    const int r = e >> 4, p = e & 15;
    if (r < rows_here)
      *reinterpret_cast<uint4*>(out + (((b * Lq) + q0 + r) * Hq + hq) * static_cast<int64_t>(D) + p * 8) =
          *reinterpret_cast<const uint4*>(&sm.q[off128(r, p)]);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int mrsa_local_attention(const void* q, const void* k, const void* v,
                                    const uint8_t* key_valid, void* out, float* lse,
                                    int64_t window, int skip_inert, int64_t chunk, float sm_scale,
                                    int64_t batch, int64_t q_len, int64_t kv_len, int64_t q_offset,
                                    int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                    mrsa_stream_t stream) {
  if (!q || !k || !v || !out) return MRSA_ERR_NULL;
  if (head_dim != D || kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads || batch < 1 ||
      q_len < 0 || kv_len < 1 || q_offset < 0 || q_heads > 65535 || batch > 65535)
    return MRSA_ERR_SHAPE;
  if (window < 0 || (skip_inert && chunk <= 0)) return MRSA_ERR_ARG;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  const int64_t blocks = (q_len + BM - 1) / BM;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  const size_t smem = sizeof(LocalSmem);
  if (cudaFuncSetAttribute(local_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(q_heads),
            static_cast<unsigned>(batch));
  local_attn_kernel<<<grid, NT, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), key_valid, static_cast<__nv_bfloat16*>(out), lse,
      window, skip_inert, static_cast<int>(chunk > 0 ? chunk : 1), sm_scale, q_len, kv_len,
      q_offset, static_cast<int>(q_heads), static_cast<int>(kv_heads));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
