// Q-Cal routing query in one kernel:
//   t       = bf16(h W_in^T)                    [64 tokens x rank 64]   (phase 1)
//   delta   = bf16(t W_out[head]^T) * scale       per head, 64 x 128      (phase 2)
//   route_q = rope(rmsnorm(bf16(invrope(q) + delta)))   fused epilogue
// Follows _qcal_delta/_finish_calibrated_query (dream_dllm_hils/attention.py:458-503)
// and qcal.rms_norm (dream_dllm_hils/qcal.py:22-26): the rank-64 intermediate and
// delta are rounded to bf16 like the reference's bf16 linear layers.
// One CTA owns 64 consecutive tokens; h streams once from HBM, W_in/W_out stay
// in L2.  Tensor work is mma.sync m16n8k16 (bf16 -> fp32).
#include <algorithm>

#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int TM = 64;      // tokens per CTA
constexpr int RANK = 64;    // Q-Cal rank
constexpr int TK = 64;      // hidden slice per pipeline stage
constexpr int NT = 128;     // threads (4 warps x 16 token rows)
constexpr int P1ST = 4;     // phase-1 stages: h streams from HBM with three tiles in flight

struct QcalSmem {
  union {
    struct {
      __nv_bfloat16 h[P1ST][TM * TK];  // 32 KB
      __nv_bfloat16 w[P1ST][RANK * TK];  // 32 KB
    } p1;
    struct {
      __nv_bfloat16 wo[2][kHeadDim * RANK];  // 32 KB
      __nv_bfloat16 q[2][TM * kHeadDim];     // 32 KB
    } p2;
  } u;
  __nv_bfloat16 t[TM * RANK];   // 8 KB, bf16(h W_in^T)
  float4 cs[TM][kHeadDim / 4 + 1];   // (cos, sin) of dims 2j, 2j+1 of token row r: {c0, s0, c1, s1}; padded row
};

// offset (elements) of 16-byte piece `p` of row `r` in a 64-column bf16 tile
__device__ __forceinline__ int off64(int r, int p) { return r * 64 + (swz(r, p) << 3); }
// same for a 128-column tile (16 pieces; swizzle inside each 8-piece half)
__device__ __forceinline__ int off128(int r, int p) {
  return r * 128 + (((p & 8) | swz(r, p & 7)) << 3);
}

__global__ void __launch_bounds__(NT) qcal_kernel(
    const __nv_bfloat16* __restrict__ hid, const __nv_bfloat16* __restrict__ q,
    const __nv_bfloat16* __restrict__ w_in, const __nv_bfloat16* __restrict__ w_out,
    const float* __restrict__ norm_w, float eps, float scale, const int64_t* __restrict__ pos_ids,
    const float* __restrict__ inv_freq, float factor, __nv_bfloat16* __restrict__ route_q,
    int64_t tokens, int hidden, int q_heads, int heads_per_cta) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  QcalSmem& sm = *reinterpret_cast<QcalSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * TM;
  const int g = lane >> 2, tq = lane & 3;

  // cos/sin table for the CTA's tokens
  for (int e = tid; e < TM * 64; e += NT) {
    const int r = e >> 6, j = e & 63;
    const int64_t tok = tok0 + r;
    float c = 0.f, s = 0.f;
    if (tok < tokens) {
      float ang = static_cast<float>(pos_ids[tok]) * __ldg(inv_freq + j);
      sincosf(ang, &s, &c);
      c *= factor;
      s *= factor;
    }
    reinterpret_cast<float2*>(&sm.cs[r][0])[j] = make_float2(c, s);
  }

  // ---------------- phase 1: t = h W_in^T -----------------------------------
  auto load_p1 = [&](int stage, int k0) {
    // h tile: 64 rows x 8 pieces; W_in tile: 64 rows x 8 pieces
    for (int e = tid; e < TM * 8; e += NT) {
      const int r = e >> 3, p = e & 7;
      const int64_t tok = tok0 + r;
      const bool ok = tok < tokens;
      cp_async16_zfill(&sm.u.p1.h[stage][off64(r, p)],
                       hid + (ok ? tok : 0) * hidden + k0 + p * 8, ok);
      cp_async16(&sm.u.p1.w[stage][off64(r, p)], w_in + static_cast<int64_t>(r) * hidden + k0 + p * 8);
    }
    cp_async_commit();
  };
  float acc1[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc1[n][i] = 0.f;

  const int ktiles = hidden / TK;
  for (int s0 = 0; s0 < P1ST - 1 && s0 < ktiles; ++s0) load_p1(s0, s0 * TK);
  for (int kt = 0; kt < ktiles; ++kt) {
    // tile kt has landed once at most min(P1ST - 1, tiles after it) groups are pending
    if (kt + P1ST - 1 < ktiles) {
      load_p1((kt + P1ST - 1) % P1ST, (kt + P1ST - 1) * TK);
      cp_async_wait<P1ST - 1>();
    } else if (ktiles - 1 - kt >= 2) {
      cp_async_wait<2>();
    } else if (ktiles - 1 - kt == 1) {
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* hs = sm.u.p1.h[kt % P1ST];
    const __nv_bfloat16* ws = sm.u.p1.w[kt % P1ST];
#pragma unroll
    for (int ks = 0; ks < TK / 16; ++ks) {
      uint32_t a[4];
      {
        const int r = warp * 16 + (lane & 15), p = ks * 2 + (lane >> 4);
        ldsm_x4(a[0], a[1], a[2], a[3], hs + off64(r, p));
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), p = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, ws + off64(r, p));
        mma_bf16(acc1[2 * np], a, b0, b1);
        mma_bf16(acc1[2 * np + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  // t -> bf16 smem (A operand of phase 2)
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int col = n * 8 + tq * 2;
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    *reinterpret_cast<uint32_t*>(&sm.t[off64(r0, col >> 3) + (col & 7)]) = pack_bf16x2(acc1[n][0], acc1[n][1]);
    *reinterpret_cast<uint32_t*>(&sm.t[off64(r1, col >> 3) + (col & 7)]) = pack_bf16x2(acc1[n][2], acc1[n][3]);
  }
  __syncthreads();

  // A fragments of t stay in registers for all heads
  uint32_t ta[RANK / 16][4];
#pragma unroll
  for (int ks = 0; ks < RANK / 16; ++ks) {
    const int r = warp * 16 + (lane & 15), p = ks * 2 + (lane >> 4);
    ldsm_x4(ta[ks][0], ta[ks][1], ta[ks][2], ta[ks][3], sm.t + off64(r, p));
  }

  // ---------------- phase 2: per head ----------------------------------------
  auto load_p2 = [&](int stage, int head) {
    const __nv_bfloat16* wsrc = w_out + static_cast<int64_t>(head) * kHeadDim * RANK;
    for (int e = tid; e < kHeadDim * 8; e += NT) {   // W_out rows of this head: 128 x 64
      const int r = e >> 3, p = e & 7;
      cp_async16(&sm.u.p2.wo[stage][off64(r, p)], wsrc + r * RANK + p * 8);
    }
    for (int e = tid; e < TM * 16; e += NT) {        // q tile: 64 tokens x 128
      const int r = e >> 4, p = e & 15;
      const int64_t tok = tok0 + r;
      const bool ok = tok < tokens;
      cp_async16_zfill(&sm.u.p2.q[stage][off128(r, p)],
                       q + ((ok ? tok : 0) * q_heads + head) * kHeadDim + p * 8, ok);
    }
    cp_async_commit();
  };

  const int r0 = warp * 16 + g, r1 = r0 + 8;
  // this thread's RMSNorm weights (dims n*8 + 2 tq + e and +64), held for all heads
  float nw_lo[8][2], nw_hi[8][2];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      nw_lo[n][e] = __ldg(norm_w + n * 8 + tq * 2 + e);
      nw_hi[n][e] = __ldg(norm_w + n * 8 + tq * 2 + e + 64);
    }
  // this CTA's heads (all of them unless few token tiles split the heads over CTAs)
  const int h_begin = static_cast<int>(blockIdx.y) * heads_per_cta;
  const int h_end = min(q_heads, h_begin + heads_per_cta);
  load_p2(0, h_begin);
  for (int head = h_begin; head < h_end; ++head) {
    const int st = (head - h_begin) & 1;
    if (head + 1 < h_end) {
      load_p2(st ^ 1, head + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float acc[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
    const __nv_bfloat16* wo = sm.u.p2.wo[st];
#pragma unroll
    for (int ks = 0; ks < RANK / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), p = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, wo + off64(r, p));
        mma_bf16(acc[2 * np], ta[ks], b0, b1);
        mma_bf16(acc[2 * np + 1], ta[ks], b2, b3);
      }
    }
    // epilogue: rows r0 (acc[..][0..1]) and r1 (acc[..][2..3])
    __nv_bfloat16* qs = sm.u.p2.q[st];
    float comb[2][16][2];
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? r1 : r0;
#pragma unroll
      for (int n = 0; n < 8; ++n) {     // n-tile n (dims < 64) pairs with n+8
        const int d = n * 8 + tq * 2;
        const float4 cs4 = sm.cs[r][n * 4 + tq];
        float2 x_lo = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&qs[off128(r, d >> 3) + (d & 7)]));
        float2 x_hi = unpack_bf16x2(
            *reinterpret_cast<const uint32_t*>(&qs[off128(r, (d + 64) >> 3) + (d & 7)]));
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float c = e ? cs4.z : cs4.x, s = e ? cs4.w : cs4.y;
          const float xl = e ? x_lo.y : x_lo.x, xh = e ? x_hi.y : x_hi.x;
          float dl = round_bf16(acc[n][half * 2 + e]);
          float dh = round_bf16(acc[n + 8][half * 2 + e]);
          if (scale != 1.0f) {
            dl = round_bf16(dl * scale);
            dh = round_bf16(dh * scale);
          }
          const float ul = round_bf16(xl * c + xh * s);   // invert_rotary_pos_emb
          const float uh = round_bf16(xh * c - xl * s);
          const float cl = round_bf16(ul + dl), ch = round_bf16(uh + dh);
          comb[half][n][e] = cl;
          comb[half][n + 8][e] = ch;
          ss[half] += cl * cl + ch * ch;
        }
      }
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      ss[half] += __shfl_xor_sync(0xffffffffu, ss[half], 1);
      ss[half] += __shfl_xor_sync(0xffffffffu, ss[half], 2);
    }
    __syncwarp();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? r1 : r0;
      const float inv = rsqrtf(ss[half] / static_cast<float>(kHeadDim) + eps);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int d = n * 8 + tq * 2;
        const float4 cs4 = sm.cs[r][n * 4 + tq];
        float ol[2], oh[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float c = e ? cs4.z : cs4.x, s = e ? cs4.w : cs4.y;
          const float nl = round_bf16(nw_lo[n][e] * (comb[half][n][e] * inv));
          const float nh = round_bf16(nw_hi[n][e] * (comb[half][n + 8][e] * inv));
          ol[e] = nl * c - nh * s;                         // apply_rotary_pos_emb
          oh[e] = nh * c + nl * s;
        }
        *reinterpret_cast<uint32_t*>(&qs[off128(r, d >> 3) + (d & 7)]) = pack_bf16x2(ol[0], ol[1]);
        *reinterpret_cast<uint32_t*>(&qs[off128(r, (d + 64) >> 3) + (d & 7)]) = pack_bf16x2(oh[0], oh[1]);
      }
    }
    __syncthreads();
    for (int e = tid; e < TM * 16; e += NT) {
      const int r = e >> 4, p = e & 15;
      const int64_t tok = tok0 + r;
      if (tok < tokens)
        *reinterpret_cast<uint4*>(route_q + (tok * q_heads + head) * kHeadDim + p * 8) =
            *reinterpret_cast<const uint4*>(&qs[off128(r, p)]);
    }
    __syncthreads();
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int mrsa_qcal_route_query(const void* hidden, const void* q, const void* w_in,
                                     const void* w_out, const float* norm_weight, float eps,
                                     float scale, const int64_t* position_ids,
                                     const float* inv_freq, float attention_factor, void* route_q,
                                     int64_t batch, int64_t seq_len, int64_t hidden_size,
                                     int64_t rank, int64_t q_heads, int64_t head_dim,
                                     mrsa_stream_t stream) {
  if (!hidden || !q || !w_in || !w_out || !norm_weight || !position_ids || !inv_freq || !route_q)
    return MRSA_ERR_NULL;
  if (head_dim != kHeadDim || rank != RANK || hidden_size <= 0 || hidden_size % TK ||
      q_heads <= 0 || batch <= 0 || seq_len < 0)
    return MRSA_ERR_SHAPE;
  if (!(eps > 0.f)) return MRSA_ERR_ARG;
  if (!aligned16(hidden) || !aligned16(q) || !aligned16(w_in) || !aligned16(w_out) || !aligned16(route_q))
    return MRSA_ERR_ALIGN;
  const int64_t tokens = batch * seq_len;
  if (tokens == 0) return MRSA_OK;
  const int64_t blocks = (tokens + TM - 1) / TM;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  // With fewer token tiles than SMs (decode-sized calls) the heads are split
  // over CTAs, each recomputing its tile's h W_in^T (L2-resident), so the
  // per-head epilogues run side by side instead of in one CTA's loop; every
  // head's result is computed exactly as in the one-CTA loop.
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int groups = 1;
  if (blocks < sms) groups = static_cast<int>(std::min<int64_t>(q_heads, (sms + blocks - 1) / blocks));
  const int heads_per_cta = static_cast<int>((q_heads + groups - 1) / groups);
  groups = static_cast<int>((q_heads + heads_per_cta - 1) / heads_per_cta);
  const size_t smem = sizeof(QcalSmem);
  if (cudaFuncSetAttribute(qcal_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(groups));
  qcal_kernel<<<grid, NT, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(hidden), static_cast<const __nv_bfloat16*>(q),
      static_cast<const __nv_bfloat16*>(w_in), static_cast<const __nv_bfloat16*>(w_out),
      norm_weight, eps, scale, position_ids, inv_freq, attention_factor,
      static_cast<__nv_bfloat16*>(route_q), tokens, static_cast<int>(hidden_size),
      static_cast<int>(q_heads), heads_per_cta);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
