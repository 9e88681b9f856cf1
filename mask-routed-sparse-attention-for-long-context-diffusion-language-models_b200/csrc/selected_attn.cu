// Weighted per-chunk-softmax attention over routed chunks, fused with the
// local branch.  Semantics of the HiLS forward (ops/hils_fwd_bwd_head.py:21-93
// torch reference, kernel :423-559): every selected chunk is normalised on
// its own (landmark slot 63 and invalid keys masked), its probabilities are
// scaled by the route weight, and P.V accumulates in fp32 on fp16 operands
// (the reference rounds P to bf16; fp16 keeps 3 more bits, and bf16 V
// converts to fp16 exactly for |v| < 65504); the epilogue applies fuse_hils_outputs
// (ops/hils_bidir_output_fusion_tilelang.py:15-37): bf16(bf16(remote) + w_l*local).
//
// CTA = 16 queries x one KV head.  Each warp owns a fixed pair of queries,
// i.e. one m16 MMA tile whose rows are (query, head-in-group) with the group
// padded to 8 rows.  The CTA walks the union of its queries' chunk lists in
// ascending order, streaming each 64x128 K and V tile once into shared
// memory (cp.async, double buffered); only warps whose queries selected the
// chunk run the two MMAs on it.
#include "common.cuh"

using namespace mrsa;

namespace {

constexpr int QB = 16, NW = 8, NT = NW * 32;
constexpr int D = kHeadDim, S = kChunk;
constexpr int KMAX = 32;

__device__ __forceinline__ int off128(int r, int p) {
  return r * 128 + (((p & 8) | swz(r, p & 7)) << 3);
}

struct SelSmem {
  __nv_bfloat16 q[QB * 8 * D];      // 32 KB: rows (query, head slot 0..7)
  __nv_bfloat16 k[2][S * D];        // 32 KB
  __nv_bfloat16 v[2][S * D];        // 32 KB
  __nv_bfloat16 w[QB][8][KMAX];     //  8 KB route weights
  int idx[QB][KMAX];                //  2 KB selected chunk ids
  int ulist[QB * KMAX];             //  2 KB union of the chunk lists
  uint8_t kvalid[2][S];
  int nu;
  uint32_t bitmap[1];               // [ceil(C/32)] words, dynamic tail
};

struct SelArgs {
  const __nv_bfloat16 *q, *k, *v;
  const uint8_t* key_valid;
  const __nv_bfloat16* w;
  const int32_t* indices;
  const __nv_bfloat16 *local_out, *local_w;
  __nv_bfloat16* out;
  float sm_scale;
  int mask_last;
  int64_t Lq, Lk;
  int Hkv, G, K, C;
};

__global__ void __launch_bounds__(NT, 2) selected_attn_kernel(SelArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  SelSmem& sm = *reinterpret_cast<SelSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, tq = lane & 3;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * QB;
  const int G = a.G, K = a.K, C = a.C, Hq = a.Hkv * a.G;
  const int nwords = (C + 31) >> 5;

  // ---- stage Q rows, indices, weights; build the union bitmap --------------
  for (int e = tid; e < QB * 8 * 16; e += NT) {
    const int r = e >> 4, p = e & 15;          // r = query*8 + head slot
    const int qi = r >> 3, gs = r & 7;
    const bool ok = gs < G && q0 + qi < a.Lq;
    const int64_t src = ((b * a.Lq + (ok ? q0 + qi : 0)) * Hq + hk * G + (ok ? gs : 0)) * (int64_t)D + p * 8;
    cp_async16_zfill(&sm.q[off128(r, p)], a.q + src, ok);
  }
  cp_async_commit();
  for (int e = tid; e < nwords; e += NT) sm.bitmap[e] = 0u;
  for (int e = tid; e < QB * KMAX; e += NT) {
    const int qi = e / KMAX, kk = e % KMAX;
    int c = -1;
    if (kk < K && q0 + qi < a.Lq) {
      c = a.indices[((b * a.Lq + q0 + qi) * a.Hkv + hk) * K + kk];
      if (c >= C) c = -1;
    }
    sm.idx[qi][kk] = c < 0 ? -1 : c;
  }
  for (int e = tid; e < QB * 8 * KMAX; e += NT) {
    const int qi = e / (8 * KMAX), gs = (e / KMAX) & 7, kk = e % KMAX;
    __nv_bfloat16 wv = f2bf(0.f);
    if (gs < G && kk < K && q0 + qi < a.Lq)
      wv = a.w[((b * a.Lq + q0 + qi) * Hq + hk * G + gs) * K + kk];
    sm.w[qi][gs][kk] = wv;
  }
  __syncthreads();
  for (int e = tid; e < QB * KMAX; e += NT) {
    const int c = sm.idx[e / KMAX][e % KMAX];
    if (c >= 0) atomicOr(&sm.bitmap[c >> 5], 1u << (c & 31));
  }
  __syncthreads();
  if (warp == 0) {
    int base = 0;
    for (int wb = 0; wb < nwords; wb += 32) {
      const uint32_t word = (wb + lane < nwords) ? sm.bitmap[wb + lane] : 0u;
      const int cnt = __popc(word);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int pos = base + incl - cnt;
      uint32_t wbits = word;
      while (wbits) {
        const int bit = __ffs(wbits) - 1;
        sm.ulist[pos++] = ((wb + lane) << 5) + bit;
        wbits &= wbits - 1;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) sm.nu = base;
  }
  __syncthreads();
  const int nu = sm.nu;

  // per-lane copies of this warp's two chunk lists (lane = slot)
  const int qa_i = 2 * warp, qb_i = 2 * warp + 1;
  const int ia = lane < K ? sm.idx[qa_i][lane] : -1;
  const int ib = lane < K ? sm.idx[qb_i][lane] : -1;

  auto load_tile = [&](int stage, int c) {
    const int64_t j0 = static_cast<int64_t>(c) * S;
    for (int e = tid; e < S * 16; e += NT) {
      const int r = e >> 4, p = e & 15;
      const int64_t src = ((b * a.Lk + j0 + r) * a.Hkv + hk) * (int64_t)D + p * 8;
      cp_async16(&sm.k[stage][off128(r, p)], a.k + src);
      cp_async16(&sm.v[stage][off128(r, p)], a.v + src);
    }
    if (tid < S) {
      bool ok = a.key_valid == nullptr || a.key_valid[b * a.Lk + j0 + tid] != 0;
      if (a.mask_last && tid == S - 1) ok = false;
      sm.kvalid[stage][tid] = ok;
    }
    cp_async_commit();
  };

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  const float sl2 = a.sm_scale * kLog2e;

  if (nu > 0) load_tile(0, sm.ulist[0]);
  for (int u = 0; u < nu; ++u) {
    const int st = u & 1;
    if (u + 1 < nu) {
      load_tile(st ^ 1, sm.ulist[u + 1]);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    tile_bf16_to_f16(sm.v[st], tid, NT);
    __syncthreads();
    const int c = sm.ulist[u];
    const uint32_t ma = __ballot_sync(0xffffffffu, ia == c);
    const uint32_t mb = __ballot_sync(0xffffffffu, ib == c);
    if (ma | mb) {
      const int slot_a = ma ? __ffs(ma) - 1 : 0, slot_b = mb ? __ffs(mb) - 1 : 0;
      float s[S / 8][4];
#pragma unroll
      for (int n = 0; n < S / 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) s[n][i] = 0.f;
      const __nv_bfloat16* ks_ = sm.k[st];
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t qa[4];
        {
          const int r = warp * 16 + (lane & 15), p = kk * 2 + (lane >> 4);
          ldsm_x4(qa[0], qa[1], qa[2], qa[3], sm.q + off128(r, p));
        }
#pragma unroll
        for (int np = 0; np < S / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3), p = kk * 2 + ((lane >> 3) & 1);
          ldsm_x4(b0, b1, b2, b3, ks_ + off128(r, p));
          mma_bf16(s[2 * np], qa, b0, b1);
          mma_bf16(s[2 * np + 1], qa, b2, b3);
        }
      }
      // rows: half 0 -> query qa_i, head g4; half 1 -> query qb_i, head g4
      const bool own[2] = {ma != 0, mb != 0};
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < S / 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int key = n * 8 + tq * 2 + (i & 1);
          const bool keep = own[i >> 1] && sm.kvalid[st][key];
          s[n][i] = keep ? s[n][i] * sl2 : -INFINITY;
          mx[i >> 1] = fmaxf(mx[i >> 1], s[n][i]);
        }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
        mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      }
      float sum[2] = {0.f, 0.f};
#pragma unroll
      for (int n = 0; n < S / 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float m = mx[i >> 1];
          s[n][i] = (m == -INFINITY) ? 0.f : exp2f(s[n][i] - m);
          sum[i >> 1] += s[n][i];
        }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        sum[hr] += __shfl_xor_sync(0xffffffffu, sum[hr], 1);
        sum[hr] += __shfl_xor_sync(0xffffffffu, sum[hr], 2);
      }
      const bool head_ok = g4 < G;
      const float w0 = (own[0] && head_ok) ? bf2f(sm.w[qa_i][g4][slot_a]) : 0.f;
      const float w1 = (own[1] && head_ok) ? bf2f(sm.w[qb_i][g4][slot_b]) : 0.f;
      const float f0 = sum[0] > 0.f ? w0 / sum[0] : 0.f;
      const float f1 = sum[1] > 0.f ? w1 / sum[1] : 0.f;
      const __nv_bfloat16* vs = sm.v[st];
#pragma unroll
      for (int kk = 0; kk < S / 16; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_f16x2(s[2 * kk][0] * f0, s[2 * kk][1] * f0);
        pa[1] = pack_f16x2(s[2 * kk][2] * f1, s[2 * kk][3] * f1);
        pa[2] = pack_f16x2(s[2 * kk + 1][0] * f0, s[2 * kk + 1][1] * f0);
        pa[3] = pack_f16x2(s[2 * kk + 1][2] * f1, s[2 * kk + 1][3] * f1);
#pragma unroll
        for (int np = 0; np < D / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), p = np * 2 + (lane >> 4);
          ldsm_x4_t(b0, b1, b2, b3, vs + off128(r, p));
          mma_f16(o[2 * np], pa, b0, b1);
          mma_f16(o[2 * np + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();   // the Q tile is still in flight when no chunk was routed

  // ---- epilogue: remote -> bf16, optional fusion with the local branch -----
  if (g4 < G) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int qi = 2 * warp + hr;
      const int64_t row = q0 + qi;
      if (row >= a.Lq) continue;
      const int64_t base = ((b * a.Lq + row) * Hq + hk * G + g4) * (int64_t)D;
      const float wl = a.local_w ? bf2f(a.local_w[(b * a.Lq + row) * Hq + hk * G + g4]) : 0.f;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        const int d = n * 8 + tq * 2;
        float r0 = round_bf16(o[n][hr * 2]), r1 = round_bf16(o[n][hr * 2 + 1]);
        if (a.local_out) {
          const float2 lo = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a.local_out + base + d));
          r0 = r0 + wl * lo.x;
          r1 = r1 + wl * lo.y;
        }
        *reinterpret_cast<uint32_t*>(a.out + base + d) = pack_bf16x2(r0, r1);
      }
    }
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int mrsa_selected_attention(const void* q, const void* k, const void* v,
                                       const uint8_t* key_valid, const void* weights,
                                       const int32_t* indices, const void* local_out,
                                       const void* local_w, void* out, float sm_scale,
                                       int mask_last_token, int64_t batch, int64_t q_len,
                                       int64_t kv_len, int64_t kv_heads, int64_t groups,
                                       int64_t head_dim, int64_t topk, int64_t chunk,
                                       mrsa_stream_t stream) {
  if (!q || !k || !v || !weights || !indices || !out) return MRSA_ERR_NULL;
  if ((local_out == nullptr) != (local_w == nullptr)) return MRSA_ERR_NULL;
  if (head_dim != D || chunk != S || groups < 1 || groups > 8 || kv_heads < 1 || batch < 1 ||
      q_len < 0 || kv_len < S || kv_len % S || topk < 1 || topk > KMAX || kv_heads > 65535 ||
      batch > 65535)
    return MRSA_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (local_out && !aligned16(local_out)))
    return MRSA_ERR_ALIGN;
  if (q_len == 0) return MRSA_OK;
  SelArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.key_valid = key_valid;
  a.w = static_cast<const __nv_bfloat16*>(weights);
  a.indices = indices;
  a.local_out = static_cast<const __nv_bfloat16*>(local_out);
  a.local_w = static_cast<const __nv_bfloat16*>(local_w);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.sm_scale = sm_scale;
  a.mask_last = mask_last_token;
  a.Lq = q_len;
  a.Lk = kv_len;
  a.Hkv = static_cast<int>(kv_heads);
  a.G = static_cast<int>(groups);
  a.K = static_cast<int>(topk);
  a.C = static_cast<int>(kv_len / S);
  const size_t smem = sizeof(SelSmem) + sizeof(uint32_t) * ((a.C + 31) / 32);
  if (smem > 110 * 1024) return MRSA_ERR_SHAPE;
  if (cudaFuncSetAttribute(selected_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return MRSA_ERR_LAUNCH;
  const int64_t blocks = (q_len + QB - 1) / QB;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(kv_heads),
            static_cast<unsigned>(batch));
  selected_attn_kernel<<<grid, NT, smem, static_cast<cudaStream_t>(stream)>>>(a);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
