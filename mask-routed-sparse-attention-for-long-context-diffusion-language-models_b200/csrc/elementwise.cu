// HBM-bound elementwise stages: YaRN RoPE (fp32), dense drop mask, output
// fusion, plus the ABI's small host helpers.
#include <math.h>

#include <cstdio>

#include "common.cuh"
#include "tc.cuh"

using namespace mrsa;

namespace {

// cos/sin of one token for the 64 frequency slots, HF rotary rule:
// ang = fp32(pos * inv_freq[j]); cos = cosf(ang) * factor.
__device__ __forceinline__ void yarn_cos_sin(int64_t pos, const float* inv_freq, float factor,
                                             int j, float& c, float& s) {
  float ang = static_cast<float>(pos) * __ldg(inv_freq + j);
  float sn, cs;
  sincosf(ang, &sn, &cs);
  c = cs * factor;
  s = sn * factor;
}

// One CTA per token.  Work item = (head, 8-dim group j in the first half):
// out[d] = x[d]cos[d] - x[d+64]sin[d], out[d+64] = x[d+64]cos[d+64] + x[d]sin[d+64].
__global__ void __launch_bounds__(256) rope_kernel(
    const __nv_bfloat16* __restrict__ x0, __nv_bfloat16* __restrict__ y0, int heads0,
    const __nv_bfloat16* __restrict__ x1, __nv_bfloat16* __restrict__ y1, int heads1,
    const int64_t* __restrict__ pos_ids, const float* __restrict__ inv_freq, float factor,
    const void* __restrict__ cos_p, const void* __restrict__ sin_p, int cs_dtype) {
  constexpr int D = kHeadDim, H = D / 2;
  __shared__ float cs_c[D], cs_s[D];
  const int64_t tok = blockIdx.x;
  if (pos_ids != nullptr) {
    if (threadIdx.x < H) {
      float c, s;
      yarn_cos_sin(pos_ids[tok], inv_freq, factor, threadIdx.x, c, s);
      cs_c[threadIdx.x] = c;
      cs_c[threadIdx.x + H] = c;
      cs_s[threadIdx.x] = s;
      cs_s[threadIdx.x + H] = s;
    }
  } else if (threadIdx.x < D) {
    if (cs_dtype == MRSA_F32) {
      cs_c[threadIdx.x] = static_cast<const float*>(cos_p)[tok * D + threadIdx.x];
      cs_s[threadIdx.x] = static_cast<const float*>(sin_p)[tok * D + threadIdx.x];
    } else {
      cs_c[threadIdx.x] = bf2f(static_cast<const __nv_bfloat16*>(cos_p)[tok * D + threadIdx.x]);
      cs_s[threadIdx.x] = bf2f(static_cast<const __nv_bfloat16*>(sin_p)[tok * D + threadIdx.x]);
    }
  }
  __syncthreads();
  const int items = (heads0 + heads1) * 8;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int head = it >> 3, j = (it & 7) * 8;
    const __nv_bfloat16* src;
    __nv_bfloat16* dst;
    if (head < heads0) {
      src = x0 + (tok * heads0 + head) * D;
      dst = y0 + (tok * heads0 + head) * D;
    } else {
      src = x1 + (tok * heads1 + (head - heads0)) * D;
      dst = y1 + (tok * heads1 + (head - heads0)) * D;
    }
    uint4 lo = *reinterpret_cast<const uint4*>(src + j);
    uint4 hi = *reinterpret_cast<const uint4*>(src + H + j);
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(&lo);
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hi);
    uint4 olo, ohi;
    uint32_t* ol = reinterpret_cast<uint32_t*>(&olo);
    uint32_t* oh = reinterpret_cast<uint32_t*>(&ohi);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float2 a = unpack_bf16x2(lw[p]), b = unpack_bf16x2(hw[p]);
      const int d = j + 2 * p;
      float a0 = a.x * cs_c[d] - b.x * cs_s[d];
      float a1 = a.y * cs_c[d + 1] - b.y * cs_s[d + 1];
      float b0 = b.x * cs_c[d + H] + a.x * cs_s[d + H];
      float b1 = b.y * cs_c[d + H + 1] + a.y * cs_s[d + H + 1];
      ol[p] = pack_bf16x2(a0, a1);
      oh[p] = pack_bf16x2(b0, b1);
    }
    *reinterpret_cast<uint4*>(dst + j) = olo;
    *reinterpret_cast<uint4*>(dst + H + j) = ohi;
  }
}

__global__ void drop_mask_kernel(const uint8_t* __restrict__ key_valid, int32_t* __restrict__ out,
                                 int64_t L, int64_t C, int64_t W, int64_t S, const int64_t* __restrict__ rows,
                                 int64_t Lq) {
  // one CTA per (query row, batch): chunk validity recomputed per chunk column;
  // row r sits at position rows[r] (rows == NULL: at position r, Lq == L)
  const int64_t r = blockIdx.x, b = blockIdx.y;
  const int64_t i = rows != nullptr ? rows[r] : r;
  const int64_t lo = (i - W > 0 ? i - W : 0) / S;
  const int64_t hi = (i + W < L - 1 ? i + W : L - 1) / S;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    bool ok = true;
    if (key_valid != nullptr) {
      ok = false;
      const uint8_t* kv = key_valid + b * L + c * S;
      for (int s = 0; s < S - 1; ++s) ok |= kv[s] != 0;
    }
    out[(b * Lq + r) * C + c] = ((c >= lo && c <= hi) || !ok) ? 1 : 0;
  }
}

__global__ void fuse_kernel(const __nv_bfloat16* __restrict__ remote,
                            const __nv_bfloat16* __restrict__ local,
                            const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                            int64_t rows, int D) {
  const int64_t n8 = rows * D / 8;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n8;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e * 8 / D;
    const float wl = bf2f(w[row]);
    uint4 r = reinterpret_cast<const uint4*>(remote)[e];
    uint4 l = reinterpret_cast<const uint4*>(local)[e];
    uint4 o;
    const uint32_t* rp = reinterpret_cast<const uint32_t*>(&r);
    const uint32_t* lp = reinterpret_cast<const uint32_t*>(&l);
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float2 a = unpack_bf16x2(rp[p]), b = unpack_bf16x2(lp[p]);
      op[p] = pack_bf16x2(a.x + wl * b.x, a.y + wl * b.y);
    }
    reinterpret_cast<uint4*>(out)[e] = o;
  }
}

// Set when mrsa_convert_bf16_to_f16 saturated a value beyond the fp16 range
// (infinities included); read and cleared through mrsa_device_error_flags() (bit 3).
__device__ int g_conv_error;

// bf16 -> fp16, eight values per thread; values beyond +-65504 saturate.
__global__ void __launch_bounds__(256) bf16_to_f16_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
                                                          int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint4 v = in[i];
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
  bool sat = false;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float f0 = __uint_as_float(w[k] << 16), f1 = __uint_as_float(w[k] & 0xffff0000u);
    const bool s0 = fabsf(f0) > 65504.f, s1 = fabsf(f1) > 65504.f;   // infinities included
    if (s0) f0 = copysignf(65504.f, f0);
    if (s1) f1 = copysignf(65504.f, f1);
    sat |= s0 | s1;
    o[k] = pack_f16x2(f0, f1);
  }
  out[i] = make_uint4(o[0], o[1], o[2], o[3]);
  if (sat) atomicOr(&g_conv_error, 1);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace mrsa {
int convert_error_flags(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_conv_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_conv_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
thread_local char g_last_error[256] = "";

void note_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
}
}  // namespace mrsa

extern "C" {

const char* mrsa_last_error(void) { return mrsa::g_last_error; }

const char* mrsa_strerror(int code) {
  switch (code) {
    case MRSA_OK: return "ok";
    case MRSA_ERR_NULL: return "a required pointer is NULL";
    case MRSA_ERR_SHAPE: return "inconsistent or unsupported shape";
    case MRSA_ERR_ALIGN: return "a pointer is not 16-byte aligned";
    case MRSA_ERR_LAUNCH: return "CUDA rejected the kernel launch";
    case MRSA_ERR_ARG: return "bad scalar argument";
    case MRSA_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown error";
  }
}

int mrsa_abi_version(void) { return 3; }

int mrsa_convert_bf16_to_f16(const void* in, void* out, int64_t n, mrsa_stream_t stream) {
  if (!in || !out) return MRSA_ERR_NULL;
  if (n < 0 || n % 8) return MRSA_ERR_SHAPE;
  if (!aligned16(in) || !aligned16(out)) return MRSA_ERR_ALIGN;
  if (n == 0) return MRSA_OK;
  const int64_t n8 = n / 8, blocks = (n8 + 255) / 256;
  if (blocks > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  bf16_to_f16_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(in), static_cast<uint4*>(out), n8);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

int mrsa_yarn_inv_freq(int dim, double base, double factor, int orig_max_pos, double beta_fast,
                       double beta_slow, int truncate, float* inv_freq_out,
                       float* attention_factor_out) {
  if (!inv_freq_out || !attention_factor_out) return MRSA_ERR_NULL;
  if (dim <= 0 || dim % 2 || base <= 1.0 || factor <= 0.0 || orig_max_pos <= 0) return MRSA_ERR_ARG;
  // Published YaRN rule (Peng et al. 2023), same arithmetic order as the
  // transformers implementation Dream uses: fp64 correction range, fp32 tables.
  auto corr = [&](double rot) {
    return (dim * log(orig_max_pos / (rot * 2.0 * M_PI))) / (2.0 * log(base));
  };
  double lo = corr(beta_fast), hi = corr(beta_slow);
  if (truncate) {
    lo = floor(lo);
    hi = ceil(hi);
  }
  if (lo < 0) lo = 0;
  if (hi > dim - 1) hi = dim - 1;
  if (lo == hi) hi += 0.001;
  const float flo = static_cast<float>(lo), fden = static_cast<float>(hi - lo);
  for (int j = 0; j < dim / 2; ++j) {
    const float expo = static_cast<float>(2 * j) / static_cast<float>(dim);
    const float pos_freq = powf(static_cast<float>(base), expo);
    const float extrap = 1.0f / pos_freq;
    const float interp = 1.0f / (static_cast<float>(factor) * pos_freq);
    float ramp = (static_cast<float>(j) - flo) / fden;
    ramp = ramp < 0.f ? 0.f : (ramp > 1.f ? 1.f : ramp);
    const float keep = 1.0f - ramp;
    inv_freq_out[j] = interp * (1.0f - keep) + extrap * keep;
  }
  *attention_factor_out = factor <= 1.0 ? 1.0f : static_cast<float>(0.1 * log(factor) + 1.0);
  return MRSA_OK;
}

int mrsa_rope(const void* x0, void* y0, int64_t heads0, const void* x1, void* y1, int64_t heads1,
              const int64_t* position_ids, const float* inv_freq, float attention_factor,
              const void* cos, const void* sin, int cs_dtype, int64_t batch, int64_t seq_len,
              int64_t head_dim, mrsa_stream_t stream) {
  if (!x0 || !y0) return MRSA_ERR_NULL;
  if (heads1 > 0 && (!x1 || !y1)) return MRSA_ERR_NULL;
  if (head_dim != kHeadDim || heads0 <= 0 || heads1 < 0 || batch <= 0 || seq_len < 0)
    return MRSA_ERR_SHAPE;
  const bool from_pos = position_ids != nullptr;
  if (from_pos && !inv_freq) return MRSA_ERR_NULL;
  if (!from_pos && (!cos || !sin)) return MRSA_ERR_NULL;
  if (!from_pos && cs_dtype != MRSA_BF16 && cs_dtype != MRSA_F32) return MRSA_ERR_ARG;
  if (!aligned16(x0) || !aligned16(y0) || (heads1 > 0 && (!aligned16(x1) || !aligned16(y1))))
    return MRSA_ERR_ALIGN;
  const int64_t tokens = batch * seq_len;
  if (tokens == 0) return MRSA_OK;
  if (tokens > 0x7fffffffLL) return MRSA_ERR_SHAPE;
  rope_kernel<<<static_cast<unsigned>(tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x0), static_cast<__nv_bfloat16*>(y0),
      static_cast<int>(heads0), static_cast<const __nv_bfloat16*>(x1),
      static_cast<__nv_bfloat16*>(y1), static_cast<int>(heads1), position_ids, inv_freq,
      attention_factor, cos, sin, cs_dtype);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

int mrsa_remote_drop_mask(const uint8_t* key_valid, int32_t* out, int64_t batch, int64_t seq_len,
                          int64_t window, int64_t chunk, mrsa_stream_t stream) {
  if (!out) return MRSA_ERR_NULL;
  if (batch <= 0 || seq_len <= 0 || chunk <= 0 || seq_len % chunk) return MRSA_ERR_SHAPE;
  if (window < 0) return MRSA_ERR_ARG;
  if (seq_len > 0x7fffffffLL || batch > 65535) return MRSA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(seq_len), static_cast<unsigned>(batch));
  drop_mask_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      key_valid, out, seq_len, seq_len / chunk, window, chunk, nullptr, seq_len);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

int mrsa_remote_drop_mask_positions(const uint8_t* key_valid, const int64_t* positions, int32_t* out,
                                    int64_t batch, int64_t seq_len, int64_t q_len, int64_t window, int64_t chunk,
                                    mrsa_stream_t stream) {
  if (!out || !positions) return MRSA_ERR_NULL;
  if (batch <= 0 || seq_len <= 0 || q_len < 0 || chunk <= 0 || seq_len % chunk) return MRSA_ERR_SHAPE;
  if (window < 0) return MRSA_ERR_ARG;
  if (q_len > 0x7fffffffLL || batch > 65535) return MRSA_ERR_SHAPE;
  if (q_len == 0) return MRSA_OK;
  dim3 grid(static_cast<unsigned>(q_len), static_cast<unsigned>(batch));
  drop_mask_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      key_valid, out, seq_len, seq_len / chunk, window, chunk, positions, q_len);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

int mrsa_fuse_outputs(const void* remote, const void* local, const void* local_w, void* out,
                      int64_t rows, int64_t head_dim, mrsa_stream_t stream) {
  if (!remote || !local || !local_w || !out) return MRSA_ERR_NULL;
  if (rows < 0 || head_dim <= 0 || head_dim % 8) return MRSA_ERR_SHAPE;
  if (!aligned16(remote) || !aligned16(local) || !aligned16(out)) return MRSA_ERR_ALIGN;
  if (rows == 0) return MRSA_OK;
  const int64_t n8 = rows * head_dim / 8;
  int blocks = static_cast<int>((n8 + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  fuse_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(remote), static_cast<const __nv_bfloat16*>(local),
      static_cast<const __nv_bfloat16*>(local_w), static_cast<__nv_bfloat16*>(out), rows,
      static_cast<int>(head_dim));
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Self-test of the bounded mbarrier wait every pipelined kernel uses: warp 0
// waits (with `rounds` rounds instead of the kernels' 4000) on a barrier
// nothing ever arrives on, so it must give up and raise the CTA's abort flag;
// warp 1 waits on a second such barrier with the full limit and must leave as
// soon as it sees the flag.  result[0] = warp 0 gave up, result[1] = abort
// flag raised, result[2] = warp 1 left through the flag.  Nothing faults or
// hangs: both waits end, and the kernel returns.
namespace {
__global__ void wait_selftest_kernel(int* result, int rounds) {
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_addr(&bar[0]), 1);
    tc::mbar_init(tc::smem_addr(&bar[1]), 1);
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* af = &abort_flag;
  if (warp == 0) {
    const bool ok = tc::wait_bounded(tc::smem_addr(&bar[0]), 0, af, rounds);
    if (lane == 0) result[0] = ok ? 0 : 1;
  } else {
    const bool ok = tc::wait_bounded(tc::smem_addr(&bar[1]), 0, af);
    if (lane == 0) result[2] = (!ok && *af) ? 1 : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) result[1] = abort_flag;
}
}  // namespace

extern "C" int mrsa_wait_selftest(int* result, int rounds, mrsa_stream_t stream) {
  if (!result) return MRSA_ERR_NULL;
  if (rounds < 1 || rounds > 4000) return MRSA_ERR_ARG;
  wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(result, rounds);
  MRSA_CHECK_LAUNCH();
  return MRSA_OK;
}
