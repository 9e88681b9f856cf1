// Whole route layer on one device: the stage sequence of
// KernelDreamFullHiLSAttention.forward (dream_dllm_hils/attention.py:1358-1774)
// from the projected q/k/v/h to the input of o_proj, as six launches on the
// caller's stream over a caller-provided workspace.
#include "common.cuh"

namespace {

constexpr size_t kAlign = 256;

inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct LayerPlan {
  size_t q, k, v16, route_q, lmk, entropy, prior, chunk_ok, local_out, local_lse, indices, scores,
      remote_w, local_w, route_keys, total;
};

LayerPlan plan(const mrsa_route_layer_args* a) {
  const size_t B = a->batch, L = a->seq_len, Hq = a->q_heads, Hkv = a->kv_heads,
               D = a->head_dim, K = a->topk, C = L / mrsa::kChunk;
  LayerPlan p{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align_up(bytes);
    return o;
  };
  p.q = take(B * L * Hq * D * 2);
  p.k = take(B * L * Hkv * D * 2);
  p.v16 = take(B * L * Hkv * D * 2);        // V in fp16 for the local and selected kernels
  p.route_q = take(B * L * Hq * D * 2);
  p.lmk = take(B * C * Hq * D * 2);
  p.entropy = take(B * C * Hq * 4);
  p.prior = take(B * C * Hq * 4);
  p.chunk_ok = take(B * C);
  p.local_out = take(B * L * Hq * D * 2);
  p.local_lse = take(B * L * Hq * 4);
  p.indices = take(B * L * Hkv * K * 4);
  p.scores = take(B * L * Hq * K * 2);
  p.remote_w = take(B * L * Hq * K * 2);
  p.local_w = take(B * L * Hq * 2);
  p.route_keys = take(mrsa_route_topk_workspace_size(B, L, C, Hkv, Hq / Hkv, MRSA_BF16));
  p.total = off;
  return p;
}

bool shape_ok(const mrsa_route_layer_args* a) {
  return a->batch > 0 && a->seq_len > 0 && a->seq_len % mrsa::kChunk == 0 && a->kv_heads > 0 &&
         a->q_heads % a->kv_heads == 0 && a->q_heads / a->kv_heads <= 8 &&
         a->head_dim == mrsa::kHeadDim && a->topk >= 1 && a->topk <= 32 && a->local_window >= 0 &&
         a->hidden_size > 0 && a->rank == 64;
}

}  // namespace

extern "C" size_t mrsa_route_layer_workspace_size(const mrsa_route_layer_args* a) {
  if (a == nullptr || !shape_ok(a)) return 0;
  return plan(a).total;
}

extern "C" int mrsa_route_layer_forward(const mrsa_route_layer_args* a, void* workspace,
                                        size_t ws_bytes, mrsa_stream_t stream) {
  if (a == nullptr) return MRSA_ERR_NULL;
  mrsa::DeviceScope device_scope(a->q_pre);
  if (!a->q_pre || !a->k_pre || !a->v || !a->hidden || !a->position_ids || !a->inv_freq ||
      !a->w_in || !a->w_out || !a->norm_weight || !a->out)
    return MRSA_ERR_NULL;
  if (!shape_ok(a)) return MRSA_ERR_SHAPE;
  const LayerPlan p = plan(a);
  if (workspace == nullptr || ws_bytes < p.total) return MRSA_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % kAlign) return MRSA_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  void* q = ws + p.q;
  void* k = ws + p.k;
  void* v16 = ws + p.v16;
  void* route_q = ws + p.route_q;
  void* lmk = ws + p.lmk;
  float* entropy = reinterpret_cast<float*>(ws + p.entropy);
  float* prior = reinterpret_cast<float*>(ws + p.prior);
  uint8_t* chunk_ok = reinterpret_cast<uint8_t*>(ws + p.chunk_ok);
  void* local_out = ws + p.local_out;
  float* local_lse = reinterpret_cast<float*>(ws + p.local_lse);
  int32_t* indices = reinterpret_cast<int32_t*>(ws + p.indices);
  void* scores = ws + p.scores;
  void* remote_w = ws + p.remote_w;
  void* local_w = ws + p.local_w;
  void* route_keys = ws + p.route_keys;

  const int64_t B = a->batch, L = a->seq_len, Hq = a->q_heads, Hkv = a->kv_heads,
                D = a->head_dim, G = Hq / Hkv, C = L / mrsa::kChunk;
  const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
  int rc;
  rc = mrsa_rope(a->q_pre, q, Hq, a->k_pre, k, Hkv, a->position_ids, a->inv_freq,
                 a->attention_factor, nullptr, nullptr, MRSA_F32, B, L, D, stream);
  if (rc) return rc;
  // V in fp16: both attention kernels then carry P as one fp16 tile instead
  // of bf16 hi + lo
  rc = mrsa_convert_bf16_to_f16(a->v, v16, B * L * Hkv * D, stream);
  if (rc) return rc;
  rc = mrsa_local_attention_f16v(q, k, v16, a->key_valid, local_out, local_lse,
                            a->local_window + mrsa::kChunk - 1, 1, mrsa::kChunk, sm_scale, B, L, L,
                            0, Hq, Hkv, D, stream);
  if (rc) return rc;
  rc = mrsa_qcal_route_query(a->hidden, q, a->w_in, a->w_out, a->norm_weight, a->rms_eps,
                             a->qcal_scale, a->position_ids, a->inv_freq, a->attention_factor,
                             route_q, B, L, a->hidden_size, a->rank, Hq, D, stream);
  if (rc) return rc;
  const __nv_bfloat16* mu = static_cast<const __nv_bfloat16*>(route_q) + (mrsa::kChunk - 1) * Hq * D;
  rc = mrsa_chunk_pool(mu, L * Hq * D, mrsa::kChunk * Hq * D, k, a->key_valid, sm_scale,
                       a->bias_scale, lmk, entropy, prior, chunk_ok, B, C, Hkv, G, D, stream);
  if (rc) return rc;
  rc = mrsa_route_topk(route_q, lmk, 1, local_lse, prior, nullptr, chunk_ok, a->local_window, 0,
                       indices, scores, MRSA_BF16, remote_w, local_w, MRSA_WEIGHTS_AFFINE,
                       a->temperature, a->gate_scale, a->gate_offset, B, L, C, Hkv, G, D,
                       a->topk, route_keys, mrsa_route_topk_workspace_size(B, L, C, Hkv, G, MRSA_BF16),
                       stream);
  if (rc) return rc;
  return mrsa_selected_attention_f16v(q, k, v16, a->key_valid, remote_w, indices, local_out, local_w,
                                 a->out, sm_scale, 1, B, L, L, Hkv, G, D, a->topk, mrsa::kChunk,
                                 stream);
}
