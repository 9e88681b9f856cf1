/*
 * mrsa.h -- C ABI of the B200 (sm_100a) MRSA route-layer / SWA-layer forward.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream, launches on that stream, never allocates, frees or synchronises,
 * and returns 0 or a negative MRSA_ERR_* code (no exceptions, no aborts).
 * Tensors are dense row-major in the reference's BLHD layouts:
 *   q            [B, L, Hq, D]   bf16        (Hq = Hkv * G, D = 128)
 *   k, v         [B, L, Hkv, D]  bf16
 *   key_valid    [B, L]          uint8 (0/1), NULL = every key valid
 *   landmarks    [B, C, Hkv, G, D] bf16      (C = L / 64 chunks)
 *   prior/entropy[B, C, Hkv, G]  fp32
 *   local_lse    [B, L, Hq]      fp32 (natural log)
 *   indices      [B, L, Hkv, K]  int32, ascending, -1 last
 *   scores / remote weights [B, L, Hq, K] bf16; local weight [B, L, Hq] bf16
 * Pointers (key_valid included) must be 16-byte aligned.  Entry points are
 * stateless and re-entrant (any host thread, any stream) with two
 * exceptions, described at their declarations: mrsa_route_layer_forward_noalloc
 * shares one scratch area per device between calls, and the device error
 * flags read by mrsa_device_error_flags are process-wide.
 */
#ifndef MRSA_B200_H
#define MRSA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* mrsa_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum {
  MRSA_OK = 0,
  MRSA_ERR_NULL = -1,      /* a required pointer is NULL */
  MRSA_ERR_SHAPE = -2,     /* inconsistent or unsupported shape */
  MRSA_ERR_ALIGN = -3,     /* a pointer is not 16-byte aligned */
  MRSA_ERR_LAUNCH = -4,    /* CUDA rejected the launch */
  MRSA_ERR_ARG = -5,       /* bad scalar argument */
  MRSA_ERR_WORKSPACE = -6  /* workspace missing or too small */
};

enum { MRSA_BF16 = 0, MRSA_F32 = 1 };                 /* cos/sin and score dtypes */
enum { MRSA_WEIGHTS_AFFINE = 0, MRSA_WEIGHTS_SOFTMAX = 1 };
enum { MRSA_GEMM_PLAIN = 0, MRSA_GEMM_SWIGLU = 1, MRSA_GEMM_RESIDUAL = 2 };   /* mrsa_gemm_bf16 epilogues */

const char* mrsa_strerror(int code);
/* The CUDA error (name, message and the entry point or step that met it)
 * behind the last MRSA_ERR_LAUNCH returned on the calling host thread; "" if
 * none.  The string stays valid until the thread's next failing call. */
const char* mrsa_last_error(void);
int mrsa_abi_version(void);

/* YaRN inverse frequencies [dim/2] and attention factor, host-side.
 * Replaces transformers ROPE_INIT_FUNCTIONS['yarn'] as used by Dream's rotary
 * module (dream_dllm_hils/train_fulltext.py:2873-2888). */
int mrsa_yarn_inv_freq(int dim, double base, double factor, int orig_max_pos, double beta_fast,
                       double beta_slow, int truncate, float* inv_freq_out,
                       float* attention_factor_out);

/* fp32 rotate-half RoPE on one or two BLHD bf16 tensors (x1 may be NULL).
 * cos/sin come either from position_ids [B,L] int64 + inv_freq [D/2] fp32 +
 * attention_factor (HF rotary rule: fp32 pos*inv_freq, cos*factor), or from
 * explicit cos/sin [B,L,D] of dtype cs_dtype.  y may alias x.
 * Replaces ops/rope_tilelang_fp32.py:84 rope_rotary_pos_emb and :173
 * single_tensor_rope_autograd (forward), and the torch RoPE of
 * dream_dllm_hils/attention.py:41-52 / :384-393. */
int mrsa_rope(const void* x0, void* y0, int64_t heads0, const void* x1, void* y1, int64_t heads1,
              const int64_t* position_ids, const float* inv_freq, float attention_factor,
              const void* cos, const void* sin, int cs_dtype, int64_t batch, int64_t seq_len,
              int64_t head_dim, mrsa_stream_t stream);

/* Q-Cal routing query: route_q = rope(rmsnorm(invrope(q) + scale*bf16(bf16(h W_in^T) W_out^T))),
 * q the RoPE'd query, h [B,L,hidden], W_in [rank,hidden], W_out [Hq*D,rank] bf16,
 * norm_weight [D] fp32, cos/sin from position_ids (as in mrsa_rope).
 * Replaces _qcal_delta + _finish_calibrated_query (dream_dllm_hils/attention.py:458-511). */
int mrsa_qcal_route_query(const void* hidden, const void* q, const void* w_in, const void* w_out,
                          const float* norm_weight, float eps, float scale,
                          const int64_t* position_ids, const float* inv_freq,
                          float attention_factor, void* route_q, int64_t batch, int64_t seq_len,
                          int64_t hidden_size, int64_t rank, int64_t q_heads, int64_t head_dim,
                          mrsa_stream_t stream);

/* Landmark attention pool + entropy prior.  mu_q element (b,c,h,g,d) is read at
 * mu_q + b*mu_stride_b + c*mu_stride_c + (h*G+g)*D + d (elements); k [B,C*64,Hkv,D].
 * Writes landmarks, entropy, optionally prior = entropy*bias_scale[h*G+g] and
 * chunk_ok [B,C] (1 = chunk has a valid non-landmark key).
 * Replaces ops/chunk_attn_pool_gqa_tilelang.py:425 chunk_attn_pool_gqa (forward). */
int mrsa_chunk_pool(const void* mu_q, int64_t mu_stride_b, int64_t mu_stride_c, const void* k,
                    const uint8_t* key_valid, float sm_scale, const float* bias_scale,
                    void* landmarks, float* entropy, float* prior, uint8_t* chunk_ok,
                    int64_t batch, int64_t chunks, int64_t kv_heads, int64_t groups,
                    int64_t head_dim, mrsa_stream_t stream);

/* Dense 1 = drop mask [B,L,C] int32 (chunk overlaps the chunk-aligned local
 * window or has no valid non-landmark key).
 * Replaces dream_dllm_hils/kernel_utils.py:102 remote_drop_mask (allowed_mask=None). */
int mrsa_remote_drop_mask(const uint8_t* key_valid, int32_t* out, int64_t batch, int64_t seq_len,
                          int64_t window, int64_t chunk, mrsa_stream_t stream);

/* The rows of that mask for query rows at cache positions `positions`
 * [q_len] int64 (each in [0, seq_len)): out [B,q_len,C] int32.  The Fast-dLLM
 * cached step's drop mask, remote_drop_mask(...).index_select(1, positions)
 * (dream_dllm_hils/fastdllm_attention.py:279-283), without the dense [B,L,C]. */
int mrsa_remote_drop_mask_positions(const uint8_t* key_valid, const int64_t* positions, int32_t* out,
                                    int64_t batch, int64_t seq_len, int64_t q_len, int64_t window, int64_t chunk,
                                    mrsa_stream_t stream);

/* Post-softmax max-pooled top-K chunk routing + optional route weights.
 * route_q [B,Lq,Hq,D] (query rows at global positions q_offset..), landmarks
 * [B,C,Hkv,G,D] (lmk_per_qhead=1) or [B,C,Hkv,D] (0), local_lse [B,Lq,Hq],
 * bias [B,C,Hq] or NULL.  Dropped chunks: drop_mask [B,Lq,C] int32 if given,
 * else the inline rule from chunk_ok [B,C] (NULL = all valid) and window
 * (window < 0: nothing dropped).  scores_out dtype: scores_dtype.
 * remote_w/local_w (both or neither) get the route weights of
 * mode MRSA_WEIGHTS_AFFINE (_route_weights_torch with gate scale/offset) or
 * MRSA_WEIGHTS_SOFTMAX (route_weights).
 * workspace: at least mrsa_route_topk_workspace_size() bytes of device memory
 * (the fp32 max-pooled keys [B,Lq,Hkv,C] and the raw scores [B,Lq,Hq,C] in the
 * scores dtype), 16-byte aligned; MRSA_ERR_WORKSPACE when missing or short.
 * Replaces ops/topk_head_softmax.py:15 ref_softmax_topk_max_pooling and :1242
 * online_softmax_topk_head (post_softmax, non-causal), dream_dllm_hils/routing.py:52
 * route_topk_g7, and fuses dream_dllm_hils/attention.py:126 _route_weights_torch. */
int mrsa_route_topk(const void* route_q, const void* landmarks, int lmk_per_qhead,
                    const float* local_lse, const float* bias, const int32_t* drop_mask,
                    const uint8_t* chunk_ok, int64_t window, int64_t q_offset,
                    int32_t* indices, void* scores_out, int scores_dtype, void* remote_w,
                    void* local_w, int weight_mode, float temperature, float gate_scale,
                    float gate_offset, int64_t batch, int64_t q_len, int64_t chunks,
                    int64_t kv_heads, int64_t groups, int64_t head_dim, int64_t topk,
                    void* workspace, size_t workspace_bytes, mrsa_stream_t stream);

/* Device workspace bytes of mrsa_route_topk (0 for an invalid shape).  No
 * reference counterpart: the reference materialises its scores instead. */
size_t mrsa_route_topk_workspace_size(int64_t batch, int64_t q_len, int64_t chunks,
                                      int64_t kv_heads, int64_t groups, int scores_dtype);

/* Route weights from scores [B,L,Hq,K] bf16, indices [B,L,Hkv,K] int32,
 * prior [B,C,Hkv,G] fp32, local_lse [B,L,Hq] fp32.
 * Replaces ops/hils_bidir_route_weights_tilelang.py:276 route_weights (any K<=32)
 * and dream_dllm_hils/attention.py:126 _route_weights_torch (no Gumbel / value bonus). */
int mrsa_route_weights(const void* scores, const int32_t* indices, const float* prior,
                       const float* local_lse, void* remote_w, void* local_w, int weight_mode,
                       float temperature, float gate_scale, float gate_offset, int64_t batch,
                       int64_t seq_len, int64_t chunks, int64_t kv_heads, int64_t groups,
                       int64_t topk, mrsa_stream_t stream);

/* Bidirectional banded GQA attention: query row i (global position q_offset+i)
 * attends keys j with |pos_i - j| <= window.  Keys that are invalid or, with
 * skip_inert, landmark slots ((j+1)%chunk==0) have K and V treated as zero
 * (logit 0, no value).  Writes out [B,Lq,Hq,D] bf16 and lse [B,Lq,Hq] fp32 (or NULL).
 * Replaces dream_dllm_hils/local_attention.py:110 bidir_local_attention (flash-attn
 * window (W,W)) and, with skip_inert=0, the SWA layer's call at attention.py:1210. */
int mrsa_local_attention(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                         void* out, float* lse, int64_t window, int skip_inert, int64_t chunk,
                         float sm_scale, int64_t batch, int64_t q_len, int64_t kv_len,
                         int64_t q_offset, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                         mrsa_stream_t stream);

/* mrsa_local_attention with V given in fp16 ([B,Lk,Hkv,D] fp16): P then
 * travels as one fp16 tile instead of bf16 hi + lo (half the P.V work).  No
 * counterpart in the reference: the fused layer uses it after
 * mrsa_convert_bf16_to_f16 on V. */
int mrsa_local_attention_f16v(const void* q, const void* k, const void* v_f16, const uint8_t* key_valid,
                              void* out, float* lse, int64_t window, int skip_inert, int64_t chunk,
                              float sm_scale, int64_t batch, int64_t q_len, int64_t kv_len,
                              int64_t q_offset, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                              mrsa_stream_t stream);

/* mrsa_local_attention for query rows at arbitrary positions of the K/V
 * cache: row i sits at query_positions[i] (int64 [q_len], shared by the batch,
 * each in [0, kv_len)) and attends keys j with |query_positions[i] - j| <=
 * window, with the same zeroed-key rules.  Replaces
 * dream_dllm_hils/local_attention.py:147 cached_local_attention (the
 * Fast-dLLM cached decode step). */
int mrsa_local_attention_positions(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                                   const int64_t* query_positions, void* out, float* lse, int64_t window,
                                   int skip_inert, int64_t chunk, float sm_scale, int64_t batch,
                                   int64_t q_len, int64_t kv_len, int64_t q_heads, int64_t kv_heads,
                                   int64_t head_dim, mrsa_stream_t stream);

/* Causal chunk-expanded window attention: query row i sits at absolute
 * position p = kv_start + (kv_len - q_len) + i and sees keys j (absolute
 * kv_start + j) in [start, p], start = p - window + 1, rounded down to a
 * multiple of chunk when expand_to_chunk; with mask_lmk the landmark slots
 * ((kv_start + j + 1) % chunk == 0) are excluded from the softmax.  Writes
 * out [B,Lq,Hq,D] bf16 and lse [B,Lq,Hq] fp32 natural log (or NULL); rows
 * without a visible key give 0 and -inf.  q_len <= kv_len, sm_scale > 0.
 * Replaces ops/flex_attn_tilelang.py:1261 flex_attn_tl (forward). */
int mrsa_flex_attention(const void* q, const void* k, const void* v, void* out, float* lse,
                        int64_t window, int64_t chunk, int mask_lmk, int expand_to_chunk,
                        int64_t kv_start, float sm_scale, int64_t batch, int64_t q_len,
                        int64_t kv_len, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                        mrsa_stream_t stream);

/* Weighted per-chunk-softmax attention over the selected chunks, optionally
 * fused with the local branch: out = bf16(bf16(remote) + local_w*local) when
 * local_out and local_w are given, else bf16(remote).
 * weights [B,Lq,Hq,K] bf16, indices [B,Lq,Hkv,K] int32, k/v [B,Lk,Hkv,D].
 * Replaces ops/hils_fwd_bwd_head.py:1113 HiLS_block_M_head (forward),
 * dream_dllm_hils/routing.py:305 selected_attention_g7 and
 * ops/hils_bidir_output_fusion_tilelang.py:138 fuse_hils_outputs. */
int mrsa_selected_attention(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                            const void* weights, const int32_t* indices, const void* local_out,
                            const void* local_w, void* out, float sm_scale, int mask_last_token,
                            int64_t batch, int64_t q_len, int64_t kv_len, int64_t kv_heads,
                            int64_t groups, int64_t head_dim, int64_t topk, int64_t chunk,
                            mrsa_stream_t stream);

/* mrsa_selected_attention with V given in fp16 ([B,Lk,Hkv,D] fp16, every
 * other argument as above).  P then travels as one fp16 tile (11 significant
 * bits) instead of bf16 hi + lo, which halves the P.V work.  No counterpart in the reference: the fused
 * layer uses it after mrsa_convert_bf16_to_f16 on V. */
int mrsa_selected_attention_f16v(const void* q, const void* k, const void* v_f16, const uint8_t* key_valid,
                                 const void* weights, const int32_t* indices, const void* local_out,
                                 const void* local_w, void* out, float sm_scale, int mask_last_token,
                                 int64_t batch, int64_t q_len, int64_t kv_len, int64_t kv_heads,
                                 int64_t groups, int64_t head_dim, int64_t topk, int64_t chunk,
                                 mrsa_stream_t stream);

/* Backward of mrsa_selected_attention (bf16 q, k, v; no local merge, no token
 * refinement): given grad_out [B,Lq,Hq,D] bf16 writes dq [B,Lq,Hq,D], dk and
 * dv [B,Lk,Hkv,D] in fp32 (every element, dk/dv of unselected keys 0) and dw
 * [B,Lq,Hq,K] bf16 (dw of slot k = sum_s P dP over its chunk; 0 for an empty
 * slot).  The softmax gradient dS and w*P are rounded to bf16 before their
 * GEMMs.  dK/dV are summed per chunk over an inverted chunk -> (query, slot)
 * index in query order (no atomics: every run gives the same bits).  workspace: at least
 * mrsa_selected_attention_backward_workspace() bytes, 16-byte aligned.
 * Sets bit 4 of mrsa_device_error_flags if a CTA gave up on a bounded wait.
 * Replaces the backward of ops/hils_fwd_bwd_head.py:915-1098
 * (_hils_block_M_attention_inverse, kernel :573-910). */
int mrsa_selected_attention_backward(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                                     const void* weights, const int32_t* indices, const void* grad_out,
                                     float* dq, float* dk, float* dv, void* dw, float sm_scale,
                                     int mask_last_token, int64_t batch, int64_t q_len, int64_t kv_len,
                                     int64_t kv_heads, int64_t groups, int64_t head_dim, int64_t topk,
                                     int64_t chunk, void* workspace, size_t ws_bytes, mrsa_stream_t stream);
/* Workspace of mrsa_selected_attention_backward: chunk counts and offsets
 * (B*Hkv*C int32 each), per-256-query-block chunk counts (B*Hkv*ceil(Lq/256)*C
 * int32) and the inverted index (B*Lq*Hkv*K int32). */
size_t mrsa_selected_attention_backward_workspace(int64_t batch, int64_t q_len, int64_t kv_len,
                                                  int64_t kv_heads, int64_t topk);

/* Backward of mrsa_chunk_pool (landmarks and entropy): mu_q [B,C,Hkv,G,D]
 * bf16 contiguous, k [B,C*64,Hkv,D] bf16, key_valid as in the forward,
 * grad_landmarks [B,C,Hkv,G,D] bf16 and grad_entropy [B,C,Hkv,G] fp32 (either
 * NULL = zero) -> d_mu [B,C,Hkv,G,D] and d_k [B,C*64,Hkv,D] bf16.  The pool
 * probabilities and entropy are recomputed; the softmax gradient is rounded to
 * bf16 before its GEMMs, as in the reference kernel.  G <= 16, D = 128.
 * Replaces the backward of ops/chunk_attn_pool_gqa_tilelang.py:328-393
 * (_ChunkAttnPoolGQA, kernel _pool_gqa_bwd :183-325). */
int mrsa_chunk_pool_backward(const void* mu_q, const void* k, const uint8_t* key_valid,
                             const void* grad_landmarks, const float* grad_entropy, void* d_mu, void* d_k,
                             float sm_scale, int64_t batch, int64_t chunks, int64_t kv_heads, int64_t groups,
                             int64_t head_dim, mrsa_stream_t stream);

/* Backward of mrsa_route_weights: grad_remote [B,L,Hq,K] and grad_local
 * [B,L,Hq] bf16 -> d_scores [B,L,Hq,K] fp32 (0 on empty slots), d_prior
 * [B,C,Hkv,G] fp32 (cleared, then summed over the slots that selected each
 * chunk), d_local_lse [B,L,Hq] fp32 and d_gate[2] fp32 = the gradients of
 * gate_scale and gate_offset (cleared, then summed over rows; in
 * MRSA_WEIGHTS_SOFTMAX mode d_gate[0] = 0).  Rows whose logits are all
 * masked get zero gradients; a row with no selected chunk adds 0 to
 * d_gate[0] (torch autograd of the reference gives NaN there).
 * Replaces the backward of ops/hils_bidir_route_weights_tilelang.py:190-255
 * (_RouteWeights, kernel :97-166) and torch autograd through
 * dream_dllm_hils/attention.py:126-227 _route_weights_torch (affine gate). */
int mrsa_route_weights_backward(const void* scores, const int32_t* indices, const float* prior,
                                const float* local_lse, const void* grad_remote, const void* grad_local,
                                float* d_scores, float* d_prior, float* d_local_lse, float* d_gate,
                                int weight_mode, float temperature, float gate_scale, float gate_offset,
                                int64_t batch, int64_t seq_len, int64_t chunks, int64_t kv_heads,
                                int64_t groups, int64_t topk, mrsa_stream_t stream);

/* Backward of the gathered routing scores s[b,l,hq,k] = q[b,l,hq] .
 * landmarks[b,c_k,hq] * sm_scale (c_k = indices[b,l,hq/G,k]): q [B,L,Hq,D]
 * and landmarks [B,C,Hkv,G,D] bf16, grad_scores [B,L,Hq,K] bf16 -> d_q
 * [B,L,Hq,D] and d_landmarks [B,C,Hkv,G,D] fp32 (every element written); G <= 8.
 * d_landmarks is summed per chunk over an inverted index built in
 * workspace (mrsa_route_scores_backward_workspace bytes, 16-byte aligned).
 * Replaces ops/topk_head_softmax.py:1071-1122 (SoftmaxTopKMaxPooling
 * backward, per-query-head landmarks). */
int mrsa_route_scores_backward(const void* q, const void* landmarks, const int32_t* indices,
                               const void* grad_scores, float* d_q, float* d_landmarks, float sm_scale,
                               int64_t batch, int64_t q_len, int64_t chunks, int64_t kv_heads, int64_t groups,
                               int64_t head_dim, int64_t topk, void* workspace, size_t ws_bytes,
                               mrsa_stream_t stream);
size_t mrsa_route_scores_backward_workspace(int64_t batch, int64_t q_len, int64_t chunks, int64_t kv_heads,
                                            int64_t topk);

/* Backward of mrsa_fuse_outputs: d_remote = bf16(g), d_local = bf16(g * w),
 * d_local_w = bf16(sum_d g * local) over rows = B*L*H rows of head_dim.
 * Replaces ops/hils_bidir_output_fusion_tilelang.py:38-99,117-130. */
int mrsa_fuse_outputs_backward(const void* local, const void* local_w, const void* grad_out, void* d_remote,
                               void* d_local, void* d_local_w, int64_t rows, int64_t head_dim,
                               mrsa_stream_t stream);

/* Backward of mrsa_local_attention (bf16 V): from the forward's inputs q
 * [B,L,Hq,D], k, v [B,L,Hkv,D] bf16 (q and k as the forward took them), key
 * validity, its output `out` [B,L,Hq,D] bf16 and natural-log `lse` [B,L,Hq]
 * fp32, and grad_out [B,L,Hq,D] bf16 plus grad_lse [B,L,Hq] fp32 (NULL =
 * zero), writes dq [B,L,Hq,D] and dk, dv [B,L,Hkv,D] in fp32 (every element;
 * zeroed keys -- invalid, or landmark slots with skip_inert -- get 0).  The
 * softmax gradient dS and P are rounded to bf16 before their GEMMs.
 * `window` is the effective window (|i - j| <= window), L % 64 == 0, G <= 8.
 * workspace: mrsa_local_attention_backward_workspace() bytes (the per-row
 * dO.O - dlse terms).  Sets bit 6 of mrsa_device_error_flags if a CTA gave up
 * on a bounded wait.  Replaces the backward of the flash-attn call inside
 * dream_dllm_hils/local_attention.py:110-144 bidir_local_attention. */
int mrsa_local_attention_backward(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                                  const void* out, const float* lse, const void* grad_out, const float* grad_lse,
                                  float* dq, float* dk, float* dv, void* workspace, size_t ws_bytes,
                                  int64_t window, int skip_inert, int64_t chunk, float sm_scale, int64_t batch,
                                  int64_t seq_len, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                  mrsa_stream_t stream);
size_t mrsa_local_attention_backward_workspace(int64_t batch, int64_t seq_len, int64_t q_heads);

/* Dense bf16 GEMM of the Dream-shaped forward's projections and MLP (no
 * reference counterpart: the reference runs them in Dream's remote modeling
 * code through torch): C = A[M,K] . B[N,K]^T with fp32 accumulation and a
 * fused epilogue -- MRSA_GEMM_PLAIN: C[M,N] = bf16(acc + bias[N]) (bias may
 * be NULL); MRSA_GEMM_SWIGLU: B's rows interleaved per 256-row block as
 * [gate n0..n0+127 ; up n0..n0+127], C[M,N/2] = bf16(bf16(silu(bf16(gate))) *
 * bf16(up)); MRSA_GEMM_RESIDUAL: C[M,N] = bf16(residual[M,N] + bf16(acc)).
 * N % 8 == 0 (N % 256 == 0 for SwiGLU), K % 64 == 0, row-major, 16-byte
 * aligned pointers.  Sets bit 5
 * of mrsa_device_error_flags if a CTA gave up on a bounded wait. */
int mrsa_gemm_bf16(const void* a, const void* b, const void* bias, const void* residual, void* c, int64_t m,
                   int64_t n, int64_t k, int epilogue, mrsa_stream_t stream);

/* Qwen2RMSNorm over rows of dim bf16 values: y = w * bf16(x * rsqrt(mean(x^2)
 * + eps)) with fp32 statistics (dim % 8 == 0). */
int mrsa_rms_norm(const void* x, const void* weight, void* y, int64_t rows, int64_t dim, float eps,
                  mrsa_stream_t stream);

/* Candidate token scores [B,Lq,Hkv,K,S] fp32: for chunk c = indices[b,l,h,i]
 * and slot s, max over the G = q_heads/kv_heads heads of the group of
 * q_g . k[c*S+s] * sm_scale; -inf when c < 0 (or c >= kv_len/S), s == S-1 or
 * key_valid (uint8 [B,Lk], NULL = all valid) is 0.  q [B,Lq,Hq,D], k
 * [B,Lk,Hkv,D] bf16, indices [B,Lq,Hkv,K] int32; S >= 16, kv_len % S == 0,
 * G <= 16.  Replaces ops/hils_token_score_gqa_tilelang.py:174
 * candidate_token_scores_gqa. */
int mrsa_candidate_token_scores(const void* q, const void* k, const int32_t* indices,
                                const uint8_t* key_valid, float* scores, float sm_scale,
                                int64_t batch, int64_t q_len, int64_t kv_len, int64_t q_heads,
                                int64_t kv_heads, int64_t head_dim, int64_t selected, int64_t chunk,
                                mrsa_stream_t stream);

/* Exact selected-token GQA attention: query row (b,l) attends the tokens
 * indices[b,l,t] (int32, clamped to [0, kv_len)) whose valid[b,l,t] (uint8)
 * is nonzero; fp32 softmax of q.k*sm_scale, probabilities rounded to bf16,
 * fp32 P.V; rows without a valid token are 0.  q [B,Lq,Hq,D], k/v
 * [B,Lk,Hkv,D] bf16, out like q; G <= 16 and the kernel's shared memory
 * (mrsa_selected_token_attention_smem) at most 227 KB.
 * Replaces ops/dsa_selected_attention_tilelang.py:593
 * selected_token_attention_tilelang (forward). */
int mrsa_selected_token_attention(const void* q, const void* k, const void* v, const int32_t* indices,
                                  const uint8_t* valid, void* out, float sm_scale, int64_t batch,
                                  int64_t q_len, int64_t kv_len, int64_t q_heads, int64_t kv_heads,
                                  int64_t head_dim, int64_t topk, mrsa_stream_t stream);

/* Dynamic shared memory bytes mrsa_selected_token_attention needs for
 * `groups` heads per KV head and `topk` tokens per row (0 if out of range). */
size_t mrsa_selected_token_attention_smem(int64_t groups, int64_t topk);

/* mrsa_selected_attention (v_f16 = 0) or mrsa_selected_attention_f16v
 * (v_f16 != 0) with token refinement: token_keep [B,Lq,Hkv,K,chunk] int8
 * (16-byte aligned) drops key s of slot k for query l and KV head h where it
 * is 0, on top of the key-validity and landmark masks; a chunk whose keys are
 * all dropped contributes nothing.  A chunk listed twice by one query uses
 * the keep row of its first slot.  Replaces the token_keep argument of
 * ops/hils_fwd_bwd_head.py:1113 HiLS_block_M_head (kernel :453-507) and
 * dream_dllm_hils/routing.py:305 selected_attention_g7. */
int mrsa_selected_attention_keep(const void* q, const void* k, const void* v, const uint8_t* key_valid,
                                 const void* weights, const int32_t* indices, const int8_t* token_keep,
                                 const void* local_out, const void* local_w, void* out, float sm_scale,
                                 int mask_last_token, int v_f16, int64_t batch, int64_t q_len,
                                 int64_t kv_len, int64_t kv_heads, int64_t groups, int64_t head_dim,
                                 int64_t topk, int64_t chunk, mrsa_stream_t stream);

/* n bf16 values (n a multiple of 8, 16-byte aligned buffers) to fp16, round to
 * nearest; values beyond +-65504 (infinities too) saturate and set bit 3 of
 * mrsa_device_error_flags.  No counterpart in the reference (V preparation
 * for mrsa_selected_attention_f16v). */
int mrsa_convert_bf16_to_f16(const void* in, void* out, int64_t n, mrsa_stream_t stream);

/* Self-test of the bounded in-kernel waits (failure detection without a GPU
 * fault): one CTA whose warp 0 waits on an mbarrier nothing arrives on, with
 * `rounds` (1..4000) bounded rounds, and whose warp 1 waits on another with
 * the kernels' full limit.  Writes result[0] = 1 (warp 0 gave up), result[1] =
 * 1 (the CTA's abort flag was raised), result[2] = 1 (warp 1 left through the
 * flag) to the device ints `result[0..2]`.  No reference counterpart. */
int mrsa_wait_selftest(int* result, int rounds, mrsa_stream_t stream);

/* Bit mask of device-side failures recorded since the last clear: bit 0 = a
 * selected-attention CTA gave up waiting on one of its internal barriers (its
 * output rows are then incomplete); bit 1 = a routing key CTA did (its keys,
 * hence its selections, are then incomplete); bit 2 = a local-window CTA did;
 * bit 3 = mrsa_convert_bf16_to_f16 saturated a value; bit 4 = a CTA of the
 * selected-attention backward gave up on a wait (its gradients are then
 * incomplete); bit 5 = a GEMM CTA did; bit 6 = a CTA of the local-window
 * backward did.  Synchronises the current device; with
 * clear != 0 also resets the mask.  Negative on a CUDA error.  Replaces the
 * reference's host-side kernel-fallback reporting (dream_dllm_hils/attention.py:932-940). */
int mrsa_device_error_flags(int clear);

/* Measurement helper with no reference counterpart: the L2 -> shared-memory
 * ceiling of the selected-attention loads.  One CTA per SM loads
 * `items_per_cta` work items, each the 64-row K and V tiles of a pseudo-random
 * (chunk, KV head) of k, v [kv_len, kv_heads, 128] (2-byte elements) plus
 * `owners` (0..8) 8-row boxes of q [q_rows, 128] -- the selected kernel's
 * tensor-map boxes -- and computes nothing.  Bytes moved per launch = SMs x
 * items_per_cta x (32768 + 2048 x owners).  Sets *status (device int) to 1 if
 * a CTA gave up on a bounded wait. */
int mrsa_probe_tile_gather(const void* k, const void* v, const void* q, int64_t kv_len, int64_t kv_heads,
                           int64_t q_rows, int owners, int64_t items_per_cta, int* status,
                           mrsa_stream_t stream);

/* out = bf16(remote + local_w * local) over rows = B*L*H, each of head_dim.
 * Replaces ops/hils_bidir_output_fusion_tilelang.py:138 fuse_hils_outputs. */
int mrsa_fuse_outputs(const void* remote, const void* local, const void* local_w, void* out,
                      int64_t rows, int64_t head_dim, mrsa_stream_t stream);

/* ---------------------------------------------------------------- layers */
typedef struct {
  /* inputs (device) */
  const void* q_pre;          /* [B,L,Hq,D] bf16, before RoPE */
  const void* k_pre;          /* [B,L,Hkv,D] bf16, before RoPE */
  const void* v;              /* [B,L,Hkv,D] bf16 */
  const void* hidden;         /* [B,L,hidden] bf16 (Q-Cal input) */
  const int64_t* position_ids;/* [B,L] */
  const uint8_t* key_valid;   /* [B,L] or NULL */
  const float* inv_freq;      /* [D/2] */
  const void* w_in;           /* [rank,hidden] bf16 */
  const void* w_out;          /* [Hq*D,rank] bf16 */
  const float* norm_weight;   /* [D] */
  const float* bias_scale;    /* [Hq] entropy_bias_scale */
  /* output */
  void* out;                  /* [B,L,Hq,D] bf16, pre o_proj */
  /* scalars */
  float attention_factor, rms_eps, qcal_scale, temperature, gate_scale, gate_offset;
  int64_t batch, seq_len, q_heads, kv_heads, head_dim, hidden_size, rank;
  int64_t topk, local_window;
} mrsa_route_layer_args;

/* Bytes of workspace mrsa_route_layer_forward needs (256-byte aligned pieces). */
size_t mrsa_route_layer_workspace_size(const mrsa_route_layer_args* a);

/* Whole route layer on one device: RoPE, local branch, Q-Cal, landmark pool,
 * routing + weights, selected attention fused with the local branch.
 * Replaces KernelDreamFullHiLSAttention.forward (dream_dllm_hils/attention.py:1313-1774)
 * from the projected q/k/v/h to the input of o_proj.  The attention kernels
 * take V in fp16 (the layer converts it once): V values beyond +-65504 (and
 * infinities) saturate to +-65504 and set bit 3 of mrsa_device_error_flags,
 * so a caller that cannot rule such values out reads the flags after the
 * call. */
int mrsa_route_layer_forward(const mrsa_route_layer_args* a, void* workspace, size_t ws_bytes,
                             mrsa_stream_t stream);

/* Size of the device scratch built into the library for
 * mrsa_route_layer_forward_noalloc (held by every GPU that loads it). */
#define MRSA_NOALLOC_SCRATCH_BYTES (32u << 20)

/* The route layer of mrsa_route_layer_forward for callers that cannot
 * allocate device memory (a plugin inside a framework that owns all device
 * allocations, a server with a fixed memory pool).  It has no counterpart in
 * the reference.  Instead of a caller
 * workspace it uses MRSA_NOALLOC_SCRATCH_BYTES of scratch inside the library
 * image: problems whose mrsa_route_layer_workspace_size exceeds that (about
 * 1200 tokens of the Dream shape) are rejected with MRSA_ERR_WORKSPACE before
 * anything runs.  Runs on the current device; its first call on a device
 * looks up the scratch address (cudaGetSymbolAddress), so make that first
 * call before any stream capture; the address is looked up again when the
 * device's context has changed since (after a cudaDeviceReset).  All calls on a device share the scratch:
 * calls whose GPU work overlaps race, so order them on one stream.  Nothing
 * in the scratch needs to start at zero.  Allocates and frees nothing. */
int mrsa_route_layer_forward_noalloc(const mrsa_route_layer_args* a, mrsa_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MRSA_B200_H */
