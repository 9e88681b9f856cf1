"""CPU restatement of the MRSA route-layer and SWA-layer forward (oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU legs of ``bench.py``; never by the product package.

Every function restates, in plain torch on the CPU, one step of the
reference's own PyTorch path for the route layer
(``dream_dllm_hils/attention.py:1313-1820``, eval mode, canonical config) and
cites the reference file:line it follows.  Storage dtypes follow the
reference (bf16 activations, fp32 statistics); math is fp32.  Two documented
choices:

* RoPE math is fp32 with fp32 cos/sin and one bf16 rounding, i.e. the
  semantics of the reference's ``ops/rope_tilelang_fp32.py:14-88`` kernel.
  The live reference path rounds cos/sin and every product to bf16
  (``dream_dllm_hils/attention.py:41-52``); ``rope_precision="bf16"`` selects
  that chain instead.
* The local window branch is a restatement of
  ``dream_dllm_hils/local_attention.py:35-107``: the reference calls the
  third-party ``flash_attn_func`` there, which has no CPU implementation.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

__all__ = [
    "MRSAConfig",
    "yarn_inv_freq",
    "landmark_position_ids",
    "rope_cos_sin",
    "rotate_half",
    "apply_rope",
    "invert_rope",
    "rms_norm",
    "qcal_route_query",
    "chunk_pool",
    "remote_drop_mask",
    "route_topk",
    "route_topk_blocked",
    "route_weights_affine",
    "route_weights_plain",
    "local_attention",
    "selected_attention",
    "fuse_outputs",
    "make_route_layer_inputs",
    "route_layer_forward",
    "route_layer_shared",
    "route_layer_rows",
    "remote_drop_mask_rows",
    "swa_layer_forward",
    "topk_set_agreement",
    "route_keys",
    "route_scores_at",
]


@dataclass(frozen=True)
class MRSAConfig:
    """Hot-path constants of the canonical config
    (``configs/from_dense16k/hils-s2-qcal-rmsnorm-rand-s1000-jingneng.json``)."""

    chunk: int = 64            # chunk_size
    topk: int = 32             # hils_topk
    local_window: int = 256    # local_window (route layers)
    swa_window: int = 1280     # swa_local_window (the 21 other layers)
    head_dim: int = 128
    q_heads: int = 28
    kv_heads: int = 4
    qcal_rank: int = 64
    rope_theta: float = 1.0e6
    yarn_factor: float = 8.0
    yarn_orig_max_pos: int = 2048
    rms_eps: float = 1e-6
    qcal_scale: float = 1.0    # qcal_scale (attention.py:473-475)
    route_temperature: float = 1.0
    rope_precision: str = "fp32"

    @property
    def groups(self) -> int:
        return self.q_heads // self.kv_heads


# ---------------------------------------------------------------- RoPE / YaRN
def yarn_inv_freq(dim: int, base: float, factor: float, orig_max_pos: int,
                  beta_fast: float = 32.0, beta_slow: float = 1.0,
                  truncate: bool = True):
    """YaRN inverse frequencies and attention factor.

    Restates the published YaRN rule (Peng et al. 2023) as implemented by the
    third-party ``transformers`` ``ROPE_INIT_FUNCTIONS['yarn']`` (5.5.0 here;
    the reference pins no version) that Dream's rotary module uses
    (``dream_dllm_hils/train_fulltext.py:2873-2888``, config lines 4-9).
    """
    def corr_dim(rot):
        return dim * math.log(orig_max_pos / (rot * 2 * math.pi)) / (2 * math.log(base))

    lo, hi = corr_dim(beta_fast), corr_dim(beta_slow)
    if truncate:
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, dim - 1)
    if lo == hi:
        hi += 0.001
    pos_freqs = base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim)
    extrap = 1.0 / pos_freqs
    interp = 1.0 / (factor * pos_freqs)
    ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
    keep_extrap = 1 - ramp
    inv_freq = interp * (1 - keep_extrap) + extrap * keep_extrap
    attn_factor = 1.0 if factor <= 1 else 0.1 * math.log(factor) + 1.0
    return inv_freq, float(attn_factor)


def landmark_position_ids(batch: int, seq_len: int, chunk: int = 64) -> torch.Tensor:
    """Position ids of the landmark layout (``dream_dllm_hils/data.py:1000-1012``):
    text slot s<chunk-1 of chunk c sits at c*(chunk-1)+s, and the landmark at
    the last text position + 1, i.e. slot i -> i - i//chunk."""
    i = torch.arange(seq_len, dtype=torch.long)
    return (i - i // chunk).unsqueeze(0).expand(batch, seq_len).contiguous()


def rope_cos_sin(position_ids: torch.Tensor, inv_freq: torch.Tensor, attn_factor: float,
                 dtype=torch.float32):
    """cos/sin ``[B, L, D]`` as the HF rotary module computes them: fp32
    ``pos * inv_freq``, duplicated halves, times the attention factor, cast
    to ``dtype``."""
    freqs = position_ids.to(torch.float32)[..., None] * inv_freq.to(torch.float32)
    emb = torch.cat((freqs, freqs), dim=-1)
    return (emb.cos() * attn_factor).to(dtype), (emb.sin() * attn_factor).to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """``dream_dllm_hils/attention.py:35-38``."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               precision: str = "fp32") -> torch.Tensor:
    """RoPE on BLHD ``x`` with ``[B, L, D]`` cos/sin.

    ``fp32``: ``ops/rope_tilelang_fp32.py:14-88`` (fp32 math, one rounding).
    ``bf16``: ``dream_dllm_hils/attention.py:41-52`` evaluated in bf16.
    """
    c, s = cos[:, :, None, :], sin[:, :, None, :]
    if precision == "bf16":
        c, s = c.to(torch.bfloat16), s.to(torch.bfloat16)
        return (x * c) + (rotate_half(x) * s)
    xf = x.float()
    return (xf * c.float() + rotate_half(xf) * s.float()).to(x.dtype)


def invert_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                precision: str = "fp32") -> torch.Tensor:
    """``invert_rotary_pos_emb`` (``dream_dllm_hils/attention.py:55-63``):
    ``x*cos - rotate_half(x)*sin``.  With YaRN's attention factor this is
    not an exact inverse; it is reproduced literally."""
    c, s = cos[:, :, None, :], sin[:, :, None, :]
    if precision == "bf16":
        c, s = c.to(torch.bfloat16), s.to(torch.bfloat16)
        return (x * c) - (rotate_half(x) * s)
    xf = x.float()
    return (xf * c.float() - rotate_half(xf) * s.float()).to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``dream_dllm_hils/qcal.py:22-26``."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + float(eps))
    return (weight.float() * xf).to(x.dtype)


def qcal_route_query(hidden: torch.Tensor, q: torch.Tensor, w_in: torch.Tensor,
                     w_out: torch.Tensor, norm_weight: torch.Tensor, cos, sin, *,
                     eps: float = 1e-6, scale: float = 1.0,
                     precision: str = "fp32") -> torch.Tensor:
    """Q-Cal routing query ``rope(rmsnorm(invrope(q) + scale*W_out W_in h))``.

    Follows ``_qcal_delta`` and ``_finish_calibrated_query``
    (``dream_dllm_hils/attention.py:458-503``): the two bias-free bf16 linear
    layers round their outputs to bf16, the residual add is a bf16 add, the
    RMSNorm runs in fp32 and returns bf16.
    """
    b, l, hq, d = q.shape
    t = (hidden.float() @ w_in.float().t()).to(torch.bfloat16)
    delta = (t.float() @ w_out.float().t()).to(torch.bfloat16).view(b, l, hq, d)
    if scale != 1.0:
        delta = delta * float(scale)
    q_unrot = invert_rope(q, cos, sin, precision)
    combined = (q_unrot.float() + delta.float()).to(torch.bfloat16)
    combined = rms_norm(combined, norm_weight, eps)
    return apply_rope(combined, cos, sin, precision)


# ------------------------------------------------------------ landmark pool
def chunk_pool(mu_q: torch.Tensor, k_chunked: torch.Tensor, key_valid: torch.Tensor,
               sm_scale: float | None = None):
    """Attention-pool chunk summaries plus entropy prior.

    ``_compact_pool_torch`` (``ops/chunk_attn_pool_gqa_tilelang.py:17-37``):
    ``mu_q [B,C,Hkv,G,D]``, ``k_chunked [B,C,S,Hkv,D]``, ``key_valid [B,C,S]``;
    softmax over the valid non-landmark slots, ``lmk = sum p k`` (bf16),
    ``entropy = -sum p ln p`` (fp32).  A chunk with no valid slot gives zeros.
    """
    d = mu_q.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(d)
    logits = torch.einsum("bckgd,bcskd->bckgs", mu_q.float(), k_chunked.float()) * sm_scale
    ok = key_valid.bool().clone()
    ok[..., -1] = False
    logits = logits.masked_fill(~ok[:, :, None, None, :], float("-inf"))
    p = torch.nan_to_num(torch.softmax(logits, dim=-1), nan=0.0)
    lmk = torch.einsum("bckgs,bcskd->bckgd", p, k_chunked.float())
    plogp = torch.where(p > 0, p * p.clamp_min(1e-30).log(), torch.zeros_like(p))
    return lmk.to(k_chunked.dtype), -plogp.sum(dim=-1)


def remote_drop_mask(key_valid: torch.Tensor, window: int, chunk: int) -> torch.Tensor:
    """1 = chunk not routable for the query (``dream_dllm_hils/kernel_utils.py:75-161``):
    it overlaps the chunk-aligned local window
    ``[floor(max(i-W,0)/S)*S, (floor(min(i+W,L-1)/S)+1)*S)`` or it has no valid
    non-landmark key.  Returns int32 ``[B, L, C]``."""
    b, l = key_valid.shape
    c = l // chunk
    pos = torch.arange(l)
    real = (pos + 1) % chunk != 0
    chunk_ok = (key_valid.bool() & real[None]).view(b, c, chunk).any(-1)
    lo = (pos - window).clamp_min(0) // chunk
    hi = (pos + window).clamp_max(l - 1) // chunk
    cid = torch.arange(c)
    local = (cid[None, :] >= lo[:, None]) & (cid[None, :] <= hi[:, None])
    return (local[None] | ~chunk_ok[:, None, :]).to(torch.int32)


def remote_drop_mask_rows(key_valid: torch.Tensor, window: int, chunk: int, qs: slice) -> torch.Tensor:
    """The rows ``qs`` of :func:`remote_drop_mask` (the same rule evaluated
    for those query positions only; the whole mask is 1 GB at 131072
    tokens)."""
    b, l = key_valid.shape
    c = l // chunk
    real = (torch.arange(l) + 1) % chunk != 0
    chunk_ok = (key_valid.bool() & real[None]).view(b, c, chunk).any(-1)
    pos = torch.arange(l)[qs]
    lo = (pos - window).clamp_min(0) // chunk
    hi = (pos + window).clamp_max(l - 1) // chunk
    cid = torch.arange(c)
    local = (cid[None, :] >= lo[:, None]) & (cid[None, :] <= hi[:, None])
    return (local[None] | ~chunk_ok[:, None, :]).to(torch.int32)


# ---------------------------------------------------------------- routing
def route_topk(q5: torch.Tensor, lmks: torch.Tensor, lse_local: torch.Tensor, topk: int,
               drop_mask: torch.Tensor | None, bias: torch.Tensor | None):
    """Post-softmax max-pooled top-k chunk selection, eval mode.

    ``ref_softmax_topk_max_pooling`` (``ops/topk_head_softmax.py:15-156``)
    with ``is_causal=False``, per-query-head landmarks, no Gumbel noise:
    ``x = q.lmk/sqrt(D) + bias``; ``T = logaddexp(lse_local, logsumexp_c x)``;
    ``key_c = max_g (x - T)``; dropped chunks ``-inf``; top-k; unselectable
    slots ``-1``; indices sorted ascending with ``-1`` last; scores are the
    raw ``q.lmk/sqrt(D)`` (no bias) per query head, ``-inf`` at ``-1``.

    q5 ``[B,L,Hkv,G,D]``; lmks ``[B,C,Hkv*G,D]``; lse_local ``[B,L,Hkv,G]``;
    bias ``[B,C,Hkv,G]``; drop_mask ``[B,L,C]``.  Returns indices
    ``[B,L,Hkv,K]`` int64 and scores ``[B,L,Hkv,G,K]`` fp32.
    """
    b, l, hkv, g, d = q5.shape
    c = lmks.shape[1]
    lm = lmks.view(b, c, hkv, g, d).float()
    raw = torch.einsum("blhgd,bchgd->blhgc", q5.float(), lm) * (1.0 / math.sqrt(d))
    x = raw if bias is None else raw + bias.float().permute(0, 2, 3, 1)[:, None]
    total = torch.logaddexp(lse_local.float(), torch.logsumexp(x, dim=-1))
    key = (x - total[..., None]).max(dim=3).values                    # [B,L,Hkv,C]
    if drop_mask is not None:
        key = key.masked_fill(drop_mask.bool()[:, :, None, :], float("-inf"))
    kk = min(topk, c)
    vals, idx = torch.topk(key, kk, dim=-1, sorted=False)
    idx[vals == float("-inf")] = -1
    if kk < topk:
        idx = torch.cat((idx, idx.new_full((b, l, hkv, topk - kk), -1)), dim=-1)
    big = c + 1000
    idx = torch.where(idx < 0, torch.full_like(idx, big), idx).sort(dim=-1).values
    idx[idx >= c] = -1
    safe = idx.clamp_min(0)[:, :, :, None, :].expand(b, l, hkv, g, topk)
    scores = torch.gather(raw, -1, safe)
    scores = scores.masked_fill(idx[:, :, :, None, :] < 0, float("-inf"))
    return idx, scores


def route_topk_blocked(route_q: torch.Tensor, lmks5: torch.Tensor, local_lse4: torch.Tensor,
                       prior_bias: torch.Tensor, drop_mask: torch.Tensor, topk: int,
                       block: int = 1024):
    """``route_topk_g7(training=False)`` (``dream_dllm_hils/routing.py:132-171``):
    1024-query blocks through :func:`route_topk`; scores cast to the query
    dtype (bf16).  route_q ``[B,L,Hq,D]``, lmks5 ``[B,C,Hkv,G,D]``.
    Returns indices ``[B,L,Hkv,K]`` int64, scores ``[B,L,Hq,K]`` bf16."""
    b, l, hq, d = route_q.shape
    c, hkv, g = lmks5.shape[1:4]
    lm = lmks5.reshape(b, c, hq, d)
    out_i, out_s = [], []
    for s in range(0, l, block):
        e = min(s + block, l)
        i, sc = route_topk(route_q[:, s:e].reshape(b, e - s, hkv, g, d), lm,
                           local_lse4[:, s:e], topk, drop_mask[:, s:e], prior_bias)
        out_i.append(i)
        out_s.append(sc.reshape(b, e - s, hq, topk).to(route_q.dtype))
    return torch.cat(out_i, 1), torch.cat(out_s, 1)


def route_keys(route_q: torch.Tensor, lmks5: torch.Tensor, local_lse4: torch.Tensor,
               prior_bias: torch.Tensor, drop_mask: torch.Tensor) -> torch.Tensor:
    """The max-pooled selection key ``[B,L,Hkv,C]`` of :func:`route_topk`
    (dropped chunks ``-inf``), for gap-aware selection comparisons."""
    b, l, hq, d = route_q.shape
    c, hkv, g = lmks5.shape[1:4]
    raw = torch.einsum("blhgd,bchgd->blhgc", route_q.float().view(b, l, hkv, g, d),
                       lmks5.float()) * (1.0 / math.sqrt(d))
    x = raw + prior_bias.float().permute(0, 2, 3, 1)[:, None]
    total = torch.logaddexp(local_lse4.float(), torch.logsumexp(x, dim=-1))
    key = (x - total[..., None]).max(dim=3).values
    return key.masked_fill(drop_mask.bool()[:, :, None, :], float("-inf"))


def route_scores_at(route_q: torch.Tensor, lmks5: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Raw scaled scores ``[B,L,Hq,K]`` (bf16, ``-inf`` at ``-1``) of given
    selections, as :func:`route_topk` gathers them."""
    b, l, hq, d = route_q.shape
    c, hkv, g = lmks5.shape[1:4]
    k = indices.shape[-1]
    raw = torch.einsum("blhgd,bchgd->blhgc", route_q.float().view(b, l, hkv, g, d),
                       lmks5.float()) * (1.0 / math.sqrt(d))
    idx = indices.long()
    sc = torch.gather(raw, -1, idx.clamp_min(0)[:, :, :, None, :].expand(b, l, hkv, g, k))
    sc = sc.masked_fill(idx[:, :, :, None, :] < 0, float("-inf"))
    return sc.reshape(b, l, hq, k).to(route_q.dtype)


def route_weights_affine(scores: torch.Tensor, indices: torch.Tensor, prior_bias: torch.Tensor,
                         local_lse: torch.Tensor, *, temperature: float = 1.0,
                         gate_offset: float = 0.0, gate_scale: float = 1.0):
    """Route weights of the live path, ``_route_weights_torch`` affine-gate
    branch (``dream_dllm_hils/attention.py:126-227``, taken because
    ``fusion_gate_scale`` exists, ``:913-914``).

    ``r_k = score_k + bias[idx_k]`` (``-inf`` for ``idx<0``);
    ``gate = scale*(logsumexp(r/T) - local_lse/T) + offset``; ``m = sigmoid``;
    ``remote = softmax(r/T)*m``, ``local = 1-m`` (both bf16)."""
    b, l, hq, k = scores.shape
    c, hkv, g = prior_bias.shape[1:4]
    idx = indices.long().repeat_interleave(g, dim=2)
    valid = (idx >= 0) & (idx < c)
    safe = idx.clamp(0, c - 1)
    bias_h = prior_bias.reshape(b, c, hq).permute(0, 2, 1)[:, None].expand(b, l, hq, c)
    r = (scores.float() + torch.gather(bias_h, -1, safe)).masked_fill(~valid, float("-inf"))
    logits = torch.cat((r, local_lse.float()[..., None]), -1) / float(temperature)
    all_masked = torch.isneginf(logits).all(-1, keepdim=True)
    logits = torch.where(all_masked, torch.zeros_like(logits), logits)
    gate = torch.logsumexp(logits[..., :k], -1) - logits[..., k]
    m = torch.sigmoid(float(gate_scale) * gate + float(gate_offset))
    inner = torch.softmax(r / float(temperature), -1)
    inner = torch.where((~valid).all(-1, keepdim=True), torch.zeros_like(inner), inner)
    remote = (inner * m[..., None]).to(scores.dtype)
    local = (1.0 - m).to(scores.dtype)
    remote = torch.where(all_masked, torch.zeros_like(remote), remote)
    local = torch.where(all_masked[..., 0], torch.zeros_like(local), local)
    return remote, local


def route_weights_plain(scores, indices, prior_bias, local_lse):
    """``route_weights`` (``ops/hils_bidir_route_weights_tilelang.py:15-95,276``):
    one softmax over ``[score_k + bias[idx_k] (k<K), local_lse]``; remote
    weights are its first K entries, the local weight its last."""
    b, l, hq, k = scores.shape
    c, hkv, g = prior_bias.shape[1:4]
    idx = indices.long().repeat_interleave(g, dim=2)
    valid = (idx >= 0) & (idx < c)
    bias_h = prior_bias.reshape(b, c, hq).permute(0, 2, 1)[:, None].expand(b, l, hq, c)
    r = (scores.float() + torch.gather(bias_h, -1, idx.clamp(0, c - 1))).masked_fill(~valid, float("-inf"))
    p = torch.softmax(torch.cat((r, local_lse.float()[..., None]), -1), -1)
    p = torch.nan_to_num(p, nan=0.0)
    return p[..., :k].to(torch.bfloat16), p[..., k].to(torch.bfloat16)


# ------------------------------------------------------------ attention
def local_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, key_valid: torch.Tensor,
                    window: int, chunk: int, skip_inert_slots: bool, block: int = 256):
    """Bidirectional banded GQA attention with natural-log LSE.

    ``bidir_local_attention`` (``dream_dllm_hils/local_attention.py:110-144``):
    keys at invalid slots (and, with ``skip_inert_slots``, at landmark slots)
    have K and V multiplied by zero -- still in the softmax with logit 0 --
    and the window is ``W + chunk - 1`` with ``skip_inert_slots`` else ``W``
    (``:35-64``); keys with ``|i - j| <= window`` attend (flash-attn
    ``window_size=(W, W)``).  Returns o ``[B,L,Hq,D]`` bf16, lse ``[B,L,Hq]`` fp32.
    """
    b, l, hq, d = q.shape
    hkv = k.shape[2]
    g = hq // hkv
    valid = key_valid.bool()
    if skip_inert_slots:
        pos = torch.arange(l)
        valid = valid & ((pos + 1) % chunk != 0)[None]
    w = window + chunk - 1 if skip_inert_slots else window
    scale = valid.to(k.dtype)[:, :, None, None]
    kz, vz = k * scale, v * scale
    out = torch.empty(b, l, hq, d, dtype=q.dtype)
    lse = torch.empty(b, l, hq, dtype=torch.float32)
    for s in range(0, l, block):
        e = min(s + block, l)
        ks, ke = max(0, s - w), min(l, e - 1 + w + 1)
        qb = q[:, s:e].float()                                      # [B,n,Hq,D]
        kb = kz[:, ks:ke].float().repeat_interleave(g, dim=2)        # [B,m,Hq,D]
        vb = vz[:, ks:ke].float().repeat_interleave(g, dim=2)
        sc = torch.einsum("bnhd,bmhd->bhnm", qb, kb) / math.sqrt(d)
        qi = torch.arange(s, e)[:, None]
        kj = torch.arange(ks, ke)[None, :]
        sc = sc.masked_fill(((qi - kj).abs() > w)[None, None], float("-inf"))
        lse_b = torch.logsumexp(sc, dim=-1)                          # [B,Hq,n]
        p = torch.exp(sc - lse_b[..., None])
        out[:, s:e] = torch.einsum("bhnm,bmhd->bnhd", p, vb).to(q.dtype)
        lse[:, s:e] = lse_b.permute(0, 2, 1)
    return out, lse


def selected_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, weights: torch.Tensor,
                       indices: torch.Tensor, key_valid: torch.Tensor | None, chunk: int,
                       block: int = 128, out_dtype=torch.bfloat16, token_keep: torch.Tensor | None = None):
    """Weighted per-chunk softmax attention over the selected chunks.

    ``hils_torch_ref`` (``ops/hils_fwd_bwd_head.py:21-93``, ``block_q=1``,
    ``mask_last_token=True``) with the key-validity mask of the kernel it
    checks (``ops/hils_fwd_bwd_head.py:440-446``):
    ``out = sum_k w_k * softmax_s(q.K_{idx_k,s}/sqrt(D))_{s valid, s!=S-1} V_{idx_k,s}``.
    Slots with ``idx<0`` and chunks with no valid key contribute nothing.
    ``token_keep`` ``[B,L,Hkv,K,S]`` (token refinement) further masks key s of
    slot k per (query, KV head) where it is zero (``:453-507``; the weighted
    per-chunk reference of ``unittests/test_hils_non_power_two_topk.py:122-135``).
    """
    b, l, hq, d = q.shape
    hkv = k.shape[2]
    g = hq // hkv
    c = k.shape[1] // chunk
    kc = k[:, : c * chunk].view(b, c, chunk, hkv, d).float()
    vc = v[:, : c * chunk].view(b, c, chunk, hkv, d).float()
    ok = torch.ones(b, c, chunk, dtype=torch.bool) if key_valid is None else \
        key_valid.bool()[:, : c * chunk].view(b, c, chunk).clone()
    ok[..., -1] = False
    out = torch.empty(b, l, hq, d, dtype=out_dtype)
    kidx = indices.shape[-1]
    for s in range(0, l, block):
        e = min(s + block, l)
        idx = indices[:, s:e].long()                                 # [B,n,Hkv,K]
        sel = idx >= 0
        safe = idx.clamp_min(0)
        bi = torch.arange(b)[:, None, None, None]
        hi = torch.arange(hkv)[None, None, :, None]
        kg = kc[bi, safe, :, hi]                                     # [B,n,Hkv,K,S,D]
        vg = vc[bi, safe, :, hi]
        okg = ok[bi, safe]                                           # [B,n,Hkv,K,S]
        if token_keep is not None:
            okg = okg & (token_keep[:, s:e] != 0)
        qg = q[:, s:e].float().view(b, e - s, hkv, g, d)
        sc = torch.einsum("bnhgd,bnhksd->bnhgks", qg, kg) / math.sqrt(d)
        sc = sc.masked_fill(~okg[:, :, :, None], float("-inf"))
        p = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
        ok_k = torch.einsum("bnhgks,bnhksd->bnhgkd", p, vg)
        w = weights[:, s:e].float().view(b, e - s, hkv, g, kidx)
        w = w.masked_fill(~sel[:, :, :, None, :], 0.0)
        out[:, s:e] = torch.einsum("bnhgkd,bnhgk->bnhgd", ok_k, w).reshape(b, e - s, hq, d).to(out_dtype)
    return out


def fuse_outputs(remote: torch.Tensor, local: torch.Tensor, local_weight: torch.Tensor) -> torch.Tensor:
    """``fuse_hils_outputs`` (``ops/hils_bidir_output_fusion_tilelang.py:15-37``):
    ``bf16(remote + w_local * local)`` in fp32."""
    return (remote.float() + local_weight.float()[..., None] * local.float()).to(torch.bfloat16)


# ------------------------------------------------------------ whole layers
def make_route_layer_inputs(batch: int, seq_len: int, cfg: MRSAConfig = MRSAConfig(), *,
                            hidden: int = 3584, seed: int = 0, dtype=torch.bfloat16,
                            key_valid: torch.Tensor | None = None):
    """Seeded synthetic inputs of the BASELINE route-layer configs.

    A CPU ``torch.Generator`` seeded with ``seed`` draws, in this order:
    h ``[B,L,hidden]`` ~ N(0,1); q_pre ``[B,L,Hq,D]``, k_pre, v ``[B,L,Hkv,D]``
    ~ N(0,1)/sqrt(D); W_in ``[rank,hidden]`` and W_out ``[Hq*D,rank]`` ~
    N(0,0.02); a role offset ``[hidden]`` ~ N(0,0.02) added to h at landmark
    slots (the landmark type embedding, ``train_fulltext.py:2339-2351``).
    RMSNorm weight 1, entropy-bias scale 1, gate offset 0 / scale 1; position
    ids follow the landmark layout; key_valid all True unless given.
    """
    gen = torch.Generator().manual_seed(seed)
    hq, hkv, d = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    h = torch.randn(batch, seq_len, hidden, generator=gen)
    q = torch.randn(batch, seq_len, hq, d, generator=gen) / math.sqrt(d)
    k = torch.randn(batch, seq_len, hkv, d, generator=gen) / math.sqrt(d)
    v = torch.randn(batch, seq_len, hkv, d, generator=gen) / math.sqrt(d)
    w_in = torch.randn(cfg.qcal_rank, hidden, generator=gen) * 0.02
    w_out = torch.randn(hq * d, cfg.qcal_rank, generator=gen) * 0.02
    role = torch.randn(hidden, generator=gen) * 0.02
    lmk_slot = (torch.arange(seq_len) + 1) % cfg.chunk == 0
    h[:, lmk_slot] += role
    if key_valid is None:
        key_valid = torch.ones(batch, seq_len, dtype=torch.bool)
    return {
        "hidden": h.to(dtype), "q_pre": q.to(dtype), "k_pre": k.to(dtype), "v": v.to(dtype),
        "w_in": w_in.to(dtype), "w_out": w_out.to(dtype),
        "norm_weight": torch.ones(d, dtype=torch.float32),
        "entropy_bias_scale": torch.ones(hq, dtype=torch.float32),
        "gate_offset": 0.0, "gate_scale": 1.0,
        "position_ids": landmark_position_ids(batch, seq_len, cfg.chunk),
        "key_valid": key_valid,
    }


def route_layer_forward(inp: dict, cfg: MRSAConfig = MRSAConfig(), *, keep: bool = True,
                        query_slice: slice | None = None, indices: torch.Tensor | None = None,
                        shared: dict | None = None):
    """Route-layer forward from post-projection q/k/v/h to the pre-``o_proj``
    output, in the order of ``KernelDreamFullHiLSAttention.forward``
    (``dream_dllm_hils/attention.py:1358-1774``): RoPE, local branch, Q-Cal,
    landmark pool + entropy prior, drop mask, routing, route weights,
    selected attention, fusion.  ``query_slice`` restricts the per-query
    stages (local, routing, weights, selected, fusion) to a query range, the
    landmark pool still covers every chunk.  ``indices`` (for the sliced rows)
    replaces the oracle's own selection -- scores, weights and outputs are
    then evaluated on those chunks, which decouples near-tie selection flips
    from the attention comparison.  ``shared`` is the result of
    :func:`route_layer_shared` for the same inputs (computed here when not
    given).  Returns a dict of every intermediate (``keep``) plus ``out``.

    With a ``query_slice`` smaller than the sequence, the returned ``q`` and
    ``route_q`` hold only the rows that slice needs (the slice and the
    landmark rows; zero elsewhere): RoPE and Q-Cal are per-row maps, so the
    rows computed are exactly those of the whole-sequence result.
    """
    l = inp["q_pre"].shape[1]
    qs = query_slice or slice(0, l)
    if shared is None:
        shared = route_layer_shared(inp, cfg, query_slice=qs)
    return route_layer_rows(inp, shared, cfg, qs, keep=keep, indices=indices)


def route_layer_shared(inp: dict, cfg: MRSAConfig = MRSAConfig(), *,
                       query_slice: slice | None = None, rows: torch.Tensor | None = None):
    """The stages every query row shares: YaRN cos/sin, RoPE of K, Q-Cal of
    the landmark rows, landmark pool and entropy prior
    (``dream_dllm_hils/attention.py:1358-1430``).  RoPE and Q-Cal of the query
    rows run on ``rows`` (a bool ``[L]`` mask; default: the landmark rows plus
    ``query_slice``, or every row) only."""
    chunk, d = cfg.chunk, cfg.head_dim
    q_pre, k_pre = inp["q_pre"], inp["k_pre"]
    b, l, hq, _ = q_pre.shape
    hkv = k_pre.shape[2]
    g = hq // hkv
    c = l // chunk
    inv_freq, af = yarn_inv_freq(d, cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
    cos, sin = rope_cos_sin(inp["position_ids"], inv_freq, af)
    prec = cfg.rope_precision
    k = apply_rope(k_pre, cos, sin, prec)
    if rows is None:
        rows = torch.zeros(l, dtype=torch.bool)
        rows[query_slice or slice(0, l)] = True
        rows[chunk - 1::chunk] = True
    ridx = rows.nonzero().squeeze(1)
    full = bool(rows.all())
    q_rows = apply_rope(q_pre if full else q_pre[:, ridx], cos if full else cos[:, ridx],
                        sin if full else sin[:, ridx], prec)
    rq_rows = qcal_route_query(inp["hidden"] if full else inp["hidden"][:, ridx], q_rows,
                               inp["w_in"], inp["w_out"], inp["norm_weight"],
                               cos if full else cos[:, ridx], sin if full else sin[:, ridx],
                               eps=cfg.rms_eps, scale=cfg.qcal_scale, precision=prec)
    if full:
        q, route_q = q_rows, rq_rows
    else:
        q = torch.zeros_like(q_pre)
        q[:, ridx] = q_rows
        route_q = torch.zeros_like(q_pre)
        route_q[:, ridx] = rq_rows
    key_valid = inp["key_valid"].bool()
    mu_q = route_q[:, chunk - 1::chunk].reshape(b, c, hkv, g, d)
    lmk, entropy = chunk_pool(mu_q, k.view(b, c, chunk, hkv, d), key_valid.view(b, c, chunk))
    prior = entropy * inp["entropy_bias_scale"].float().view(1, 1, hkv, g)
    return {"q": q, "k": k, "route_q": route_q, "rows": rows, "lmk": lmk, "entropy": entropy,
            "prior_bias": prior, "cos": cos, "sin": sin, "key_valid": key_valid}


def route_layer_rows(inp: dict, shared: dict, cfg: MRSAConfig, qs: slice, *, keep: bool = True,
                     indices: torch.Tensor | None = None):
    """The per-query stages of the route layer on the query rows ``qs``
    (local branch, drop mask, routing, route weights, selected attention,
    fusion; ``dream_dllm_hils/attention.py:1380-1774``) over the shared
    stages of :func:`route_layer_shared`."""
    chunk = cfg.chunk
    v = inp["v"]
    q, k, route_q, lmk, prior = shared["q"], shared["k"], shared["route_q"], shared["lmk"], shared["prior_bias"]
    key_valid = shared["key_valid"]
    b, l, hq, _ = q.shape
    hkv = k.shape[2]
    g = hq // hkv
    assert bool(shared["rows"][qs].all()), "the shared stages did not compute these query rows"
    local_o, local_lse = _local_rows(q, k, v, key_valid, cfg.local_window, chunk, True, qs)
    drop = remote_drop_mask_rows(key_valid, cfg.local_window, chunk, qs)
    idx, scores = route_topk_blocked(route_q[:, qs], lmk, local_lse.view(b, -1, hkv, g), prior, drop, cfg.topk)
    if indices is not None:
        idx = indices.long().cpu()
        scores = route_scores_at(route_q[:, qs], lmk, idx)
    rw, lw = route_weights_affine(scores, idx, prior, local_lse, temperature=cfg.route_temperature,
                                  gate_offset=inp["gate_offset"], gate_scale=inp["gate_scale"])
    remote = _selected_rows(q, k, v, rw, idx, key_valid, chunk, qs)
    out = fuse_outputs(remote, local_o, lw)
    res = {"out": out}
    if keep:
        res.update(route_key=route_keys(route_q[:, qs], lmk, local_lse.view(b, -1, hkv, g), prior, drop))
        res.update(q=q, k=k, route_q=route_q, lmk=lmk, entropy=shared["entropy"], prior_bias=prior,
                   local_out=local_o, local_lse=local_lse, indices=idx, scores=scores,
                   remote_weights=rw, local_weight=lw, remote_out=remote, cos=shared["cos"],
                   sin=shared["sin"], rows=shared["rows"])
    return res


def _local_rows(q, k, v, key_valid, window, chunk, skip, qs):
    """:func:`local_attention` evaluated on the query rows ``qs`` only."""
    l = q.shape[1]
    start, stop = qs.start or 0, qs.stop if qs.stop is not None else l
    if start == 0 and stop == l:
        return local_attention(q, k, v, key_valid, window, chunk, skip)
    w = window + chunk - 1 if skip else window
    ks, ke = max(0, start - w) // chunk * chunk, min(l, stop + w)
    o, lse = local_attention(_pad_rows(q, ks, ke, start, stop), k[:, ks:ke], v[:, ks:ke],
                             key_valid[:, ks:ke], window, chunk, skip)
    return o[:, start - ks:stop - ks], lse[:, start - ks:stop - ks]


def _pad_rows(q, ks, ke, start, stop):
    out = torch.zeros(q.shape[0], ke - ks, *q.shape[2:], dtype=q.dtype)
    out[:, start - ks:stop - ks] = q[:, start:stop]
    return out


def _selected_rows(q, k, v, rw, idx, key_valid, chunk, qs):
    return selected_attention(q[:, qs], k, v, rw, idx, key_valid, chunk)


def swa_layer_forward(inp: dict, cfg: MRSAConfig = MRSAConfig(), window: int | None = None):
    """SWA layer (``KernelDreamSlidingWindowAttention.forward``,
    ``dream_dllm_hils/attention.py:1168-1220``): RoPE then
    ``bidir_local_attention(window=1280, skip_inert_slots=False)``."""
    d = cfg.head_dim
    inv_freq, af = yarn_inv_freq(d, cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
    cos, sin = rope_cos_sin(inp["position_ids"], inv_freq, af)
    q = apply_rope(inp["q_pre"], cos, sin, cfg.rope_precision)
    k = apply_rope(inp["k_pre"], cos, sin, cfg.rope_precision)
    o, lse = local_attention(q, k, inp["v"], inp["key_valid"], window or cfg.swa_window,
                             cfg.chunk, False)
    return {"out": o, "lse": lse, "q": q, "k": k}


# ------------------------------------------------------------ comparators
def topk_set_agreement(key: torch.Tensor, idx_a: torch.Tensor, idx_b: torch.Tensor,
                       topk: int, gap: float = 1e-3):
    """Gap-aware comparison of two top-k selections over the same ``key``
    ``[..., C]`` (the max-pooled routing key).  For each row: every chunk whose
    key is at least ``t33 + gap`` must be selected by both, and every chunk at
    most ``t32 - gap`` by neither (``t32``/``t33``: the 32nd/33rd largest
    key).  Returns ``(violations, exact_match_fraction)``."""
    c = key.shape[-1]
    srt = key.sort(dim=-1, descending=True).values
    t32 = srt[..., topk - 1] if c >= topk else torch.full(key.shape[:-1], float("-inf"))
    t33 = srt[..., topk] if c > topk else torch.full(key.shape[:-1], float("-inf"))

    def member(idx):
        # scatter_add: "-1" slots map to chunk 0 with weight 0 and never erase it
        m = torch.zeros(*key.shape, dtype=torch.int32)
        m.scatter_add_(-1, idx.clamp_min(0).long(), (idx >= 0).to(torch.int32))
        return m > 0

    ma, mb = member(idx_a), member(idx_b)
    must_in = (key >= t33[..., None] + gap) & torch.isfinite(key)
    must_out = key <= t32[..., None] - gap
    viol = (must_in & ~(ma & mb)) | (must_out & (ma | mb))
    exact = (ma == mb).all(-1).float().mean().item()
    return int(viol.sum().item()), exact
