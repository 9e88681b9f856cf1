"""CPU oracle for the token-granular ops and the causal flex window.

TEST INFRASTRUCTURE ONLY (same rules as ``oracle/route_layer.py``): the
checker for ``mrsa_b200.token_ops`` and ``mrsa_b200.local_attention.flex_attn_tl``,
never part of the product path.  Plain torch on the CPU, fp32 math on the
bf16 values.  Pinned against the reference's own torch functions by
``tests/golden/{token_scores,dsa,flex}.pt`` (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math

import torch


def candidate_token_scores(q: torch.Tensor, k: torch.Tensor, indices: torch.Tensor,
                           key_valid: torch.Tensor, chunk: int) -> torch.Tensor:
    """``[B, Lq, Hkv, K, S]`` fp32: max over the query group of the raw
    ``q_g . k`` of every slot of each selected chunk, divided by ``sqrt(D)``;
    ``-inf`` where the chunk index is outside ``[0, C)``, the slot is the
    chunk's last one or the key is invalid.
    Follows ``dream_dllm_hils/token_refinement.py:10-93``
    (``candidate_token_scores_reference``) and the kernel
    ``ops/hils_token_score_gqa_tilelang.py:61-114``."""
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    g = hq // hkv
    c = lk // chunk
    sel = indices.shape[-1]
    idx = indices.long()
    ok_chunk = (idx >= 0) & (idx < c)
    safe = idx.clamp(0, max(c - 1, 0))
    kc = k.float().view(b, c, chunk, hkv, d)
    qg = q.float().view(b, lq, hkv, g, d)
    out = torch.empty(b, lq, hkv, sel, chunk)
    valid = key_valid.bool().view(b, c, chunk)
    for bi in range(b):
        for h in range(hkv):
            keys = kc[bi, safe[bi, :, h], :, h]                       # [Lq, K, S, D]
            raw = torch.einsum("lgd,lksd->lksg", qg[bi, :, h], keys)   # [Lq, K, S, G]
            sc = raw.amax(-1) / math.sqrt(d)
            ok = valid[bi, safe[bi, :, h]] & ok_chunk[bi, :, h, :, None]
            ok[..., -1] = False
            out[bi, :, h] = torch.where(ok, sc, torch.full_like(sc, -math.inf))
    return out


def selected_token_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                             valid: torch.Tensor, sm_scale: float | None = None) -> torch.Tensor:
    """Exact GQA attention over per-row token lists, bf16 ``[B, Lq, Hq, D]``.
    Indices clamp to ``[0, Lk)``; invalid entries are ``-inf``; the fp32
    softmax (NaN rows -> 0) is rounded to the value dtype before ``P.V``.
    Follows ``dream_dllm_hils/dsa_attention.py:498-540``
    (``selected_token_attention_reference``, dropout off) and the kernel
    ``ops/dsa_selected_attention_tilelang.py:113-248``."""
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    g = hq // hkv
    scale = d ** -0.5 if sm_scale is None else sm_scale
    safe = indices.long().clamp(0, lk - 1)
    bidx = torch.arange(b)[:, None, None]
    ks = k[bidx, safe].float()                                        # [B, Lq, T, Hkv, D]
    vs = v[bidx, safe].float()
    qg = q.float().view(b, lq, hkv, g, d)
    scores = torch.einsum("blhgd,blthd->blhgt", qg, ks) * scale
    scores = scores.masked_fill(~valid.bool()[:, :, None, None, :], -math.inf)
    p = torch.nan_to_num(torch.softmax(scores, dim=-1), nan=0.0)
    p = p.to(v.dtype).float()
    out = torch.einsum("blhgt,blthd->blhgd", p, vs)
    return out.reshape(b, lq, hq, d).to(q.dtype)


def flex_window_mask(q_len: int, kv_len: int, window: int, chunk: int, mask_lmk: bool,
                     expand_to_chunk: bool, kv_start: int = 0) -> torch.Tensor:
    """``[Lq, Lk]`` bool: key j visible to query row i.  Row i sits at
    absolute position ``p = kv_start + Lk - Lq + i``; key j at
    ``kv_start + j``.  Follows ``ops/flex_attn_tilelang.py:115-215`` (and the
    torch mask of ``:1355-1380``)."""
    p = kv_start + (kv_len - q_len) + torch.arange(q_len)[:, None]
    j = kv_start + torch.arange(kv_len)[None, :]
    start = p - window + 1
    if expand_to_chunk:
        start = torch.div(start, chunk, rounding_mode="floor") * chunk
    keep = (j >= start) & (j <= p)
    if mask_lmk:
        keep = keep & ((j + 1) % chunk != 0)
    return keep


def flex_window_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int, chunk: int,
                          mask_lmk: bool = True, expand_to_chunk: bool = True, kv_start: int = 0,
                          sm_scale: float | None = None):
    """``(o [B, Lq, Hq, D] fp32, lse [B, Lq, Hq] natural log)`` of the causal
    chunk-expanded window: masked softmax over the visible keys, rows without
    one give 0 and ``-inf`` (``ops/flex_attn_tilelang.py:245-251``)."""
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    g = hq // hkv
    scale = d ** -0.5 if sm_scale is None else sm_scale
    keep = flex_window_mask(lq, lk, window, chunk, mask_lmk, expand_to_chunk, kv_start)
    qf = q.float().view(b, lq, hkv, g, d)
    s = torch.einsum("blhgd,bjhd->bhglj", qf, k.float()) * scale     # [B, Hkv, G, Lq, Lk]
    s = s.masked_fill(~keep, -math.inf)
    lse = torch.logsumexp(s, dim=-1)                                 # -inf on empty rows
    p = torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))[..., None])
    p = torch.where(keep, p, torch.zeros_like(p))
    o = torch.einsum("bhglj,bjhd->blhgd", p, v.float()).reshape(b, lq, hq, d)
    return o, lse.permute(0, 3, 1, 2).reshape(b, lq, hq)
