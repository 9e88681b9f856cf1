"""CPU restatement of the Fast-dLLM cached decode step (oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``; never by the product
package.

``cached_route_layer_step`` follows ``dream_dllm_hils/fastdllm_attention.py:
70-382 cached_attention_forward`` for a HiLS route layer, composed from the
oracle's own per-op restatements (each pinned to the reference by the golden
fixtures): RoPE of the partial rows, the cache update (``fastdllm_cache.py:
100-127``), the local branch at the rows' cache positions
(``local_attention.py:147 cached_local_attention``), Q-Cal of the partial
rows, the landmark refresh of the affected chunks (``:254-312``), the drop
mask rows, routing (``route_topk_g7(training=False)``), one softmax over
remote and local logits (``_route_weights_torch`` with no gate, temperature
1 -- ``:292-303``), selected attention over the cache and the fusion.
"""

from __future__ import annotations

import math

import torch

from . import route_layer as orc

__all__ = ["cached_local_rows", "cached_route_layer_step", "cached_swa_layer_step"]


def cached_local_rows(q, key, value, key_valid, positions, window: int, chunk: int, skip_inert_slots: bool):
    """Banded attention of query rows at cache ``positions`` (``[M]``) over the
    cache: the rows of :func:`oracle.route_layer.local_attention` at those
    positions (``dream_dllm_hils/local_attention.py:147-197``)."""
    b, m, hq, d = q.shape
    l, hkv = key.shape[1], key.shape[2]
    g = hq // hkv
    valid = key_valid.bool().clone()
    if skip_inert_slots:
        valid = valid & ((torch.arange(l) + 1) % chunk != 0)[None]
    w = window + chunk - 1 if skip_inert_slots else window
    sc = valid.to(key.dtype)[:, :, None, None]
    kz, vz = key * sc, value * sc
    out = torch.empty(b, m, hq, d, dtype=q.dtype)
    lse = torch.empty(b, m, hq, dtype=torch.float32)
    for r in range(m):
        p = int(positions[r])
        ks, ke = max(0, p - w), min(l, p + w + 1)
        kb = kz[:, ks:ke].float().repeat_interleave(g, dim=2)           # [B,n,Hq,D]
        vb = vz[:, ks:ke].float().repeat_interleave(g, dim=2)
        s = torch.einsum("bhd,bnhd->bhn", q[:, r].float(), kb) / math.sqrt(d)
        ls = torch.logsumexp(s, dim=-1)
        out[:, r] = torch.einsum("bhn,bnhd->bhd", torch.exp(s - ls[..., None]), vb).to(q.dtype)
        lse[:, r] = ls
    return out, lse


def _apply_update(cache, q_pre, k_pre, v, position_ids, query_positions, kv_update_positions, cfg):
    inv, af = orc.yarn_inv_freq(q_pre.shape[-1], cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
    cos, sin = orc.rope_cos_sin(position_ids, inv, af)
    q = orc.apply_rope(q_pre, cos, sin)
    k = orc.apply_rope(k_pre, cos, sin)
    cache = {n: (t.clone() if isinstance(t, torch.Tensor) else t) for n, t in cache.items()}
    rows = torch.searchsorted(query_positions, kv_update_positions)
    cache["key"].index_copy_(1, kv_update_positions, k.index_select(1, rows))
    cache["value"].index_copy_(1, kv_update_positions, v.index_select(1, rows).to(cache["value"].dtype))
    return q, cos, sin, cache


def cached_route_layer_step(cache: dict, q_pre, k_pre, v, hidden, position_ids, query_positions,
                            kv_update_positions, affected_chunks, weights: dict, cfg=orc.MRSAConfig()):
    """One cached step of a route layer.  ``cache``: ``key``/``value``
    ``[1,L,Hkv,D]``, ``key_valid [1,L]``, ``landmark_keys [1,C,Hkv,G,D]``,
    ``prior_bias [1,C,Hkv,G]``; ``weights``: ``w_in``, ``w_out``,
    ``norm_weight``, ``entropy_bias_scale``.  Returns ``(out [1,M,Hq,D] bf16,
    new cache, intermediates)``."""
    q, cos, sin, cache = _apply_update(cache, q_pre, k_pre, v, position_ids, query_positions,
                                       kv_update_positions, cfg)
    _, m, hq, d = q.shape
    hkv = cache["key"].shape[2]
    g = hq // hkv
    chunk = cfg.chunk
    local_o, local_lse = cached_local_rows(q, cache["key"], cache["value"], cache["key_valid"], query_positions,
                                           cfg.local_window, chunk, True)
    route_q = orc.qcal_route_query(hidden, q, weights["w_in"], weights["w_out"], weights["norm_weight"], cos, sin,
                                   eps=cfg.rms_eps, scale=cfg.qcal_scale)
    if affected_chunks.numel():
        lrows = torch.searchsorted(query_positions, affected_chunks * chunk + chunk - 1)
        mu = route_q.index_select(1, lrows).reshape(1, -1, hkv, g, d)
        span = (affected_chunks[:, None] * chunk + torch.arange(chunk)[None]).reshape(-1)
        kc = cache["key"].index_select(1, span).reshape(1, -1, chunk, hkv, d)
        vc = cache["key_valid"].index_select(1, span).reshape(1, -1, chunk)
        lmk, ent = orc.chunk_pool(mu, kc, vc)
        prior = ent * weights["entropy_bias_scale"].float().view(1, 1, hkv, g)
        cache["landmark_keys"].index_copy_(1, affected_chunks, lmk)
        cache["prior_bias"].index_copy_(1, affected_chunks, prior)
    drop = orc.remote_drop_mask(cache["key_valid"], cfg.local_window, chunk).index_select(1, query_positions)
    idx, scores = orc.route_topk_blocked(route_q, cache["landmark_keys"], local_lse.view(1, m, hkv, g),
                                         cache["prior_bias"], drop, cfg.topk)
    rw, lw = orc.route_weights_plain(scores, idx, cache["prior_bias"], local_lse)
    remote = orc.selected_attention(q, cache["key"], cache["value"], rw, idx, cache["key_valid"], chunk)
    out = orc.fuse_outputs(remote, local_o, lw)
    inter = {"q": q, "route_q": route_q, "local_out": local_o, "local_lse": local_lse, "drop": drop,
             "indices": idx, "scores": scores, "remote_weights": rw, "local_weight": lw,
             "route_key": orc.route_keys(route_q, cache["landmark_keys"], local_lse.view(1, m, hkv, g),
                                         cache["prior_bias"], drop)}
    return out, cache, inter


def cached_route_layer_rows_with(cache: dict, q, route_q, local_o, local_lse, indices, chunk: int = 64):
    """The steps after routing for given selections (to compare attention
    independently of near-tie routing flips): scores, one-softmax weights,
    selected attention over the cache, fusion."""
    scores = orc.route_scores_at(route_q, cache["landmark_keys"], indices)
    rw, lw = orc.route_weights_plain(scores, indices, cache["prior_bias"], local_lse)
    remote = orc.selected_attention(q, cache["key"], cache["value"], rw, indices, cache["key_valid"], chunk)
    return orc.fuse_outputs(remote, local_o, lw)


def cached_swa_layer_step(cache: dict, q_pre, k_pre, v, position_ids, query_positions, kv_update_positions,
                          window: int = 1280, cfg=orc.MRSAConfig()):
    """The sliding-window branch (``fastdllm_attention.py:214-244``)."""
    q, _, _, cache = _apply_update(cache, q_pre, k_pre, v, position_ids, query_positions, kv_update_positions, cfg)
    out, _ = cached_local_rows(q, cache["key"], cache["value"], cache["key_valid"], query_positions, window,
                               cfg.chunk, False)
    return out, cache
