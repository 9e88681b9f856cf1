"""CPU restatement of the backward passes of the MRSA route-layer ops (oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``; never by the product
package.

Each function differentiates, with torch autograd in fp32 on the CPU, a
restatement of one forward op of the route layer, and names the reference
backward it stands for.  The reference's backward kernels round some
intermediates to bf16 (the softmax gradient tiles of the selected and pool
kernels); these restatements keep fp32 throughout, so GPU results are
compared against them within tolerances written in the tests.
"""

from __future__ import annotations

import math

import torch

__all__ = ["selected_attention_grads", "pool_grads", "route_weights_grads", "route_scores_grads", "fuse_grads",
           "local_attention_grads", "dense_local_attention"]


def _selected_fp32(q, k, v, w, idx, ok, chunk, scale):
    """out[l, hq] = sum_k w[l,hq,k] softmax_s(q.K[c_k,s] * scale ; ok) . V[c_k,s]
    for one block of queries (``ops/hils_fwd_bwd_head.py:21-93``)."""
    b, n, hq, d = q.shape
    hkv = k.shape[2]
    g = hq // hkv
    c = k.shape[1] // chunk
    kc = k[:, : c * chunk].reshape(b, c, chunk, hkv, d)
    vc = v[:, : c * chunk].reshape(b, c, chunk, hkv, d)
    sel = idx >= 0
    safe = idx.clamp_min(0)
    bi = torch.arange(b)[:, None, None, None]
    hi = torch.arange(hkv)[None, None, :, None]
    kg = kc[bi, safe, :, hi]                                       # [B,n,Hkv,K,S,D]
    vg = vc[bi, safe, :, hi]
    okg = ok[bi, safe]                                             # [B,n,Hkv,K,S]
    qg = q.reshape(b, n, hkv, g, d)
    sc = torch.einsum("bnhgd,bnhksd->bnhgks", qg, kg) * scale
    sc = sc.masked_fill(~okg[:, :, :, None], float("-inf"))
    p = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
    o_k = torch.einsum("bnhgks,bnhksd->bnhgkd", p, vg)
    wm = w.reshape(b, n, hkv, g, -1).masked_fill(~sel[:, :, :, None, :], 0.0)
    return torch.einsum("bnhgkd,bnhgk->bnhgd", o_k, wm).reshape(b, n, hq, d)


def selected_attention_grads(q, k, v, weights, indices, key_valid, chunk: int, grad_out, *,
                             mask_last_token: bool = True, sm_scale: float | None = None, block: int = 32):
    """(dq, dk, dv, dweights) in fp32: autograd of the selected-chunk
    attention forward, the quantities the reference's backward kernel
    ``hierarchical_sparse_attention_bwd_dqkv_block_M_inverse``
    (``ops/hils_fwd_bwd_head.py:573-910``) returns.  Queries run in blocks of
    ``block`` so the gathered chunk tiles stay small; dK and dV sum over the
    blocks.  An empty slot (index < 0 or >= C) has dweights 0."""
    b, l, hq, d = q.shape
    lk = k.shape[1]
    c = lk // chunk
    scale = d ** -0.5 if sm_scale is None else float(sm_scale)
    ok = torch.ones(b, c, chunk, dtype=torch.bool) if key_valid is None else \
        key_valid.bool()[:, : c * chunk].reshape(b, c, chunk).clone()
    if mask_last_token:
        ok[..., -1] = False
    idx_all = indices.long().clone()
    idx_all[idx_all >= c] = -1
    kf = k.float().detach().requires_grad_()
    vf = v.float().detach().requires_grad_()
    dq = torch.zeros(b, l, hq, d)
    dw = torch.zeros(weights.shape)
    dk = torch.zeros(kf.shape)
    dv = torch.zeros(vf.shape)
    for s in range(0, l, block):
        e = min(s + block, l)
        qf = q[:, s:e].float().detach().requires_grad_()
        wf = weights[:, s:e].float().detach().requires_grad_()
        out = _selected_fp32(qf, kf, vf, wf, idx_all[:, s:e], ok, chunk, scale)
        gq, gk, gv, gw = torch.autograd.grad(out, (qf, kf, vf, wf), grad_out[:, s:e].float())
        dq[:, s:e] = gq
        dw[:, s:e] = gw
        dk += gk
        dv += gv
    return dq, dk, dv, dw


def pool_grads(mu_q, k_chunked, key_valid, grad_lmk, grad_entropy, sm_scale: float | None = None):
    """(d_mu, d_k) in fp32: autograd of the landmark pool
    ``ops/chunk_attn_pool_gqa_tilelang.py:17-37 _compact_pool_torch`` (lmk =
    sum_s p k, entropy = -sum_s p ln p, p the softmax over the chunk's valid
    non-landmark keys), the quantities of the reference's ``_pool_gqa_bwd``
    (``:183-325``).  ``grad_lmk`` / ``grad_entropy`` may be None."""
    d = mu_q.shape[-1]
    scale = d ** -0.5 if sm_scale is None else float(sm_scale)
    mu = mu_q.float().detach().requires_grad_()
    k = k_chunked.float().detach().requires_grad_()
    valid = key_valid.bool().clone()
    valid[..., -1] = False
    sc = torch.einsum("bnkgd,bnskd->bnkgs", mu, k) * scale
    sc = sc.masked_fill(~valid[:, :, None, None, :], float("-inf"))
    p = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
    lmk = torch.einsum("bnkgs,bnskd->bnkgd", p, k)
    logp = torch.where(p > 0, p.clamp_min(1e-30).log(), torch.zeros_like(p))
    ent = -(p * logp).sum(-1)
    outs, grads = [], []
    if grad_lmk is not None:
        outs.append(lmk)
        grads.append(grad_lmk.float())
    if grad_entropy is not None:
        outs.append(ent)
        grads.append(grad_entropy.float())
    dmu, dk = torch.autograd.grad(outs, (mu, k), grads)
    return dmu, dk


def route_weights_grads(scores, indices, prior_bias, local_lse, grad_remote, grad_local, *, affine: bool,
                        temperature: float = 1.0, gate_scale: float = 1.0, gate_offset: float = 0.0):
    """(d_scores, d_prior, d_local_lse, d_gate_scale, d_gate_offset) in fp32:
    autograd of the route weights.

    ``affine``: the live affine-gate branch of
    ``dream_dllm_hils/attention.py:126-227 _route_weights_torch``
    (m = sigmoid(scale * (lse(r / T) - local / T) + offset), remote =
    softmax(r / T) * m, local = 1 - m).  Otherwise one softmax over
    ``[r, local - offset] / T`` (its non-affine branch, and with offset 0 the
    ``ops/hils_bidir_route_weights_tilelang.py`` kernel).  r = score + prior of
    the selected chunk, -inf on empty slots.  Rows whose logits are all masked
    have zero gradients; a row without a selected chunk contributes 0 to the
    gate-scale gradient (autograd of the reference gives NaN there)."""
    b, l, hq, k = scores.shape
    _, c, hkv, g = prior_bias.shape
    sc = scores.float().detach().requires_grad_()
    pb = prior_bias.float().detach().requires_grad_()
    ll = local_lse.float().detach().requires_grad_()
    gs = torch.tensor(float(gate_scale), requires_grad=True)
    go = torch.tensor(float(gate_offset), requires_grad=True)
    idx = indices.long().repeat_interleave(g, dim=2)
    valid = (idx >= 0) & (idx < c)
    safe = idx.clamp(0, c - 1)
    bias = pb.reshape(b, c, hq).permute(0, 2, 1)[:, None].expand(b, l, hq, c)
    sel_bias = torch.gather(bias, -1, safe)
    ninf = torch.tensor(float("-inf"))
    r = torch.where(valid, sc + sel_bias, ninf) / temperature
    any_r = valid.any(-1)
    if affine:
        lt = ll / temperature
        masked = ~any_r & torch.isneginf(lt)
        rs = torch.where(any_r[..., None], r, torch.zeros_like(r))
        ri = torch.where(any_r[..., None], torch.softmax(rs.masked_fill(~valid, float("-inf")), -1),
                         torch.zeros_like(r))
        lse = torch.logsumexp(rs.masked_fill(~valid, float("-inf")), -1)
        diff = torch.where(any_r & ~torch.isneginf(lt), lse - lt, torch.zeros_like(lt))
        # rows with an empty remote side: gate -> -inf (m = 0) for a positive scale
        gate = gs * diff + go
        m = torch.where(any_r, torch.sigmoid(gate), torch.zeros_like(gate))
        m = torch.where(any_r & torch.isneginf(lt), torch.ones_like(m), m)
        rw = ri * m[..., None]
        lw = 1 - m
        rw = torch.where(masked[..., None], torch.zeros_like(rw), rw)
        lw = torch.where(masked, torch.zeros_like(lw), lw)
    else:
        lt = (ll - go) / temperature
        logits = torch.cat((r, lt[..., None]), -1)
        masked = torch.isneginf(logits).all(-1)
        logits = torch.where(masked[..., None], torch.zeros_like(logits), logits)
        p = torch.softmax(logits, -1)
        p = torch.where(masked[..., None], torch.zeros_like(p), p)
        rw, lw = p[..., :k], p[..., k]
    loss = (rw * grad_remote.float()).sum() + (lw * grad_local.float()).sum()
    d_sc, d_pb, d_ll, d_gs, d_go = torch.autograd.grad(loss, (sc, pb, ll, gs, go), allow_unused=True)
    z = torch.zeros(())
    return (d_sc, d_pb, d_ll, z if d_gs is None else d_gs, z if d_go is None else d_go)


def route_scores_grads(q, landmarks, indices, grad_scores, sm_scale: float | None = None):
    """(d_q, d_landmarks) in fp32 of the gathered routing scores
    s[l, hq, k] = q[l, hq] . lmk[c_k, hq] * scale: the dense scatter + GEMM of
    ``ops/topk_head_softmax.py:1071-1122`` (per-query-head landmarks), in fp32.
    q [B,L,Hq,D], landmarks [B,C,Hkv,G,D], indices [B,L,Hkv,K], grad [B,L,Hq,K]."""
    b, l, hq, d = q.shape
    _, c, hkv, g, _ = landmarks.shape
    scale = d ** -0.5 if sm_scale is None else float(sm_scale)
    idx = indices.long().repeat_interleave(g, dim=2)                 # [B,L,Hq,K]
    valid = (idx >= 0) & (idx < c)
    dense = torch.zeros(b, l, hq, c)
    dense.scatter_add_(-1, idx.clamp(0, c - 1), torch.where(valid, grad_scores.float() * scale,
                                                            torch.zeros(())))
    lmk = landmarks.float().reshape(b, c, hq, d)
    dq = torch.einsum("blhc,bchd->blhd", dense, lmk)
    dl = torch.einsum("blhc,blhd->bchd", dense, q.float()).reshape(b, c, hkv, g, d)
    return dq, dl


def fuse_grads(local, local_weight, grad_out):
    """(d_remote, d_local, d_local_weight) of out = remote + w * local
    (``ops/hils_bidir_output_fusion_tilelang.py:38-99``), fp32."""
    gf = grad_out.float()
    return gf, gf * local_weight.float()[..., None], (gf * local.float()).sum(-1)


def local_attention_grads(q, k, v, key_valid, window: int, chunk: int, skip_inert_slots: bool, grad_out,
                          grad_lse=None):
    """(dq, dk, dv) in fp32: autograd of the oracle's banded attention
    (:func:`oracle.route_layer.local_attention`, the restatement of
    ``dream_dllm_hils/local_attention.py:35-144`` that hands the window to
    flash-attn), including the gradient that reaches its LSE output.
    ``window`` is the layer's window (the oracle widens it by chunk - 1 with
    ``skip_inert_slots``)."""
    from . import route_layer as orc

    qf, kf, vf = (t.float().detach().requires_grad_() for t in (q, k, v))
    out, lse = orc.local_attention(qf, kf, vf, key_valid, window, chunk, skip_inert_slots)
    outs, grads = [out], [grad_out.float()]
    if grad_lse is not None:
        outs.append(lse)
        grads.append(grad_lse.float())
    return torch.autograd.grad(outs, (qf, kf, vf), grads)


def dense_local_attention(q, k, v, key_valid, window: int, chunk: int, skip_inert_slots: bool):
    """The same banded attention written densely over the whole [L, L] score
    matrix (an independent formulation for pinning :func:`local_attention_grads`
    on small inputs): keys zeroed where invalid (and at landmark slots with
    ``skip_inert_slots``), ``|i - j| <= window (+ chunk - 1)``."""
    b, l, hq, d = q.shape
    g = hq // k.shape[2]
    valid = key_valid.bool()
    if skip_inert_slots:
        valid = valid & ((torch.arange(l) + 1) % chunk != 0)[None]
    w = window + chunk - 1 if skip_inert_slots else window
    z = valid.to(k.dtype)[:, :, None, None]
    kz = (k * z).repeat_interleave(g, dim=2)
    vz = (v * z).repeat_interleave(g, dim=2)
    s = torch.einsum("bihd,bjhd->bhij", q, kz) / math.sqrt(d)
    band = (torch.arange(l)[:, None] - torch.arange(l)[None, :]).abs() <= w
    s = s.masked_fill(~band[None, None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    out = torch.einsum("bhij,bjhd->bihd", torch.softmax(s, dim=-1), vz)
    return out, lse.permute(0, 2, 1)
