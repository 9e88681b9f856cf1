"""Query -> chunk routing on the B200 kernels.

Drop-ins for ``ops/topk_head_softmax.py`` (``ref_softmax_topk_max_pooling``
:15, ``online_softmax_topk_head`` :1242 with its scores backward :1071),
``dream_dllm_hils/routing.py``
(``route_topk_g7`` :52) and ``dream_dllm_hils/kernel_utils.py``
(``remote_drop_mask`` :102).  The fused route layer does not materialise the
dense drop mask; it evaluates the same rule inline.
"""

from __future__ import annotations

import torch

from . import _lib

_LOGICAL_G = 7


def remote_drop_mask(valid_mask: torch.Tensor, window: int, chunk_size: int,
                     allowed_mask: torch.Tensor | None = None) -> torch.Tensor:
    """1 = drop chunk for the query: overlaps the chunk-aligned local window or
    has no valid real key (``dream_dllm_hils/kernel_utils.py:102-161``)."""
    if valid_mask.ndim != 2:
        raise ValueError(f"valid_mask must have shape [B, L], got {tuple(valid_mask.shape)}")
    batch, seq_len = valid_mask.shape
    if chunk_size <= 0 or seq_len % chunk_size != 0:
        raise ValueError(f"sequence length {seq_len} must be divisible by chunk_size={chunk_size}")
    if valid_mask.device.type != "cuda":
        raise ValueError("remote_drop_mask requires a CUDA tensor")
    valid = valid_mask.to(torch.bool).contiguous()
    out = torch.empty(batch, seq_len, seq_len // chunk_size, device=valid.device, dtype=torch.int32)
    _lib.call("mrsa_remote_drop_mask", _lib.ptr(valid), _lib.ptr(out), batch, seq_len, int(window),
              int(chunk_size), _lib.stream_of(valid))
    if allowed_mask is not None:
        if allowed_mask.shape != (batch, seq_len, seq_len):
            raise ValueError("allowed_mask must have shape "
                             f"{(batch, seq_len, seq_len)}, got {tuple(allowed_mask.shape)}")
        lmk = torch.arange(chunk_size - 1, seq_len, chunk_size, device=valid.device)
        out |= (~allowed_mask.to(torch.bool).index_select(-1, lmk)).to(torch.int32)
    return out


def _route(q5: torch.Tensor, k_lmks: torch.Tensor, lse: torch.Tensor, topk: int,
           drop_mask, bias, scores_dtype, *, chunk_ok=None, window=-1, q_offset=0,
           weights=None):
    """Shared launcher.  q5 ``[B,L,Hkv,G,D]``; k_lmks ``[B,S,Hkv,D]`` or
    ``[B,S,Hkv*G,D]``; lse ``[B,L,Hq]`` or ``[B,L,Hkv,G]``."""
    b, l, hkv, g, d = q5.shape
    s = k_lmks.shape[1]
    lh = k_lmks.shape[2]
    if lh == hkv:
        per_q = 0
    elif lh == hkv * g:
        per_q = 1
    else:
        raise AssertionError(
            f"k_lmks h dim ({lh}) must be either h_kv ({hkv}) or h_kv*G ({hkv * g})")
    if q5.device.type != "cuda":
        raise ValueError("routing requires CUDA tensors")
    dev = q5.device
    q = q5.to(torch.bfloat16).contiguous()
    lm = k_lmks.to(torch.bfloat16).contiguous()
    lse_f = lse.to(device=dev, dtype=torch.float32).contiguous()
    if lse_f.numel() != b * l * hkv * g:
        raise ValueError(f"invalid lse_swa shape {tuple(lse.shape)}")
    bias_f = None
    if bias is not None:
        bias_f = bias.to(device=dev, dtype=torch.float32).contiguous()
        if bias_f.numel() != b * s * hkv * g:
            raise AssertionError(f"bias must be [B, S, h_q] or [B, S, h_kv, G], got {tuple(bias.shape)}")
    drop = None
    if drop_mask is not None:
        if drop_mask.shape != (b, l, s):
            raise ValueError(f"invalid drop_mask shape {tuple(drop_mask.shape)}")
        drop = drop_mask.to(device=dev, dtype=torch.int32).contiguous()
    idx = torch.empty(b, l, hkv, topk, device=dev, dtype=torch.int32)
    sc = torch.empty(b, l, hkv * g, topk, device=dev, dtype=scores_dtype)
    rw = lw = None
    mode, temp, gs, go = _lib.WEIGHTS_AFFINE, 1.0, 1.0, 0.0
    if weights is not None:
        mode, temp, gs, go = weights
        rw = torch.empty(b, l, hkv * g, topk, device=dev, dtype=torch.bfloat16)
        lw = torch.empty(b, l, hkv * g, device=dev, dtype=torch.bfloat16)
    sdt = _lib.F32 if scores_dtype == torch.float32 else _lib.BF16
    ws_bytes = _lib.load().mrsa_route_topk_workspace_size(b, l, s, hkv, g, sdt)
    ws = torch.empty(max(ws_bytes, 16), device=dev, dtype=torch.uint8)
    _lib.call("mrsa_route_topk", _lib.ptr(q), _lib.ptr(lm), per_q, _lib.ptr(lse_f), _lib.ptr(bias_f),
              _lib.ptr(drop), _lib.ptr(chunk_ok), int(window), int(q_offset), _lib.ptr(idx),
              _lib.ptr(sc), _lib.F32 if scores_dtype == torch.float32 else _lib.BF16,
              _lib.ptr(rw), _lib.ptr(lw), int(mode), float(temp), float(gs), float(go),
              b, l, s, hkv, g, d, int(topk), _lib.ptr(ws), ws.numel(), _lib.stream_of(q))
    return idx, sc, rw, lw


def route_scores_backward(q, landmarks, indices, grad_scores, sm_scale=None):
    """``(d_q [B,L,Hq,D], d_landmarks [B,C,Hkv,G,D])`` in fp32 for the gathered
    routing scores ``q . lmk[c_k] * sm_scale``: the backward of
    ``ops/topk_head_softmax.py:1005 SoftmaxTopKMaxPoolingFusedFn``
    (``:1071-1122``) with per-query-head landmarks."""
    b, l, hq, d = q.shape
    _, c, hkv, g, _ = landmarks.shape
    topk = indices.shape[-1]
    dev = q.device
    qq = q.to(torch.bfloat16).contiguous()
    lm = landmarks.to(torch.bfloat16).contiguous()
    idx = indices.to(device=dev, dtype=torch.int32).contiguous()
    gs = grad_scores.to(torch.bfloat16).reshape(b, l, hq, topk).contiguous()
    d_q = torch.empty(b, l, hq, d, dtype=torch.float32, device=dev)
    d_l = torch.empty(b, c, hkv, g, d, dtype=torch.float32, device=dev)
    scale = d ** -0.5 if sm_scale is None else float(sm_scale)
    lib = _lib.load()
    ws_bytes = lib.mrsa_route_scores_backward_workspace(b, l, c, hkv, topk)
    ws = torch.empty(max(int(ws_bytes), 16), dtype=torch.uint8, device=dev)
    _lib.call("mrsa_route_scores_backward", _lib.ptr(qq), _lib.ptr(lm), _lib.ptr(idx), _lib.ptr(gs),
              _lib.ptr(d_q), _lib.ptr(d_l), scale, b, l, c, hkv, g, d, topk, _lib.ptr(ws), int(ws_bytes),
              _lib.stream_of(qq))
    return d_q, d_l


class _RouteScores(torch.autograd.Function):
    """Routing with the B200 backward of the gathered scores (indices carry
    no gradient): ``ops/topk_head_softmax.py:1005-1122``."""

    @staticmethod
    def forward(ctx, q5, k_lmks, lse, drop_mask, bias, topk, scores_dtype):
        idx, sc, _, _ = _route(q5, k_lmks, lse, topk, drop_mask, bias, scores_dtype)
        ctx.mark_non_differentiable(idx)
        ctx.save_for_backward(q5, k_lmks, idx)
        return idx, sc

    @staticmethod
    def backward(ctx, grad_idx, grad_sc):
        q5, k_lmks, idx = ctx.saved_tensors
        b, l, hkv, g, d = q5.shape
        s = k_lmks.shape[1]
        per_q = k_lmks.shape[2] == hkv * g
        lm = k_lmks.view(b, s, hkv, g, d) if per_q else k_lmks[:, :, :, None, :].expand(b, s, hkv, g, d)
        d_q, d_l = route_scores_backward(q5.reshape(b, l, hkv * g, d), lm, idx, grad_sc)
        d_l = d_l.reshape(b, s, hkv * g, d) if per_q else d_l.sum(3)
        return d_q.view(q5.shape).to(q5.dtype), d_l.to(k_lmks.dtype), None, None, None, None, None


def _route_autograd(q5, k_lmks, lse, topk, drop_mask, bias, scores_dtype):
    if torch.is_grad_enabled() and (q5.requires_grad or k_lmks.requires_grad):
        return _RouteScores.apply(q5, k_lmks, lse, drop_mask, bias, topk, scores_dtype)
    idx, sc, _, _ = _route(q5, k_lmks, lse, topk, drop_mask, bias, scores_dtype)
    return idx, sc


def ref_softmax_topk_max_pooling(q, k_lmks, lse_swa, topk, block_size, window_size, is_causal=False,
                                 q_offset=0, drop_mask=None, bias=None, gumbel_noise=None,
                                 selection_mode="post_softmax"):
    """Post-softmax max-pooled top-k (``ops/topk_head_softmax.py:15``), on the GPU.

    Returns ``indices [B,L,h_kv,topk]`` (int64, ascending, -1 last) and
    ``scores [B,L,h_kv,G,topk]`` fp32 raw scaled q.lmk (-inf at -1)."""
    if selection_mode not in {"post_softmax", "pre_softmax"}:
        raise ValueError(f"unsupported selection_mode={selection_mode}")
    if selection_mode != "post_softmax" or is_causal or gumbel_noise is not None:
        raise ValueError("the B200 routing kernel implements the eval path: post_softmax, "
                         "non-causal, no Gumbel noise")
    b, l, hkv, g, d = q.shape
    idx, sc, _, _ = _route(q, k_lmks, lse_swa, topk, drop_mask, bias, torch.float32)
    return idx.long(), sc.view(b, l, hkv, g, topk)


def online_softmax_topk_head(q, lmks, lse_swa, topk, block_size, window_size, is_causal=True,
                             q_offset=0, is_training=True, drop_mask=None, sm_scale=None, bias=None,
                             use_gumbel=False, gumbel_noise=None, G=1):
    """Fused routing entry (``ops/topk_head_softmax.py:1242``): the non-causal,
    Gumbel-free selection.  ``q [B,L,Hq,D]``; returns ``(indices
    [B,L,Hkv,topk] int32, scores [B,L,Hq,topk] bf16)``; the scores carry the
    B200 backward to q and lmks when those require grad."""
    if is_causal or use_gumbel or gumbel_noise is not None:
        raise ValueError("the B200 routing kernel implements non-causal, Gumbel-free routing")
    if sm_scale is not None and abs(sm_scale - q.shape[-1] ** -0.5) > 1e-12:
        raise ValueError("only sm_scale = 1/sqrt(D) is supported")
    b, l, hq, d = q.shape
    hkv = hq // G
    idx, sc = _route_autograd(q.view(b, l, hkv, G, d), lmks, lse_swa, topk, drop_mask, bias, torch.bfloat16)
    return idx, sc


def route_topk_g7(q, lmks, local_lse, prior_bias, drop_mask, topk, chunk_size, window, *,
                  training=True, use_gumbel=False, gumbel_scale=1.0, return_selected_gumbel=False,
                  selection_mode="post_softmax"):
    """``dream_dllm_hils/routing.py:52`` for G=7 (deterministic eval path).

    Returns ``indices [B,L,Hkv,K]`` int64 and ``scores [B,L,Hq,K]`` in q's dtype."""
    if q.ndim != 4 or lmks.ndim != 5:
        raise ValueError(f"expected q [B,L,Hq,D] and lmks [B,C,Hkv,7,D], got "
                         f"{tuple(q.shape)} and {tuple(lmks.shape)}")
    batch, seq_len, h_q, dim = q.shape
    if lmks.shape[0] != batch or lmks.shape[3:] != (_LOGICAL_G, dim):
        raise ValueError(f"invalid landmark shape {tuple(lmks.shape)} for q {tuple(q.shape)}")
    chunks, h_kv = lmks.shape[1:3]
    if h_q != h_kv * _LOGICAL_G:
        raise ValueError(f"expected {h_kv * _LOGICAL_G} query heads, got {h_q}")
    if local_lse.shape != (batch, seq_len, h_kv, _LOGICAL_G):
        raise ValueError(f"invalid local_lse shape {tuple(local_lse.shape)}")
    if prior_bias.shape != (batch, chunks, h_kv, _LOGICAL_G):
        raise ValueError(f"invalid prior_bias shape {tuple(prior_bias.shape)}")
    if drop_mask.shape != (batch, seq_len, chunks):
        raise ValueError(f"invalid drop_mask shape {tuple(drop_mask.shape)}")
    if topk <= 0:
        raise ValueError(f"topk must be positive, got {topk}")
    if selection_mode != "post_softmax" or (use_gumbel and training):
        raise ValueError("the B200 routing kernel implements post_softmax routing without Gumbel")
    idx, sc = _route_autograd(q.view(batch, seq_len, h_kv, _LOGICAL_G, dim),
                              lmks.reshape(batch, chunks, h_q, dim), local_lse, topk, drop_mask,
                              prior_bias, torch.bfloat16)
    idx = idx.long()
    sc = sc.to(q.dtype)
    if return_selected_gumbel:
        return idx, sc, None
    return idx, sc


def route_topk_fused(route_q, landmarks, local_lse, prior, chunk_ok, topk, window, *,
                     q_offset=0, temperature=1.0, gate_scale=1.0, gate_offset=0.0,
                     weight_mode=_lib.WEIGHTS_AFFINE):
    """Routing of the fused layer: inline drop rule, route weights fused.

    Returns ``(indices int32, scores bf16, remote_w bf16, local_w bf16)``."""
    b, l, hq, d = route_q.shape
    c, hkv, g = landmarks.shape[1:4]
    return _route(route_q.view(b, l, hkv, g, d), landmarks.reshape(b, c, hq, d), local_lse, topk,
                  None, prior, torch.bfloat16, chunk_ok=chunk_ok, window=window,
                  q_offset=q_offset, weights=(weight_mode, temperature, gate_scale, gate_offset))
