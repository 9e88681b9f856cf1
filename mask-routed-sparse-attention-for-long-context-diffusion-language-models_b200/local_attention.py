"""Bidirectional window attention on the B200 kernel.

Drop-in for ``dream_dllm_hils/local_attention.py:110 bidir_local_attention``
with its backward (``window_attention_backward``; flash-attn's in the
reference); ``cached_local_attention`` and ``flex_attn_tl`` are forward-only
and raise when a gradient would be needed
(the reference hands this to third-party flash-attn with
``window_size=(W, W)``): keys that are invalid or, with ``skip_inert_slots``,
landmark slots get zero K and V -- they stay in the softmax with logit 0 --
and the window widens to ``W + chunk - 1`` with ``skip_inert_slots``.
"""

from __future__ import annotations

import torch

from . import _lib


def _no_backward(*tensors) -> None:
    # calls without a B200 backward refuse rather than drop the gradient
    if _wants_grad(*tensors):
        raise NotImplementedError("this window attention call has no backward on the B200 kernels; "
                                  "call it under torch.no_grad() or with inputs that do not require grad")


def _wants_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def window_attention_backward(q, k, v, key_valid, out, lse, grad_out, grad_lse=None, *, window: int,
                              skip_inert: bool, chunk: int = 64, sm_scale=None):
    """``(dq, dk, dv)`` in fp32 of :func:`window_attention` (query rows = the
    key rows, bf16 V): the backward of the flash-attn call inside
    ``dream_dllm_hils/local_attention.py:110-144``, including the gradient
    that reaches the LSE output (``grad_lse``, e.g. from the route weights).
    ``window`` is the effective window; zeroed keys get zero dk / dv."""
    b, l, hq, d = q.shape
    hkv = k.shape[2]
    dev = q.device
    if v.dtype != torch.bfloat16 or q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise ValueError("the window-attention backward requires BF16 q, k and v")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    kv = None if key_valid is None else key_valid.to(device=dev, dtype=torch.bool).contiguous()
    o = out.to(torch.bfloat16).contiguous()
    ls = lse.to(torch.float32).contiguous()
    go = grad_out.to(torch.bfloat16).contiguous()
    gl = None if grad_lse is None else grad_lse.to(torch.float32).contiguous()
    dq = torch.empty(b, l, hq, d, dtype=torch.float32, device=dev)
    dk = torch.empty(b, l, hkv, d, dtype=torch.float32, device=dev)
    dv = torch.empty_like(dk)
    ws_bytes = int(_lib.load().mrsa_local_attention_backward_workspace(b, l, hq))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    scale = float(d) ** -0.5 if sm_scale is None else float(sm_scale)
    _lib.call("mrsa_local_attention_backward", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(kv), _lib.ptr(o),
              _lib.ptr(ls), _lib.ptr(go), _lib.ptr(gl), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(ws),
              ws_bytes, int(window), int(bool(skip_inert)), int(chunk), scale, b, l, hq, hkv, d, _lib.stream_of(q))
    return dq, dk, dv


class _WindowAttention(torch.autograd.Function):
    """Window attention with the B200 backward (flash-attn's role in the reference)."""

    @staticmethod
    def forward(ctx, q, k, v, key_valid, window, skip_inert, chunk):
        with torch.no_grad():
            out, lse = _window_forward(q, k, v, key_valid, window, skip_inert=skip_inert, chunk=chunk)
        ctx.save_for_backward(q, k, v, key_valid, out, lse)
        ctx.cfg = (window, skip_inert, chunk)
        return out, lse

    @staticmethod
    def backward(ctx, grad_out, grad_lse):
        q, k, v, key_valid, out, lse = ctx.saved_tensors
        window, skip_inert, chunk = ctx.cfg
        if grad_out is None:
            grad_out = torch.zeros_like(out)
        dq, dk, dv = window_attention_backward(q, k, v, key_valid, out, lse, grad_out, grad_lse, window=window,
                                               skip_inert=skip_inert, chunk=chunk)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None, None


def _validate_layout(q, k, v, key_valid) -> None:
    # mirrors dream_dllm_hils/local_attention.py:15-32
    if q.device.type != "cuda":
        raise ValueError("local attention requires CUDA tensors")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("local attention requires BF16 q, k, and v")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must have BLHD layout")
    batch, seq_len, h_q, dim = q.shape
    if k.shape[0] != batch or v.shape != k.shape:
        raise ValueError(f"q/k/v batch mismatch: {q.shape}, {k.shape}, {v.shape}")
    if k.shape[-1] != dim or h_q % k.shape[2] != 0:
        raise ValueError("query heads must be divisible by KV heads with equal head_dim")
    if key_valid.shape[0] != batch or key_valid.shape[-1] != k.shape[1]:
        raise ValueError(f"key_valid must have shape {(batch, k.shape[1])}, got {tuple(key_valid.shape)}")


def window_attention(q, k, v, key_valid, window: int, *, skip_inert: bool, chunk: int = 64,
                     q_offset: int = 0, out=None, lse=None, need_lse: bool = True):
    """Banded attention of query rows at global positions ``q_offset..`` over
    the full key range of ``k``/``v``; ``window`` is the effective flash window.
    ``v`` in fp16 runs the one-tile fp16 P kernel, bf16 the hi + lo one.
    When an input requires grad (query rows = key rows, bf16 V, no output
    buffers) the call records the B200 backward."""
    if _wants_grad(q, k, v):
        if q_offset != 0 or q.shape[1] != k.shape[1] or out is not None or lse is not None or \
                v.dtype != torch.bfloat16:
            _no_backward(q, k, v)
        return _WindowAttention.apply(q, k, v, key_valid, int(window), bool(skip_inert), int(chunk))
    return _window_forward(q, k, v, key_valid, window, skip_inert=skip_inert, chunk=chunk, q_offset=q_offset,
                           out=out, lse=lse, need_lse=need_lse)


def _window_forward(q, k, v, key_valid, window: int, *, skip_inert: bool, chunk: int = 64,
                    q_offset: int = 0, out=None, lse=None, need_lse: bool = True):
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    kv = None if key_valid is None else key_valid.to(device=q.device, dtype=torch.bool).contiguous()
    if out is None:
        out = torch.empty_like(q)
    if lse is None and need_lse:
        lse = torch.empty(b, lq, hq, device=q.device, dtype=torch.float32)
    if v.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"v must be bf16 or fp16, got {v.dtype}")
    entry = "mrsa_local_attention_f16v" if v.dtype == torch.float16 else "mrsa_local_attention"
    _lib.call(entry, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(kv),
              _lib.ptr(out), _lib.ptr(lse), int(window), int(bool(skip_inert)), int(chunk),
              float(d) ** -0.5, b, lq, lk, int(q_offset), hq, hkv, d, _lib.stream_of(q))
    return out, lse


def bidir_local_attention(q, k, v, key_valid, window: int, chunk_size: int, allowed_mask=None,
                          skip_inert_slots: bool = False):
    """Bidirectional local GQA attention and natural-log LSE ``[B, L, Hq]``."""
    _validate_layout(q, k, v, key_valid)
    seq_len = q.shape[1]
    if k.shape[1] != seq_len:
        raise ValueError("prefill local attention requires equal Q/K lengths")
    if window < 0 or chunk_size <= 0 or seq_len % chunk_size != 0:
        raise ValueError(f"invalid window/chunk layout: L={seq_len}, W={window}, S={chunk_size}")
    if allowed_mask is not None:
        raise ValueError("bidir_local_attention only accepts 2D key_valid; "
                         "do not pass a dense L×L allowed_mask")
    eff = window + chunk_size - 1 if skip_inert_slots else window
    return window_attention(q, k, v, key_valid, eff, skip_inert=skip_inert_slots, chunk=chunk_size)


def cached_local_attention(q, k, v, key_valid, query_positions, window: int, chunk_size: int,
                           skip_inert_slots: bool = False):
    """Fast-dLLM query rows at ``query_positions`` against a windowed K/V cache
    (``dream_dllm_hils/local_attention.py:147``): each row attends the cache
    keys within the same window as :func:`bidir_local_attention` around its own
    position.  Returns ``(o [B, Lq, Hq, D] bf16, lse [B, Lq, Hq])``."""
    _no_backward(q, k, v)
    _validate_layout(q, k, v, key_valid)
    batch, query_len, h_q, dim = q.shape
    seq_len = k.shape[1]
    # mirrors dream_dllm_hils/local_attention.py:158-181
    if query_positions.shape != (query_len,):
        raise ValueError(f"query_positions must have shape {(query_len,)}, "
                         f"got {tuple(query_positions.shape)}")
    if query_positions.device != q.device or query_positions.dtype != torch.long:
        raise ValueError("query_positions must be CUDA torch.long")
    if query_len == 0:
        return q.new_empty((batch, 0, h_q, dim)), q.new_empty((batch, 0, h_q), dtype=torch.float32)
    if torch.unique(query_positions).numel() != query_len:
        raise ValueError("query_positions must be unique")
    if bool(((query_positions < 0) | (query_positions >= seq_len)).any()):
        raise ValueError("query_positions must be in cache range")
    if window < 0 or chunk_size <= 0 or seq_len % chunk_size:
        raise ValueError(f"invalid window/chunk layout: L={seq_len}, W={window}, S={chunk_size}")
    return positions_window_attention(q, k, v, key_valid, query_positions, window, chunk_size, skip_inert_slots)


def positions_window_attention(q, k, v, key_valid, query_positions, window: int, chunk_size: int,
                               skip_inert_slots: bool):
    """The launch behind :func:`cached_local_attention`, for callers that have
    already checked the query positions (unique, inside the cache) and the
    window layout; it reads nothing back from the GPU."""
    batch, query_len, h_q, dim = q.shape
    seq_len = k.shape[1]
    if query_len == 0:
        return q.new_empty((batch, 0, h_q, dim)), q.new_empty((batch, 0, h_q), dtype=torch.float32)
    eff = window + chunk_size - 1 if skip_inert_slots else window
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    kv = key_valid.to(device=q.device, dtype=torch.bool).contiguous()
    pos = query_positions.contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(batch, query_len, h_q, device=q.device, dtype=torch.float32)
    _lib.call("mrsa_local_attention_positions", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(kv),
              _lib.ptr(pos), _lib.ptr(out), _lib.ptr(lse), int(eff), int(bool(skip_inert_slots)),
              int(chunk_size), float(dim) ** -0.5, batch, query_len, seq_len, h_q, k.shape[2], dim,
              _lib.stream_of(q))
    return out, lse


def flex_attn_tl(q, k, v, window_size: int, chunk_size: int, training: bool = True, mask_lmk: bool = True,
                 expand_to_chunk: bool = True, sm_scale: float = None, kv_start: int = 0):
    """Causal chunk-expanded window attention of ``ops/flex_attn_tilelang.py:1261``
    (forward): query row i (absolute position ``kv_start + Lk - Lq + i``) sees
    keys j with ``start <= j <= i``, ``start = i - W + 1`` (rounded down to a
    chunk boundary with ``expand_to_chunk``); with ``mask_lmk`` the landmark
    slots ``(j + 1) % chunk_size == 0`` are excluded.  Returns
    ``(o [B,Lq,Hq,D] bf16, lse [B,Lq,Hq] natural log)``; rows without a
    visible key give 0 and ``-inf``."""
    if training and int(kv_start) != 0:
        raise ValueError("flex_attn_tl only supports non-zero kv_start in inference (training=False)")
    _no_backward(q, k, v)
    if q.device.type != "cuda":
        raise ValueError("flex_attn_tl requires CUDA tensors")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must have (B, L, H, D) layout")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("flex_attn_tl requires BF16 q, k, and v")
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    if k.shape[0] != b or v.shape[:3] != k.shape[:3] or k.shape[-1] != d:
        raise ValueError(f"q/k/v shape mismatch: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if v.shape[-1] != d or d != 128:
        raise ValueError("the B200 kernel supports D_qk = D_v = 128")
    if hq % hkv or hq // hkv > 8:
        raise ValueError("the B200 kernel supports query groups of at most 8 heads")
    if lq > lk:
        raise ValueError(f"q_len={lq} must not exceed kv_len={lk}")
    if chunk_size <= 0 or window_size < 0 or kv_start < 0:
        raise ValueError(f"invalid window/chunk: W={window_size}, S={chunk_size}, kv_start={kv_start}")
    scale = float(d) ** -0.5 if sm_scale is None else float(sm_scale)
    if not scale > 0.0:
        raise ValueError("the B200 kernel requires sm_scale > 0")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(b, lq, hq, device=q.device, dtype=torch.float32)
    if out.numel() == 0:
        return out, lse
    _lib.call("mrsa_flex_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(lse),
              int(window_size), int(chunk_size), int(bool(mask_lmk)), int(bool(expand_to_chunk)),
              int(kv_start), scale, b, lq, lk, hq, hkv, d, _lib.stream_of(q))
    return out, lse
