"""Bidirectional window attention on the B200 kernel.

Drop-in for ``dream_dllm_hils/local_attention.py:110 bidir_local_attention``
(the reference hands this to third-party flash-attn with
``window_size=(W, W)``): keys that are invalid or, with ``skip_inert_slots``,
landmark slots get zero K and V -- they stay in the softmax with logit 0 --
and the window widens to ``W + chunk - 1`` with ``skip_inert_slots``.
"""

from __future__ import annotations

import torch

from . import _lib


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
    ``v`` in fp16 runs the one-tile fp16 P kernel, bf16 the hi + lo one."""
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
