"""Landmark attention pool (drop-in for ``ops/chunk_attn_pool_gqa_tilelang.py``)."""

from __future__ import annotations

import math

import torch

from . import _lib


def _validate(mu_q, k_chunked, key_valid):
    # mirrors ops/chunk_attn_pool_gqa_tilelang.py:404-422
    if mu_q.device.type != "cuda":
        raise ValueError("chunk_attn_pool_gqa requires CUDA tensors")
    if mu_q.dtype != torch.bfloat16 or k_chunked.dtype != torch.bfloat16:
        raise ValueError("chunk_attn_pool_gqa requires BF16 mu_q and K")
    if mu_q.ndim != 5 or k_chunked.ndim != 5:
        raise ValueError("mu_q and k_chunked must be 5D")
    batch, chunks, kv_heads, groups, head_dim = mu_q.shape
    expected_k = (batch, chunks, k_chunked.shape[2], kv_heads, head_dim)
    if k_chunked.shape != expected_k:
        raise ValueError(f"expected compact K shape {expected_k}, got {tuple(k_chunked.shape)}")
    if key_valid.shape != (batch, chunks, k_chunked.shape[2]):
        raise ValueError(f"invalid key_valid shape {tuple(key_valid.shape)}")
    if groups > 16:
        raise ValueError(f"groups must be <= 16, got {groups}")
    if groups > 8 or head_dim != 128 or k_chunked.shape[2] != 64:
        raise ValueError("the B200 pool kernel supports groups <= 8, head_dim 128, chunk 64")


def chunk_attn_pool_gqa(mu_q: torch.Tensor, k_chunked: torch.Tensor, key_valid: torch.Tensor,
                        sm_scale: float | None = None):
    """Pool compact per-KV-head chunks into per-query-head summaries.

    Returns ``(landmarks [B,C,Hkv,G,D] bf16, entropy [B,C,Hkv,G] fp32)``
    (``ops/chunk_attn_pool_gqa_tilelang.py:425``)."""
    _validate(mu_q, k_chunked, key_valid)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(mu_q.shape[-1])
    b, c, hkv, g, d = mu_q.shape
    mu = mu_q.contiguous()
    k = k_chunked.contiguous()
    kv = key_valid.to(device=mu.device, dtype=torch.bool).contiguous()
    lmk = torch.empty_like(mu)
    ent = torch.empty(b, c, hkv, g, device=mu.device, dtype=torch.float32)
    _lib.call("mrsa_chunk_pool", _lib.ptr(mu), c * hkv * g * d, hkv * g * d, _lib.ptr(k),
              _lib.ptr(kv), float(sm_scale), None, _lib.ptr(lmk), _lib.ptr(ent), None, None,
              b, c, hkv, g, d, _lib.stream_of(mu))
    return lmk, ent
