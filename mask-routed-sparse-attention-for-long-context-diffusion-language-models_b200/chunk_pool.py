"""Landmark attention pool (drop-in for ``ops/chunk_attn_pool_gqa_tilelang.py``,
forward and backward)."""

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


def _pool_forward(mu_q, k_chunked, key_valid, sm_scale):
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


def chunk_pool_backward(mu_q, k_chunked, key_valid, grad_landmarks=None, grad_entropy=None,
                        sm_scale: float | None = None):
    """``(d_mu, d_k)`` in bf16 for the pool's landmark and entropy gradients
    (either may be None): ``_ChunkAttnPoolGQA.backward``
    (``ops/chunk_attn_pool_gqa_tilelang.py:361-393``, kernel ``:183-325``)."""
    _validate(mu_q, k_chunked, key_valid)
    b, c, hkv, g, d = mu_q.shape
    scale = 1.0 / math.sqrt(d) if sm_scale is None else float(sm_scale)
    mu = mu_q.contiguous()
    k = k_chunked.contiguous()
    kv = key_valid.to(device=mu.device, dtype=torch.bool).contiguous()
    gl = None if grad_landmarks is None else grad_landmarks.to(torch.bfloat16).contiguous()
    ge = None if grad_entropy is None else grad_entropy.to(torch.float32).contiguous()
    d_mu = torch.empty_like(mu)
    d_k = torch.empty_like(k)
    _lib.call("mrsa_chunk_pool_backward", _lib.ptr(mu), _lib.ptr(k), _lib.ptr(kv), _lib.ptr(gl), _lib.ptr(ge),
              _lib.ptr(d_mu), _lib.ptr(d_k), scale, b, c, hkv, g, d, _lib.stream_of(mu))
    return d_mu, d_k


class _ChunkPool(torch.autograd.Function):
    """``ops/chunk_attn_pool_gqa_tilelang.py:328 _ChunkAttnPoolGQA`` on the B200 kernels."""

    @staticmethod
    def forward(ctx, mu_q, k_chunked, key_valid, sm_scale):
        lmk, ent = _pool_forward(mu_q, k_chunked, key_valid, sm_scale)
        ctx.save_for_backward(mu_q, k_chunked, key_valid)
        ctx.sm_scale = sm_scale
        return lmk, ent

    @staticmethod
    def backward(ctx, grad_lmk, grad_ent):
        mu_q, k_chunked, key_valid = ctx.saved_tensors
        d_mu, d_k = chunk_pool_backward(mu_q, k_chunked, key_valid, grad_lmk, grad_ent, ctx.sm_scale)
        return d_mu, d_k, None, None


def chunk_attn_pool_gqa(mu_q: torch.Tensor, k_chunked: torch.Tensor, key_valid: torch.Tensor,
                        sm_scale: float | None = None):
    """Pool compact per-KV-head chunks into per-query-head summaries.

    Returns ``(landmarks [B,C,Hkv,G,D] bf16, entropy [B,C,Hkv,G] fp32)``
    (``ops/chunk_attn_pool_gqa_tilelang.py:425``); records the B200 backward
    when an input requires grad."""
    _validate(mu_q, k_chunked, key_valid)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(mu_q.shape[-1])
    if torch.is_grad_enabled() and (mu_q.requires_grad or k_chunked.requires_grad):
        return _ChunkPool.apply(mu_q, k_chunked, key_valid, float(sm_scale))
    return _pool_forward(mu_q, k_chunked, key_valid, sm_scale)
