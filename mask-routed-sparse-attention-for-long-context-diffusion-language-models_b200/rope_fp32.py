"""fp32 YaRN RoPE on the B200 kernels.

Drop-ins for ``ops/rope_tilelang_fp32.py``: ``rope_rotary_pos_emb`` (:84) and
``single_tensor_rope_autograd`` (:173, with its backward), plus the position-id
form used by the fused layer (cos/sin computed in the kernel from the YaRN
inverse frequencies, as Dream's rotary module computes them).
"""

from __future__ import annotations

import math

import torch

from . import _lib


def yarn_inv_freq(dim: int = 128, base: float = 1.0e6, factor: float = 8.0,
                  orig_max_pos: int = 2048, beta_fast: float = 32.0, beta_slow: float = 1.0,
                  truncate: bool = True, device=None):
    """YaRN inverse frequencies ``[dim/2]`` (fp32) and attention factor, the
    published rule as ``transformers`` ``ROPE_INIT_FUNCTIONS['yarn']`` applies
    it for Dream (``dream_dllm_hils/train_fulltext.py:2873-2888``)."""
    def corr_dim(rot):
        return dim * math.log(orig_max_pos / (rot * 2 * math.pi)) / (2 * math.log(base))

    lo, hi = corr_dim(beta_fast), corr_dim(beta_slow)
    if truncate:
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, dim - 1)
    if lo == hi:
        hi += 0.001
    pos_freqs = base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim)
    ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
    keep = 1 - ramp
    inv = (1.0 / (factor * pos_freqs)) * (1 - keep) + (1.0 / pos_freqs) * keep
    af = 1.0 if factor <= 1 else 0.1 * math.log(factor) + 1.0
    return (inv if device is None else inv.to(device)), float(af)


def _check_x(x, name):
    if x.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be BF16")
    if x.ndim != 4:
        raise ValueError(f"{name} must be (B, L, H, D)")


def _cs(cos, sin, x):
    if cos.shape != sin.shape or cos.shape != (x.shape[0], x.shape[1], x.shape[3]):
        raise ValueError(f"cos/sin must be (B, L, D) = {(x.shape[0], x.shape[1], x.shape[3])}")
    if cos.dtype not in (torch.bfloat16, torch.float32) or sin.dtype != cos.dtype:
        raise ValueError("cos/sin must both be BF16 or FP32")
    return cos.contiguous(), sin.contiguous(), (_lib.F32 if cos.dtype == torch.float32 else _lib.BF16)


def rope_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """``(q*cos + rotate_half(q)*sin, k*cos + rotate_half(k)*sin)`` in fp32
    math, bf16 out (``ops/rope_tilelang_fp32.py:84``)."""
    _check_x(q, "q")
    _check_x(k, "k")
    cos, sin, cs_dtype = _cs(cos, sin, q)
    q, k = q.contiguous(), k.contiguous()
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    b, l, hq, d = q.shape
    _lib.call("mrsa_rope", _lib.ptr(q), _lib.ptr(qo), hq, _lib.ptr(k), _lib.ptr(ko), k.shape[2],
              None, None, 0.0, _lib.ptr(cos), _lib.ptr(sin), cs_dtype, b, l, d, _lib.stream_of(q))
    return qo, ko


def _single_rope(x, x_cos, x_sin):
    _check_x(x, "x")
    cos, sin, cs_dtype = _cs(x_cos, x_sin, x)
    x = x.contiguous()
    y = torch.empty_like(x)
    b, l, h, d = x.shape
    _lib.call("mrsa_rope", _lib.ptr(x), _lib.ptr(y), h, None, None, 0, None, None, 0.0,
              _lib.ptr(cos), _lib.ptr(sin), cs_dtype, b, l, d, _lib.stream_of(x))
    return y


class _SingleTensorRoPE(torch.autograd.Function):
    """``ops/rope_tilelang_fp32.py:150 SingleTensorRoPEFunction``: the
    backward is the same rotation with -sin."""

    @staticmethod
    def forward(ctx, x, x_cos, x_sin):
        ctx.save_for_backward(x_cos, x_sin)
        return _single_rope(x, x_cos, x_sin)

    @staticmethod
    def backward(ctx, dy):
        x_cos, x_sin = ctx.saved_tensors
        return _single_rope(dy.to(torch.bfloat16).contiguous(), x_cos, -x_sin), None, None


def single_tensor_rope_autograd(x: torch.Tensor, x_cos: torch.Tensor, x_sin: torch.Tensor):
    """Single-tensor fp32 RoPE (``ops/rope_tilelang_fp32.py:173``); records
    its backward when x requires grad."""
    if torch.is_grad_enabled() and x.requires_grad:
        return _SingleTensorRoPE.apply(x, x_cos, x_sin)
    return _single_rope(x, x_cos, x_sin)


def yarn_rope_qk(q: torch.Tensor, k: torch.Tensor | None, position_ids: torch.Tensor,
                 inv_freq: torch.Tensor, attention_factor: float, out_q=None, out_k=None):
    """RoPE with cos/sin computed in-kernel from ``position_ids`` (int64
    ``[B, L]``): ``fp32(pos * inv_freq)``, ``cos * attention_factor``."""
    _check_x(q, "q")
    b, l, hq, d = q.shape
    if position_ids.shape != (b, l) or position_ids.dtype != torch.long:
        raise ValueError("position_ids must be int64 (B, L)")
    q = q.contiguous()
    pos = position_ids.to(q.device).contiguous()
    inv = inv_freq.to(device=q.device, dtype=torch.float32).contiguous()
    qo = torch.empty_like(q) if out_q is None else out_q
    ko = None
    hk = 0
    if k is not None:
        _check_x(k, "k")
        k = k.contiguous()
        ko = torch.empty_like(k) if out_k is None else out_k
        hk = k.shape[2]
    _lib.call("mrsa_rope", _lib.ptr(q), _lib.ptr(qo), hq, _lib.ptr(k), _lib.ptr(ko), hk,
              _lib.ptr(pos), _lib.ptr(inv), float(attention_factor), None, None, _lib.F32,
              b, l, d, _lib.stream_of(q))
    return qo, ko
