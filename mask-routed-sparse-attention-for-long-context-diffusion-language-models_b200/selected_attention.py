"""Selected-chunk attention (+ local merge) on the B200 kernel.

Drop-ins for ``ops/hils_fwd_bwd_head.py:1113 HiLS_block_M_head`` (forward and backward),
``dream_dllm_hils/routing.py:305 selected_attention_g7`` / ``:330
selected_attention_g7_cached`` and
``ops/hils_bidir_output_fusion_tilelang.py:138 fuse_hils_outputs``.  No
physical G=8 / power-of-two top-k padding is needed: the kernel takes the
logical group size (<= 8) and any top-k <= 32.
"""

from __future__ import annotations

import torch

from . import _lib

_LOGICAL_G = 7


def selected_attention(q, k, v, weights, indices, key_valid=None, *, chunk: int = 64,
                       local_out=None, local_weight=None, mask_last_token=True, sm_scale=None,
                       out=None, token_keep=None):
    """``out = sum_k w_k softmax_chunk(q.K_k/sqrt(D)) V_k`` (bf16), fused with
    ``+ local_weight * local_out`` when those are given.

    ``v`` in bf16 runs the exact-P kernel (P as bf16 hi + lo); ``v`` in fp16
    (see :func:`to_f16`) runs the fp16-P kernel, which does half the P.V work
    and keeps P to 11 significant bits.  ``token_keep`` (``[B, Lq, Hkv, K,
    chunk]``, nonzero = keep) additionally drops tokens of each selected chunk
    per (query, KV head, slot), as token refinement does
    (``ops/hils_fwd_bwd_head.py:453-507``); a chunk listed twice by one query
    uses its first slot's keep row."""
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    topk = indices.shape[-1]
    dev = q.device
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    w = weights.to(torch.bfloat16).contiguous()
    idx = indices.to(device=dev, dtype=torch.int32).contiguous()
    kv = None if key_valid is None else key_valid.to(device=dev, dtype=torch.bool).contiguous()
    lo = None if local_out is None else local_out.contiguous()
    lw = None if local_weight is None else local_weight.to(torch.bfloat16).contiguous()
    if out is None:
        out = torch.empty_like(q)
    scale = float(d) ** -0.5 if sm_scale is None else float(sm_scale)
    if v.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"v must be bf16 or fp16, got {v.dtype}")
    if token_keep is not None:
        if tuple(token_keep.shape) != (b, lq, hkv, topk, chunk):
            raise ValueError(f"token_keep must have shape {(b, lq, hkv, topk, chunk)}, "
                             f"got {tuple(token_keep.shape)}")
        keep = token_keep.to(device=dev, dtype=torch.int8).contiguous()
        _lib.call("mrsa_selected_attention_keep", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(kv),
                  _lib.ptr(w), _lib.ptr(idx), _lib.ptr(keep), _lib.ptr(lo), _lib.ptr(lw), _lib.ptr(out),
                  scale, int(bool(mask_last_token)), int(v.dtype == torch.float16), b, lq, lk, hkv,
                  hq // hkv, d, topk, int(chunk), _lib.stream_of(q))
        return out
    entry = "mrsa_selected_attention_f16v" if v.dtype == torch.float16 else "mrsa_selected_attention"
    _lib.call(entry, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(kv),
              _lib.ptr(w), _lib.ptr(idx), _lib.ptr(lo), _lib.ptr(lw), _lib.ptr(out), scale,
              int(bool(mask_last_token)), b, lq, lk, hkv, hq // hkv, d, topk, int(chunk),
              _lib.stream_of(q))
    return out


def selected_attention_backward(q, k, v, weights, indices, grad_out, key_valid=None, *, chunk: int = 64,
                                mask_last_token=True, sm_scale=None):
    """Gradients of :func:`selected_attention` (no local merge) for bf16 q, k,
    v: ``(dq, dk, dv)`` in fp32 and ``dweights`` in bf16, as the reference's
    backward kernel returns them before its casts
    (``ops/hils_fwd_bwd_head.py:1044-1098``).  ``dweights[l, h, k]`` is
    ``sum_s P dP`` of slot k's chunk (0 for an empty slot); the gradients of a
    chunk listed twice by a query follow the forward's shared softmax."""
    b, lq, hq, d = q.shape
    lk, hkv = k.shape[1], k.shape[2]
    topk = indices.shape[-1]
    dev = q.device
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("the selected-attention backward requires BF16 q, k and v")
    if tuple(grad_out.shape) != (b, lq, hq, d):
        raise ValueError(f"grad_out must have shape {(b, lq, hq, d)}, got {tuple(grad_out.shape)}")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    go = grad_out.to(torch.bfloat16).contiguous()
    w = weights.to(torch.bfloat16).contiguous()
    idx = indices.to(device=dev, dtype=torch.int32).contiguous()
    kv = None if key_valid is None else key_valid.to(device=dev, dtype=torch.bool).contiguous()
    dq = torch.empty(b, lq, hq, d, dtype=torch.float32, device=dev)
    dk = torch.empty(b, lk, hkv, d, dtype=torch.float32, device=dev)
    dv = torch.empty_like(dk)
    dw = torch.empty(b, lq, hq, topk, dtype=torch.bfloat16, device=dev)
    scale = float(d) ** -0.5 if sm_scale is None else float(sm_scale)
    lib = _lib.load()
    ws_bytes = lib.mrsa_selected_attention_backward_workspace(b, lq, lk, hkv, topk)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=dev)
    _lib.call("mrsa_selected_attention_backward", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(kv),
              _lib.ptr(w), _lib.ptr(idx), _lib.ptr(go), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(dw),
              scale, int(bool(mask_last_token)), b, lq, lk, hkv, hq // hkv, d, topk, int(chunk),
              _lib.ptr(ws), int(ws_bytes), _lib.stream_of(q))
    return dq, dk, dv, dw


class _SelectedAttention(torch.autograd.Function):
    """Selected-chunk attention with the B200 backward
    (``ops/hils_fwd_bwd_head.py:915-1098 _hils_block_M_attention_inverse``)."""

    @staticmethod
    def forward(ctx, q, k, v, weights, indices, key_valid, chunk, mask_last_token, sm_scale):
        out = selected_attention(q, k, v, weights, indices, key_valid, chunk=chunk,
                                 mask_last_token=mask_last_token, sm_scale=sm_scale)
        ctx.save_for_backward(q, k, v, weights, indices, key_valid)
        ctx.cfg = (chunk, mask_last_token, sm_scale)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, weights, indices, key_valid = ctx.saved_tensors
        chunk, mask_last_token, sm_scale = ctx.cfg
        dq, dk, dv, dw = selected_attention_backward(q, k, v, weights, indices, grad_out, key_valid, chunk=chunk,
                                                     mask_last_token=mask_last_token, sm_scale=sm_scale)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dw.to(weights.dtype), None, None, None, None, None


def _needs_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def selected_attention_autograd(q, k, v, weights, indices, key_valid=None, *, chunk: int = 64,
                                mask_last_token=True, sm_scale=None):
    """:func:`selected_attention` that records the B200 backward for autograd
    (bf16 q, k, v; no token refinement)."""
    return _SelectedAttention.apply(q, k, v, weights, indices, key_valid, chunk, mask_last_token, sm_scale)


def to_f16(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 -> fp16 on the GPU (round to nearest; values beyond +-65504,
    infinities included, saturate and set bit 3 of the device error flags)."""
    if x.dtype != torch.bfloat16:
        raise ValueError(f"expected bf16, got {x.dtype}")
    x = x.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    _lib.call("mrsa_convert_bf16_to_f16", _lib.ptr(x), _lib.ptr(out), x.numel(), _lib.stream_of(x))
    return out


def _validate_g7(q, k, v, weights, indices, key_valid, chunk_size):
    # mirrors dream_dllm_hils/routing.py:368-425
    if q.ndim != 4 or k.ndim != 4:
        raise ValueError(f"q and k must be BLHD tensors, got {tuple(q.shape)} and {tuple(k.shape)}")
    batch, query_len, h_q, dim = q.shape
    if k.shape[0] != batch or k.shape[-1] != dim:
        raise ValueError(f"incompatible q/k shapes {tuple(q.shape)} and {tuple(k.shape)}")
    kv_len, h_kv = k.shape[1:3]
    if h_q != h_kv * _LOGICAL_G:
        raise ValueError(f"Dream G7 requires h_q == 7 * h_kv, got h_q={h_q}, h_kv={h_kv}")
    if v.shape != k.shape:
        raise ValueError(f"v shape {tuple(v.shape)} must match k shape {tuple(k.shape)}")
    selected = indices.shape[-1]
    if indices.shape != (batch, query_len, h_kv, selected):
        raise ValueError(f"invalid indices shape {tuple(indices.shape)}")
    if weights.shape != (batch, query_len, h_q, selected):
        raise ValueError(f"invalid weights shape {tuple(weights.shape)}")
    if key_valid.shape != (batch, kv_len):
        raise ValueError(f"invalid key_valid shape {tuple(key_valid.shape)}")
    if kv_len % chunk_size != 0:
        raise ValueError(f"cache length {kv_len} must be divisible by chunk_size={chunk_size}")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("selected attention requires BF16 q, k, and v")
    if q.device != k.device or v.device != q.device:
        raise ValueError("q, k, and v must share a device")
    if weights.device != q.device or indices.device != q.device:
        raise ValueError("weights and indices must share the q device")
    if key_valid.device != q.device:
        raise ValueError("key_valid must share the q device")
    if selected <= 0:
        raise ValueError("selected attention requires at least one chunk slot")


def selected_attention_g7(q, k, v, weights, indices, key_valid, chunk_size, training,
                          token_keep=None):
    """Selected-chunk attention with compact KV (``dream_dllm_hils/routing.py:305``)."""
    _validate_g7(q, k, v, weights, indices, key_valid, chunk_size)
    if token_keep is not None:
        # mirrors dream_dllm_hils/routing.py:393-419
        expect = (q.shape[0], q.shape[1], k.shape[2], indices.shape[-1], chunk_size)
        if tuple(token_keep.shape) != expect:
            raise ValueError(f"token_keep must have shape {expect}, got {tuple(token_keep.shape)}")
        if token_keep.device != q.device:
            raise ValueError("token_keep must share the q device")
    if training and _needs_grad(q, k, v, weights):
        if token_keep is not None:
            raise ValueError("token refinement has no backward on the B200 kernels")
        return selected_attention_autograd(q, k, v, weights, indices, key_valid, chunk=chunk_size)
    return selected_attention(q, k, v, weights, indices, key_valid, chunk=chunk_size, token_keep=token_keep)


def selected_attention_g7_cached(q, k, v, weights, indices, key_valid, chunk_size, token_keep=None):
    """Partial queries against a full K/V cache (``dream_dllm_hils/routing.py:330``)."""
    return selected_attention_g7(q, k, v, weights, indices, key_valid, chunk_size, False, token_keep)


def HiLS_block_M_head(q, k, v, weights, indices, block_size=64, sm_scale=None, block_M=None,
                      mask_last_token=True, dtype="bfloat16", accum_dtype="float", num_threads=None,
                      num_threads_fwd=None, num_threads_bwd=None, is_training=True, slope=None,
                      key_valid=None, token_keep=None):
    """``ops/hils_fwd_bwd_head.py:1113`` (q may carry padded heads; padded
    weights are zero).  With ``is_training`` and an input that requires grad
    the call records the B200 backward."""
    if slope is not None:
        raise ValueError("ALiBi slope is not supported by the B200 kernel")
    hq, hkv = q.shape[2], k.shape[2]
    if hq % hkv or hq // hkv > 8:
        raise ValueError("the B200 kernel supports query groups of at most 8 heads")
    if is_training and _needs_grad(q, k, v, weights):
        if token_keep is not None:
            raise ValueError("token refinement has no backward on the B200 kernels")
        return selected_attention_autograd(q, k, v, weights, indices, key_valid, chunk=block_size,
                                           mask_last_token=mask_last_token, sm_scale=sm_scale)
    return selected_attention(q, k, v, weights, indices, key_valid, chunk=block_size,
                              mask_last_token=mask_last_token, sm_scale=sm_scale, token_keep=token_keep)


def fuse_hils_outputs(remote_output, local_output, local_weight):
    """``bf16(remote + local_weight * local)`` (fp32 math)."""
    # mirrors ops/hils_bidir_output_fusion_tilelang.py:101-135
    if remote_output.shape != local_output.shape or remote_output.ndim != 4:
        raise ValueError("remote_output and local_output must be matching BLHD tensors")
    if local_weight.shape != remote_output.shape[:-1]:
        raise ValueError("local_weight must be [B,L,H]")
    if not (remote_output.dtype == local_output.dtype == local_weight.dtype == torch.bfloat16):
        raise ValueError("fuse_hils_outputs requires BF16 tensors")
    if not (remote_output.is_contiguous() and local_output.is_contiguous() and local_weight.is_contiguous()):
        raise ValueError("fuse_hils_outputs requires contiguous tensors")
    if torch.is_grad_enabled() and (remote_output.requires_grad or local_output.requires_grad
                                    or local_weight.requires_grad):
        return _FuseOutputs.apply(remote_output, local_output, local_weight)
    return _fuse_forward(remote_output, local_output, local_weight)


def _fuse_forward(remote_output, local_output, local_weight):
    out = torch.empty_like(remote_output)
    b, l, h, d = remote_output.shape
    _lib.call("mrsa_fuse_outputs", _lib.ptr(remote_output), _lib.ptr(local_output),
              _lib.ptr(local_weight), _lib.ptr(out), b * l * h, d, _lib.stream_of(out))
    return out


def fuse_outputs_backward(local_output, local_weight, grad_out):
    """``(d_remote, d_local, d_local_weight)`` in bf16
    (``ops/hils_bidir_output_fusion_tilelang.py:38-99``)."""
    b, l, h, d = local_output.shape
    g = grad_out.to(torch.bfloat16).contiguous()
    d_r, d_l = torch.empty_like(g), torch.empty_like(g)
    d_w = torch.empty(b, l, h, dtype=torch.bfloat16, device=g.device)
    _lib.call("mrsa_fuse_outputs_backward", _lib.ptr(local_output.contiguous()),
              _lib.ptr(local_weight.contiguous()), _lib.ptr(g), _lib.ptr(d_r), _lib.ptr(d_l), _lib.ptr(d_w),
              b * l * h, d, _lib.stream_of(g))
    return d_r, d_l, d_w


class _FuseOutputs(torch.autograd.Function):
    """``ops/hils_bidir_output_fusion_tilelang.py:102 _FuseHiLSOutputs`` on the B200 kernels."""

    @staticmethod
    def forward(ctx, remote_output, local_output, local_weight):
        ctx.save_for_backward(local_output, local_weight)
        return _fuse_forward(remote_output, local_output, local_weight)

    @staticmethod
    def backward(ctx, grad_out):
        local_output, local_weight = ctx.saved_tensors
        return fuse_outputs_backward(local_output, local_weight, grad_out)
