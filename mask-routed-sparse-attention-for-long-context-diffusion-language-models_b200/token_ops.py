"""Token-granular ops off the route layer's live path, on the B200 kernels of
``csrc/token_ops.cu``:

* :func:`candidate_token_scores_gqa` -- ``ops/hils_token_score_gqa_tilelang.py:174``
  (token refinement, ``dream_dllm_hils/token_refinement.py:377-420``);
* :func:`selected_token_attention_tilelang` -- ``ops/dsa_selected_attention_tilelang.py:593``
  (the DSA / NSA baselines, ``dream_dllm_hils/dsa_attention.py:664``), forward.

Both raise ``ValueError`` on the reference's layout errors; there is no CPU
fallback.
"""

from __future__ import annotations

import torch

from . import _lib


def candidate_token_scores_gqa(q: torch.Tensor, k: torch.Tensor, indices: torch.Tensor,
                               key_valid: torch.Tensor, chunk_size: int) -> torch.Tensor:
    """FP32 ``[B, Lq, Hkv, K, S]``: per selected chunk, the max over the
    query group of ``q_g . k_s / sqrt(D)`` for every slot s, ``-inf`` for
    negative chunk indices, the landmark slot ``S - 1`` and invalid keys."""
    # mirrors ops/hils_token_score_gqa_tilelang.py:119-171
    if q.device.type != "cuda":
        raise ValueError("candidate_token_scores_gqa requires CUDA tensors")
    if not (q.device == k.device == indices.device == key_valid.device):
        raise ValueError("all token-score tensors must share one CUDA device")
    if q.ndim != 4 or k.ndim != 4 or indices.ndim != 4:
        raise ValueError("q, k, and indices must be rank-four tensors")
    batch, query_len, query_heads, head_dim = q.shape
    if k.shape[0] != batch or k.shape[-1] != head_dim:
        raise ValueError(f"incompatible q/k shapes {tuple(q.shape)} and {tuple(k.shape)}")
    kv_len, kv_heads = k.shape[1:3]
    if query_heads % kv_heads:
        raise ValueError(f"query_heads={query_heads} must divide kv_heads={kv_heads}")
    selected = indices.shape[-1]
    if indices.shape != (batch, query_len, kv_heads, selected):
        raise ValueError(f"invalid indices shape {tuple(indices.shape)}")
    if key_valid.shape != (batch, kv_len):
        raise ValueError(f"invalid key_valid shape {tuple(key_valid.shape)}")
    if chunk_size < 16 or kv_len % chunk_size:
        raise ValueError(f"kv_len={kv_len} must be divisible by chunk_size >= 16")
    if head_dim != 128:
        raise ValueError(f"the B200 kernel supports head_dim 128, got {head_dim}")
    if query_heads // kv_heads > 16:
        raise ValueError("the B200 kernel supports query groups of at most 16 heads")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise ValueError("candidate_token_scores_gqa requires BF16 q and k")
    if indices.dtype != torch.int32:
        raise ValueError("indices must be int32")
    if not (q.is_contiguous() and k.is_contiguous() and indices.is_contiguous() and key_valid.is_contiguous()):
        raise ValueError("candidate_token_scores_gqa requires contiguous tensors")
    kv = key_valid.to(dtype=torch.bool).contiguous()
    scores = torch.empty(batch, query_len, kv_heads, selected, chunk_size, device=q.device,
                         dtype=torch.float32)
    if scores.numel() == 0:
        return scores
    _lib.call("mrsa_candidate_token_scores", _lib.ptr(q), _lib.ptr(k), _lib.ptr(indices), _lib.ptr(kv),
              _lib.ptr(scores), float(head_dim) ** -0.5, batch, query_len, kv_len, query_heads, kv_heads,
              head_dim, selected, int(chunk_size), _lib.stream_of(q))
    return scores


def selected_token_attention_tilelang(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                      indices: torch.Tensor, valid: torch.Tensor, *,
                                      sm_scale: float | None = None) -> torch.Tensor:
    """Exact GQA attention of each query row over its own token list
    ``indices [B, Lq, topk]`` (clamped to ``[0, Lk)``; entries with
    ``valid == False`` are out).  fp32 softmax, probabilities rounded to bf16
    before ``P.V``; rows without a valid entry are 0.  Forward only."""
    # mirrors ops/dsa_selected_attention_tilelang.py:482-532
    if q.device.type != "cuda":
        raise ValueError("Dream DSA TileLang attention requires CUDA tensors")
    if not (q.device == k.device == v.device == indices.device == valid.device):
        raise ValueError("all Dream DSA TileLang tensors must share one device")
    if q.ndim != 4 or k.ndim != 4 or v.shape != k.shape:
        raise ValueError("q/k/v must have [B,L,H,D] GQA layouts")
    if q.shape[0] != k.shape[0] or q.shape[-1] != k.shape[-1]:
        raise ValueError("Dream DSA requires matching Q/K batch and head dims")
    if q.shape[0:2] != indices.shape[0:2] or valid.shape != indices.shape or indices.ndim != 3:
        raise ValueError("indices/valid must have shape [B,L,topk]")
    if q.shape[2] % k.shape[2]:
        raise ValueError("query heads must be divisible by KV heads")
    if q.shape[-1] != 128:
        raise ValueError(f"Dream DSA TileLang kernel currently requires head_dim=128, got {q.shape[-1]}")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("Dream DSA TileLang attention requires BF16 q/k/v")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("Dream DSA TileLang q/k/v tensors must be contiguous")
    batch, query_len, query_heads, head_dim = q.shape
    kv_len, kv_heads = k.shape[1:3]
    groups = query_heads // kv_heads
    if groups > 16:
        raise ValueError("the B200 kernel supports query groups of at most 16 heads")
    topk = indices.shape[-1]
    lib = _lib.load()
    if topk > 0 and lib.mrsa_selected_token_attention_smem(groups, topk) > 232448:
        raise ValueError(f"topk={topk} with {groups} heads per group exceeds the kernel's shared memory")
    scale = float(head_dim) ** -0.5 if sm_scale is None else float(sm_scale)
    # the reference clamps to [0, Lk-1] before its int32 cast (ops/dsa_selected_attention_tilelang.py:511-531)
    idx = indices.clamp(min=0, max=kv_len - 1).to(torch.int32).contiguous()
    keep = valid.to(torch.bool).contiguous()
    out = torch.empty_like(q)
    if out.numel() == 0:
        return out
    if topk == 0:
        return out.zero_()
    _lib.call("mrsa_selected_token_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(idx),
              _lib.ptr(keep), _lib.ptr(out), scale, batch, query_len, kv_len, query_heads, kv_heads,
              head_dim, topk, _lib.stream_of(q))
    return out
