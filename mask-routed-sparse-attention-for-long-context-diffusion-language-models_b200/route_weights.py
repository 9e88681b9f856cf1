"""Route weights on the B200 kernels (forward and backward).

Drop-ins for ``ops/hils_bidir_route_weights_tilelang.py:276 route_weights``
(one softmax over the K remote logits and the local LSE; any K <= 32, not
only K <= 31) and ``dream_dllm_hils/attention.py:126 _route_weights_torch``
(the affine-gate branch of the live path; Gumbel and value bonus are
training-only and not supported).
"""

from __future__ import annotations

import torch

from . import _lib


def _launch(scores, indices, prior_bias, local_lse, mode, temperature, gate_scale, gate_offset):
    if scores.ndim != 4 or indices.ndim != 4 or prior_bias.ndim != 4:
        raise ValueError("scores, indices, and prior_bias must be 4D")
    if local_lse.ndim != 3:
        raise ValueError("local_lse must be [B,L,Hq]")
    batch, seq_len, h_q, topk = scores.shape
    bias_batch, chunks, kv_heads, groups = prior_bias.shape
    if groups <= 0 or h_q != kv_heads * groups:
        raise ValueError(f"invalid grouped-head layout Hq={h_q}, Hkv={kv_heads}, G={groups}")
    if bias_batch != batch or chunks <= 0:
        raise ValueError(f"invalid prior_bias shape {tuple(prior_bias.shape)}")
    if indices.shape != (batch, seq_len, kv_heads, topk):
        raise ValueError(f"invalid indices shape {tuple(indices.shape)}")
    if local_lse.shape != (batch, seq_len, h_q):
        raise ValueError(f"invalid local_lse shape {tuple(local_lse.shape)}")
    if topk < 1 or topk > 32:
        raise ValueError(f"route weights support 1 <= topk <= 32, got {topk}")
    if scores.device.type != "cuda":
        raise ValueError("route_weights requires CUDA tensors")
    dev = scores.device
    sc = scores.to(torch.bfloat16).contiguous()
    idx = indices.to(device=dev, dtype=torch.int32).contiguous()
    pb = prior_bias.to(device=dev, dtype=torch.float32).contiguous()
    ll = local_lse.to(device=dev, dtype=torch.float32).contiguous()
    rw = torch.empty(batch, seq_len, h_q, topk, device=dev, dtype=torch.bfloat16)
    lw = torch.empty(batch, seq_len, h_q, device=dev, dtype=torch.bfloat16)
    _lib.call("mrsa_route_weights", _lib.ptr(sc), _lib.ptr(idx), _lib.ptr(pb), _lib.ptr(ll),
              _lib.ptr(rw), _lib.ptr(lw), mode, float(temperature), float(gate_scale),
              float(gate_offset), batch, seq_len, chunks, kv_heads, groups, topk, _lib.stream_of(sc))
    return rw, lw


def route_weights_backward(scores, indices, prior_bias, local_lse, grad_remote, grad_local, *, mode: int,
                           temperature: float = 1.0, gate_scale: float = 1.0, gate_offset: float = 0.0):
    """``(d_scores, d_prior, d_local_lse, d_gate_scale, d_gate_offset)`` in fp32
    (the gate gradients as 0-d tensors): the backward of the softmax kernel
    (``ops/hils_bidir_route_weights_tilelang.py:97-166``) or of the affine-gate
    branch of ``dream_dllm_hils/attention.py:126-227``."""
    batch, seq_len, h_q, topk = scores.shape
    _, chunks, kv_heads, groups = prior_bias.shape
    dev = scores.device
    sc = scores.to(torch.bfloat16).contiguous()
    idx = indices.to(device=dev, dtype=torch.int32).contiguous()
    pb = prior_bias.to(device=dev, dtype=torch.float32).contiguous()
    ll = local_lse.to(device=dev, dtype=torch.float32).contiguous()
    gr = (torch.zeros_like(sc) if grad_remote is None else grad_remote.to(torch.bfloat16)).contiguous()
    gl = (torch.zeros(batch, seq_len, h_q, dtype=torch.bfloat16, device=dev) if grad_local is None
          else grad_local.to(torch.bfloat16)).contiguous()
    d_sc = torch.empty(batch, seq_len, h_q, topk, dtype=torch.float32, device=dev)
    d_pb = torch.empty(batch, chunks, kv_heads, groups, dtype=torch.float32, device=dev)
    d_ll = torch.empty(batch, seq_len, h_q, dtype=torch.float32, device=dev)
    d_gate = torch.empty(2, dtype=torch.float32, device=dev)
    _lib.call("mrsa_route_weights_backward", _lib.ptr(sc), _lib.ptr(idx), _lib.ptr(pb), _lib.ptr(ll),
              _lib.ptr(gr), _lib.ptr(gl), _lib.ptr(d_sc), _lib.ptr(d_pb), _lib.ptr(d_ll), _lib.ptr(d_gate),
              mode, float(temperature), float(gate_scale), float(gate_offset), batch, seq_len, chunks,
              kv_heads, groups, topk, _lib.stream_of(sc))
    return d_sc, d_pb, d_ll, d_gate[0], d_gate[1]


class _RouteWeights(torch.autograd.Function):
    """Route weights with the B200 backward; the gate scale / offset are
    0-d tensors (or None) so that their gradients reach the module parameters."""

    @staticmethod
    def forward(ctx, scores, indices, prior_bias, local_lse, gate_scale, gate_offset, mode, temperature):
        gs = 1.0 if gate_scale is None else float(gate_scale)
        go = 0.0 if gate_offset is None else float(gate_offset)
        rw, lw = _launch(scores, indices, prior_bias, local_lse, mode, temperature, gs, go)
        ctx.save_for_backward(scores, indices, prior_bias, local_lse)
        ctx.cfg = (mode, temperature, gs, go, gate_scale is not None, gate_offset is not None, scores.dtype)
        return rw.to(scores.dtype), lw.to(scores.dtype)

    @staticmethod
    def backward(ctx, grad_rw, grad_lw):
        scores, indices, prior_bias, local_lse = ctx.saved_tensors
        mode, temperature, gs, go, has_gs, has_go, dtype = ctx.cfg
        d_sc, d_pb, d_ll, d_gs, d_go = route_weights_backward(
            scores, indices, prior_bias, local_lse, grad_rw, grad_lw, mode=mode, temperature=temperature,
            gate_scale=gs, gate_offset=go)
        need = ctx.needs_input_grad
        return (d_sc.to(dtype), None, d_pb.to(prior_bias.dtype), d_ll.to(local_lse.dtype),
                d_gs if has_gs and need[4] else None, d_go if has_go and need[5] else None, None, None)


def _wants_grad(*xs) -> bool:
    return torch.is_grad_enabled() and any(isinstance(x, torch.Tensor) and x.requires_grad for x in xs)


def route_weights(scores: torch.Tensor, indices: torch.Tensor, prior_bias: torch.Tensor,
                  local_lse: torch.Tensor):
    """Normalise selected remote branches together with the local branch."""
    if scores.dtype != torch.bfloat16:
        raise ValueError("route_weights requires BF16 scores")
    if prior_bias.dtype != torch.float32 or local_lse.dtype != torch.float32:
        raise ValueError("prior_bias and local_lse must be FP32")
    if _wants_grad(scores, prior_bias, local_lse):
        return _RouteWeights.apply(scores, indices, prior_bias, local_lse, None, None, _lib.WEIGHTS_SOFTMAX, 1.0)
    return _launch(scores, indices, prior_bias, local_lse, _lib.WEIGHTS_SOFTMAX, 1.0, 1.0, 0.0)


def route_weights_torch(scores, indices, prior_bias, local_lse, *, temperature: float,
                        selected_gumbel=None, value_bonus=None, return_gate_logit=False,
                        gate_offset=None, gate_scale=None):
    """Signature of ``_route_weights_torch``.  With ``gate_scale`` the affine
    sigmoid gate of the live path; without, one softmax over remote logits and
    ``local_lse - gate_offset``."""
    if temperature <= 0:
        raise ValueError(f"temperature must be positive, got {temperature}")
    if selected_gumbel is not None or value_bonus is not None:
        raise ValueError("selected_gumbel / value_bonus are training-only and not supported")
    if gate_scale is not None:
        mode, gs = _lib.WEIGHTS_AFFINE, float(gate_scale.detach() if isinstance(gate_scale, torch.Tensor)
                                             else gate_scale)
    else:
        mode, gs = _lib.WEIGHTS_SOFTMAX, 1.0
    go = 0.0 if gate_offset is None else float(gate_offset.detach() if isinstance(gate_offset, torch.Tensor)
                                                else gate_offset)
    if _wants_grad(scores, prior_bias, local_lse, gate_scale, gate_offset):
        as_t = (lambda x: x.reshape(()) if isinstance(x, torch.Tensor) else
                (None if x is None else torch.tensor(float(x))))
        rw, lw = _RouteWeights.apply(scores, indices, prior_bias, local_lse,
                                     as_t(gate_scale) if gate_scale is not None else None, as_t(gate_offset),
                                     mode, float(temperature))
    else:
        rw, lw = _launch(scores, indices, prior_bias, local_lse, mode, temperature, gs, go)
        rw, lw = rw.to(scores.dtype), lw.to(scores.dtype)
    if not return_gate_logit:
        return rw, lw
    w_remote = rw.float().sum(-1).clamp(1e-6, 1 - 1e-6)
    w_local = lw.float().clamp(1e-6, 1 - 1e-6)
    return rw, lw, w_remote.log() - w_local.log()
