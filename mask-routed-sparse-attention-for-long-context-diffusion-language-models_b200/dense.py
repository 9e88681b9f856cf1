"""Dense layers of the Dream-shaped forward on the B200 kernels.

``linear`` / ``swiglu`` / ``linear_residual`` run ``mrsa_gemm_bf16`` (a
tcgen05 GEMM with the epilogue fused: bias, the Qwen2 SwiGLU, the residual
add) and ``rms_norm`` runs ``mrsa_rms_norm`` (Qwen2RMSNorm).  Weights keep
``nn.Linear``'s ``[out, in]`` layout; ``interleave_gate_up`` builds the
SwiGLU operand from the gate and up weights once.
"""

from __future__ import annotations

import torch

from . import _lib


def _gemm(a, b, bias, resid, out, mode):
    m, k = a.shape
    _lib.call("mrsa_gemm_bf16", _lib.ptr(a), _lib.ptr(b), _lib.ptr(bias), _lib.ptr(resid), _lib.ptr(out),
              m, b.shape[0], k, mode, _lib.stream_of(a))
    return out


def _flat(x):
    if x.dtype != torch.bfloat16:
        raise ValueError(f"expected bf16, got {x.dtype}")
    return x.reshape(-1, x.shape[-1]).contiguous()


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(x, weight, bias)`` in bf16 (fp32 accumulation, one rounding)."""
    a = _flat(x)
    out = torch.empty(a.shape[0], weight.shape[0], dtype=torch.bfloat16, device=a.device)
    _gemm(a, weight.contiguous(), None if bias is None else bias.to(torch.bfloat16).contiguous(), None, out,
          _lib.GEMM_PLAIN)
    return out.view(*x.shape[:-1], weight.shape[0])


def linear_residual(x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """``residual + F.linear(x, weight)`` (the linear rounded to bf16 first, as torch does)."""
    a = _flat(x)
    r = _flat(residual)
    out = torch.empty_like(r)
    _gemm(a, weight.contiguous(), None, r, out, _lib.GEMM_RESIDUAL)
    return out.view(residual.shape)


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """``[2F, H]`` operand of :func:`swiglu`: per 128-row block, the gate rows
    then the up rows (F % 128 == 0)."""
    f, h = w_gate.shape
    if w_up.shape != (f, h) or f % 128:
        raise ValueError("gate and up weights must share a [F, H] shape with F % 128 == 0")
    return torch.stack((w_gate.view(f // 128, 128, h), w_up.view(f // 128, 128, h)), 1).reshape(2 * f, h).contiguous()


def swiglu(x: torch.Tensor, w_gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(F.linear(x, w_gate)) * F.linear(x, w_up)`` from the interleaved operand."""
    a = _flat(x)
    out = torch.empty(a.shape[0], w_gate_up.shape[0] // 2, dtype=torch.bfloat16, device=a.device)
    _gemm(a, w_gate_up, None, None, out, _lib.GEMM_SWIGLU)
    return out.view(*x.shape[:-1], w_gate_up.shape[0] // 2)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen2RMSNorm: ``weight * bf16(x * rsqrt(mean(x^2) + eps))``."""
    a = _flat(x)
    out = torch.empty_like(a)
    _lib.call("mrsa_rms_norm", _lib.ptr(a), _lib.ptr(weight.to(torch.bfloat16).contiguous()), _lib.ptr(out),
              a.shape[0], a.shape[1], float(eps), _lib.stream_of(a))
    return out.view(x.shape)
