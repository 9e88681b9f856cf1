"""Route layer and SWA layer forward on one device.

``RouteLayer.forward`` replaces ``KernelDreamFullHiLSAttention.forward``
(``dream_dllm_hils/attention.py:1313-1774``) from the projected q/k/v and the
hidden state (Q-Cal input) to the input of ``o_proj``; ``swa_layer_forward``
replaces ``KernelDreamSlidingWindowAttention.forward`` (``:1168-1220``).
The default path is one C-ABI call (``mrsa_route_layer_forward``: six kernels
on the current stream over a cached workspace); ``stages=True`` runs the
same kernels one by one through the op shims and returns every intermediate.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .chunk_pool import chunk_attn_pool_gqa  # noqa: F401  (re-export for callers)
from .local_attention import window_attention
from .rope_fp32 import yarn_inv_freq, yarn_rope_qk
from .routing import route_topk_fused
from .selected_attention import selected_attention, to_f16


def raise_device_errors():
    """Read and clear the device error flags (synchronises with the device);
    raise when a kernel set one: bit 3 = V outside the fp16 range (the
    attention kernels take V in fp16; larger magnitudes saturate), bits 0-2
    = a selected-attention, routing or window kernel gave up on a bounded
    wait."""
    flags = int(_lib.load().mrsa_device_error_flags(1))
    if flags < 0:
        raise RuntimeError(f"could not read the device error flags ({_lib.load().mrsa_strerror(flags).decode()})")
    if flags & 8:
        raise ValueError("V holds values beyond the fp16 range (|v| > 65504); the route layer's "
                         "attention kernels take V in fp16")
    if flags:
        raise RuntimeError(f"a route-layer kernel gave up on a bounded wait (device error flags {flags:#x})")


@dataclass
class RouteLayerConfig:
    """Hot-path constants of the canonical config
    (``configs/from_dense16k/hils-s2-qcal-rmsnorm-rand-s1000-jingneng.json``)."""

    q_heads: int = 28
    kv_heads: int = 4
    head_dim: int = 128
    chunk: int = 64
    topk: int = 32
    local_window: int = 256
    swa_window: int = 1280
    qcal_rank: int = 64
    rope_theta: float = 1.0e6
    yarn_factor: float = 8.0
    yarn_orig_max_pos: int = 2048
    rms_eps: float = 1e-6
    qcal_scale: float = 1.0
    route_temperature: float = 1.0


class RouteLayer:
    """Weights and constants of one MRSA route layer.

    ``w_in [rank, hidden]``, ``w_out [Hq*D, rank]`` (bf16), ``norm_weight [D]``
    and ``entropy_bias_scale [Hq]`` (fp32), ``gate_offset``/``gate_scale``
    (the ``fusion_gate_*`` parameters, ``attention.py:913-914``)."""

    def __init__(self, w_in, w_out, norm_weight=None, entropy_bias_scale=None, *, gate_offset=0.0,
                 gate_scale=1.0, cfg: RouteLayerConfig | None = None, check_errors: bool = True):
        self.cfg = cfg or RouteLayerConfig()
        # read the device error flags after every fused forward (one small
        # synchronous read): V beyond the fp16 range, or a kernel that gave
        # up on a bounded wait, then raises instead of returning inf/NaN rows
        self.check_errors = bool(check_errors)
        dev = w_in.device
        if dev.type != "cuda":
            raise ValueError("RouteLayer weights must live on a CUDA device")
        c = self.cfg
        self.w_in = w_in.to(torch.bfloat16).contiguous()
        self.w_out = w_out.to(torch.bfloat16).contiguous()
        self.norm_weight = (torch.ones(c.head_dim, device=dev) if norm_weight is None
                            else norm_weight.to(device=dev, dtype=torch.float32).contiguous())
        self.bias_scale = (torch.ones(c.q_heads, device=dev) if entropy_bias_scale is None
                           else entropy_bias_scale.to(device=dev, dtype=torch.float32).contiguous())
        self.gate_offset = float(gate_offset)
        self.gate_scale = float(gate_scale)
        inv, af = yarn_inv_freq(c.head_dim, c.rope_theta, c.yarn_factor, c.yarn_orig_max_pos)
        self.inv_freq = inv.to(dev)
        self.attention_factor = af
        self._ws = None

    # ------------------------------------------------------------------ fused
    def _args(self, q_pre, k_pre, v, hidden, position_ids, key_valid, out):
        c = self.cfg
        b, l, hq, d = q_pre.shape
        a = _lib.RouteLayerArgs()
        a.q_pre, a.k_pre, a.v, a.hidden = (q_pre.data_ptr(), k_pre.data_ptr(), v.data_ptr(),
                                          hidden.data_ptr())
        a.position_ids = position_ids.data_ptr()
        a.key_valid = None if key_valid is None else key_valid.data_ptr()
        a.inv_freq = self.inv_freq.data_ptr()
        a.w_in, a.w_out = self.w_in.data_ptr(), self.w_out.data_ptr()
        a.norm_weight, a.bias_scale = self.norm_weight.data_ptr(), self.bias_scale.data_ptr()
        a.out = out.data_ptr()
        a.attention_factor, a.rms_eps, a.qcal_scale = self.attention_factor, c.rms_eps, c.qcal_scale
        a.temperature, a.gate_scale, a.gate_offset = (c.route_temperature, self.gate_scale,
                                                      self.gate_offset)
        a.batch, a.seq_len, a.q_heads, a.kv_heads, a.head_dim = b, l, hq, k_pre.shape[2], d
        a.hidden_size, a.rank, a.topk, a.local_window = (hidden.shape[-1], self.w_in.shape[0],
                                                         c.topk, c.local_window)
        return a

    def workspace_bytes(self, q_pre, k_pre, v, hidden, position_ids, key_valid=None):
        a = self._args(q_pre, k_pre, v, hidden, position_ids, key_valid, q_pre)
        return int(_lib.load().mrsa_route_layer_workspace_size(C.byref(a)))

    def forward(self, q_pre, k_pre, v, hidden, position_ids, key_valid=None, *, out=None,
                stages: bool = False):
        """Route-layer output ``[B, L, Hq, D]`` bf16 (pre ``o_proj``).
        ``stages=True`` returns a dict of every intermediate instead."""
        self._validate(q_pre, k_pre, v, hidden, position_ids, key_valid)
        q_pre, k_pre, v, hidden = (t.contiguous() for t in (q_pre, k_pre, v, hidden))
        position_ids = position_ids.contiguous()
        if key_valid is not None:
            key_valid = key_valid.to(torch.bool).contiguous()
        if stages:
            return self._forward_stages(q_pre, k_pre, v, hidden, position_ids, key_valid)
        if out is None:
            out = torch.empty_like(q_pre)
        a = self._args(q_pre, k_pre, v, hidden, position_ids, key_valid, out)
        need = int(_lib.load().mrsa_route_layer_workspace_size(C.byref(a)))
        if need == 0:
            raise ValueError("unsupported route-layer shape")
        if self._ws is None or self._ws.numel() < need or self._ws.device != q_pre.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=q_pre.device)
        _lib.call("mrsa_route_layer_forward", C.byref(a), C.c_void_p(self._ws.data_ptr()),
                  C.c_size_t(self._ws.numel()), _lib.stream_of(q_pre))
        if self.check_errors:
            raise_device_errors()
        return out

    __call__ = forward

    def _validate(self, q_pre, k_pre, v, hidden, position_ids, key_valid):
        c = self.cfg
        if q_pre.ndim != 4 or k_pre.ndim != 4 or v.shape != k_pre.shape:
            raise ValueError("q/k/v must be BLHD with matching k and v")
        b, l, hq, d = q_pre.shape
        if (hq, k_pre.shape[2], d) != (c.q_heads, c.kv_heads, c.head_dim):
            raise ValueError(f"expected {c.q_heads}/{c.kv_heads} heads of dim {c.head_dim}")
        if l % c.chunk:
            raise ValueError(f"sequence length {l} must be divisible by chunk_size={c.chunk}")
        for t in (q_pre, k_pre, v, hidden):
            if t.dtype != torch.bfloat16 or t.device != self.w_in.device:
                raise ValueError("q/k/v/hidden must be BF16 on the layer's device")
        if hidden.shape[:2] != (b, l) or hidden.shape[2] != self.w_in.shape[1]:
            raise ValueError(f"hidden must be [B, L, {self.w_in.shape[1]}]")
        if position_ids.shape != (b, l) or position_ids.dtype != torch.long:
            raise ValueError("position_ids must be int64 [B, L]")
        if key_valid is not None and key_valid.shape != (b, l):
            raise ValueError("key_valid must be [B, L]")

    # ------------------------------------------------------------------ timing
    STAGES = ("rope", "local_attention", "qcal", "pool", "route", "selected_attention")

    def stage_times(self, q_pre, k_pre, v, hidden, position_ids, key_valid=None, reps: int = 5):
        """Average device milliseconds of each of the six kernels of the fused
        path, from CUDA events on the current stream around each launch."""
        res = None
        for _ in range(reps + 1):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.STAGES) + 1)]
            self._forward_stages(q_pre, k_pre, v, hidden, position_ids, key_valid, events=ev)
            torch.cuda.synchronize()
            t = [ev[i].elapsed_time(ev[i + 1]) for i in range(len(self.STAGES))]
            if res is None:
                res = [0.0] * len(t)          # first pass warms the allocator
            else:
                res = [a + b for a, b in zip(res, t)]
        return {n: v / reps for n, v in zip(self.STAGES, res)}

    # ------------------------------------------------------------------ staged
    def _forward_stages(self, q_pre, k_pre, v, hidden, position_ids, key_valid, events=None):
        c = self.cfg
        mark = (lambda i: events[i].record()) if events is not None else (lambda i: None)
        b, l, hq, d = q_pre.shape
        hkv = k_pre.shape[2]
        g = hq // hkv
        nc = l // c.chunk
        dev = q_pre.device
        st = _lib.stream_of(q_pre)
        local_out = torch.empty_like(q_pre)
        local_lse = torch.empty(b, l, hq, device=dev, dtype=torch.float32)
        route_q = torch.empty_like(q_pre)
        lmk = torch.empty(b, nc, hkv, g, d, device=dev, dtype=torch.bfloat16)
        ent = torch.empty(b, nc, hkv, g, device=dev, dtype=torch.float32)
        prior = torch.empty_like(ent)
        chunk_ok = torch.empty(b, nc, device=dev, dtype=torch.uint8)
        out = torch.empty_like(q_pre)
        mark(0)
        q, k = yarn_rope_qk(q_pre, k_pre, position_ids, self.inv_freq, self.attention_factor)
        mark(1)
        v16 = to_f16(v)                      # as the fused layer: fp16 V, one fp16 P tile
        window_attention(q, k, v16, key_valid, c.local_window + c.chunk - 1, skip_inert=True,
                         chunk=c.chunk, out=local_out, lse=local_lse)
        mark(2)
        _lib.call("mrsa_qcal_route_query", _lib.ptr(hidden), _lib.ptr(q), _lib.ptr(self.w_in),
                  _lib.ptr(self.w_out), _lib.ptr(self.norm_weight), float(c.rms_eps),
                  float(c.qcal_scale), _lib.ptr(position_ids), _lib.ptr(self.inv_freq),
                  float(self.attention_factor), _lib.ptr(route_q), b, l, hidden.shape[-1],
                  self.w_in.shape[0], hq, d, st)
        mark(3)
        mu = route_q[:, c.chunk - 1:]
        _lib.call("mrsa_chunk_pool", C.c_void_p(mu.data_ptr()), l * hq * d, c.chunk * hq * d,
                  _lib.ptr(k), _lib.ptr(key_valid), d ** -0.5, _lib.ptr(self.bias_scale),
                  _lib.ptr(lmk), _lib.ptr(ent), _lib.ptr(prior), _lib.ptr(chunk_ok),
                  b, nc, hkv, g, d, st)
        mark(4)
        idx, scores, rw, lw = route_topk_fused(route_q, lmk, local_lse, prior, chunk_ok, c.topk,
                                               c.local_window, temperature=c.route_temperature,
                                               gate_scale=self.gate_scale,
                                               gate_offset=self.gate_offset)
        mark(5)
        selected_attention(q, k, v16, rw, idx, key_valid, chunk=c.chunk, local_out=local_out,
                           local_weight=lw, out=out)
        mark(6)
        if events is not None:
            return None
        remote = selected_attention(q, k, v16, rw, idx, key_valid, chunk=c.chunk)
        return {"q": q, "k": k, "route_q": route_q, "local_out": local_out, "local_lse": local_lse,
                "lmk": lmk, "entropy": ent, "prior_bias": prior, "chunk_ok": chunk_ok,
                "indices": idx, "scores": scores, "remote_weights": rw, "local_weight": lw,
                "remote_out": remote, "out": out}


def swa_layer_forward(q_pre, k_pre, v, position_ids, key_valid=None, *, window: int = 1280,
                      cfg: RouteLayerConfig | None = None, inv_freq=None, attention_factor=None,
                      return_lse: bool = False):
    """SWA layer: YaRN RoPE then bidirectional window-``window`` attention with
    landmarks as ordinary keys (``attention.py:1208-1218``)."""
    c = cfg or RouteLayerConfig()
    if inv_freq is None:
        inv_freq, attention_factor = yarn_inv_freq(c.head_dim, c.rope_theta, c.yarn_factor,
                                                   c.yarn_orig_max_pos)
    q, k = yarn_rope_qk(q_pre, k_pre, position_ids, inv_freq.to(q_pre.device), attention_factor)
    out, lse = window_attention(q, k, v, key_valid, window, skip_inert=False, chunk=c.chunk,
                                need_lse=return_lse)
    return (out, lse) if return_lse else out
