"""Dream-7B-shaped (Qwen2, bidirectional) forward around the B200 attention.

The reference runs its attention inside Dream's remote modeling code, which is
not part of the checkout; this module is the stand-in the reference's
benchmark config describes (28 layers, hidden 3584, SwiGLU FFN 18944, 28/4
heads of 128, vocab 152064, RMSNorm eps 1e-6, route layers at
``idx % 4 == 3`` as ``dream_dllm_hils/attention.py:1823-1826`` installs them,
the other 21 layers bidirectional SWA-1280).  Around the attention it keeps
Qwen2's decoder layer: pre-norm, q/k/v projections with bias, ``o_proj``,
residuals, SwiGLU MLP, final norm and ``lm_head``.  Every stage runs on this
package's kernels: the projections, the MLP and ``lm_head`` on the tcgen05
GEMM with the bias, SwiGLU and residual epilogues fused (``dense.py``),
RMSNorm on its own kernel, and the attention on the fused route layer or on
RoPE plus the window kernel with fp16 V.  The landmark role offset is added to the input
embeddings at landmark slots (``train_fulltext.py:2339-2351``).  Weights are
random N(0, 0.02) (biases zero, norm weights one): no checkpoint is available.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .dense import interleave_gate_up, linear, linear_residual, rms_norm, swiglu
from .layer import RouteLayer, RouteLayerConfig
from .local_attention import window_attention
from .rope_fp32 import yarn_inv_freq, yarn_rope_qk
from .selected_attention import to_f16


@dataclass(frozen=True)
class DreamConfig:
    layers: int = 28
    hidden: int = 3584
    ffn: int = 18944
    q_heads: int = 28
    kv_heads: int = 4
    head_dim: int = 128
    vocab: int = 152064
    rms_eps: float = 1e-6
    chunk: int = 64
    topk: int = 32
    local_window: int = 256
    swa_window: int = 1280
    qcal_rank: int = 64
    route_every: int = 4          # route layers: idx % route_every == route_every - 1

    def is_route(self, idx: int) -> bool:
        return idx % self.route_every == self.route_every - 1

    def layer_cfg(self) -> RouteLayerConfig:
        return RouteLayerConfig(q_heads=self.q_heads, kv_heads=self.kv_heads, head_dim=self.head_dim,
                                chunk=self.chunk, topk=self.topk, local_window=self.local_window,
                                swa_window=self.swa_window, qcal_rank=self.qcal_rank, rms_eps=self.rms_eps)


def landmark_inputs(batch: int, seq_len: int, cfg: DreamConfig, *, mask_id: int, mask_frac: float = 0.3,
                    seed: int = 0, device="cuda"):
    """Token ids of the benchmark config: uniform ids, the mask token at every
    landmark slot (``(i + 1) % chunk == 0``) and on ``mask_frac`` of the other
    positions; landmark-layout position ids (text position ``c*(chunk-1)+s``)."""
    g = torch.Generator(device=device).manual_seed(seed)
    ids = torch.randint(0, cfg.vocab, (batch, seq_len), device=device, generator=g)
    masked = torch.rand(batch, seq_len, device=device, generator=g) < mask_frac
    i = torch.arange(seq_len, device=device)
    lmk = (i + 1) % cfg.chunk == 0
    ids = torch.where(masked | lmk[None], torch.full_like(ids, mask_id), ids)
    pos = (i - i // cfg.chunk).expand(batch, seq_len).contiguous()
    return ids, pos, lmk


class DreamForward:
    """Random-init Dream-shaped model; ``forward(ids, position_ids)`` returns
    logits ``[B, L, vocab]`` bf16 (or the final hidden states)."""

    def __init__(self, cfg: DreamConfig = DreamConfig(), *, seed: int = 0, device="cuda"):
        self.cfg = c = cfg
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, device=dev, generator=g) * 0.02).bfloat16()

        qd, kd = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
        self.embed = w(c.vocab, c.hidden)
        self.role = w(c.hidden)
        self.layers = []
        lcfg = c.layer_cfg()
        for idx in range(c.layers):
            lay = {
                "in_norm": torch.ones(c.hidden, device=dev, dtype=torch.bfloat16),
                "post_norm": torch.ones(c.hidden, device=dev, dtype=torch.bfloat16),
                "wq": w(qd, c.hidden), "bq": torch.zeros(qd, device=dev, dtype=torch.bfloat16),
                "wk": w(kd, c.hidden), "bk": torch.zeros(kd, device=dev, dtype=torch.bfloat16),
                "wv": w(kd, c.hidden), "bv": torch.zeros(kd, device=dev, dtype=torch.bfloat16),
                "wo": w(c.hidden, qd),
            }
            lay["wgu"] = interleave_gate_up(w(c.ffn, c.hidden), w(c.ffn, c.hidden))
            lay["wd"] = w(c.hidden, c.ffn)
            if c.is_route(idx):
                lay["route"] = RouteLayer(w(c.qcal_rank, c.hidden), w(qd, c.qcal_rank), cfg=lcfg)
            self.layers.append(lay)
        self.final_norm = torch.ones(c.hidden, device=dev, dtype=torch.bfloat16)
        self.lm_head = w(c.vocab, c.hidden)
        inv, af = yarn_inv_freq(c.head_dim, lcfg.rope_theta, lcfg.yarn_factor, lcfg.yarn_orig_max_pos)
        self.inv_freq, self.attention_factor = inv.to(dev), af

    def rms_norm(self, x, weight):
        # Qwen2RMSNorm: fp32 statistics, back to the input dtype, times the weight
        return rms_norm(x, weight, self.cfg.rms_eps)

    def gate_up(self, idx):
        """The gate and up weights ``[F, H]`` of layer ``idx`` (copies out of
        the interleaved SwiGLU operand)."""
        wgu, c = self.layers[idx]["wgu"], self.cfg
        blocks = wgu.view(c.ffn // 128, 2, 128, c.hidden)
        return blocks[:, 0].reshape(c.ffn, c.hidden), blocks[:, 1].reshape(c.ffn, c.hidden)

    def attention(self, idx, h, position_ids, key_valid):
        """Attention output of layer ``idx`` before ``o_proj``: ``[B, L, Hq*D]``."""
        c, lay = self.cfg, self.layers[idx]
        b, l, _ = h.shape
        q = linear(h, lay["wq"], lay["bq"]).view(b, l, c.q_heads, c.head_dim)
        k = linear(h, lay["wk"], lay["bk"]).view(b, l, c.kv_heads, c.head_dim)
        v = linear(h, lay["wv"], lay["bv"]).view(b, l, c.kv_heads, c.head_dim)
        if "route" in lay:
            o = lay["route"].forward(q, k, v, h, position_ids, key_valid)
        else:
            qr, kr = yarn_rope_qk(q, k, position_ids, self.inv_freq, self.attention_factor)
            o, _ = window_attention(qr, kr, to_f16(v.contiguous()), key_valid, c.swa_window,
                                    skip_inert=False, chunk=c.chunk, need_lse=False)
        return o.reshape(b, l, c.q_heads * c.head_dim)

    def layer(self, idx, x, position_ids, key_valid):
        lay = self.layers[idx]
        h = self.rms_norm(x, lay["in_norm"])
        x = linear_residual(self.attention(idx, h, position_ids, key_valid), lay["wo"], x)
        h = self.rms_norm(x, lay["post_norm"])
        return linear_residual(swiglu(h, lay["wgu"]), lay["wd"], x)

    @torch.inference_mode()
    def forward(self, ids, position_ids, key_valid=None, *, logits: bool = True, return_layer_inputs=False):
        lmk = (torch.arange(ids.shape[1], device=ids.device) + 1) % self.cfg.chunk == 0
        x = self.embed[ids]
        x = torch.where(lmk[None, :, None], x + self.role, x)
        inputs = []
        for idx in range(self.cfg.layers):
            if return_layer_inputs:
                inputs.append(x)
            x = self.layer(idx, x, position_ids, key_valid)
        out = self.rms_norm(x, self.final_norm)
        if logits:
            out = linear(out, self.lm_head)
        return (out, inputs) if return_layer_inputs else out

    __call__ = forward

    def flops_per_token(self, seq_len: int) -> float:
        """Dense GEMM FLOPs per token (projections, MLP, lm_head) plus the
        attention's algorithmic FLOPs (route: local band + selected tiles +
        routing + Q-Cal; SWA: band)."""
        c = self.cfg
        qd, kd = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
        per_layer = 2 * c.hidden * (qd + 2 * kd) + 2 * qd * c.hidden + 3 * 2 * c.hidden * c.ffn
        n_route = sum(c.is_route(i) for i in range(c.layers))
        n_swa = c.layers - n_route
        wl = c.local_window + c.chunk - 1
        route_attn = (c.q_heads * c.head_dim * 4 * (2 * wl + 1) + c.q_heads * c.topk * c.chunk * c.head_dim * 4
                      + 2 * 2 * c.q_heads * (seq_len // c.chunk) * c.head_dim
                      + 2 * (c.hidden * c.qcal_rank + c.qcal_rank * qd))
        swa_attn = c.q_heads * c.head_dim * 4 * (2 * c.swa_window + 1)
        return (c.layers * per_layer + 2 * c.hidden * c.vocab + n_route * route_attn + n_swa * swa_attn)


def model_parameters(cfg: DreamConfig) -> int:
    c = cfg
    qd, kd = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
    per_layer = c.hidden * (qd + 2 * kd) + qd + 2 * kd + qd * c.hidden + 3 * c.hidden * c.ffn + 2 * c.hidden
    n_route = sum(c.is_route(i) for i in range(c.layers))
    return (c.layers * per_layer + n_route * (c.qcal_rank * (c.hidden + qd)) + 2 * c.vocab * c.hidden
            + 2 * c.hidden)


__all__ = ["DreamConfig", "DreamForward", "landmark_inputs", "model_parameters"]
