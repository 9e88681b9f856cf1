"""Install the B200 ops into the reference's modules as drop-ins.

``KernelDreamFullHiLSAttention.forward`` imports its ops lazily inside the
call (``dream_dllm_hils/attention.py:1343-1355``), ``dream_dllm_hils/routing.py``
binds ``HiLS_block_M_head`` / ``online_softmax_topk_head`` /
``ref_softmax_topk_max_pooling`` at import (``:8-12``), and
``_route_weights_torch`` is a module global of ``attention.py``.  Replacing
those attributes is enough for the reference layer to run on these kernels.
``install(fused_layer=True)`` additionally replaces the whole route-layer
forward with :class:`RouteLayer` (one C-ABI call after the projections).
"""

from __future__ import annotations

import importlib
import sys

from . import chunk_pool, local_attention, rope_fp32, routing  # noqa: F401  (load submodules)
from . import route_weights as _rw, selected_attention as _sel, token_ops  # noqa: F401

# the package re-exports functions named like two of its modules; take the modules
route_weights = sys.modules[__package__ + ".route_weights"]
selected_attention = sys.modules[__package__ + ".selected_attention"]

# (module, attribute) -> replacement
PATCHES = {
    ("ops.chunk_attn_pool_gqa_tilelang", "chunk_attn_pool_gqa"): chunk_pool.chunk_attn_pool_gqa,
    ("ops.topk_head_softmax", "ref_softmax_topk_max_pooling"): routing.ref_softmax_topk_max_pooling,
    ("ops.topk_head_softmax", "online_softmax_topk_head"): routing.online_softmax_topk_head,
    ("ops.hils_bidir_route_weights_tilelang", "route_weights"): route_weights.route_weights,
    ("ops.hils_fwd_bwd_head", "HiLS_block_M_head"): selected_attention.HiLS_block_M_head,
    ("ops.hils_bidir_output_fusion_tilelang", "fuse_hils_outputs"): selected_attention.fuse_hils_outputs,
    ("ops.rope_tilelang_fp32", "rope_rotary_pos_emb"): rope_fp32.rope_rotary_pos_emb,
    ("ops.rope_tilelang_fp32", "single_tensor_rope_autograd"): rope_fp32.single_tensor_rope_autograd,
    ("dream_dllm_hils.kernel_utils", "remote_drop_mask"): routing.remote_drop_mask,
    ("dream_dllm_hils.local_attention", "bidir_local_attention"): local_attention.bidir_local_attention,
    ("dream_dllm_hils.routing", "route_topk_g7"): routing.route_topk_g7,
    ("dream_dllm_hils.routing", "selected_attention_g7"): selected_attention.selected_attention_g7,
    ("dream_dllm_hils.routing", "selected_attention_g7_cached"): selected_attention.selected_attention_g7_cached,
    ("dream_dllm_hils.routing", "HiLS_block_M_head"): selected_attention.HiLS_block_M_head,
    ("dream_dllm_hils.routing", "online_softmax_topk_head"): routing.online_softmax_topk_head,
    ("dream_dllm_hils.routing", "ref_softmax_topk_max_pooling"): routing.ref_softmax_topk_max_pooling,
    ("dream_dllm_hils.attention", "_route_weights_torch"): route_weights.route_weights_torch,
    ("dream_dllm_hils.local_attention", "cached_local_attention"): local_attention.cached_local_attention,
    # dream_dllm_hils/fastdllm_attention.py:16-21 binds these at import
    ("dream_dllm_hils.fastdllm_attention", "cached_local_attention"): local_attention.cached_local_attention,
    ("dream_dllm_hils.fastdllm_attention", "remote_drop_mask"): routing.remote_drop_mask,
    ("dream_dllm_hils.fastdllm_attention", "route_topk_g7"): routing.route_topk_g7,
    ("dream_dllm_hils.fastdllm_attention", "selected_attention_g7_cached"):
        selected_attention.selected_attention_g7_cached,
    ("ops.flex_attn_tilelang", "flex_attn_tl"): local_attention.flex_attn_tl,
    ("ops.hils_token_score_gqa_tilelang", "candidate_token_scores_gqa"): token_ops.candidate_token_scores_gqa,
    ("ops.dsa_selected_attention_tilelang", "selected_token_attention_tilelang"):
        token_ops.selected_token_attention_tilelang,
}

_ORIGINALS: dict = {}


def install(*, fused_layer: bool = False, strict: bool = False):
    """Patch every reference module that is importable; returns the list of
    ``module.attr`` names replaced (originals kept for :func:`uninstall`)."""
    done = []
    for (mod_name, attr), fn in PATCHES.items():
        try:
            mod = importlib.import_module(mod_name)
        except ImportError:
            if strict:
                raise
            continue
        if not hasattr(mod, attr):
            if strict:
                raise AttributeError(f"{mod_name}.{attr}")
            continue
        _ORIGINALS.setdefault((mod_name, attr), getattr(mod, attr))
        setattr(mod, attr, fn)
        done.append(f"{mod_name}.{attr}")
    if fused_layer:
        mod = importlib.import_module("dream_dllm_hils.attention")
        cls = mod.KernelDreamFullHiLSAttention
        _ORIGINALS.setdefault(("dream_dllm_hils.attention", "KernelDreamFullHiLSAttention.forward"),
                              cls.forward)
        cls.forward = _fused_forward
        done.append("dream_dllm_hils.attention.KernelDreamFullHiLSAttention.forward")
    return done


def uninstall():
    """Restore every attribute :func:`install` replaced."""
    for (mod_name, attr), orig in list(_ORIGINALS.items()):
        mod = importlib.import_module(mod_name)
        if "." in attr:
            cls_name, meth = attr.split(".")
            setattr(getattr(mod, cls_name), meth, orig)
        else:
            setattr(mod, attr, orig)
    _ORIGINALS.clear()


def _fused_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None,
                   output_attentions=False, use_cache=False, cache_position=None,
                   position_embeddings=None, **kwargs):
    """``KernelDreamFullHiLSAttention.forward`` (``attention.py:1313``) on
    :class:`RouteLayer`: the module's own q/k/v projections, the whole routed
    attention in one C-ABI call, then ``o_proj``.  Eval / prefill only: the
    reference's training-only branches are not supported."""
    import torch

    from .layer import RouteLayer, RouteLayerConfig

    if use_cache or past_key_value is not None or self.training:
        raise NotImplementedError("the fused B200 route layer is an eval/prefill forward")
    bsz, q_len, _ = hidden_states.shape
    q = self.q_proj(hidden_states).view(bsz, q_len, self.num_heads, self.head_dim)
    k = self.k_proj(hidden_states).view(bsz, q_len, self.num_key_value_heads, self.head_dim)
    v = self.v_proj(hidden_states).view(bsz, q_len, self.num_key_value_heads, self.head_dim)
    if position_ids is None:
        position_ids = torch.arange(q_len, device=hidden_states.device).expand(bsz, q_len)
    key_valid = self._key_valid_mask(attention_mask, bsz, q_len, hidden_states.device)
    layer = getattr(self, "_mrsa_b200_layer", None)
    if layer is None:
        cfg = RouteLayerConfig(q_heads=self.num_heads, kv_heads=self.num_key_value_heads,
                               head_dim=self.head_dim, chunk=self.chunk_size, topk=self.topk,
                               local_window=self.local_window,
                               qcal_scale=float(getattr(self, "qcal_scale", 1.0)),
                               route_temperature=float(self.route_temperature))
        layer = RouteLayer(self.qcal[0].weight.detach(), self.qcal[1].weight.detach(),
                           self.qcal_norm.weight.detach(), self.entropy_bias_scale.detach(),
                           gate_offset=float(self.fusion_gate_offset),
                           gate_scale=float(self.fusion_gate_scale), cfg=cfg)
        rot = getattr(self, "rotary_emb", None)
        if rot is not None and hasattr(rot, "inv_freq"):
            layer.inv_freq = rot.inv_freq.detach().float().to(hidden_states.device)
            layer.attention_factor = float(getattr(rot, "attention_scaling", 1.0))
        self._mrsa_b200_layer = layer
    out = layer(q.contiguous(), k.contiguous(), v.contiguous(), hidden_states.contiguous(),
                position_ids.to(torch.long).contiguous(), key_valid)
    return self.o_proj(out.reshape(bsz, q_len, self.hidden_size)), None, past_key_value
