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
# class attribute that keeps the reference forward of a class whose forward
# is replaced by _fused_forward (the fused path hands every case it does not
# implement back to it)
_REFERENCE_FORWARD = "_mrsa_b200_reference_forward"


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
        install_fused_forward(mod.KernelDreamFullHiLSAttention)
        _ORIGINALS.setdefault(("dream_dllm_hils.attention", "KernelDreamFullHiLSAttention.forward"),
                              getattr(mod.KernelDreamFullHiLSAttention, _REFERENCE_FORWARD))
        done.append("dream_dllm_hils.attention.KernelDreamFullHiLSAttention.forward")
    return done


def install_fused_forward(cls):
    """Replace ``cls.forward`` (the signature of
    ``KernelDreamFullHiLSAttention.forward``, ``attention.py:1313-1324``) by
    :func:`_fused_forward`, keeping the class's own forward for the cases the
    fused layer does not implement."""
    if cls.__dict__.get("forward") is _fused_forward:
        return
    setattr(cls, _REFERENCE_FORWARD, cls.forward)
    cls.forward = _fused_forward


def uninstall():
    """Restore every attribute :func:`install` replaced."""
    for (mod_name, attr), orig in list(_ORIGINALS.items()):
        mod = importlib.import_module(mod_name)
        if "." in attr:
            cls_name, meth = attr.split(".")
            cls = getattr(mod, cls_name)
            setattr(cls, meth, orig)
            if _REFERENCE_FORWARD in cls.__dict__:
                delattr(cls, _REFERENCE_FORWARD)
        else:
            setattr(mod, attr, orig)
    _ORIGINALS.clear()


def fused_unsupported(self, hidden_states, attention_mask=None, position_ids=None,
                      past_key_value=None, use_cache=False, position_embeddings=None):
    """Why :func:`_fused_forward` cannot reproduce the reference forward of
    ``self`` for this call (``None`` when it can).

    The fused layer is the eval / prefill forward of the canonical config
    (``attention.py:1358-1774`` with the defaults of ``:906-920``): attention
    pooled chunk summaries with the entropy prior, landmark slots skipped in
    the local branch, Q-Cal with RMSNorm, post-softmax routing, the affine
    fusion gate, no token refinement, no forced or ablated routes, no hooks
    and no prefill capture, cos/sin from the module's rotary embedding, and
    no gradient requested."""
    import torch

    if self.training:
        return "training forward"
    if torch.is_grad_enabled() and (getattr(hidden_states, "requires_grad", False) or
                                    any(p.requires_grad for p in self.parameters())):
        return "gradient requested (the fused layer is forward-only)"
    if use_cache or past_key_value is not None:
        return "KV cache requested"
    validate = getattr(self, "_validate_kernel_call", None)
    if validate is not None:
        reason = validate(hidden_states, attention_mask)
        if reason is not None:
            return str(reason)
    if hidden_states.device.type != "cuda" or hidden_states.dtype != torch.bfloat16:
        return "hidden states must be BF16 on a CUDA device"
    if attention_mask is not None and not isinstance(attention_mask, str) and attention_mask.ndim != 2:
        return "4-D allowed mask (routed through remote_drop_mask by the reference)"
    if position_embeddings is not None:
        return "explicit position_embeddings"
    if position_ids is None:
        return "no position_ids"
    if (self.chunk_size, self.head_dim) != (64, 128):
        return "chunk_size 64 and head_dim 128 only"
    if self.num_heads % self.num_key_value_heads or self.num_heads // self.num_key_value_heads > 8:
        return "query heads per KV head must be at most 8"
    checks = (
        (getattr(self, "skip_inert_slots", True) is not True, "skip_inert_slots=False"),
        (str(getattr(self, "chunk_summary", "attn")) != "attn", "chunk_summary != 'attn'"),
        (not bool(getattr(self, "entropy_prior", True)), "entropy_prior=False"),
        (callable(getattr(self, "_lmk_keys_intervene", None)), "landmark intervention hook"),
        (callable(getattr(self, "_lmk_summary_hook", None)), "landmark summary hook"),
        (bool(getattr(self, "_prefill_capture", False)), "prefill cache capture"),
        (getattr(self, "route_query_positions", None) is not None, "route_query_positions"),
        (str(getattr(self, "route_selection_mode", "post_softmax")) != "post_softmax",
         "route_selection_mode != 'post_softmax'"),
        (getattr(self, "force_remote_query_mask", None) is not None, "forced remote routes"),
        (bool(getattr(self, "force_remote_oracle_route", False)), "oracle routes"),
        (float(getattr(self, "value_fusion_beta", 0.0) or 0.0) > 0, "value-aware fusion"),
        (int(getattr(self, "token_budget", 0) or 0) > 0, "token refinement"),
        (float(getattr(self, "route_residual_weight", 0.0) or 0.0) > 0, "soft route residual"),
        (not hasattr(self, "qcal"), "no Q-Cal (route_q = q)"),
        (getattr(self, "qcal_norm", None) is None, "Q-Cal without RMSNorm"),
        (getattr(getattr(self, "rotary_emb", None), "inv_freq", None) is None,
         "no rotary_emb.inv_freq"),
    )
    for bad, why in checks:
        if bad:
            return why
    qc = self.qcal
    try:
        w_in, w_out = qc[0].weight, qc[1].weight
    except (TypeError, IndexError, AttributeError):
        return "Q-Cal is not a two-layer Sequential"
    if len(qc) != 2 or getattr(qc[0], "bias", None) is not None or getattr(qc[1], "bias", None) is not None:
        return "Q-Cal is not two bias-free linear layers"
    if w_in.shape[0] != 64 or w_out.shape != (self.num_heads * self.head_dim, 64):
        return "Q-Cal rank must be 64"
    if w_in.shape[1] != hidden_states.shape[-1]:
        return "Q-Cal input width differs from the hidden size"
    return None


def _fused_layer_for(self, device):
    """The module's :class:`RouteLayer`, rebuilt whenever a parameter it
    copies from changed (storage or in-place version)."""
    import torch

    from .layer import RouteLayer, RouteLayerConfig

    norm = self.qcal_norm
    rot = self.rotary_emb
    srcs = [self.qcal[0].weight, self.qcal[1].weight, norm.weight, self.entropy_bias_scale,
            rot.inv_freq]
    gate_off = getattr(self, "fusion_gate_offset", None)
    gate_scale = getattr(self, "fusion_gate_scale", None)
    srcs += [t for t in (gate_off, gate_scale) if isinstance(t, torch.Tensor)]
    sig = tuple((t.data_ptr(), t._version) for t in srcs) + (str(device),)
    layer = getattr(self, "_mrsa_b200_layer", None)
    if layer is not None and getattr(self, "_mrsa_b200_sig", None) == sig:
        return layer
    # topk < 32 takes the reference's route_weights kernel: a plain softmax over
    # [routed logits, local LSE], i.e. the affine gate at scale 1, offset 0, T = 1
    affine = self.topk >= 32
    cfg = RouteLayerConfig(q_heads=self.num_heads, kv_heads=self.num_key_value_heads,
                           head_dim=self.head_dim, chunk=self.chunk_size, topk=self.topk,
                           local_window=self.local_window, rms_eps=float(norm.eps),
                           qcal_scale=float(getattr(self, "qcal_scale", 1.0)),
                           route_temperature=float(self.route_temperature) if affine else 1.0)
    layer = RouteLayer(self.qcal[0].weight.detach().to(device), self.qcal[1].weight.detach().to(device),
                       norm.weight.detach(), self.entropy_bias_scale.detach(),
                       gate_offset=float(gate_off) if (affine and gate_off is not None) else 0.0,
                       gate_scale=float(gate_scale) if (affine and gate_scale is not None) else 1.0,
                       cfg=cfg)
    layer.inv_freq = rot.inv_freq.detach().float().to(device).contiguous()
    layer.attention_factor = float(getattr(rot, "attention_scaling", 1.0))
    self._mrsa_b200_layer = layer
    self._mrsa_b200_sig = sig
    return layer


def _reference_forward(self):
    for klass in type(self).__mro__:
        fwd = klass.__dict__.get(_REFERENCE_FORWARD)
        if fwd is not None:
            return fwd
    raise RuntimeError("the fused route-layer forward is installed without a reference forward")


def _fused_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None,
                   output_attentions=False, use_cache=False, cache_position=None,
                   position_embeddings=None, **kwargs):
    """``KernelDreamFullHiLSAttention.forward`` (``attention.py:1313``) on
    :class:`RouteLayer`: the module's own q/k/v projections, the whole routed
    attention in one C-ABI call, then ``o_proj``.  Every call the fused layer
    does not reproduce exactly (:func:`fused_unsupported`: training, caches,
    4-D masks, explicit cos/sin, non-default summaries, hooks, forced routes,
    token refinement, ...) goes to the reference forward instead, which runs
    on the drop-in ops."""
    import torch

    why = fused_unsupported(self, hidden_states, attention_mask, position_ids, past_key_value, use_cache,
                            position_embeddings)
    if why is not None:
        return _reference_forward(self)(self, hidden_states, attention_mask, position_ids, past_key_value,
                                        output_attentions, use_cache, cache_position, position_embeddings,
                                        **kwargs)
    bsz, q_len, _ = hidden_states.shape
    q = self.q_proj(hidden_states).view(bsz, q_len, self.num_heads, self.head_dim)
    k = self.k_proj(hidden_states).view(bsz, q_len, self.num_key_value_heads, self.head_dim)
    v = self.v_proj(hidden_states).view(bsz, q_len, self.num_key_value_heads, self.head_dim)
    key_valid = self._key_valid_mask(attention_mask, bsz, q_len, hidden_states.device)
    layer = _fused_layer_for(self, hidden_states.device)
    pos = position_ids.to(device=hidden_states.device, dtype=torch.long).expand(bsz, q_len).contiguous()
    out = layer(q.contiguous(), k.contiguous(), v.contiguous(), hidden_states.contiguous(), pos, key_valid)
    return self.o_proj(out.reshape(bsz, q_len, self.num_heads * self.head_dim)), None, past_key_value
