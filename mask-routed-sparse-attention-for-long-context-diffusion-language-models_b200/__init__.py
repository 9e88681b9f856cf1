"""MRSA route-layer / SWA-layer forward for B200 (sm_100a).

Hand-written CUDA kernels behind the C ABI of ``include/mrsa.h``
(``libmrsa_b200.so``), with Python shims that keep the reference's op
signatures (``ops/*`` and ``dream_dllm_hils/{routing,local_attention}.py``)
so ``dream_dllm_hils/attention.py`` can call them as drop-ins (see
``dropin.install``).  There is no CPU fallback: the ops raise when the
library is missing.
"""

from . import _lib
from .chunk_pool import chunk_attn_pool_gqa, chunk_pool_backward
from .dream_forward import DreamConfig, DreamForward
from .layer import RouteLayer, RouteLayerConfig, swa_layer_forward
from .local_attention import (bidir_local_attention, cached_local_attention, flex_attn_tl,
                              window_attention, window_attention_backward)
from .rope_fp32 import rope_rotary_pos_emb, single_tensor_rope_autograd, yarn_inv_freq, yarn_rope_qk
from .route_weights import route_weights, route_weights_backward, route_weights_torch
from .routing import (online_softmax_topk_head, ref_softmax_topk_max_pooling, remote_drop_mask,
                      route_scores_backward, route_topk_fused, route_topk_g7)
from .selected_attention import (HiLS_block_M_head, fuse_hils_outputs, fuse_outputs_backward, selected_attention,
                                 selected_attention_autograd, selected_attention_backward,
                                 selected_attention_g7, selected_attention_g7_cached, to_f16)
from .token_ops import candidate_token_scores_gqa, selected_token_attention_tilelang

__all__ = [
    "DreamConfig", "DreamForward", "RouteLayer", "RouteLayerConfig", "swa_layer_forward", "chunk_attn_pool_gqa",
    "bidir_local_attention", "cached_local_attention", "window_attention", "rope_rotary_pos_emb",
    "single_tensor_rope_autograd", "yarn_inv_freq", "yarn_rope_qk", "route_weights",
    "route_weights_torch", "online_softmax_topk_head", "ref_softmax_topk_max_pooling",
    "remote_drop_mask", "route_topk_fused", "route_topk_g7", "HiLS_block_M_head",
    "fuse_hils_outputs", "selected_attention", "selected_attention_autograd", "selected_attention_backward",
    "selected_attention_g7",
    "selected_attention_g7_cached", "to_f16", "flex_attn_tl", "candidate_token_scores_gqa",
    "selected_token_attention_tilelang", "load_library", "chunk_pool_backward", "route_weights_backward",
    "route_scores_backward", "fuse_outputs_backward", "window_attention_backward",
]


def load_library():
    """Load ``libmrsa_b200.so`` now (it is otherwise loaded on first use)."""
    return _lib.load()
