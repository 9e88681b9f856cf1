"""CPU: the drop-in installer patches the reference's modules (when the
reference checkout is importable on this host) and restores them."""

import importlib
import os
import sys

import pytest

REF = os.environ.get("MRSA_REFERENCE_PATH", "/root/reference")


@pytest.fixture
def reference_on_path():
    if not os.path.isdir(os.path.join(REF, "dream_dllm_hils")):
        pytest.skip("reference checkout not present on this host")
    sys.path.insert(0, REF)
    try:
        importlib.import_module("dream_dllm_hils.routing")
    except Exception as exc:  # pragma: no cover - environment dependent
        sys.path.remove(REF)
        pytest.skip(f"reference not importable here: {exc}")
    yield
    sys.path.remove(REF)


def test_patch_table_names_reference_signatures(mrsa):
    from mrsa_b200 import dropin

    names = {attr for (_, attr) in dropin.PATCHES}
    for n in ("chunk_attn_pool_gqa", "ref_softmax_topk_max_pooling", "route_weights",
              "HiLS_block_M_head", "fuse_hils_outputs", "rope_rotary_pos_emb",
              "bidir_local_attention", "route_topk_g7", "selected_attention_g7",
              "_route_weights_torch", "remote_drop_mask", "flex_attn_tl", "cached_local_attention",
              "candidate_token_scores_gqa", "selected_token_attention_tilelang"):
        assert n in names


def test_install_and_uninstall_on_reference(mrsa, reference_on_path):
    from mrsa_b200 import dropin

    routing = importlib.import_module("dream_dllm_hils.routing")
    attention = importlib.import_module("dream_dllm_hils.attention")
    orig_route, orig_cls_fwd = routing.route_topk_g7, attention.KernelDreamFullHiLSAttention.forward
    done = dropin.install(fused_layer=True)
    try:
        assert "dream_dllm_hils.routing.route_topk_g7" in done
        assert routing.route_topk_g7 is mrsa.route_topk_g7
        assert routing.HiLS_block_M_head is mrsa.HiLS_block_M_head
        assert attention._route_weights_torch is mrsa.route_weights_torch
        assert attention.KernelDreamFullHiLSAttention.forward is dropin._fused_forward
    finally:
        dropin.uninstall()
    assert routing.route_topk_g7 is orig_route
    assert attention.KernelDreamFullHiLSAttention.forward is orig_cls_fwd


def test_install_reaches_the_cached_decode_bindings(mrsa, reference_on_path):
    """``fastdllm_attention.py`` binds its ops at import (``:16-21``); the
    installer patches those names too."""
    from mrsa_b200 import dropin

    try:
        fast = importlib.import_module("dream_dllm_hils.fastdllm_attention")
    except Exception as exc:  # pragma: no cover - environment dependent
        pytest.skip(f"fastdllm_attention not importable here: {exc}")
    orig = fast.cached_local_attention
    done = dropin.install()
    try:
        assert fast.cached_local_attention is mrsa.cached_local_attention
        assert fast.route_topk_g7 is mrsa.route_topk_g7
        assert fast.selected_attention_g7_cached is mrsa.selected_attention_g7_cached
        assert "ops.flex_attn_tilelang.flex_attn_tl" in done
    finally:
        dropin.uninstall()
    assert fast.cached_local_attention is orig
