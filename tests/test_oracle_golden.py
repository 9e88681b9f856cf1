"""CPU: the oracle against golden fixtures produced by the reference itself
(``tests/golden/make_golden.py``)."""

import math

import pytest
import torch

from conftest import load_golden
from oracle import route_layer as orc


def test_yarn_matches_transformers():
    g = load_golden("yarn.pt")
    inv, af = orc.yarn_inv_freq(g["dim"], g["base"], g["factor"], g["orig"])
    assert torch.equal(inv, g["inv_freq"])
    assert af == pytest.approx(g["attention_factor"], abs=0)


def test_landmark_positions_follow_layout():
    pos = orc.landmark_position_ids(1, 192, 64)[0]
    assert pos[:63].tolist() == list(range(63))
    assert pos[63].item() == 63            # landmark = last text position + 1
    assert pos[64].item() == 63            # next chunk's first text token
    assert pos[127].item() == 126


def test_pool_matches_compact_pool_torch():
    g = load_golden("pool.pt")
    lmk, ent = orc.chunk_pool(g["mu_q"], g["k_chunked"], g["key_valid"])
    assert torch.equal(lmk, g["lmk"])
    torch.testing.assert_close(ent, g["entropy"], atol=1e-6, rtol=1e-5)
    assert torch.count_nonzero(lmk[:, 3]) == 0 and torch.count_nonzero(ent[:, 3]) == 0


def test_drop_mask_matches_reference():
    g = load_golden("drop.pt")
    for w, ref in g["masks"].items():
        assert torch.equal(orc.remote_drop_mask(g["key_valid"], w, 64).bool(), ref), w


def test_route_topk_matches_route_topk_g7():
    g = load_golden("route.pt")
    b, l, hq, d = g["q"].shape
    c, hkv, gg = g["lmk"].shape[1:4]
    idx, sc = orc.route_topk_blocked(g["q"], g["lmk"], g["local_lse"], g["bias"], g["drop"], g["topk"])
    assert torch.equal(idx, g["indices"])
    assert torch.equal(sc, g["scores"])
    assert (idx[0, 9] == -1).all()
    assert (idx[0, 7, :, :20] >= 0).all() and (idx[0, 7, :, 20:] == -1).all()


@pytest.mark.parametrize("off,scale", [(0.0, 1.0), (0.3, 1.7)])
def test_route_weights_match_route_weights_torch(off, scale):
    r, w = load_golden("route.pt"), load_golden("weights.pt")
    rw, lw = orc.route_weights_affine(r["scores"], r["indices"], r["bias"], w["local_lse"],
                                      gate_offset=off, gate_scale=scale)
    ref_rw, ref_lw = w["outs"][(off, scale)]
    assert torch.equal(rw, ref_rw)
    assert torch.equal(lw, ref_lw)


def test_selected_matches_hils_torch_ref():
    g = load_golden("selected.pt")
    out = orc.selected_attention(g["q"], g["k"], g["v"], g["weights"], g["indices"], None, 64,
                                 out_dtype=torch.float32)
    torch.testing.assert_close(out, g["out"], atol=2e-6, rtol=1e-5)
    assert torch.count_nonzero(out[:, 6]) == 0


def test_qcal_chain_bf16_matches_reference():
    g = load_golden("qcal.pt")
    q_roped = orc.apply_rope(g["q"], g["cos"], g["sin"], "bf16")
    assert torch.equal(q_roped, g["q_roped"])
    unrot = orc.invert_rope(q_roped, g["cos"], g["sin"], "bf16")
    assert torch.equal(unrot, g["unrot"])
    comb = orc.rms_norm(unrot + g["delta"], torch.ones(128), 1e-6)
    assert torch.equal(orc.apply_rope(comb, g["cos"], g["sin"], "bf16"), g["route_q"])


def test_qcal_fp32_rope_close_to_bf16_chain():
    g = load_golden("qcal.pt")
    yarn = load_golden("yarn.pt")
    cos, sin = orc.rope_cos_sin(g["position_ids"], yarn["inv_freq"], yarn["attention_factor"])
    q_roped = orc.apply_rope(g["q"], cos, sin, "fp32")
    torch.testing.assert_close(q_roped.float(), g["q_roped"].float(), atol=2e-2, rtol=2e-2)


def test_local_mask_semantics():
    g = load_golden("local_mask.pt")
    for skip, ref in g["out"].items():
        pos = torch.arange(g["k"].shape[1])
        valid = g["key_valid"] & ((pos + 1) % 64 != 0) if skip else g["key_valid"]
        assert torch.equal(valid, ref["valid"])
        sc = valid.to(g["k"].dtype)[:, :, None, None]
        assert torch.equal(g["k"] * sc, ref["k"]) and torch.equal(g["v"] * sc, ref["v"])
        assert ref["window"] == (256 + 63 if skip else 256)


def test_local_attention_matches_dense_masked_softmax():
    """The banded restatement equals a dense masked softmax (the flash-attn
    window semantics) on a small case with ragged validity."""
    gen = torch.Generator().manual_seed(1)
    b, l, hq, hkv, d, w = 1, 320, 14, 2, 128, 40
    q = torch.randn(b, l, hq, d, generator=gen).bfloat16()
    k = torch.randn(b, l, hkv, d, generator=gen).bfloat16()
    v = torch.randn(b, l, hkv, d, generator=gen).bfloat16()
    valid = torch.rand(b, l, generator=gen) > 0.1
    o, lse = orc.local_attention(q, k, v, valid, w, 64, True, block=64)
    pos = torch.arange(l)
    keep = valid & ((pos + 1) % 64 != 0)
    kz = (k * keep[:, :, None, None].to(k.dtype)).float().repeat_interleave(7, 2)
    vz = (v * keep[:, :, None, None].to(v.dtype)).float().repeat_interleave(7, 2)
    sc = torch.einsum("bihd,bjhd->bhij", q.float(), kz) / math.sqrt(d)
    band = (pos[:, None] - pos[None, :]).abs() <= w + 63
    sc = sc.masked_fill(~band, float("-inf"))
    ref_lse = torch.logsumexp(sc, -1).permute(0, 2, 1)
    ref_o = torch.einsum("bhij,bjhd->bihd", torch.softmax(sc, -1), vz)
    torch.testing.assert_close(lse, ref_lse, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(o.float(), ref_o, atol=1e-2, rtol=1e-2)


def test_whole_layer_matches_reference_composition():
    """Whole route layer (bf16 RoPE chain, as on the live path) against the
    composition of the reference's own functions."""
    g = load_golden("layer.pt")
    cfg = orc.MRSAConfig(q_heads=g["q_heads"], kv_heads=g["kv_heads"], rope_precision="bf16")
    inp = orc.make_route_layer_inputs(g["batch"], g["seq_len"], cfg, hidden=g["hidden"], seed=g["seed"])
    res = orc.route_layer_forward(inp, cfg)
    rows = g["rows"]
    assert torch.equal(res["q"][:, rows], g["q"])
    assert torch.equal(res["k"][:, rows], g["k"])
    assert torch.equal(res["route_q"][:, rows], g["route_q"])
    assert torch.equal(res["lmk"], g["lmk"])
    torch.testing.assert_close(res["entropy"], g["entropy"], atol=1e-6, rtol=1e-5)
    assert torch.equal(res["indices"], g["indices"])
    # the reference's bf16 CPU linear layers may round a few route_q entries
    # differently from fp32-accumulate-then-round: allow 1-ulp score flips
    fin = torch.isfinite(g["scores"].float())
    assert torch.equal(fin, torch.isfinite(res["scores"].float()))
    ds = (res["scores"].float() - g["scores"].float())[fin]
    assert ds.abs().max().item() <= 2.5e-4 and (ds != 0).float().mean().item() < 5e-3
    torch.testing.assert_close(res["remote_weights"].float(), g["remote_weights"].float(),
                               atol=4e-3, rtol=1e-2)
    torch.testing.assert_close(res["local_weight"].float(), g["local_weight"].float(),
                               atol=4e-3, rtol=1e-2)
    d = (res["out"].float() - g["out"].float()).abs()
    assert d.max().item() <= 2e-2
    assert d.mean().item() / g["out"].float().abs().mean().item() <= 1e-3


def test_query_slice_equals_full_layer():
    cfg = orc.MRSAConfig(q_heads=7, kv_heads=1)
    inp = orc.make_route_layer_inputs(1, 1024, cfg, hidden=256, seed=3)
    full = orc.route_layer_forward(inp, cfg)
    part = orc.route_layer_forward(inp, cfg, query_slice=slice(320, 640))
    assert torch.equal(part["indices"], full["indices"][:, 320:640])
    # fp32 sums over differently sized key windows: rare 1-ulp bf16 flips
    torch.testing.assert_close(part["out"].float(), full["out"][:, 320:640].float(),
                               atol=1e-4, rtol=1e-2)


def test_topk_set_agreement_flags_real_differences():
    gen = torch.Generator().manual_seed(0)
    key = torch.randn(4, 100, generator=gen)
    top = key.topk(32, -1).indices.sort(-1).values
    viol, exact = orc.topk_set_agreement(key, top, top, 32)
    assert viol == 0 and exact == 1.0
    worst = key.topk(32, -1, largest=False).indices.sort(-1).values
    viol, exact = orc.topk_set_agreement(key, top, worst, 32)
    assert viol > 0 and exact == 0.0


def test_candidate_token_scores_match_reference():
    from oracle import token_ops as tok

    g = load_golden("token_scores.pt")
    out = tok.candidate_token_scores(g["q"], g["k"], g["indices"], g["key_valid"], g["chunk"])
    ref = g["out"]
    assert torch.equal(torch.isinf(out), torch.isinf(ref))
    fin = torch.isfinite(ref)
    torch.testing.assert_close(out[fin], ref[fin], atol=1e-5, rtol=1e-5)
    assert torch.isinf(out[:, 4, 0]).all() and torch.isinf(out[..., -1]).all()


def test_selected_token_attention_matches_reference():
    from oracle import token_ops as tok

    g = load_golden("dsa.pt")
    out = tok.selected_token_attention(g["q"], g["k"], g["v"], g["indices"], g["valid"])
    # both round P to bf16 and the output to bf16; the einsum order may differ by one bf16 ulp
    torch.testing.assert_close(out.float(), g["out"].float(), atol=1e-2, rtol=1e-2)
    assert (out.float() - g["out"].float()).abs().mean() < 1e-4
    assert torch.count_nonzero(out[:, 0]) == 0


def test_flex_window_matches_torch_flex_attention():
    from oracle import token_ops as tok

    for case in load_golden("flex.pt")["cases"]:
        o, lse = tok.flex_window_attention(case["q"], case["k"], case["v"], case["window"], case["chunk"],
                                           case["mask_lmk"], case["expand"])
        torch.testing.assert_close(o, case["o"], atol=2e-5, rtol=1e-4, msg=case["name"])
        fin = torch.isfinite(case["lse"])
        assert torch.equal(fin, torch.isfinite(lse)), case["name"]
        torch.testing.assert_close(lse[fin], case["lse"][fin], atol=2e-5, rtol=1e-5, msg=case["name"])


def test_flex_mask_kv_start_is_a_shift():
    """With a truncated cache (kv_start > 0) the mask equals the full-prefix
    mask restricted to the kept keys (absolute positions throughout)."""
    from oracle import token_ops as tok

    full = tok.flex_window_mask(8, 200, 70, 32, True, True, 0)
    part = tok.flex_window_mask(8, 136, 70, 32, True, True, 64)
    assert torch.equal(full[:, 64:], part)
    assert not full[:, :64].any()


def test_local_window_matches_reference_bidir_local_attention():
    """The reference's own bidir_local_attention (masking helpers, window rule,
    LSE layout), with its GPU-only flash-attn call replaced by torch's
    flex_attention under flash-attn's |i - j| <= W window."""
    for case in load_golden("local_window.pt")["cases"]:
        o, lse = orc.local_attention(case["q"], case["k"], case["v"], case["key_valid"], case["window"], 64,
                                     case["skip"])
        d = (o.float() - case["o"].float()).abs()
        assert d.max() <= 2 ** -6 and (d > 0).float().mean() < 0.02, (case["window"], case["skip"], d.max())
        torch.testing.assert_close(lse, case["lse"], atol=2e-5, rtol=1e-5)


def test_cached_rows_match_reference_cached_local_attention():
    """dream_dllm_hils/local_attention.py:147 cached_local_attention (same
    stand-in for flash-attn): rows at arbitrary cache positions equal the
    full-window oracle's rows at those positions."""
    g = load_golden("local_window.pt")["cached"]
    pos = g["positions"]
    q_full = torch.zeros(1, g["k"].shape[1], *g["q"].shape[2:], dtype=g["q"].dtype)
    q_full[:, pos] = g["q"]
    for run in g["runs"]:
        o, lse = orc.local_attention(q_full, g["k"], g["v"], g["key_valid"], run["window"], 64, run["skip"])
        d = (o[:, pos].float() - run["o"].float()).abs()
        assert d.max() <= 2 ** -6, (run["window"], d.max())
        torch.testing.assert_close(lse[:, pos], run["lse"], atol=2e-5, rtol=1e-5)
