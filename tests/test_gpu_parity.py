"""GPU parity of every hot-path stage against the CPU oracle and the golden
fixtures made by the reference itself.

Tolerances (bf16 outputs, from the BASELINE north_star): attention outputs
max-abs <= 2e-2 and mean-rel <= 1e-3; routing: no selection differs where the
key gap to the top-K boundary exceeds 1e-3.
"""

import math

import pytest
import torch

from conftest import load_golden
from oracle import route_layer as orc

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def close_bf16(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all()
    d = (got - ref).abs()
    rel = d.mean().item() / max(ref.abs().mean().item(), 1e-30)
    assert d.max().item() <= max_abs and rel <= mean_rel, (d.max().item(), rel)


def ulp_close(got, ref, frac=1e-3, floor=2.0 ** -20):
    """bf16 results of fp32 math done in a different order: at most one ulp
    apart (or ``floor`` apart where cancellation leaves a result near zero),
    and almost always identical."""
    got, ref = got.float().cpu(), ref.float().cpu()
    d = (got - ref).abs()
    _, e = torch.frexp(torch.maximum(got.abs(), ref.abs()))
    ulp = torch.ldexp(torch.ones_like(d), e - 8)          # bf16 spacing at that magnitude
    assert ((d <= ulp) | (d <= floor)).all(), d.max().item()
    assert (d > 0).float().mean().item() <= frac


@pytest.fixture(scope="module")
def dev(cuda_device):
    return cuda_device


# ---------------------------------------------------------------- RoPE
def test_rope_positions_match_oracle(mrsa, dev):
    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(2, 640, cfg, hidden=64, seed=2)
    inv, af = orc.yarn_inv_freq(128, cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
    cos, sin = orc.rope_cos_sin(inp["position_ids"], inv, af)
    q, k = mrsa.yarn_rope_qk(inp["q_pre"].to(dev), inp["k_pre"].to(dev), inp["position_ids"].to(dev),
                             inv.to(dev), af)
    ulp_close(q, orc.apply_rope(inp["q_pre"], cos, sin))
    ulp_close(k, orc.apply_rope(inp["k_pre"], cos, sin))


@pytest.mark.parametrize("cs_dtype", [torch.float32, torch.bfloat16])
def test_rope_cossin_dropins(mrsa, dev, cs_dtype):
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, 96, 5, 128, generator=g).bfloat16()
    k = torch.randn(1, 96, 3, 128, generator=g).bfloat16()
    cos = torch.randn(1, 96, 128, generator=g).to(cs_dtype)
    sin = torch.randn(1, 96, 128, generator=g).to(cs_dtype)
    qo, ko = mrsa.rope_rotary_pos_emb(q.to(dev), k.to(dev), cos.to(dev), sin.to(dev))
    ref_q = (q.float() * cos.float()[:, :, None] + orc.rotate_half(q.float()) * sin.float()[:, :, None]).bfloat16()
    ref_k = (k.float() * cos.float()[:, :, None] + orc.rotate_half(k.float()) * sin.float()[:, :, None]).bfloat16()
    ulp_close(qo, ref_q)
    ulp_close(ko, ref_k)
    xo = mrsa.single_tensor_rope_autograd(q.to(dev), cos.to(dev), sin.to(dev))
    assert torch.equal(xo, qo)


# ---------------------------------------------------------------- pool / drop
def test_pool_matches_reference_golden(mrsa, dev):
    g = load_golden("pool.pt")
    lmk, ent = mrsa.chunk_attn_pool_gqa(g["mu_q"].to(dev), g["k_chunked"].to(dev), g["key_valid"].to(dev))
    ulp_close(lmk, g["lmk"], frac=2e-3)
    torch.testing.assert_close(ent.cpu(), g["entropy"], atol=2e-5, rtol=2e-5)
    assert torch.count_nonzero(lmk[:, 3]) == 0 and torch.count_nonzero(ent[:, 3]) == 0


def test_drop_mask_matches_reference_golden(mrsa, dev):
    g = load_golden("drop.pt")
    for w, ref in g["masks"].items():
        got = mrsa.remote_drop_mask(g["key_valid"].to(dev), w, 64)
        assert got.dtype == torch.int32 and torch.equal(got.cpu().bool(), ref), w


# ---------------------------------------------------------------- routing
def test_route_topk_g7_matches_reference_golden(mrsa, dev):
    g = load_golden("route.pt")
    idx, sc = mrsa.route_topk_g7(g["q"].to(dev), g["lmk"].to(dev), g["local_lse"].to(dev),
                                 g["bias"].to(dev), g["drop"].to(dev), g["topk"], 64, 512,
                                 training=False)
    b, l, hq, d = g["q"].shape
    key = orc.route_keys(g["q"], g["lmk"], g["local_lse"], g["bias"], g["drop"])
    viol, exact = orc.topk_set_agreement(key, idx.cpu(), g["indices"], g["topk"])
    assert viol == 0
    assert exact >= 0.98
    same = (idx.cpu() == g["indices"]).all(-1)[..., None, None].expand(-1, -1, 1, 7, g["topk"])
    s_ref = g["scores"].float().view(b, l, 1, 7, -1)
    s_got = sc.float().cpu().view(b, l, 1, 7, -1)
    fin = torch.isfinite(s_ref) & same
    assert torch.equal(torch.isinf(s_got) & same, torch.isinf(s_ref) & same)
    torch.testing.assert_close(s_got[fin], s_ref[fin], atol=2e-4, rtol=1e-2)
    # sorted ascending, -1 last, ragged availability
    i = idx.cpu()
    assert (i[0, 9] == -1).all()
    assert (i[0, 7, :, :20] >= 0).all() and (i[0, 7, :, 20:] == -1).all()
    srt = torch.where(i < 0, torch.full_like(i, 1 << 30), i)
    assert torch.equal(srt, srt.sort(-1).values)


@pytest.mark.parametrize("c", [600, 2000])
@pytest.mark.parametrize("tiers", [0, 1, 2])
def test_route_ties_take_lowest_chunk_ids(mrsa, dev, c, tiers):
    """Keys equal at the top-K boundary: the lowest chunk ids win.  Zero
    landmarks make every key a function of its chunk's bias alone, so chunks
    with equal bias tie exactly (on the GPU and in the oracle).  tiers=0: every
    key ties; 1: the boundary falls inside the lowest of three tiers (hundreds
    of equal keys, more than the filtered search keeps); 2: 20 chunks above
    a tier of 40 equal keys that holds the boundary, every other key distinct
    and lower, so the filtered candidate search finds the threshold and the
    tie is broken by the chunk-order pass."""
    gen = torch.Generator().manual_seed(c + tiers)
    b, l, hkv, g, d, topk = 1, 96, 2, 7, 128, 32
    q = torch.randn(b, l, hkv * g, d, generator=gen).bfloat16()
    lmk = torch.zeros(b, c, hkv, g, d).bfloat16()
    lse = torch.randn(b, l, hkv, g, generator=gen)
    bias = torch.zeros(b, c, hkv, g)
    if tiers == 1:
        perm = torch.randperm(c, generator=gen)
        bias[:, perm[:5]] = 2.0
        bias[:, perm[5:25]] = 1.0
    elif tiers == 2:
        perm = torch.randperm(c, generator=gen)
        bias[:] = (-1.0 - torch.rand(c, generator=gen))[None, :, None, None]
        bias[:, perm[:20]] = 2.0
        bias[:, perm[20:60]] = 1.0
    drop = (torch.rand(b, l, c, generator=gen) < 0.2).int()
    idx, _ = mrsa.route_topk_g7(q.to(dev), lmk.to(dev), lse.to(dev), bias.to(dev), drop.to(dev),
                                topk, 64, 512, training=False)
    key = orc.route_keys(q, lmk, lse, bias, drop)                      # [b, l, hkv, c]
    # order by key descending, then chunk id ascending (a stable sort keeps
    # equal keys in chunk order); dropped chunks never
    order = torch.sort(key, dim=-1, descending=True, stable=True).indices
    top = order[..., :topk]
    top = torch.where(torch.gather(key, -1, top).isfinite(), top, torch.full_like(top, 1 << 30))
    want = top.sort(-1).values
    want = torch.where(want == (1 << 30), torch.full_like(want, -1), want)
    assert torch.equal(idx.cpu(), want)


@pytest.mark.parametrize("c,topk,ties", [(300, 32, False), (512, 31, False), (1000, 32, False),
                                          (2048, 32, False), (2048, 7, False), (1000, 32, True),
                                          (2048, 32, True)])
def test_route_selection_exact_on_the_kernels_own_keys(mrsa, dev, c, topk, ties):
    """The selection kernel against an exact top-K of the keys the key kernel
    wrote (read back from the workspace): bit-exact indices, ties broken
    towards the lowest chunk ids, ascending, -1 last.  Covers the 16-, 32- and
    64-keys-per-lane kernels and, with ``ties``, keys drawn from a few
    distinct values so that rows also take the paths for ties at the
    threshold and for filters that keep too many keys."""
    lib = mrsa._lib
    gen = torch.Generator().manual_seed(c * 3 + topk + ties)
    b, l, hkv, g, d = 1, 80, 2, 7, 128
    q = (torch.randn(b, l, hkv * g, d, generator=gen) * 0.3).bfloat16()
    if ties:
        lmk = torch.zeros(b, c, hkv, g, d).bfloat16()
        bias = torch.randint(0, 40, (b, c, hkv, g), generator=gen).float() * 0.25
    else:
        lmk = (torch.randn(b, c, hkv, g, d, generator=gen) * 0.3).bfloat16()
        bias = torch.randn(b, c, hkv, g, generator=gen) * 0.5
    lse = torch.randn(b, l, hkv * g, generator=gen)
    drop = (torch.rand(b, l, c, generator=gen) < 0.2).int()
    qd, ld, lsed, bd, dd = (t.to(dev).contiguous() for t in (q, lmk, lse, bias, drop))
    idx = torch.empty(b, l, hkv, topk, device=dev, dtype=torch.int32)
    sc = torch.empty(b, l, hkv * g, topk, device=dev, dtype=torch.bfloat16)
    ws_bytes = lib.load().mrsa_route_topk_workspace_size(b, l, c, hkv, g, lib.BF16)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    lib.call("mrsa_route_topk", lib.ptr(qd), lib.ptr(ld), 1, lib.ptr(lsed), lib.ptr(bd), lib.ptr(dd), None,
             -1, 0, lib.ptr(idx), lib.ptr(sc), lib.BF16, None, None, lib.WEIGHTS_AFFINE, 1.0, 1.0, 0.0,
             b, l, c, hkv, g, d, topk, lib.ptr(ws), ws.numel(), lib.stream_of(qd))
    torch.cuda.synchronize(dev)
    keys = ws[: b * l * hkv * c * 4].view(torch.float32).view(b, l, hkv, c).cpu().double()
    assert torch.isneginf(keys[drop.bool()[:, :, None, :].expand_as(keys)]).all()
    # the K largest finite keys, equal keys in ascending chunk id, output ascending
    flat = keys.reshape(-1, c)
    want = torch.full((flat.shape[0], topk), -1, dtype=torch.int64)
    for r in range(flat.shape[0]):
        fin = torch.nonzero(torch.isfinite(flat[r])).flatten()
        top = sorted(fin.tolist(), key=lambda ch: (-flat[r, ch].item(), ch))[:topk]
        want[r, :len(top)] = torch.tensor(sorted(top), dtype=torch.int64)
    assert torch.equal(idx.cpu().long().reshape(-1, topk), want)


def test_ref_softmax_topk_dropin_shared_landmarks(mrsa, dev):
    """per-KV-head (GQA-shared) landmarks, fp32 scores, no bias"""
    gen = torch.Generator().manual_seed(8)
    b, l, hkv, g, d, c, topk = 1, 200, 2, 7, 128, 50, 16
    q = torch.randn(b, l, hkv, g, d, generator=gen).bfloat16()
    lm = torch.randn(b, c, hkv, d, generator=gen).bfloat16()
    lse = torch.randn(b, l, hkv * g, generator=gen)
    drop = (torch.rand(b, l, c, generator=gen) < 0.2).int()
    idx, sc = mrsa.ref_softmax_topk_max_pooling(q.to(dev), lm.to(dev), lse.to(dev), topk, 64, 0,
                                                drop_mask=drop.to(dev))
    lm_h = lm[:, :, :, None].expand(b, c, hkv, g, d).reshape(b, c, hkv * g, d)
    ref_i, ref_s = orc.route_topk(q, lm_h, lse.view(b, l, hkv, g), topk, drop, None)
    key = orc.route_keys(q.view(b, l, hkv * g, d), lm_h.view(b, c, hkv, g, d), lse.view(b, l, hkv, g),
                         torch.zeros(b, c, hkv, g), drop)
    viol, exact = orc.topk_set_agreement(key, idx.cpu(), ref_i, topk)
    assert viol == 0 and exact >= 0.98
    assert idx.dtype == torch.int64 and sc.dtype == torch.float32 and sc.shape == ref_s.shape


@pytest.mark.parametrize("off,scale", [(0.0, 1.0), (0.3, 1.7)])
def test_route_weights_torch_dropin_matches_golden(mrsa, dev, off, scale):
    r, w = load_golden("route.pt"), load_golden("weights.pt")
    rw, lw = mrsa.route_weights_torch(r["scores"].to(dev), r["indices"].to(dev), r["bias"].to(dev),
                                      w["local_lse"].to(dev), temperature=1.0,
                                      gate_offset=torch.tensor(off), gate_scale=torch.tensor(scale))
    ref_rw, ref_lw = w["outs"][(off, scale)]
    torch.testing.assert_close(rw.float().cpu(), ref_rw.float(), atol=4e-3, rtol=8e-3)
    torch.testing.assert_close(lw.float().cpu(), ref_lw.float(), atol=4e-3, rtol=8e-3)


def test_route_weights_softmax_dropin_allows_topk32(mrsa, dev):
    r, w = load_golden("route.pt"), load_golden("weights.pt")
    rw, lw = mrsa.route_weights(r["scores"].to(dev), r["indices"].to(dev), r["bias"].to(dev),
                                w["local_lse"].to(dev))
    ref_rw, ref_lw = orc.route_weights_plain(r["scores"], r["indices"], r["bias"], w["local_lse"])
    torch.testing.assert_close(rw.float().cpu(), ref_rw.float(), atol=4e-3, rtol=8e-3)
    torch.testing.assert_close(lw.float().cpu(), ref_lw.float(), atol=4e-3, rtol=8e-3)
    tot = rw.float().sum(-1) + lw.float()
    assert ((tot - 1).abs() < 0.05).all()


# ---------------------------------------------------------------- attention
def test_selected_matches_hils_torch_ref_golden(mrsa, dev):
    g = load_golden("selected.pt")
    lk = g["k"].shape[1]
    valid = torch.ones(1, lk, dtype=torch.bool, device=dev)
    out = mrsa.selected_attention_g7(g["q"].to(dev), g["k"].to(dev), g["v"].to(dev), g["weights"].to(dev),
                                     g["indices"].to(dev), valid, 64, False)
    close_bf16(out, g["out"].bfloat16())
    assert torch.count_nonzero(out[:, 6]) == 0


def test_selected_with_invalid_keys_matches_oracle(mrsa, dev):
    """reference unit test pattern (unittests/test_hils_non_power_two_topk.py:95-142):
    contiguous chunks, invalid key every 97th, topk 31, first query routed nowhere"""
    gen = torch.Generator().manual_seed(79)
    lq, lk, hkv, g, d, topk = 2048, 2048, 4, 7, 128, 31
    q = torch.randn(1, lq, hkv * g, d, generator=gen).bfloat16()
    k = torch.randn(1, lk, hkv, d, generator=gen).bfloat16()
    v = torch.randn(1, lk, hkv, d, generator=gen).bfloat16()
    idx = torch.arange(topk, dtype=torch.int32).expand(1, lq, hkv, -1).clone()
    idx[:, 0] = -1
    w = torch.randn(1, lq, hkv * g, topk, generator=gen).softmax(-1).bfloat16()
    w[:, 0] = 0
    valid = torch.ones(1, lk, dtype=torch.bool)
    valid[:, ::97] = False
    out = mrsa.selected_attention_g7(q.to(dev), k.to(dev), v.to(dev), w.to(dev), idx.to(dev),
                                     valid.to(dev), 64, False)
    rows = torch.tensor([0, 1, 777, lq // 2, lq - 1])
    ref = orc.selected_attention(q[:, rows], k, v, w[:, rows], idx[:, rows], valid, 64)
    close_bf16(out[:, rows.to(dev)], ref)
    assert torch.equal(out[:, 0].cpu(), torch.zeros_like(out[:, 0].cpu()))


@pytest.mark.parametrize("vdt", ["bf16", "f16"])
@pytest.mark.parametrize("g,topk,lq", [(7, 32, 1000), (8, 13, 777), (3, 32, 96)])
def test_selected_random_routing_duplicates_ragged(mrsa, dev, g, topk, lq, vdt):
    """random chunk lists with empty (-1) and repeated slots, a query length that
    is not a multiple of the 32-query block, batch 2, several group sizes; the
    oracle (``hils_torch_ref`` semantics) counts a repeated chunk once per slot"""
    gen = torch.Generator().manual_seed(1000 * g + topk)
    b, lk, hkv, d = 2, 2048, 2, 128
    c = lk // 64
    q = torch.randn(b, lq, hkv * g, d, generator=gen).bfloat16()
    k = torch.randn(b, lk, hkv, d, generator=gen).bfloat16()
    v = torch.randn(b, lk, hkv, d, generator=gen).bfloat16()
    idx = torch.randint(0, c, (b, lq, hkv, topk), generator=gen, dtype=torch.int32)
    idx[torch.rand(idx.shape, generator=gen) < 0.1] = -1
    idx[:, ::5, :, 1] = idx[:, ::5, :, 0]                    # repeated chunk in a query's list
    idx[:, ::7, :, -1] = idx[:, ::7, :, 0]
    w = torch.rand(b, lq, hkv * g, topk, generator=gen).bfloat16()
    valid = torch.rand(b, lk, generator=gen) > 0.05
    vd = v.to(dev) if vdt == "bf16" else mrsa.to_f16(v.to(dev))   # fp16 V: the one-tile fp16 P kernel
    out = mrsa.selected_attention(q.to(dev), k.to(dev), vd, w.to(dev), idx.to(dev), valid.to(dev))
    rows = torch.unique(torch.cat([torch.arange(0, lq, 37), torch.tensor([lq - 1, 0, 5, 35])]))
    ref = orc.selected_attention(q[:, rows], k, v, w[:, rows], idx[:, rows], valid, 64, block=16)
    close_bf16(out[:, rows.to(dev)], ref)


@pytest.mark.parametrize("cached", [False, True])
@pytest.mark.parametrize("filtered", [False, True])
def test_selected_k31_token_keep_matches_oracle(mrsa, dev, cached, filtered):
    """unittests/test_hils_non_power_two_topk.py:95-142: K=31 (not a power of
    two), the first query without chunks, every 97th key invalid, and with
    ``filtered`` a random token_keep mask (token refinement)."""
    g = torch.Generator().manual_seed(79)
    lq, lk, hkv, gg, d, topk, size = (35 if cached else 2048), 2048, 4, 7, 128, 31, 64
    q = torch.randn(1, lq, hkv * gg, d, generator=g).bfloat16()
    k = torch.randn(1, lk, hkv, d, generator=g).bfloat16()
    v = torch.randn(1, lk, hkv, d, generator=g).bfloat16()
    idx = torch.arange(topk, dtype=torch.int32).expand(1, lq, hkv, -1).clone()
    idx[:, 0] = -1
    w = torch.randn(1, lq, hkv * gg, topk, generator=g).softmax(-1).bfloat16()
    w[:, 0] = 0
    valid = torch.ones(1, lk, dtype=torch.bool)
    valid[:, ::97] = False
    keep = (torch.rand(1, lq, hkv, topk, size, generator=g) > 0.4) if filtered else None
    args = [t.to(dev) for t in (q, k, v, w, idx, valid)] + [size]
    dkeep = None if keep is None else keep.to(dev)
    got = (mrsa.selected_attention_g7_cached(*args, token_keep=dkeep) if cached else
           mrsa.selected_attention_g7(*args, training=False, token_keep=dkeep))
    assert torch.count_nonzero(got[:, 0]) == 0
    ref = orc.selected_attention(q, k, v, w, idx, valid, size, token_keep=keep)
    close_bf16(got, ref)
    if filtered:   # the fp16-V kernel reads the same keep rows
        got16 = mrsa.selected_attention(q.to(dev), k.to(dev), mrsa.to_f16(v.to(dev)), w.to(dev), idx.to(dev),
                                        valid.to(dev), chunk=size, token_keep=dkeep)
        close_bf16(got16, ref)


@pytest.mark.parametrize("vdt", ["bf16", "f16"])
def test_selected_all_queries_same_chunks(mrsa, dev, vdt):
    """every query of a block selects the same chunks: items of 8 owners, 4 per chunk"""
    gen = torch.Generator().manual_seed(5)
    lq, lk, hkv, g, d, topk = 256, 4096, 4, 7, 128, 32
    q = torch.randn(1, lq, hkv * g, d, generator=gen).bfloat16()
    k = torch.randn(1, lk, hkv, d, generator=gen).bfloat16()
    v = torch.randn(1, lk, hkv, d, generator=gen).bfloat16()
    idx = (torch.arange(topk, dtype=torch.int32) * 2).expand(1, lq, hkv, -1).contiguous()
    w = torch.randn(1, lq, hkv * g, topk, generator=gen).softmax(-1).bfloat16()
    vd = v.to(dev) if vdt == "bf16" else mrsa.to_f16(v.to(dev))
    local = torch.randn(1, lq, hkv * g, d, generator=gen).bfloat16()
    lw = torch.rand(1, lq, hkv * g, generator=gen).bfloat16()
    out = mrsa.selected_attention(q.to(dev), k.to(dev), vd, w.to(dev), idx.to(dev),
                                  local_out=local.to(dev), local_weight=lw.to(dev))
    rows = torch.tensor([0, 31, 32, 100, 255])
    ref = orc.selected_attention(q[:, rows], k, v, w[:, rows], idx[:, rows], None, 64, block=8)
    ref = orc.fuse_outputs(ref, local[:, rows], lw[:, rows])
    close_bf16(out[:, rows.to(dev)], ref)


def test_convert_bf16_to_f16_exact_and_saturating(mrsa, dev):
    """in-range values convert with round-to-nearest; |x| > 65504 (and
    infinities) saturate to +-65504 and raise bit 3 of the device flags"""
    lib = mrsa._lib.load()
    gen = torch.Generator().manual_seed(16)
    x = (torch.randn(4096, generator=gen) * 300).bfloat16()
    x[:8] = torch.tensor([70000., -70000., 65504., -65504., 1e-6, 0., float("inf"), 3e-8]).bfloat16()
    lib.mrsa_device_error_flags(1)
    y = mrsa.to_f16(x.to(dev)).cpu()
    want = x.float().clamp(-65504., 65504.).half()
    assert torch.equal(y, want)
    assert lib.mrsa_device_error_flags(1) & 8
    y2 = mrsa.to_f16(x[8:].to(dev)).cpu()                 # nothing out of range
    assert torch.equal(y2, x[8:].float().half())
    assert lib.mrsa_device_error_flags(1) & 8 == 0


@pytest.mark.parametrize("window,skip", [(256, True), (1280, False), (40, True)])
def test_local_attention_matches_oracle(mrsa, dev, window, skip):
    _local_case(mrsa, dev, window, skip, f16v=False)


@pytest.mark.parametrize("window,skip", [(256, True), (1280, False)])
def test_local_attention_f16v_matches_oracle(mrsa, dev, window, skip):
    """V in fp16: P as one fp16 tile (11 significant bits) instead of bf16 hi + lo"""
    _local_case(mrsa, dev, window, skip, f16v=True)


@pytest.mark.parametrize("hq,l", [(4, 300), (8, 157), (16, 1), (32, 200), (28, 37), (28, 73)])
def test_local_attention_group_sizes_and_ragged_lengths(mrsa, dev, hq, l):
    """The window kernel packs 128 // G queries x G head rows per query tile and
    runs two tiles per CTA: group sizes 1, 2, 4, 8 and 7 (tiles of 128, 64, 32,
    16 and 18 queries), lengths that leave a CTA's second tile partial or
    empty, bf16 V (hi + lo P) and fp16 V."""
    gen = torch.Generator().manual_seed(hq * 1000 + l)
    b, hkv, d, window = 2, 4, 128, 40
    q = torch.randn(b, l, hq, d, generator=gen).bfloat16()
    k = torch.randn(b, l, hkv, d, generator=gen).bfloat16()
    v = torch.randn(b, l, hkv, d, generator=gen).bfloat16()
    valid = torch.rand(b, l, generator=gen) > 0.1
    ro, rl = orc.local_attention(q, k, v, valid, window, 64, True)
    # the kernel entry directly: the reference's layout check wants L % 64 == 0
    o, lse = mrsa.window_attention(q.to(dev), k.to(dev), v.to(dev), valid.to(dev), window + 63,
                                   skip_inert=True, chunk=64)
    close_bf16(o, ro)
    torch.testing.assert_close(lse.cpu(), rl, atol=2e-4, rtol=1e-5)
    o16, lse16 = mrsa.window_attention(q.to(dev), k.to(dev), mrsa.to_f16(v.to(dev)), valid.to(dev), window + 63,
                                       skip_inert=True, chunk=64)
    close_bf16(o16, ro)
    torch.testing.assert_close(lse16.cpu(), rl, atol=2e-4, rtol=1e-5)


def _local_case(mrsa, dev, window, skip, f16v):
    gen = torch.Generator().manual_seed(window)
    b, l, hq, hkv, d = 2, 2048 + 64, 28, 4, 128
    q = (torch.randn(b, l, hq, d, generator=gen)).bfloat16()
    k = (torch.randn(b, l, hkv, d, generator=gen)).bfloat16()
    v = torch.randn(b, l, hkv, d, generator=gen).bfloat16()
    valid = torch.rand(b, l, generator=gen) > 0.05
    valid[1, 1900:] = False
    if f16v:
        eff = window + 63 if skip else window    # bidir_local_attention's effective window
        o, lse = mrsa.window_attention(q.to(dev), k.to(dev), mrsa.to_f16(v.to(dev)), valid.to(dev), eff,
                                       skip_inert=skip, chunk=64)
    else:
        o, lse = mrsa.bidir_local_attention(q.to(dev), k.to(dev), v.to(dev), valid.to(dev), window, 64,
                                            skip_inert_slots=skip)
    sl = slice(1024, 1536)
    ro, rl = orc._local_rows(q, k, v, valid, window, 64, skip, sl)
    close_bf16(o[:, sl], ro)
    torch.testing.assert_close(lse[:, sl].cpu(), rl, atol=2e-4, rtol=1e-5)
    ro2, rl2 = orc._local_rows(q, k, v, valid, window, 64, skip, slice(0, 256))
    close_bf16(o[:, :256], ro2)
    torch.testing.assert_close(lse[:, :256].cpu(), rl2, atol=2e-4, rtol=1e-5)


def test_fuse_outputs_dropin(mrsa, dev):
    gen = torch.Generator().manual_seed(1)
    r = torch.randn(1, 64, 28, 128, generator=gen).bfloat16()
    lo = torch.randn(1, 64, 28, 128, generator=gen).bfloat16()
    w = torch.rand(1, 64, 28, generator=gen).bfloat16()
    got = mrsa.fuse_hils_outputs(r.to(dev), lo.to(dev), w.to(dev))
    assert torch.equal(got.cpu(), orc.fuse_outputs(r, lo, w))


# ---------------------------------------------------------------- layers
def _layer_case(mrsa, dev, l, cfg, hidden, seed, key_valid=None, batch=1):
    inp = orc.make_route_layer_inputs(batch, l, cfg, hidden=hidden, seed=seed, key_valid=key_valid)
    lc = mrsa.RouteLayerConfig(q_heads=cfg.q_heads, kv_heads=cfg.kv_heads)
    layer = mrsa.RouteLayer(inp["w_in"].to(dev), inp["w_out"].to(dev), cfg=lc)
    args = [inp[n].to(dev) for n in ("q_pre", "k_pre", "v", "hidden", "position_ids")]
    return inp, layer, args


def _check_layer(mrsa, dev, l, cfg, hidden, seed, sl, key_valid=None, batch=1, min_exact=0.9):
    inp, layer, args = _layer_case(mrsa, dev, l, cfg, hidden, seed, key_valid, batch)
    kv = inp["key_valid"].to(dev)
    st = layer.forward(*args, kv, stages=True)
    fused = layer.forward(*args, kv)
    assert torch.equal(fused, st["out"]), "fused C-ABI layer differs from the staged ops"
    ref = orc.route_layer_forward(inp, cfg, query_slice=sl)
    rows = ref["rows"].nonzero().squeeze(1)           # the query rows the oracle computed
    ulp_close(st["q"][:, rows.to(dev)], ref["q"][:, rows])
    ulp_close(st["k"], ref["k"])
    rq_rows = torch.arange(cfg.chunk - 1, l, cfg.chunk)
    # route_q is RMS-normalised (|x| up to ~8): one bf16 ulp there is 3.1e-2
    close_bf16(st["route_q"][:, rq_rows], ref["route_q"][:, rq_rows], max_abs=6.5e-2, mean_rel=2e-3)
    close_bf16(st["lmk"], ref["lmk"], max_abs=2e-2, mean_rel=2e-3)
    torch.testing.assert_close(st["entropy"].cpu(), ref["entropy"], atol=2e-3, rtol=1e-3)
    close_bf16(st["local_out"][:, sl], ref["local_out"])
    torch.testing.assert_close(st["local_lse"][:, sl].cpu(), ref["local_lse"], atol=5e-4, rtol=1e-5)
    viol, exact = orc.topk_set_agreement(ref["route_key"], st["indices"][:, sl].cpu(), ref["indices"], cfg.topk)
    assert viol == 0
    assert exact >= min_exact, exact
    # attention parity on the kernel's own selection (decouples near-tie flips)
    ref_own = orc.route_layer_forward(inp, cfg, query_slice=sl, indices=st["indices"][:, sl].cpu())
    close_bf16(st["remote_weights"][:, sl], ref_own["remote_weights"], max_abs=2e-2, mean_rel=2e-3)
    close_bf16(st["local_weight"][:, sl], ref_own["local_weight"], max_abs=2e-2, mean_rel=2e-3)
    close_bf16(st["remote_out"][:, sl], ref_own["remote_out"])
    close_bf16(st["out"][:, sl], ref_own["out"])
    return st, ref


def test_route_layer_dream_shape_matches_oracle(mrsa, dev):
    cfg = orc.MRSAConfig()
    _check_layer(mrsa, dev, 4096, cfg, 3584, 0, slice(2048, 2560))


def test_route_layer_ragged_validity_and_batch(mrsa, dev):
    cfg = orc.MRSAConfig()
    l = 2112                                   # 33 chunks, not a multiple of 16 queries x 64
    kv = torch.ones(2, l, dtype=torch.bool)
    kv[0, 640:703] = False                     # chunk 10: only its landmark valid -> never routed
    kv[1, 1500:] = False                       # ragged tail
    kv[1, ::37] = False
    st, ref = _check_layer(mrsa, dev, l, cfg, 256, 5, slice(1024, 1408), key_valid=kv, batch=2)
    assert not (st["indices"][0] == 10).any()


def test_route_layer_short_sequence_pads_with_minus_one(mrsa, dev):
    """9 chunks: the local window drops most of them, fewer than 32 remain."""
    cfg = orc.MRSAConfig(q_heads=7, kv_heads=1)
    st, _ = _check_layer(mrsa, dev, 576, cfg, 128, 9, slice(0, 576), min_exact=0.97)
    i = st["indices"].cpu()
    assert (i[..., -1] == -1).all()


def test_route_layer_vs_reference_composition_golden(mrsa, dev):
    """against the reference's own functions composed on the live path (bf16
    RoPE chain there, fp32 RoPE here)"""
    g = load_golden("layer.pt")
    cfg = orc.MRSAConfig(q_heads=g["q_heads"], kv_heads=g["kv_heads"])
    inp, layer, args = _layer_case(mrsa, dev, g["seq_len"], cfg, g["hidden"], g["seed"])
    st = layer.forward(*args, inp["key_valid"].to(dev), stages=True)
    key = orc.route_layer_forward(
        orc.make_route_layer_inputs(1, g["seq_len"], cfg, hidden=g["hidden"], seed=g["seed"]),
        orc.MRSAConfig(q_heads=7, kv_heads=1, rope_precision="bf16"))["route_key"]
    viol, exact = orc.topk_set_agreement(key, st["indices"].cpu(), g["indices"], 32, gap=2e-3)
    assert viol == 0 and exact >= 0.8
    same = (st["indices"].cpu() == g["indices"]).all(-1).all(-1)[0]
    rows = same.nonzero().squeeze(1)
    close_bf16(st["out"][:, rows.to(dev)], g["out"][:, rows], max_abs=3e-2, mean_rel=6e-3)


def test_route_layer_deterministic(mrsa, dev):
    cfg = orc.MRSAConfig()
    inp, layer, args = _layer_case(mrsa, dev, 2048, cfg, 512, 3)
    a = layer(*args)
    b = layer(*args)
    assert torch.equal(a, b)


def test_swa_layer_matches_oracle(mrsa, dev):
    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(2, 3072, cfg, hidden=64, seed=6)
    out, lse = mrsa.swa_layer_forward(*[inp[n].to(dev) for n in ("q_pre", "k_pre", "v", "position_ids")],
                                      inp["key_valid"].to(dev), return_lse=True)
    inv, af = orc.yarn_inv_freq(128, cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
    cos, sin = orc.rope_cos_sin(inp["position_ids"], inv, af)
    q, k = orc.apply_rope(inp["q_pre"], cos, sin), orc.apply_rope(inp["k_pre"], cos, sin)
    sl = slice(1280, 1792)
    ro, rl = orc._local_rows(q, k, inp["v"], inp["key_valid"], 1280, 64, False, sl)
    close_bf16(out[:, sl], ro)
    torch.testing.assert_close(lse[:, sl].cpu(), rl, atol=5e-4, rtol=1e-5)


def test_no_device_side_wait_gave_up(mrsa, dev):
    """every bounded in-kernel wait of the runs above completed"""
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0


@pytest.mark.parametrize("rows", [1, 33, 200, 1000])
def test_qcal_head_split_for_few_tokens_is_bit_equal(mrsa, dev, rows):
    """Q-Cal with fewer 64-token tiles than SMs splits the heads over CTAs
    (each recomputing its tile's h W_in^T).  Every token's route query must be
    the same bits as the same token computed inside a large call, where one
    CTA walks all heads."""
    lib = mrsa._lib
    gen = torch.Generator().manual_seed(rows)
    l, hq, d, hidden, rank = 16384, 28, 128, 3584, 64
    h = torch.randn(1, l, hidden, generator=gen).bfloat16().to(dev)
    q = (torch.randn(1, l, hq, d, generator=gen) / d ** 0.5).bfloat16().to(dev)
    w_in = (torch.randn(rank, hidden, generator=gen) * 0.02).bfloat16().to(dev)
    w_out = (torch.randn(hq * d, rank, generator=gen) * 0.02).bfloat16().to(dev)
    norm = torch.ones(d, device=dev)
    i = torch.arange(l, device=dev)
    pos = (i - i // 64).view(1, -1).contiguous()
    inv, af = mrsa.yarn_inv_freq(d, 1.0e6, 8.0, 2048)
    inv = inv.to(dev)

    def qcal(hh, qq, pp):
        out = torch.empty_like(qq)
        lib.call("mrsa_qcal_route_query", lib.ptr(hh), lib.ptr(qq), lib.ptr(w_in), lib.ptr(w_out), lib.ptr(norm),
                 1e-6, 1.0, lib.ptr(pp), lib.ptr(inv), float(af), lib.ptr(out), 1, qq.shape[1], hidden, rank, hq, d,
                 lib.stream_of(qq))
        return out

    full = qcal(h, q, pos)
    start = 5000 + rows % 37                  # not on a 64-token tile boundary
    sl = slice(start, start + rows)
    part = qcal(h[:, sl].contiguous(), q[:, sl].contiguous(), pos[:, sl].contiguous())
    torch.cuda.synchronize(dev)
    assert torch.equal(part, full[:, sl])
