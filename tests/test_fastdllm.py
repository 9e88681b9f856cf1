"""Fast-dLLM cached decode step (``dream_dllm_hils/fastdllm_attention.py:70-382``).

CPU: the oracle's cached step reproduces the oracle's full-sequence route
layer on the same rows when the step changes nothing (the cache holds the
prefill and the partial rows carry the prefill's own values) -- the
property that makes the cached step an exact replacement for a re-run.

GPU: ``mrsa_b200.fastdllm.cached_route_layer_step`` (every stage on this
package's kernels) against the oracle's step with new values at the
updated rows: cache K/V, refreshed landmarks and prior, routing (gap-aware
set agreement) and the output (max-abs 2e-2 / mean-rel 1e-3 on the kernel's
own selection); and the sliding-window branch.
"""

import pytest
import torch

from oracle import fastdllm as ofd
from oracle import route_layer as orc


def _prefill_cache(inp, cfg):
    """Cache state after a prefill: RoPE'd K, V, validity, landmarks, prior."""
    l = inp["q_pre"].shape[1]
    rows = torch.zeros(l, dtype=torch.bool)
    rows[cfg.chunk - 1::cfg.chunk] = True
    sh = orc.route_layer_shared(inp, cfg, rows=rows)
    cache = {"key": sh["k"].clone(), "value": inp["v"].clone(), "key_valid": inp["key_valid"].clone(),
             "landmark_keys": sh["lmk"].clone(), "prior_bias": sh["prior_bias"].clone()}
    return cache, sh


def _weights(inp):
    return {n: inp[n] for n in ("w_in", "w_out", "norm_weight", "entropy_bias_scale")}


def _query_positions(l, chunk=64):
    """Two decode blocks of 32 rows plus the landmark slots of the chunks they touch."""
    blocks = [torch.arange(l // 4 + 16, l // 4 + 48), torch.arange(l // 2 + 40, l // 2 + 72)]
    upd = torch.cat(blocks)
    aff = torch.unique(upd // chunk)
    qp = torch.unique(torch.cat([upd, aff * chunk + chunk - 1]))
    return qp, upd, aff


def test_oracle_cached_step_without_changes_equals_the_prefill_rows():
    cfg = orc.MRSAConfig()
    l = 1024
    inp = orc.make_route_layer_inputs(1, l, cfg, hidden=3584, seed=3)
    inp["key_valid"][0, 600:620] = False
    cache, _ = _prefill_cache(inp, cfg)
    qp, upd, aff = _query_positions(l)
    pos = orc.landmark_position_ids(1, l)
    sel = lambda t: t.index_select(1, qp)
    out, new_cache, inter = ofd.cached_route_layer_step(cache, sel(inp["q_pre"]), sel(inp["k_pre"]), sel(inp["v"]),
                                                        sel(inp["hidden"]), sel(pos), qp, upd, aff, _weights(inp), cfg)
    # the cache is unchanged by a step that writes back the prefill's own values
    assert torch.equal(new_cache["key"], cache["key"]) and torch.equal(new_cache["value"], cache["value"])
    torch.testing.assert_close(new_cache["landmark_keys"], cache["landmark_keys"], atol=0, rtol=0)
    torch.testing.assert_close(new_cache["prior_bias"], cache["prior_bias"], atol=0, rtol=0)
    # the rows equal the full layer's rows (default gate: the affine gate is the plain softmax)
    full = orc.route_layer_forward(inp, cfg)
    assert torch.equal(inter["indices"], full["indices"].index_select(1, qp))
    torch.testing.assert_close(out.float(), full["out"].index_select(1, qp).float(), atol=2e-2, rtol=0)
    d = (out.float() - full["out"].index_select(1, qp).float()).abs()
    assert d.mean() / full["out"].float().abs().mean() < 1e-3


def _step_case(l, seed):
    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(1, l, cfg, hidden=3584, seed=seed)
    inp["key_valid"][0, l // 3:l // 3 + 25] = False
    cache, _ = _prefill_cache(inp, cfg)
    qp, upd, aff = _query_positions(l)
    g = torch.Generator().manual_seed(seed + 100)
    m = qp.numel()
    pos = orc.landmark_position_ids(1, l).index_select(1, qp)
    new = {"q_pre": (torch.randn(1, m, 28, 128, generator=g) / 128 ** 0.5).bfloat16(),
           "k_pre": (torch.randn(1, m, 4, 128, generator=g) / 128 ** 0.5).bfloat16(),
           "v": (torch.randn(1, m, 4, 128, generator=g) / 128 ** 0.5).bfloat16(),
           "hidden": torch.randn(1, m, 3584, generator=g).bfloat16(), "position_ids": pos}
    return cfg, inp, cache, qp, upd, aff, new


@pytest.mark.gpu
def test_cached_route_layer_step_matches_the_oracle_step(mrsa, cuda_device):
    from mrsa_b200.fastdllm import LayerKVCache, cached_route_layer_step

    dev = cuda_device
    cfg, inp, cache, qp, upd, aff, new = _step_case(4096, seed=12)
    ref_out, ref_cache, inter = ofd.cached_route_layer_step(cache, new["q_pre"], new["k_pre"], new["v"],
                                                            new["hidden"], new["position_ids"], qp, upd, aff,
                                                            _weights(inp), cfg)
    gc = LayerKVCache(*(cache[n].to(dev) for n in ("key", "value", "key_valid", "landmark_keys", "prior_bias")))
    layer = mrsa.RouteLayer(inp["w_in"].to(dev), inp["w_out"].to(dev))
    out, stats = cached_route_layer_step(layer, *(new[n].to(dev) for n in ("q_pre", "k_pre", "v", "hidden",
                                                                           "position_ids")),
                                         qp.to(dev), upd.to(dev), aff.to(dev), gc)
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0
    assert stats.routing_calls == 1 and torch.equal(stats.refreshed_chunks.cpu(), aff)
    # cache K/V at the updated rows (RoPE: one bf16 rounding of fp32 math on both sides)
    torch.testing.assert_close(gc.key.float().cpu(), ref_cache["key"].float(), atol=1e-2, rtol=8e-3)
    assert torch.equal(gc.value.cpu(), ref_cache["value"])
    # refreshed landmarks and prior of the affected chunks; the others untouched
    torch.testing.assert_close(gc.landmark_keys.float().cpu(), ref_cache["landmark_keys"].float(),
                               atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(gc.prior_bias.cpu(), ref_cache["prior_bias"], atol=2e-3, rtol=1e-3)
    untouched = torch.ones(gc.prior_bias.shape[1], dtype=torch.bool)
    untouched[aff] = False
    assert torch.equal(gc.prior_bias.cpu()[:, untouched], cache["prior_bias"][:, untouched])
    # a second run on a fresh copy of the cache: same bits, and its stages
    gc2 = LayerKVCache(*(cache[n].to(dev) for n in ("key", "value", "key_valid", "landmark_keys", "prior_bias")))
    out2, _, st = cached_route_layer_step(layer, *(new[n].to(dev) for n in ("q_pre", "k_pre", "v", "hidden",
                                                                            "position_ids")),
                                          qp.to(dev), upd.to(dev), aff.to(dev), gc2, stages=True)
    assert torch.equal(out, out2), "the cached step is deterministic"
    close = dict(atol=2e-2, rtol=0)
    torch.testing.assert_close(st["local_out"].float().cpu(), inter["local_out"].float(), **close)
    torch.testing.assert_close(st["local_lse"].cpu(), inter["local_lse"], atol=5e-4, rtol=1e-5)
    assert torch.equal(st["drop"].cpu(), inter["drop"])
    # routing: no selection differs where the key gap exceeds 1e-3
    idx = st["indices"].long().cpu()
    viol, exact = orc.topk_set_agreement(inter["route_key"], idx, inter["indices"], cfg.topk)
    assert viol == 0 and exact >= 0.9, (viol, exact)
    # output on the kernel's own selection
    want = ofd.cached_route_layer_rows_with(ref_cache, inter["q"], inter["route_q"], inter["local_out"],
                                            inter["local_lse"], idx)
    got, want = out.float().cpu(), want.float()
    d = (got - want).abs()
    assert d.max() <= 2e-2 and d.mean() / want.abs().mean() <= 1e-3, (d.max().item(), d.mean().item())


@pytest.mark.gpu
def test_cached_swa_layer_step_matches_the_oracle_step(mrsa, cuda_device):
    from mrsa_b200.fastdllm import LayerKVCache, cached_swa_layer_step

    dev = cuda_device
    cfg, inp, cache, qp, upd, aff, new = _step_case(4096, seed=13)
    ref_out, ref_cache = ofd.cached_swa_layer_step(cache, new["q_pre"], new["k_pre"], new["v"],
                                                   new["position_ids"], qp, upd, 1280, cfg)
    gc = LayerKVCache(cache["key"].to(dev), cache["value"].to(dev), cache["key_valid"].to(dev))
    out, stats = cached_swa_layer_step(*(new[n].to(dev) for n in ("q_pre", "k_pre", "v", "position_ids")),
                                       qp.to(dev), upd.to(dev), gc)
    assert stats.routing_calls == 0
    d = (out.float().cpu() - ref_out.float()).abs()
    assert d.max() <= 2e-2 and d.mean() / ref_out.float().abs().mean() <= 1e-3


def test_layer_kv_cache_validates_like_the_reference(mrsa):
    from mrsa_b200.fastdllm import LayerKVCache

    k = torch.zeros(1, 128, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        LayerKVCache(k, k, torch.ones(1, 128))                       # key_valid must be bool
    with pytest.raises(ValueError):
        LayerKVCache(k, k, torch.ones(1, 128, dtype=torch.bool), torch.zeros(1, 2, 4, 7, 128, dtype=torch.bfloat16))
    c = LayerKVCache(k.clone(), k.clone(), torch.ones(1, 128, dtype=torch.bool))
    with pytest.raises(ValueError):
        c.replace(torch.tensor([3, 3]), k[:, :2], k[:, :2])           # positions must be unique
    c.replace(torch.tensor([5, 9]), torch.ones(1, 2, 4, 128, dtype=torch.bfloat16), k[:, :2])
    assert c.key[0, 5].float().sum() == 512 and c.key[0, 9].float().sum() == 512 and c.key[0, 6].float().sum() == 0


@pytest.mark.parametrize("case,msg", [
    ("dup_query", "query_positions must be unique"),
    ("range_query", "query_positions must be in range"),
    ("count", "query position count must match partial hidden length"),
    ("unsorted", "query_positions must be sorted"),
    ("dup_update", "kv_update_positions must be unique"),
    ("not_owned", "all owned positions must also be query positions"),
    ("pos_shape", "position_ids must have shape (1, 4)"),
    ("first_wins", "query_positions must be unique"),
])
def test_cached_step_position_checks_raise_like_the_reference(mrsa, case, msg):
    """The cached step's position checks, read back from the device in one
    transfer, raise the reference's first failing check (same order, same
    message) before anything is computed or written; CPU tensors suffice."""
    from mrsa_b200.fastdllm import LayerKVCache, _prepare

    k = torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16)
    cache = LayerKVCache(k.clone(), k.clone(), torch.ones(1, 256, dtype=torch.bool))
    q = torch.zeros(1, 4, 28, 128, dtype=torch.bfloat16)
    kv = torch.zeros(1, 4, 4, 128, dtype=torch.bfloat16)
    qp, up, pos = torch.tensor([3, 9, 63, 100]), torch.tensor([3, 9]), torch.zeros(1, 4, dtype=torch.long)
    if case == "dup_query":
        qp = torch.tensor([3, 9, 9, 100])
    elif case == "range_query":
        qp = torch.tensor([3, 9, 63, 256])
    elif case == "count":
        qp = torch.tensor([3, 9, 63])
    elif case == "unsorted":
        qp = torch.tensor([9, 3, 63, 100])
    elif case == "dup_update":
        up = torch.tensor([3, 3])
    elif case == "not_owned":
        up = torch.tensor([3, 10])
    elif case == "pos_shape":
        pos = torch.zeros(4, dtype=torch.long)
    elif case == "first_wins":                   # also unsorted and a bad position_ids shape
        qp, pos = torch.tensor([9, 9, 3, 100]), torch.zeros(4, dtype=torch.long)
    before = cache.key.clone()
    with pytest.raises(ValueError, match=msg.replace("(", r"\(").replace(")", r"\)")):
        _prepare(q, kv, kv, pos, qp, up, cache, torch.ones(64), 1.0)
    assert torch.equal(cache.key, before)
