"""GPU parity of the ops off the route layer's live path -- the causal flex
window (``flex_attn_tl``), the cached (Fast-dLLM) local rows, candidate token
scores and selected-token (DSA) attention -- against the CPU oracle, which
``test_oracle_golden.py`` pins to the reference's own functions (the cached
local rows through ``cached_local_attention`` with a CPU stand-in for its
flash-attn call).

Tolerances: bf16 attention outputs max-abs <= 2e-2 and mean-rel <= 1e-3 (as
for the route layer), plus the reference tests' own bars where they state
one (DSA relative L2 < 1e-2, ``unittests/test_dream_dsa_fastdllm.py:86-90``);
fp32 token scores within 1e-4 (accumulation order only), the -inf pattern
exact.
"""

import math

import pytest
import torch

from oracle import token_ops as tok

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def close_bf16(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all()
    d = (got - ref).abs()
    rel = d.mean().item() / max(ref.abs().mean().item(), 1e-30)
    assert d.max().item() <= max_abs and rel <= mean_rel, (d.max().item(), rel)


@pytest.fixture(scope="module")
def dev(cuda_device):
    return cuda_device


# ------------------------------------------------------------ flex_attn_tl
# the reference's own case list (ops/flex_attn_tilelang.py:1405-1525), D = 128
FLEX = [
    # name, training, batch, hq, hkv, L_k, L_q, window, chunk, mask_lmk, expand, kv_start
    ("train_lmk_expand", True, 1, 8, 2, 512, 512, 128, 64, True, True, 0),
    ("train_no_flags", True, 1, 8, 2, 512, 512, 128, 64, False, False, 0),
    ("train_lmk_only", True, 1, 8, 2, 512, 512, 128, 64, True, False, 0),
    ("train_expand_only", True, 1, 8, 2, 512, 512, 128, 64, False, True, 0),
    ("train_dream_g7_batch2", True, 2, 28, 4, 640, 640, 320, 64, True, True, 0),
    ("train_w_lt_cs", True, 1, 8, 2, 512, 512, 32, 64, True, True, 0),
    ("train_w_not_mult", True, 1, 8, 2, 384, 384, 100, 64, True, True, 0),
    ("train_w_ge_seq", True, 1, 8, 2, 256, 256, 512, 64, True, True, 0),
    ("train_seq_not_block", True, 1, 8, 2, 200, 200, 128, 64, True, True, 0),
    ("infer_prefill_half", False, 1, 8, 2, 512, 256, 128, 64, True, True, 0),
    ("infer_prefill_small", False, 1, 8, 2, 512, 64, 128, 64, True, True, 0),
    ("infer_decode_q1", False, 1, 8, 2, 512, 1, 128, 64, True, True, 0),
    ("infer_decode_q1_long", False, 1, 8, 2, 2048, 1, 512, 128, True, True, 0),
    ("infer_gqa_g4_q1", False, 1, 8, 2, 512, 1, 128, 64, True, True, 0),
    ("infer_gqa_g8_q1", False, 1, 8, 1, 512, 1, 128, 64, True, True, 0),
    ("infer_q_non_aligned", False, 1, 8, 2, 1024, 100, 256, 64, True, True, 0),
    ("infer_noexp_lmk_k333", False, 1, 8, 2, 333, 1, 512, 64, True, False, 0),
    ("infer_kv_start", False, 1, 8, 2, 448, 96, 200, 64, True, True, 64),
    ("infer_kv_start_odd", False, 1, 8, 2, 300, 37, 150, 64, True, False, 17),
    ("train_chunk65_long", True, 1, 8, 2, 2080, 2080, 512, 65, True, True, 0),
    ("train_chunk65_nonmultiple", True, 1, 8, 2, 1000, 1000, 512, 65, True, True, 0),
    ("infer_chunk65_nonmultiple", False, 1, 8, 2, 1000, 333, 512, 65, True, True, 0),
    ("train_L16_lt_chunk", True, 1, 8, 2, 16, 16, 512, 64, True, True, 0),
]


@pytest.mark.parametrize("case", FLEX, ids=[c[0] for c in FLEX])
def test_flex_attn_tl_matches_oracle(mrsa, dev, case):
    name, training, b, hq, hkv, lk, lq, w, c, lmk, exp, kv_start = case
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    q = (torch.randn(b, lq, hq, 128, generator=g) * 0.5).bfloat16()
    k = (torch.randn(b, lk, hkv, 128, generator=g) * 0.5).bfloat16()
    v = (torch.randn(b, lk, hkv, 128, generator=g) * 0.5).bfloat16()
    o, lse = mrsa.flex_attn_tl(q.to(dev), k.to(dev), v.to(dev), window_size=w, chunk_size=c,
                               training=training, mask_lmk=lmk, expand_to_chunk=exp, kv_start=kv_start)
    ro, rl = tok.flex_window_attention(q, k, v, w, c, lmk, exp, kv_start)
    close_bf16(o, ro.to(torch.bfloat16))     # both sides rounded to the bf16 output
    lse = lse.cpu()
    assert torch.equal(torch.isfinite(lse), torch.isfinite(rl)), name
    fin = torch.isfinite(rl)
    torch.testing.assert_close(lse[fin], rl[fin], atol=1e-3, rtol=1e-5)
    assert torch.count_nonzero(o.cpu()[~fin]) == 0


def test_flex_attn_tl_rejects_reference_errors(mrsa, dev):
    q = torch.zeros(1, 64, 8, 128, dtype=torch.bfloat16, device=dev)
    k = torch.zeros(1, 64, 2, 128, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError, match="kv_start"):
        mrsa.flex_attn_tl(q, k, k, 32, 64, training=True, kv_start=4)
    with pytest.raises(ValueError):
        mrsa.flex_attn_tl(q.float(), k, k, 32, 64)
    with pytest.raises(ValueError):
        mrsa.flex_attn_tl(torch.zeros(1, 65, 8, 128, dtype=torch.bfloat16, device=dev), k, k, 32, 64)


# ------------------------------------------------ cached (Fast-dLLM) local rows
@pytest.mark.parametrize("positions", [
    list(range(512, 544)),                                   # one decode block
    [1023, 5, 700, 64, 63, 300, 301, 999, 0, 511, 128, 127, 640, 641, 642, 900, 17],   # scattered, unsorted
])
@pytest.mark.parametrize("window,skip", [(256, True), (1280, False)])
def test_cached_local_attention_matches_oracle(mrsa, dev, positions, window, skip):
    from oracle import route_layer as orc

    g = torch.Generator().manual_seed(len(positions) + window)
    b, l, hq, hkv, d = 2, 1024, 28, 4, 128
    pos = torch.tensor(positions, dtype=torch.long)
    q = torch.randn(b, len(positions), hq, d, generator=g).bfloat16()
    k = torch.randn(b, l, hkv, d, generator=g).bfloat16()
    v = torch.randn(b, l, hkv, d, generator=g).bfloat16()
    valid = torch.rand(b, l, generator=g) > 0.05
    valid[1, 900:] = False
    o, lse = mrsa.cached_local_attention(q.to(dev), k.to(dev), v.to(dev), valid.to(dev), pos.to(dev),
                                         window, 64, skip_inert_slots=skip)
    # the reference places the rows at their positions and runs the full window
    # (dream_dllm_hils/local_attention.py:183-197)
    q_full = torch.zeros(b, l, hq, d, dtype=torch.bfloat16)
    q_full[:, pos] = q
    ro, rl = orc.local_attention(q_full, k, v, valid, window, 64, skip)
    close_bf16(o, ro[:, pos])
    torch.testing.assert_close(lse.cpu(), rl[:, pos], atol=2e-4, rtol=1e-5)


def test_cached_local_attention_rejects_reference_errors(mrsa, dev):
    q = torch.zeros(1, 3, 28, 128, dtype=torch.bfloat16, device=dev)
    k = torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16, device=dev)
    valid = torch.ones(1, 256, dtype=torch.bool, device=dev)
    with pytest.raises(ValueError, match="unique"):
        mrsa.cached_local_attention(q, k, k, valid, torch.tensor([1, 1, 2], device=dev), 256, 64)
    with pytest.raises(ValueError, match="cache range"):
        mrsa.cached_local_attention(q, k, k, valid, torch.tensor([1, 2, 256], device=dev), 256, 64)
    with pytest.raises(ValueError, match="torch.long"):
        mrsa.cached_local_attention(q, k, k, valid, torch.tensor([1, 2, 3], device=dev, dtype=torch.int32),
                                    256, 64)


# ------------------------------------------------------ candidate token scores
@pytest.mark.parametrize("b,lq,lk,hq,hkv,sel,chunk", [
    (1, 96, 2048, 28, 4, 32, 64),      # Dream route-layer shape (K=32 of 32 chunks)
    (2, 37, 1024, 28, 4, 8, 64),       # batch, ragged query count
    (1, 20, 650, 16, 1, 5, 65),        # 16-head group, odd chunk
    (1, 9, 256, 4, 2, 3, 16),          # smallest chunk the reference accepts
])
def test_candidate_token_scores_match_oracle(mrsa, dev, b, lq, lk, hq, hkv, sel, chunk):
    g = torch.Generator().manual_seed(lq * 7 + sel)
    q = (torch.randn(b, lq, hq, 128, generator=g) / math.sqrt(128)).bfloat16()
    k = torch.randn(b, lk, hkv, 128, generator=g).bfloat16()
    c = lk // chunk
    idx = torch.randint(0, c, (b, lq, hkv, sel), generator=g).to(torch.int32)
    idx[:, 1, :, : sel // 2] = -1
    idx[:, 2, 0, 0] = c            # out of range: -inf like a negative index
    valid = torch.ones(b, lk, dtype=torch.bool)
    valid[:, chunk + 3: chunk + 11] = False
    valid[-1, -chunk // 2:] = False
    got = mrsa.candidate_token_scores_gqa(q.to(dev), k.to(dev), idx.to(dev), valid.to(dev), chunk).cpu()
    ref = tok.candidate_token_scores(q, k, idx, valid, chunk)
    assert torch.equal(torch.isinf(got), torch.isinf(ref))
    fin = torch.isfinite(ref)
    torch.testing.assert_close(got[fin], ref[fin], atol=1e-4, rtol=1e-4)


def test_candidate_token_scores_rejects_reference_errors(mrsa, dev):
    q = torch.zeros(1, 4, 28, 128, dtype=torch.bfloat16, device=dev)
    k = torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16, device=dev)
    idx = torch.zeros(1, 4, 4, 2, dtype=torch.int32, device=dev)
    valid = torch.ones(1, 256, dtype=torch.bool, device=dev)
    with pytest.raises(ValueError, match="int32"):
        mrsa.candidate_token_scores_gqa(q, k, idx.long(), valid, 64)
    with pytest.raises(ValueError, match="chunk_size"):
        mrsa.candidate_token_scores_gqa(q, k, idx, valid, 8)
    with pytest.raises(ValueError, match="indices shape"):
        mrsa.candidate_token_scores_gqa(q, k, idx[..., :1].expand(1, 4, 4, 3).contiguous()[:, :3], valid, 64)


# ------------------------------------------------ selected-token attention (DSA)
@pytest.mark.parametrize("lq,lk,topk,hq,hkv", [
    (1, 128, 64, 28, 4),               # unittests/test_dream_dsa_fastdllm.py:75 cases
    (35, 2048, 1024, 28, 4),
    (67, 32768, 1024, 28, 4),
    (19, 4096, 2560, 28, 4),           # the Dream DSA layer's top-k
    (23, 1000, 101, 16, 1),            # 16-head group, top-k not a multiple of 4
])
def test_selected_token_attention_matches_oracle(mrsa, dev, lq, lk, topk, hq, hkv):
    g = torch.Generator().manual_seed(23 + topk)
    q = torch.randn(1, lq, hq, 128, generator=g).bfloat16()
    k = torch.randn(1, lk, hkv, 128, generator=g).bfloat16()
    v = torch.randn(1, lk, hkv, 128, generator=g).bfloat16()
    indices = torch.randint(-2, lk + 2, (1, lq, topk), generator=g)      # clamped by both sides
    valid = torch.rand(1, lq, topk, generator=g) > 0.2
    valid[:, 0] = False
    got = mrsa.selected_token_attention_tilelang(q.to(dev), k.to(dev), v.to(dev), indices.to(dev),
                                                 valid.to(dev)).cpu()
    ref = tok.selected_token_attention(q, k, v, indices, valid)
    close_bf16(got, ref)
    rel_l2 = (got.float() - ref.float()).norm() / ref.float().norm().clamp_min(1e-6)
    assert rel_l2 < 0.01
    assert torch.count_nonzero(got[:, 0]) == 0


def test_selected_token_attention_empty_and_custom_scale(mrsa, dev):
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 6, 28, 128, generator=g).bfloat16()
    k = torch.randn(1, 64, 4, 128, generator=g).bfloat16()
    v = torch.randn(1, 64, 4, 128, generator=g).bfloat16()
    none = torch.zeros(1, 6, 0, dtype=torch.long)
    out = mrsa.selected_token_attention_tilelang(q.to(dev), k.to(dev), v.to(dev), none.to(dev),
                                                 none.bool().to(dev))
    assert out.shape == q.shape and torch.count_nonzero(out) == 0
    idx = torch.randint(0, 64, (1, 6, 40), generator=g)
    valid = torch.ones(1, 6, 40, dtype=torch.bool)
    got = mrsa.selected_token_attention_tilelang(q.to(dev), k.to(dev), v.to(dev), idx.to(dev), valid.to(dev),
                                                 sm_scale=0.02).cpu()
    close_bf16(got, tok.selected_token_attention(q, k, v, idx, valid, sm_scale=0.02))


def test_token_ops_left_no_device_error(mrsa, dev):
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0


def test_bounded_wait_gives_up_and_context_survives(mrsa, dev):
    """Failure detection without a fault: a wait nothing ever satisfies gives up
    after its bounded rounds, raises the CTA's abort flag, a second waiter
    leaves through that flag, and the context keeps working afterwards."""
    res = torch.full((3,), -1, dtype=torch.int32, device=dev)
    mrsa._lib.call("mrsa_wait_selftest", mrsa._lib.ptr(res), 20, mrsa._lib.stream_of(res))
    torch.cuda.synchronize()
    assert res.tolist() == [1, 1, 1]
    x = torch.randn(1024, device=dev).bfloat16()
    assert torch.equal(mrsa.to_f16(x).float(), x.float())
    with pytest.raises(ValueError):
        mrsa._lib.call("mrsa_wait_selftest", mrsa._lib.ptr(res), 0, mrsa._lib.stream_of(res))
