"""Backward of the selected-chunk attention (and, below, of the other route-layer ops).

CPU: the fp32 autograd oracle (``oracle/backward.py``) against gradients of
the reference's own torch function (``tests/golden/selected_bwd.pt``, made by
``tests/golden/make_golden.py`` from ``ops/hils_fwd_bwd_head.py:21
hils_torch_ref``).

GPU: ``mrsa_selected_attention_backward`` (dQ/dW kernel + inverted-index
dK/dV kernel) against the oracle.  The kernels round dS and w*P to bf16
before their GEMMs, as the reference's backward kernel does
(``ops/hils_fwd_bwd_head.py:846-881``), so each gradient is compared by its
relative L2 error (<= 1e-2) and its largest element error (<= 2e-2 of the
largest reference element).
"""

import pytest
import torch

from conftest import load_golden
from oracle import backward as obw

REL_L2, MAX_FRAC = 1e-2, 2e-2


def close_grad(got, ref, name, rel_l2=REL_L2, max_frac=MAX_FRAC):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all(), name
    scale = ref.abs().max().item()
    if scale == 0.0:
        assert got.abs().max().item() == 0.0, name
        return
    err = (got - ref).norm().item() / max(ref.norm().item(), 1e-30)
    mx = (got - ref).abs().max().item() / scale
    assert err <= rel_l2 and mx <= max_frac, (name, err, mx)


def test_selected_grads_oracle_matches_reference_autograd():
    g, gb = load_golden("selected.pt"), load_golden("selected_bwd.pt")
    dq, dk, dv, dw = obw.selected_attention_grads(g["q"], g["k"], g["v"], g["weights"], g["indices"], None, 64,
                                                  gb["grad_out"])
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv"), (dw, "dw")):
        torch.testing.assert_close(got, gb[name], atol=2e-5, rtol=1e-4, msg=name)


def _sel_case(b, lq, lk, hkv, g, topk, seed, *, holes=True, dup=True):
    gen = torch.Generator().manual_seed(seed)
    c = lk // 64
    q = torch.randn(b, lq, hkv * g, 128, generator=gen).bfloat16()
    k = torch.randn(b, lk, hkv, 128, generator=gen).bfloat16()
    v = torch.randn(b, lk, hkv, 128, generator=gen).bfloat16()
    idx = torch.stack([torch.randperm(c, generator=gen)[:topk].sort().values for _ in range(b * lq * hkv)])
    idx = idx.view(b, lq, hkv, topk).to(torch.int32)
    if holes:
        idx[:, 3, :, topk // 2:] = -1                     # ragged list
        idx[:, 4] = -1                                    # nothing selected
    if dup:
        idx[0, 5, 0, 1] = idx[0, 5, 0, 0]                 # a chunk listed twice
    w = torch.softmax(torch.randn(b, lq, hkv * g, topk, generator=gen), -1).bfloat16()
    valid = torch.ones(b, lk, dtype=torch.bool)
    if holes:
        valid[:, 70:90] = False                           # ragged validity
        valid[-1, 128:192] = False                        # a chunk with no usable key
    go = torch.randn(b, lq, hkv * g, 128, generator=gen).bfloat16()
    return q, k, v, w, idx, valid, go


def _check_selected_bwd(mrsa, dev, case, mask_last=True):
    q, k, v, w, idx, valid, go = case
    dq, dk, dv, dw = mrsa.selected_attention_backward(q.to(dev), k.to(dev), v.to(dev), w.to(dev), idx.to(dev),
                                                      go.to(dev), valid.to(dev), mask_last_token=mask_last)
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0
    rq, rk, rv, rw = obw.selected_attention_grads(q, k, v, w, idx, valid, 64, go, mask_last_token=mask_last)
    close_grad(dq, rq, "dq")
    close_grad(dk, rk, "dk")
    close_grad(dv, rv, "dv")
    close_grad(dw, rw, "dw", rel_l2=1e-2, max_frac=2e-2)
    # empty slots carry no weight gradient
    empty = (idx < 0).repeat_interleave(q.shape[2] // k.shape[2], dim=2)
    assert (dw.cpu()[empty] == 0).all()


@pytest.mark.gpu
def test_selected_backward_matches_reference_autograd(mrsa, cuda_device):
    g, gb = load_golden("selected.pt"), load_golden("selected_bwd.pt")
    dev = cuda_device
    dq, dk, dv, dw = mrsa.selected_attention_backward(g["q"].to(dev), g["k"].to(dev), g["v"].to(dev),
                                                      g["weights"].to(dev), g["indices"].to(dev),
                                                      gb["grad_out"].to(dev))
    close_grad(dq, gb["dq"], "dq")
    close_grad(dk, gb["dk"], "dk")
    close_grad(dv, gb["dv"], "dv")
    close_grad(dw, gb["dw"], "dw")


@pytest.mark.gpu
@pytest.mark.parametrize("b,lq,lk,hkv,g,topk,mask_last", [
    (2, 200, 4096, 4, 7, 32, True),      # Dream shape, ragged query block, holes, a repeated chunk
    (1, 96, 2048, 2, 8, 16, False),      # a full 8-head group, landmark key kept
    (1, 40, 1024, 1, 3, 5, True),        # small group, top-k not a multiple of 4
])
def test_selected_backward_matches_oracle(mrsa, cuda_device, b, lq, lk, hkv, g, topk, mask_last):
    _check_selected_bwd(mrsa, cuda_device, _sel_case(b, lq, lk, hkv, g, topk, seed=lq + topk), mask_last)


@pytest.mark.gpu
def test_selected_backward_is_deterministic(mrsa, cuda_device):
    """The inverted index is built in query order, so two runs give the same bits."""
    dev = cuda_device
    q, k, v, w, idx, valid, go = (t.to(dev) for t in _sel_case(1, 512, 2048, 4, 7, 32, seed=5))
    first = mrsa.selected_attention_backward(q, k, v, w, idx, go, valid)
    second = mrsa.selected_attention_backward(q, k, v, w, idx, go, valid)
    for a, b2 in zip(first, second):
        assert torch.equal(a, b2)


@pytest.mark.gpu
def test_selected_backward_many_owners_per_chunk(mrsa, cuda_device):
    """Few chunks: every chunk is selected by most queries (8 owners per item,
    many 16-pair tiles per chunk in the dK/dV kernel)."""
    q, k, v, w, idx, valid, go = _sel_case(1, 256, 512, 4, 7, 6, seed=3, holes=False, dup=False)
    _check_selected_bwd(mrsa, cuda_device, (q, k, v, w, idx, valid, go))


@pytest.mark.gpu
def test_hils_block_m_head_autograd_uses_the_backward(mrsa, cuda_device):
    dev = cuda_device
    q, k, v, w, idx, valid, go = _sel_case(1, 64, 1024, 1, 7, 8, seed=11, holes=False, dup=False)
    qd, kd, vd, wd = (t.to(dev).requires_grad_() for t in (q, k, v, w))
    out = mrsa.HiLS_block_M_head(qd, kd, vd, wd, idx.to(dev), block_size=64, is_training=True,
                                 key_valid=valid.to(dev))
    out.backward(go.to(dev))
    dq, dk, dv, dw = mrsa.selected_attention_backward(q.to(dev), k.to(dev), v.to(dev), w.to(dev), idx.to(dev),
                                                      go.to(dev), valid.to(dev))
    assert torch.equal(qd.grad, dq.bfloat16()) and torch.equal(kd.grad, dk.bfloat16())
    assert torch.equal(vd.grad, dv.bfloat16()) and torch.equal(wd.grad, dw)
    # no grad requested: the forward-only kernel, no autograd node
    with torch.no_grad():
        out2 = mrsa.HiLS_block_M_head(qd, kd, vd, wd, idx.to(dev), block_size=64, key_valid=valid.to(dev))
    assert out2.grad_fn is None and torch.equal(out2, out.detach())


# ---------------------------------------------------------------- pool, weights, scores, fusion
def test_pool_grads_oracle_matches_reference_autograd():
    g, gb = load_golden("pool.pt"), load_golden("pool_bwd.pt")
    dmu, dk = obw.pool_grads(g["mu_q"], g["k_chunked"], g["key_valid"], gb["grad_lmk"], gb["grad_entropy"])
    torch.testing.assert_close(dmu, gb["d_mu"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(dk, gb["d_k"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("case", [(True, 1.0, 0.3, 1.7), (True, 0.7, -0.2, 0.8), (False, 1.0, 0.0, None),
                                  (False, 0.7, 0.4, None)])
def test_route_weights_grads_oracle_matches_reference_autograd(case):
    r, w, gb = load_golden("route.pt"), load_golden("weights.pt"), load_golden("weights_bwd.pt")
    affine, temp, off, scl = case
    got = obw.route_weights_grads(gb["scores"], gb["indices"], r["bias"], w["local_lse"], gb["grad_remote"],
                                  gb["grad_local"], affine=affine, temperature=temp,
                                  gate_scale=1.0 if scl is None else scl, gate_offset=off)
    want = gb["cases"][case]
    for i, name in enumerate(("d_scores", "d_prior", "d_local", "d_offset")):
        torch.testing.assert_close(got[4 if i == 3 else i], want[i], atol=1e-5, rtol=1e-4, msg=name)
    if affine:
        torch.testing.assert_close(got[3], want[4], atol=1e-4, rtol=1e-4)


def test_route_scores_grads_oracle_matches_reference_backward():
    r, gb = load_golden("route.pt"), load_golden("scores_bwd.pt")
    dq, dl = obw.route_scores_grads(r["q"], r["lmk"], r["indices"], gb["grad_scores"])
    torch.testing.assert_close(dq, gb["d_q"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(dl, gb["d_lmk"], atol=1e-5, rtol=1e-4)


@pytest.mark.gpu
def test_pool_backward_matches_reference_autograd(mrsa, cuda_device):
    """The kernel rounds p and the softmax gradient to bf16 (as the reference
    kernel does) and returns bf16; the golden is the fp32 autograd."""
    from mrsa_b200.chunk_pool import chunk_pool_backward

    g, gb = load_golden("pool.pt"), load_golden("pool_bwd.pt")
    dev = cuda_device
    d_mu, d_k = chunk_pool_backward(g["mu_q"].to(dev), g["k_chunked"].to(dev), g["key_valid"].to(dev),
                                    gb["grad_lmk"].to(dev), gb["grad_entropy"].to(dev))
    close_grad(d_mu, gb["d_mu"], "d_mu", rel_l2=2e-2, max_frac=3e-2)
    close_grad(d_k, gb["d_k"], "d_k", rel_l2=2e-2, max_frac=3e-2)


@pytest.mark.gpu
def test_pool_backward_dream_shape_and_autograd(mrsa, cuda_device):
    dev = cuda_device
    gen = torch.Generator().manual_seed(29)
    b, c, hkv, gg, d = 2, 24, 4, 7, 128
    mu = torch.randn(b, c, hkv, gg, d, generator=gen).bfloat16()
    k = (torch.randn(b, c, 64, hkv, d, generator=gen) / d ** 0.5).bfloat16()
    valid = torch.rand(b, c, 64, generator=gen) > 0.1
    valid[0, 5, :-1] = False                       # only the landmark valid -> zero gradients
    g_l = torch.randn(b, c, hkv, gg, d, generator=gen).bfloat16()
    g_e = torch.randn(b, c, hkv, gg, generator=gen)
    rmu, rk = obw.pool_grads(mu, k, valid, g_l, g_e)
    mud, kd = mu.to(dev).requires_grad_(), k.to(dev).requires_grad_()
    lmk, ent = mrsa.chunk_attn_pool_gqa(mud, kd, valid.to(dev))
    torch.autograd.backward((lmk, ent), (g_l.to(dev), g_e.to(dev)))
    close_grad(mud.grad, rmu, "d_mu", rel_l2=2e-2, max_frac=3e-2)
    close_grad(kd.grad, rk, "d_k", rel_l2=2e-2, max_frac=3e-2)
    assert (mud.grad[0, 5] == 0).all()
    # only the entropy gradient
    from mrsa_b200.chunk_pool import chunk_pool_backward

    # only the entropy gradient: ln(bf16(p)) (the reference kernel's rounding)
    # weighs more here than in the landmark gradient
    d_mu, d_k = chunk_pool_backward(mu.to(dev), k.to(dev), valid.to(dev), None, g_e.to(dev))
    emu, ek = obw.pool_grads(mu, k, valid, None, g_e)
    close_grad(d_mu, emu, "d_mu(entropy)", rel_l2=3e-2, max_frac=3e-2)
    close_grad(d_k, ek, "d_k(entropy)", rel_l2=3e-2, max_frac=3e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("case", [(True, 1.0, 0.3, 1.7), (True, 0.7, -0.2, 0.8), (False, 1.0, 0.0, None),
                                  (False, 0.7, 0.4, None)])
def test_route_weights_backward_matches_reference_autograd(mrsa, cuda_device, case):
    from mrsa_b200 import _lib
    from mrsa_b200.route_weights import route_weights_backward

    r, w, gb = load_golden("route.pt"), load_golden("weights.pt"), load_golden("weights_bwd.pt")
    affine, temp, off, scl = case
    dev = cuda_device
    got = route_weights_backward(gb["scores"].to(dev), gb["indices"].to(dev), r["bias"].to(dev),
                                 w["local_lse"].to(dev), gb["grad_remote"].to(dev), gb["grad_local"].to(dev),
                                 mode=_lib.WEIGHTS_AFFINE if affine else _lib.WEIGHTS_SOFTMAX, temperature=temp,
                                 gate_scale=1.0 if scl is None else scl, gate_offset=off)
    want = gb["cases"][case]
    torch.testing.assert_close(got[0].cpu(), want[0], atol=2e-5, rtol=1e-3)
    torch.testing.assert_close(got[1].cpu(), want[1], atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(got[2].cpu(), want[2], atol=2e-5, rtol=1e-3)
    torch.testing.assert_close(got[4].cpu(), want[3], atol=1e-3, rtol=1e-3)
    if affine:
        torch.testing.assert_close(got[3].cpu(), want[4], atol=1e-3, rtol=1e-3)


@pytest.mark.gpu
def test_route_weights_torch_autograd_with_empty_rows(mrsa, cuda_device):
    """The live affine gate under autograd: gradients reach scores, prior,
    local LSE and the gate parameters; rows without a selected chunk give
    finite (zero gate-scale) contributions."""
    dev = cuda_device
    gen = torch.Generator().manual_seed(31)
    b, l, hkv, gg, k, c = 1, 96, 4, 7, 32, 48
    idx = torch.stack([torch.randperm(c, generator=gen)[:k].sort().values for _ in range(b * l * hkv)])
    idx = idx.view(b, l, hkv, k).to(torch.int32)
    idx[0, 3] = -1
    idx[0, 4, :, 5:] = -1
    sc = torch.randn(b, l, hkv * gg, k, generator=gen).bfloat16()
    pb = torch.randn(b, c, hkv, gg, generator=gen)
    ll = torch.randn(b, l, hkv * gg, generator=gen)
    g_rw = torch.randn(b, l, hkv * gg, k, generator=gen).bfloat16()
    g_lw = torch.randn(b, l, hkv * gg, generator=gen).bfloat16()
    scd, pbd, lld = (t.to(dev).requires_grad_() for t in (sc, pb, ll))
    gs = torch.tensor(1.3, device=dev, requires_grad=True)
    go = torch.tensor(0.2, device=dev, requires_grad=True)
    rw, lw = mrsa.route_weights_torch(scd, idx.to(dev), pbd, lld, temperature=1.0, gate_offset=go, gate_scale=gs)
    torch.autograd.backward((rw, lw), (g_rw.to(dev), g_lw.to(dev)))
    want = obw.route_weights_grads(sc, idx, pb, ll, g_rw, g_lw, affine=True, temperature=1.0, gate_scale=1.3,
                                   gate_offset=0.2)
    close_grad(scd.grad, want[0], "d_scores")
    close_grad(pbd.grad, want[1], "d_prior", rel_l2=1e-3, max_frac=1e-3)
    close_grad(lld.grad, want[2], "d_local", rel_l2=1e-3, max_frac=1e-3)
    torch.testing.assert_close(gs.grad.cpu(), want[3], atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(go.grad.cpu(), want[4], atol=1e-3, rtol=1e-3)


@pytest.mark.gpu
def test_route_scores_backward_matches_reference_backward(mrsa, cuda_device):
    r, gb = load_golden("route.pt"), load_golden("scores_bwd.pt")
    dev = cuda_device
    d_q, d_l = mrsa.route_scores_backward(r["q"].to(dev), r["lmk"].to(dev), r["indices"].to(dev),
                                          gb["grad_scores"].to(dev))
    torch.testing.assert_close(d_q.cpu(), gb["d_q"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(d_l.cpu(), gb["d_lmk"], atol=1e-4, rtol=1e-4)


@pytest.mark.gpu
def test_routing_autograd_dream_shape(mrsa, cuda_device):
    """route_topk_g7 under autograd: the scores' gradients reach q and the
    landmarks through the B200 backward (indices carry none)."""
    dev = cuda_device
    gen = torch.Generator().manual_seed(37)
    b, l, hkv, gg, d, c, k = 1, 256, 4, 7, 128, 64, 32
    q = torch.randn(b, l, hkv * gg, d, generator=gen).bfloat16()
    lmk = torch.randn(b, c, hkv, gg, d, generator=gen).bfloat16()
    lse = torch.randn(b, l, hkv, gg, generator=gen)
    bias = torch.randn(b, c, hkv, gg, generator=gen)
    drop = torch.zeros(b, l, c, dtype=torch.int32)
    drop[:, :, :3] = 1
    qd, ld = q.to(dev).requires_grad_(), lmk.to(dev).requires_grad_()
    idx, sc = mrsa.route_topk_g7(qd, ld, lse.to(dev), bias.to(dev), drop.to(dev), k, 64, 256)
    g = torch.randn(sc.shape, generator=gen).bfloat16()
    g[torch.isinf(sc.float().cpu())] = 0
    sc.backward(g.to(dev))
    rq, rl = obw.route_scores_grads(q, lmk, idx.cpu(), g)
    close_grad(qd.grad, rq, "d_q")
    close_grad(ld.grad, rl, "d_lmk")


@pytest.mark.gpu
def test_fusion_and_rope_backward(mrsa, cuda_device):
    dev = cuda_device
    gen = torch.Generator().manual_seed(41)
    b, l, h, d = 2, 64, 28, 128
    rem, loc = (torch.randn(b, l, h, d, generator=gen).bfloat16() for _ in range(2))
    w = torch.rand(b, l, h, generator=gen).bfloat16()
    go = torch.randn(b, l, h, d, generator=gen).bfloat16()
    rd, ldv, wd = (t.to(dev).requires_grad_() for t in (rem, loc, w))
    out = mrsa.fuse_hils_outputs(rd, ldv, wd)
    out.backward(go.to(dev))
    e_r, e_l, e_w = obw.fuse_grads(loc, w, go)
    assert torch.equal(rd.grad.cpu(), e_r.bfloat16())
    assert torch.equal(ldv.grad.cpu(), e_l.bfloat16())
    torch.testing.assert_close(wd.grad.float().cpu(), e_w, atol=2e-2, rtol=8e-3)
    # single-tensor RoPE: the gradient is the same rotation with -sin
    from oracle import route_layer as orc

    x = torch.randn(b, l, 4, d, generator=gen).bfloat16()
    pos = orc.landmark_position_ids(b, l)
    inv, af = orc.yarn_inv_freq(d, 1.0e6, 8.0, 2048)
    cos, sin = orc.rope_cos_sin(pos, inv, af)
    xd = x.to(dev).requires_grad_()
    y = mrsa.single_tensor_rope_autograd(xd, cos.to(dev), sin.to(dev))
    gy = torch.randn(y.shape, generator=gen).bfloat16()
    y.backward(gy.to(dev))
    want = orc.apply_rope(gy, cos, -sin)
    torch.testing.assert_close(xd.grad.float().cpu(), want.float(), atol=1e-2, rtol=8e-3)


def test_local_grads_oracle_matches_a_dense_formulation():
    """The banded oracle's gradients (block-wise softmax with an LSE output)
    equal autograd of the dense [L, L] formulation."""
    g = torch.Generator().manual_seed(43)
    b, l, hkv, gg, d = 1, 256, 1, 3, 128
    q = torch.randn(b, l, hkv * gg, d, generator=g)
    k = torch.randn(b, l, hkv, d, generator=g) / d ** 0.5
    v = torch.randn(b, l, hkv, d, generator=g)
    valid = torch.ones(b, l, dtype=torch.bool)
    valid[0, 90:100] = False
    go = torch.randn(b, l, hkv * gg, d, generator=g)
    gl = torch.randn(b, l, hkv * gg, generator=g)
    for window, skip in ((40, True), (70, False)):
        got = obw.local_attention_grads(q, k, v, valid, window, 64, skip, go, gl)
        qf, kf, vf = (t.clone().requires_grad_() for t in (q, k, v))
        out, lse = obw.dense_local_attention(qf, kf, vf, valid, window, 64, skip)
        want = torch.autograd.grad((out, lse), (qf, kf, vf), (go, gl))
        for a, w_ in zip(got, want):
            torch.testing.assert_close(a, w_, atol=2e-5, rtol=1e-4)


def _local_case(b, l, hkv, g, seed):
    gen = torch.Generator().manual_seed(seed)
    q = (torch.randn(b, l, hkv * g, 128, generator=gen) / 2).bfloat16()
    k = (torch.randn(b, l, hkv, 128, generator=gen) / 2).bfloat16()
    v = torch.randn(b, l, hkv, 128, generator=gen).bfloat16()
    valid = torch.ones(b, l, dtype=torch.bool)
    valid[:, 150:190] = False
    valid[-1, l - 100:] = False
    go = torch.randn(b, l, hkv * g, 128, generator=gen).bfloat16()
    gl = torch.randn(b, l, hkv * g, generator=gen)
    return q, k, v, valid, go, gl


@pytest.mark.gpu
@pytest.mark.parametrize("b,l,hkv,g,window,skip", [
    (2, 1024, 2, 7, 256, True),       # the route layer's local branch (effective window 319)
    (1, 2048, 1, 7, 1280, False),     # an SWA layer
    (1, 512, 2, 8, 40, True),         # a full 8-head group, a short window
])
def test_local_window_backward_matches_oracle(mrsa, cuda_device, b, l, hkv, g, window, skip):
    dev = cuda_device
    q, k, v, valid, go, gl = _local_case(b, l, hkv, g, seed=l + window)
    eff = window + 63 if skip else window
    qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
    out, lse = mrsa.bidir_local_attention(qd, kd, vd, valid.to(dev), window, 64, skip_inert_slots=skip)
    torch.autograd.backward((out, lse), (go.to(dev), gl.to(dev)))
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0
    rq, rk, rv = obw.local_attention_grads(q, k, v, valid, window, 64, skip, go, gl)
    close_grad(qd.grad, rq, "dq")
    close_grad(kd.grad, rk, "dk")
    close_grad(vd.grad, rv, "dv")
    # zeroed keys get no gradient
    zero = ~valid
    if skip:
        zero = zero | ((torch.arange(l) + 1) % 64 == 0)[None]
    assert (kd.grad.cpu()[zero] == 0).all() and (vd.grad.cpu()[zero] == 0).all()
    # the direct call with the same inputs gives the same bits
    dq, dk, dv = mrsa.window_attention_backward(q.to(dev), k.to(dev), v.to(dev), valid.to(dev), out.detach(),
                                                lse.detach(), go.to(dev), gl.to(dev), window=eff, skip_inert=skip)
    assert torch.equal(dq.bfloat16(), qd.grad) and torch.equal(dk.bfloat16(), kd.grad)


def test_local_window_refuses_to_drop_a_gradient(mrsa):
    """Calls without a backward (cached rows, the causal flex window, output
    buffers) raise instead of returning a result that silently carries no
    gradient."""
    from mrsa_b200.local_attention import _no_backward

    x = torch.zeros(2, requires_grad=True)
    with pytest.raises(NotImplementedError):
        _no_backward(x, None)
    with torch.no_grad():
        _no_backward(x)
    _no_backward(torch.zeros(2))


@pytest.mark.gpu
def test_route_layer_training_step_matches_oracle_autograd(mrsa, cuda_device):
    """A whole route layer trained through the drop-ins -- RoPE, local window,
    Q-Cal (torch, as the reference module computes it), landmark pool,
    routing scores, affine-gate route weights, selected attention and fusion,
    each with its B200 backward -- against fp32 autograd of the oracle's
    composition on the kernel's own selection (routing indices carry no
    gradient).  Gradients of q, k, v, the hidden state and the Q-Cal weights
    within relative L2 5e-2 (bf16 roundings on every stage of the GPU side)."""
    from oracle import route_layer as orc

    dev = cuda_device
    cfg = orc.MRSAConfig()
    l, topk = 1024, 8
    inp = orc.make_route_layer_inputs(1, l, cfg, hidden=3584, seed=17)
    inp["key_valid"][0, 700:720] = False
    pos = orc.landmark_position_ids(1, l)
    inv, af = orc.yarn_inv_freq(128, cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
    cos, sin = orc.rope_cos_sin(pos, inv, af)
    valid = inp["key_valid"]
    gen = torch.Generator().manual_seed(5)
    gout = torch.randn(1, l, 28, 128, generator=gen)
    names = ("q_pre", "k_pre", "v", "hidden", "w_in", "w_out")

    # ---- GPU: the drop-ins under autograd
    leaves = {n: inp[n].to(dev).requires_grad_() for n in names}
    c, s = cos.to(dev), sin.to(dev)
    vd = valid.to(dev)
    q = mrsa.single_tensor_rope_autograd(leaves["q_pre"], c, s)
    k = mrsa.single_tensor_rope_autograd(leaves["k_pre"], c, s)
    lo, lse = mrsa.bidir_local_attention(q, k, leaves["v"], vd, cfg.local_window, 64, skip_inert_slots=True)
    t = (leaves["hidden"] @ leaves["w_in"].t())
    delta = (t @ leaves["w_out"].t()).view(1, l, 28, 128)
    comb = (mrsa.single_tensor_rope_autograd(q, c, -s).float() + delta.float()).bfloat16()
    cf = comb.float()
    normed = (cf * torch.rsqrt(cf.pow(2).mean(-1, keepdim=True) + cfg.rms_eps)).bfloat16()
    route_q = mrsa.single_tensor_rope_autograd(normed, c, s)
    n_chunks = l // 64
    mu = route_q[:, 63::64].reshape(1, n_chunks, 4, 7, 128)
    lmk, ent = mrsa.chunk_attn_pool_gqa(mu, k.view(1, n_chunks, 64, 4, 128), vd.view(1, n_chunks, 64))
    prior = ent * 1.0
    drop = mrsa.remote_drop_mask(vd, cfg.local_window, 64)
    idx, sc = mrsa.route_topk_g7(route_q, lmk, lse.view(1, l, 4, 7), prior, drop, topk, 64, cfg.local_window)
    rw, lw = mrsa.route_weights_torch(sc, idx, prior, lse, temperature=1.0, gate_offset=torch.tensor(0.3),
                                      gate_scale=torch.tensor(1.2))
    remote = mrsa.HiLS_block_M_head(q, k, leaves["v"], rw, idx, key_valid=vd)
    out = mrsa.fuse_hils_outputs(remote, lo, lw)
    (out.float() * gout.to(dev)).sum().backward()
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0

    # ---- CPU: the oracle's composition in fp32 on the same selection
    ref = {n: inp[n].float().requires_grad_() for n in names}
    rq = orc.apply_rope(ref["q_pre"], cos, sin)
    rk = orc.apply_rope(ref["k_pre"], cos, sin)
    rlo, rlse = orc.local_attention(rq, rk, ref["v"], valid, cfg.local_window, 64, True)
    rroute = orc.qcal_route_query(ref["hidden"], rq, ref["w_in"], ref["w_out"], torch.ones(128), cos, sin,
                                  eps=cfg.rms_eps)
    rmu = rroute[:, 63::64].reshape(1, n_chunks, 4, 7, 128)
    rlmk, rent = orc.chunk_pool(rmu, rk.view(1, n_chunks, 64, 4, 128), valid.view(1, n_chunks, 64))
    ridx = idx.long().cpu()
    rsc = orc.route_scores_at(rroute, rlmk, ridx)
    rrw, rlw = orc.route_weights_affine(rsc, ridx, rent, rlse, gate_offset=0.3, gate_scale=1.2)
    rremote = orc.selected_attention(rq, rk, ref["v"], rrw, ridx, valid, 64, out_dtype=torch.float32)
    rout = rremote + rlw[..., None] * rlo
    (rout * gout).sum().backward()
    for n in names:
        close_grad(leaves[n].grad, ref[n].grad, n, rel_l2=5e-2, max_frac=1.0)
