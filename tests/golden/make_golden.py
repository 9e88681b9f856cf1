"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (read-only) and
``transformers``::

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py

Each fixture stores seeded inputs (or the seed that regenerates them) and the
outputs of the reference's OWN functions, imported from the checkout:

* ``yarn.pt``      transformers ``ROPE_INIT_FUNCTIONS['yarn']`` (Dream's rotary)
* ``pool.pt``      ``ops/chunk_attn_pool_gqa_tilelang.py:17 _compact_pool_torch``
* ``drop.pt``      ``dream_dllm_hils/kernel_utils.py:102 remote_drop_mask``
* ``route.pt``     ``dream_dllm_hils/routing.py:52 route_topk_g7(training=False)``
* ``weights.pt``   ``dream_dllm_hils/attention.py:126 _route_weights_torch``
* ``selected.pt``  ``ops/hils_fwd_bwd_head.py:21 hils_torch_ref``
* ``selected_bwd.pt`` gradients of ``hils_torch_ref`` (torch autograd on fp32
  leaves): the quantities of the backward kernel ``:573-910``
* ``pool_bwd.pt``  gradients of ``_compact_pool_torch`` (autograd, fp32 leaves)
* ``weights_bwd.pt`` gradients of ``_route_weights_torch`` (autograd, fp32
  leaves; affine gate and the plain softmax branch)
* ``scores_bwd.pt`` ``ops/topk_head_softmax.py:1071 SoftmaxTopKMaxPoolingFusedFn.backward``
  run on the CPU (its torch scatter + bmm), per-query-head landmarks
* ``qcal.pt``      ``attention.py:41-63`` RoPE / inverse RoPE + ``qcal.py:22 rms_norm``
* ``local_mask.pt`` ``dream_dllm_hils/local_attention.py:35-64`` K/V masking + window
* ``layer.pt``     a whole route layer composed from the functions above (the
  flash-attn local branch, GPU-only in the reference, comes from the oracle)
* ``token_scores.pt`` ``dream_dllm_hils/token_refinement.py:10 candidate_token_scores_reference``
* ``dsa.pt``       ``dream_dllm_hils/dsa_attention.py:498 selected_token_attention_reference``
* ``flex.pt``      ``ops/flex_attn_tilelang.py:1355 _torch_ref_flex_attn`` (torch
  flex_attention with the reference's mask; its block mask is built on the CPU)
* ``local_window.pt`` ``dream_dllm_hils/local_attention.py:110 bidir_local_attention``
  run end to end, with its third-party ``flash_attn_func`` (GPU only) replaced by
  torch ``flex_attention`` under flash-attn's window rule ``|i - j| <= W``

The fixtures are consumed by ``tests/test_oracle_golden.py`` (CPU) and by the
GPU parity tests; nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import route_layer as orc  # noqa: E402


def _save(name, obj):
    path = os.path.join(HERE, name)
    torch.save(obj, path)
    print(f"wrote {name}: {os.path.getsize(path) / 1024:.1f} KiB")


def gen_yarn():
    from transformers import Qwen2Config
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    cfg = Qwen2Config(
        hidden_size=3584, num_attention_heads=28, num_key_value_heads=4,
        max_position_embeddings=16384, rope_theta=1.0e6,
        rope_scaling={"rope_type": "yarn", "factor": 8.0,
                      "original_max_position_embeddings": 2048},
    )
    inv_freq, af = ROPE_INIT_FUNCTIONS["yarn"](cfg, "cpu")
    _save("yarn.pt", {"inv_freq": inv_freq.float(), "attention_factor": float(af),
                      "dim": 128, "base": 1.0e6, "factor": 8.0, "orig": 2048})


def gen_pool():
    from ops.chunk_attn_pool_gqa_tilelang import _compact_pool_torch

    g = torch.Generator().manual_seed(11)
    b, c, s, hkv, gg, d = 1, 6, 64, 2, 7, 128
    mu = (torch.randn(b, c, hkv, gg, d, generator=g)).bfloat16()
    k = (torch.randn(b, c, s, hkv, d, generator=g) / math.sqrt(d)).bfloat16()
    valid = torch.ones(b, c, s, dtype=torch.bool)
    valid[:, 1, ::5] = False          # ragged validity
    valid[:, 3, :-1] = False          # chunk with only its landmark valid -> zeros
    valid[:, 4, 0] = False            # first slot invalid
    lmk, ent = _compact_pool_torch(mu, k, valid, 1.0 / math.sqrt(d))
    _save("pool.pt", {"mu_q": mu, "k_chunked": k, "key_valid": valid, "lmk": lmk, "entropy": ent})


def gen_drop():
    from dream_dllm_hils.kernel_utils import remote_drop_mask

    b, l = 2, 1024
    valid = torch.ones(b, l, dtype=torch.bool)
    valid[0, 128:191] = False          # chunk 2 of batch 0: only its landmark stays valid
    valid[1, 640:] = False             # ragged tail in batch 1
    out = {}
    for w in (0, 63, 64, 256, 1280):
        out[w] = remote_drop_mask(valid, w, 64).bool()
    _save("drop.pt", {"key_valid": valid, "masks": out})


def gen_route():
    from dream_dllm_hils.routing import route_topk_g7

    g = torch.Generator().manual_seed(74)
    b, l, c, hkv, gg, d, topk = 1, 300, 40, 1, 7, 128, 32
    q = torch.randn(b, l, hkv * gg, d, generator=g).bfloat16()
    lmk = torch.randn(b, c, hkv, gg, d, generator=g).bfloat16()
    lse = torch.randn(b, l, hkv, gg, generator=g)
    bias = torch.randn(b, c, hkv, gg, generator=g)
    drop = torch.zeros(b, l, c, dtype=torch.int32)
    drop[:, ::11, 3] = 1
    drop[:, 7, :20] = 1               # 20 available chunks -> 12 slots of -1
    drop[:, 9, :] = 1                 # nothing routable
    idx, sc = route_topk_g7(q, lmk, lse, bias, drop, topk, 64, 512, training=False)
    _save("route.pt", {"q": q, "lmk": lmk, "local_lse": lse, "bias": bias, "drop": drop,
                       "topk": topk, "indices": idx, "scores": sc})


def gen_weights():
    from dream_dllm_hils.attention import _route_weights_torch

    r = torch.load(os.path.join(HERE, "route.pt"))
    b, l, hq, k = r["scores"].shape
    g = torch.Generator().manual_seed(5)
    local_lse = torch.randn(b, l, hq, generator=g)
    outs = {}
    for off, sc in ((0.0, 1.0), (0.3, 1.7)):
        rw, lw = _route_weights_torch(
            r["scores"], r["indices"], r["bias"].contiguous(), local_lse, temperature=1.0,
            gate_offset=torch.tensor(off), gate_scale=torch.tensor(sc))
        outs[(off, sc)] = (rw, lw)
    _save("weights.pt", {"local_lse": local_lse, "outs": outs})


def gen_selected():
    from ops.hils_fwd_bwd_head import hils_torch_ref

    g = torch.Generator().manual_seed(79)
    b, lq, lk, hkv, gg, d, topk, s = 1, 48, 1024, 1, 7, 128, 8, 64
    q = torch.randn(b, lq, hkv * gg, d, generator=g).bfloat16()
    k = torch.randn(b, lk, hkv, d, generator=g).bfloat16()
    v = torch.randn(b, lk, hkv, d, generator=g).bfloat16()
    c = lk // s
    idx = torch.stack([torch.randperm(c, generator=g)[:topk].sort().values for _ in range(lq)])
    idx = idx.view(b, lq, hkv, topk).to(torch.int32)
    idx[:, 5, :, 5:] = -1
    idx[:, 6] = -1
    w = torch.softmax(torch.randn(b, lq, hkv * gg, topk, generator=g), -1).bfloat16()
    out = hils_torch_ref(q, k, v, w, idx, chunk_size=s, sm_scale=d ** -0.5, block_q=1)
    _save("selected.pt", {"q": q, "k": k, "v": v, "weights": w, "indices": idx, "out": out})


def gen_selected_bwd():
    from ops.hils_fwd_bwd_head import hils_torch_ref

    r = torch.load(os.path.join(HERE, "selected.pt"))
    g = torch.Generator().manual_seed(83)
    q, k, v, w = (r[n].float().requires_grad_() for n in ("q", "k", "v", "weights"))
    d = q.shape[-1]
    out = hils_torch_ref(q, k, v, w, r["indices"], chunk_size=64, sm_scale=d ** -0.5, block_q=1)
    grad_out = torch.randn(out.shape, generator=g).bfloat16()
    dq, dk, dv, dw = torch.autograd.grad(out, (q, k, v, w), grad_out.float())
    _save("selected_bwd.pt", {"grad_out": grad_out, "dq": dq, "dk": dk, "dv": dv, "dw": dw})


def gen_pool_bwd():
    from ops.chunk_attn_pool_gqa_tilelang import _compact_pool_torch

    r = torch.load(os.path.join(HERE, "pool.pt"))
    g = torch.Generator().manual_seed(17)
    mu = r["mu_q"].float().requires_grad_()
    k = r["k_chunked"].float().requires_grad_()
    lmk, ent = _compact_pool_torch(mu, k, r["key_valid"], 1.0 / math.sqrt(mu.shape[-1]))
    g_lmk = torch.randn(lmk.shape, generator=g).bfloat16()
    g_ent = torch.randn(ent.shape, generator=g)
    d_mu, d_k = torch.autograd.grad((lmk, ent), (mu, k), (g_lmk.float(), g_ent))
    _save("pool_bwd.pt", {"grad_lmk": g_lmk, "grad_entropy": g_ent, "d_mu": d_mu, "d_k": d_k})


def gen_weights_bwd():
    from dream_dllm_hils.attention import _route_weights_torch

    r = torch.load(os.path.join(HERE, "route.pt"))
    w = torch.load(os.path.join(HERE, "weights.pt"))
    idx = r["indices"].clone()
    scores = r["scores"].clone()
    # every row keeps at least one selected chunk with a finite score (autograd
    # of the affine gate is NaN for gate_scale on a row without one)
    empty = idx[..., 0] < 0
    idx[..., 0] = idx[..., 0].clamp_min(0)
    scores[..., 0] = torch.where(empty.repeat_interleave(scores.shape[2] // idx.shape[2], dim=2),
                                 torch.zeros((), dtype=scores.dtype), scores[..., 0])
    g = torch.Generator().manual_seed(19)
    b, l, hq, k = scores.shape
    g_rw = torch.randn(b, l, hq, k, generator=g).bfloat16()
    g_lw = torch.randn(b, l, hq, generator=g).bfloat16()
    out = {"indices": idx, "scores": scores, "grad_remote": g_rw, "grad_local": g_lw, "cases": {}}
    for affine, temp, off, scl in ((True, 1.0, 0.3, 1.7), (True, 0.7, -0.2, 0.8), (False, 1.0, 0.0, None),
                                   (False, 0.7, 0.4, None)):
        sc = scores.float().requires_grad_()
        pb = r["bias"].float().contiguous().requires_grad_()
        ll = w["local_lse"].float().requires_grad_()
        go = torch.tensor(off, requires_grad=True)
        gs = torch.tensor(scl, requires_grad=True) if affine else None
        rw, lw = _route_weights_torch(sc, idx, pb, ll, temperature=temp, gate_offset=go, gate_scale=gs)
        loss = (rw * g_rw.float()).sum() + (lw * g_lw.float()).sum()
        leaves = (sc, pb, ll, go) + ((gs,) if affine else ())
        grads = torch.autograd.grad(loss, leaves)
        out["cases"][(affine, temp, off, scl)] = grads
    _save("weights_bwd.pt", out)


def gen_scores_bwd():
    from ops.topk_head_softmax import SoftmaxTopKMaxPoolingFusedFn

    r = torch.load(os.path.join(HERE, "route.pt"))
    b, l, hq, d = r["q"].shape
    _, c, hkv, gg, _ = r["lmk"].shape
    g = torch.Generator().manual_seed(23)
    grad = torch.randn(b, l, hq, r["topk"], generator=g).bfloat16()

    class Ctx:
        pass

    ctx = Ctx()
    ctx.saved_tensors = (r["q"].float().view(b, l, hkv, gg, d), r["lmk"].float().reshape(b, c, hq, d),
                         r["indices"].to(torch.int32))
    ctx.h_kv, ctx.G, ctx.shapes, ctx.sm_scale, ctx.per_qhead_lmks = hkv, gg, (b, l, c, hkv, d), None, True
    res = SoftmaxTopKMaxPoolingFusedFn.backward(ctx, None, grad.float().view(b, l, hkv, gg, -1))
    _save("scores_bwd.pt", {"grad_scores": grad, "d_q": res[0].reshape(b, l, hq, d),
                            "d_lmk": res[1].reshape(b, c, hkv, gg, d)})


def gen_qcal():
    from dream_dllm_hils.attention import apply_rotary_pos_emb, invert_rotary_pos_emb
    from dream_dllm_hils.qcal import rms_norm

    yarn = torch.load(os.path.join(HERE, "yarn.pt"))
    g = torch.Generator().manual_seed(3)
    b, l, hq, d = 1, 128, 4, 128
    pos = orc.landmark_position_ids(b, l)
    cos, sin = orc.rope_cos_sin(pos, yarn["inv_freq"], yarn["attention_factor"], torch.bfloat16)
    q = (torch.randn(b, l, hq, d, generator=g) / math.sqrt(d)).bfloat16()
    delta = (torch.randn(b, l, hq, d, generator=g) * 0.05).bfloat16()
    q_roped, _ = apply_rotary_pos_emb(q.transpose(1, 2), q.transpose(1, 2), cos, sin)
    q_roped = q_roped.transpose(1, 2).contiguous()
    unrot = invert_rotary_pos_emb(q_roped.transpose(1, 2), cos, sin).transpose(1, 2)
    comb = rms_norm(unrot + delta, torch.ones(d), 1e-6)
    rq, _ = apply_rotary_pos_emb(comb.transpose(1, 2), comb.transpose(1, 2), cos, sin)
    _save("qcal.pt", {"q": q, "delta": delta, "position_ids": pos, "cos": cos, "sin": sin,
                      "q_roped": q_roped, "unrot": unrot.contiguous(),
                      "route_q": rq.transpose(1, 2).contiguous()})


def gen_local_mask():
    from dream_dllm_hils.local_attention import _apply_key_valid, _flash_window, _window_key_valid

    g = torch.Generator().manual_seed(9)
    b, l, hkv, d = 1, 256, 1, 8
    k = torch.randn(b, l, hkv, d, generator=g).bfloat16()
    v = torch.randn(b, l, hkv, d, generator=g).bfloat16()
    valid = torch.ones(b, l, dtype=torch.bool)
    valid[:, 100:110] = False
    out = {}
    for skip in (False, True):
        vmask = _window_key_valid(valid, chunk_size=64, skip_inert_slots=skip)
        mk, mv = _apply_key_valid(k, v, vmask)
        out[skip] = {"valid": vmask, "k": mk, "v": mv, "window": _flash_window(256, skip, 64)}
    _save("local_mask.pt", {"k": k, "v": v, "key_valid": valid, "out": out})


def gen_layer():
    """Whole route layer, composed from the reference's functions in the order
    of ``attention.py:1358-1774`` (bf16 RoPE chain of the live path)."""
    from dream_dllm_hils.attention import (
        _route_weights_torch, apply_rotary_pos_emb, invert_rotary_pos_emb)
    from dream_dllm_hils.kernel_utils import remote_drop_mask
    from dream_dllm_hils.qcal import rms_norm
    from dream_dllm_hils.routing import route_topk_g7
    from ops.chunk_attn_pool_gqa_tilelang import _compact_pool_torch
    from ops.hils_fwd_bwd_head import hils_torch_ref

    cfg = orc.MRSAConfig(q_heads=7, kv_heads=1, rope_precision="bf16")
    b, l, hidden, seed = 1, 1024, 512, 1234
    inp = orc.make_route_layer_inputs(b, l, cfg, hidden=hidden, seed=seed)
    yarn = torch.load(os.path.join(HERE, "yarn.pt"))
    cos, sin = orc.rope_cos_sin(inp["position_ids"], yarn["inv_freq"], yarn["attention_factor"],
                                torch.bfloat16)
    qt, kt = apply_rotary_pos_emb(inp["q_pre"].transpose(1, 2), inp["k_pre"].transpose(1, 2), cos, sin)
    q, k, v = qt.transpose(1, 2).contiguous(), kt.transpose(1, 2).contiguous(), inp["v"]
    hq, hkv, d, chunk = 7, 1, 128, 64
    c = l // chunk
    valid = inp["key_valid"]
    local_o, local_lse = orc.local_attention(q, k, v, valid, 256, chunk, True)
    # Q-Cal (attention.py:458-503)
    t = torch.nn.functional.linear(inp["hidden"], inp["w_in"])
    delta = torch.nn.functional.linear(t, inp["w_out"]).view(b, l, hq, d)
    unrot = invert_rotary_pos_emb(q.transpose(1, 2), cos, sin).transpose(1, 2)
    comb = rms_norm(unrot + delta, inp["norm_weight"], 1e-6)
    rqt, _ = apply_rotary_pos_emb(comb.transpose(1, 2), comb.transpose(1, 2), cos, sin)
    route_q = rqt.transpose(1, 2).contiguous()
    mu = route_q[:, chunk - 1::chunk].reshape(b, c, hkv, 7, d)
    lmk, ent = _compact_pool_torch(mu, k.reshape(b, c, chunk, hkv, d), valid.reshape(b, c, chunk),
                                   1.0 / math.sqrt(d))
    prior = ent * inp["entropy_bias_scale"].view(1, 1, hkv, 7)
    drop = remote_drop_mask(valid, 256, chunk)
    idx, sc = route_topk_g7(route_q, lmk, local_lse.reshape(b, l, hkv, 7), prior.contiguous(), drop,
                            32, chunk, 256, training=False)
    rw, lw = _route_weights_torch(sc, idx, prior.contiguous(), local_lse.float().contiguous(),
                                  temperature=1.0, gate_offset=torch.tensor(0.0),
                                  gate_scale=torch.tensor(1.0))
    remote = hils_torch_ref(q, k, v, rw, idx.to(torch.int32), chunk_size=chunk,
                            sm_scale=d ** -0.5, block_q=1).to(torch.bfloat16)
    out = (remote.float() + lw.float()[..., None] * local_o.float()).to(torch.bfloat16)
    rows = torch.arange(7, l, 8)      # every 8th row, landmark rows (63 mod 64) included
    _save("layer.pt", {"seed": seed, "batch": b, "seq_len": l, "hidden": hidden,
                       "q_heads": hq, "kv_heads": hkv, "rows": rows, "q": q[:, rows],
                       "k": k[:, rows], "route_q": route_q[:, rows],
                       "lmk": lmk, "entropy": ent, "indices": idx, "scores": sc,
                       "remote_weights": rw, "local_weight": lw, "local_lse": local_lse,
                       "out": out})


def gen_token_scores():
    from dream_dllm_hils.token_refinement import candidate_token_scores_reference

    g = torch.Generator().manual_seed(41)
    b, lq, lk, hkv, gg, d, sel, s = 1, 12, 512, 2, 7, 32, 5, 64
    q = torch.randn(b, lq, hkv * gg, d, generator=g).bfloat16()
    k = torch.randn(b, lk, hkv, d, generator=g).bfloat16()
    c = lk // s
    idx = torch.randint(0, c, (b, lq, hkv, sel), generator=g).to(torch.int32)
    idx[:, 3, 1, 2] = -1
    idx[:, 4, 0] = -1
    valid = torch.ones(b, lk, dtype=torch.bool)
    valid[:, 70:90] = False
    out = candidate_token_scores_reference(q, k, idx, valid, s)
    _save("token_scores.pt", {"q": q, "k": k, "indices": idx, "key_valid": valid, "chunk": s,
                              "out": out})


def gen_dsa():
    from dream_dllm_hils.dsa_attention import selected_token_attention_reference

    g = torch.Generator().manual_seed(23)
    b, lq, lk, hkv, gg, d, topk = 1, 9, 256, 2, 7, 32, 101
    q = torch.randn(b, lq, hkv * gg, d, generator=g).bfloat16()
    k = torch.randn(b, lk, hkv, d, generator=g).bfloat16()
    v = torch.randn(b, lk, hkv, d, generator=g).bfloat16()
    idx = torch.randint(-3, lk + 3, (b, lq, topk), generator=g)
    valid = torch.rand(b, lq, topk, generator=g) > 0.2
    valid[:, 0] = False
    out = selected_token_attention_reference(q, k, v, idx, valid)
    _save("dsa.pt", {"q": q, "k": k, "v": v, "indices": idx, "valid": valid, "out": out})


FLEX_CASES = [
    # (name, q_len, kv_len, window, chunk, mask_lmk, expand_to_chunk)
    ("lmk_expand", 192, 192, 48, 32, True, True),
    ("no_flags", 192, 192, 48, 32, False, False),
    ("lmk_only", 192, 192, 48, 32, True, False),
    ("expand_only", 192, 192, 48, 32, False, True),
    ("prefill_part", 40, 192, 48, 32, True, True),
    ("decode_q1", 1, 192, 100, 32, True, False),
    ("chunk65", 150, 150, 100, 65, True, True),
    ("window_ge_seq", 64, 64, 512, 32, True, True),
]


def gen_flex():
    import functools

    import torch.nn.attention.flex_attention as fa
    from ops.flex_attn_tilelang import _torch_ref_flex_attn

    # the reference builds its block mask on the default CUDA device; build it on the CPU
    orig = fa.create_block_mask
    fa.create_block_mask = functools.partial(orig, device="cpu")
    try:
        cases = []
        for i, (name, lq, lk, w, c, lmk, exp) in enumerate(FLEX_CASES):
            g = torch.Generator().manual_seed(100 + i)
            hq, hkv, d = 4, 2, 32
            q = (torch.randn(1, lq, hq, d, generator=g) * 0.5).bfloat16()
            k = (torch.randn(1, lk, hkv, d, generator=g) * 0.5).bfloat16()
            v = (torch.randn(1, lk, hkv, d, generator=g) * 0.5).bfloat16()
            o, lse = _torch_ref_flex_attn(q.float(), k.float(), v.float(), w, c, lmk, exp)
            cases.append({"name": name, "window": w, "chunk": c, "mask_lmk": lmk, "expand": exp,
                          "q": q, "k": k, "v": v, "o": o.transpose(1, 2).contiguous(),
                          "lse": lse.transpose(1, 2).contiguous()})
    finally:
        fa.create_block_mask = orig
    _save("flex.pt", {"cases": cases})


def _cpu_flash_attn_module():
    """A stand-in ``flash_attn`` module for the CPU: ``flash_attn_func`` with
    flash-attn's non-causal sliding window (keys j with |i - j| <= W) and its
    return convention (out [B,L,H,D], lse [B,H,L]), computed by torch's
    ``flex_attention``."""
    import functools
    import types

    import torch.nn.attention.flex_attention as fa

    def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                        return_softmax_lse=False):
        assert dropout_p == 0.0 and not causal
        wl, wr = window_size
        lq, lk = q.shape[1], k.shape[1]

        def mask_mod(b, h, qi, kj):
            return (kj >= qi - wl) & (kj <= qi + wr)

        bm = fa.create_block_mask(mask_mod, B=None, H=None, Q_LEN=lq, KV_LEN=lk, device="cpu")
        o, lse = fa.flex_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(), v.transpose(1, 2).float(),
                                   block_mask=bm, scale=softmax_scale, enable_gqa=True, return_lse=True)
        return o.transpose(1, 2).to(q.dtype), lse

    mod = types.ModuleType("flash_attn")
    mod.flash_attn_func = flash_attn_func
    _ = functools
    return mod


def gen_local_window():
    import dream_dllm_hils.local_attention as la

    saved = sys.modules.get("flash_attn")
    sys.modules["flash_attn"] = _cpu_flash_attn_module()
    # the reference's layout check demands CUDA tensors (local_attention.py:15-17);
    # the rest of bidir_local_attention runs unchanged on the CPU
    check = la._validate_layout
    la._validate_layout = lambda *args: None
    bidir_local_attention = la.bidir_local_attention
    try:
        cases = []
        for i, (l, w, skip) in enumerate([(256, 40, True), (256, 40, False), (320, 100, True)]):
            g = torch.Generator().manual_seed(200 + i)
            hq, hkv, d = 4, 2, 32
            q = torch.randn(1, l, hq, d, generator=g).bfloat16()
            k = torch.randn(1, l, hkv, d, generator=g).bfloat16()
            v = torch.randn(1, l, hkv, d, generator=g).bfloat16()
            valid = torch.rand(1, l, generator=g) > 0.1
            o, lse = bidir_local_attention(q, k, v, valid, w, 64, skip_inert_slots=skip)
            cases.append({"q": q, "k": k, "v": v, "key_valid": valid, "window": w, "skip": skip,
                          "o": o, "lse": lse})
        # the Fast-dLLM cached rows (local_attention.py:147-197) on the same helpers
        g = torch.Generator().manual_seed(300)
        l, hq, hkv, d = 256, 4, 2, 32
        pos = torch.tensor([130, 3, 255, 64, 63, 200, 201, 17])
        q = torch.randn(1, pos.numel(), hq, d, generator=g).bfloat16()
        k = torch.randn(1, l, hkv, d, generator=g).bfloat16()
        v = torch.randn(1, l, hkv, d, generator=g).bfloat16()
        valid = torch.rand(1, l, generator=g) > 0.1
        cached = []
        for w, skip in [(40, True), (100, False)]:
            o, lse = la.cached_local_attention(q, k, v, valid, pos, w, 64, skip_inert_slots=skip)
            cached.append({"window": w, "skip": skip, "o": o, "lse": lse})
    finally:
        la._validate_layout = check
        if saved is None:
            sys.modules.pop("flash_attn", None)
        else:
            sys.modules["flash_attn"] = saved
    _save("local_window.pt", {"cases": cases, "cached": {"q": q, "k": k, "v": v, "key_valid": valid,
                                                          "positions": pos, "runs": cached}})


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gen_yarn()
    gen_pool()
    gen_drop()
    gen_route()
    gen_weights()
    gen_selected()
    gen_selected_bwd()
    gen_pool_bwd()
    gen_weights_bwd()
    gen_scores_bwd()
    gen_qcal()
    gen_local_mask()
    gen_layer()
    gen_token_scores()
    gen_dsa()
    gen_flex()
    gen_local_window()
    print("done")
