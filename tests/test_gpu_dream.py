"""GPU: the Dream-shaped forward (Qwen2 decoder layers around the B200
attention) against the CPU oracle, layer by layer with the GPU's own layer
inputs (teacher forcing, so an early rounding difference cannot grow), and
end to end on a small model.

Tolerances: a layer's update of the residual stream within mean-rel 2e-2 of
the oracle's (bf16 projections and MLP on both sides, rounded in a different
order; a near-tie routing flip moves a few rows), final logits with cosine
similarity above 0.999.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import route_layer as orc

pytestmark = pytest.mark.gpu


def _oracle_layer(model, idx, x, pos, valid):
    c, lay = model.cfg, model.layers[idx]
    cpu = {k: v.cpu() for k, v in lay.items() if torch.is_tensor(v)}
    cpu["wg"], cpu["wu"] = (w.cpu() for w in model.gate_up(idx))

    def norm(t, w):
        tf = t.float()
        tf = tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + c.rms_eps)
        return w * tf.to(t.dtype)

    b, l, _ = x.shape
    h = norm(x, cpu["in_norm"])
    q = F.linear(h, cpu["wq"], cpu["bq"]).view(b, l, c.q_heads, c.head_dim)
    k = F.linear(h, cpu["wk"], cpu["bk"]).view(b, l, c.kv_heads, c.head_dim)
    v = F.linear(h, cpu["wv"], cpu["bv"]).view(b, l, c.kv_heads, c.head_dim)
    ocfg = orc.MRSAConfig(q_heads=c.q_heads, kv_heads=c.kv_heads, head_dim=c.head_dim, chunk=c.chunk,
                          topk=c.topk, local_window=c.local_window, swa_window=c.swa_window)
    inp = {"hidden": h, "q_pre": q, "k_pre": k, "v": v, "position_ids": pos, "key_valid": valid}
    if "route" in lay:
        rl = lay["route"]
        inp.update(w_in=rl.w_in.cpu(), w_out=rl.w_out.cpu(), norm_weight=rl.norm_weight.cpu(),
                   entropy_bias_scale=rl.bias_scale.cpu(), gate_offset=0.0, gate_scale=1.0)
        o = orc.route_layer_forward(inp, ocfg, keep=False)["out"]
    else:
        o = orc.swa_layer_forward(inp, ocfg)["out"]
    x = x + F.linear(o.reshape(b, l, -1), cpu["wo"])
    h = norm(x, cpu["post_norm"])
    return x + F.linear(F.silu(F.linear(h, cpu["wg"])) * F.linear(h, cpu["wu"]), cpu["wd"])


def test_dream_forward_layers_match_oracle(mrsa, cuda_device):
    from mrsa_b200.dream_forward import DreamConfig, DreamForward, landmark_inputs

    cfg = DreamConfig(layers=4, hidden=896, ffn=1024, q_heads=7, kv_heads=1, vocab=512, swa_window=300)
    model = DreamForward(cfg, seed=3, device=cuda_device)
    ids, pos, _ = landmark_inputs(1, 1024, cfg, mask_id=cfg.vocab - 1, device=cuda_device)
    valid = torch.ones(1, 1024, dtype=torch.bool, device=cuda_device)
    logits, xs = model(ids, pos, valid, return_layer_inputs=True)
    assert logits.shape == (1, 1024, cfg.vocab) and torch.isfinite(logits).all()
    outs = xs[1:] + [None]
    for idx in range(cfg.layers):
        x_in = xs[idx].cpu()
        if outs[idx] is None:
            with torch.inference_mode():
                outs[idx] = model.layer(idx, xs[idx], pos, valid)
        got = outs[idx].cpu()
        ref = _oracle_layer(model, idx, x_in, pos.cpu(), valid.cpu())
        d_got, d_ref = (got.float() - x_in.float()), (ref.float() - x_in.float())
        rel = (d_got - d_ref).abs().mean() / d_ref.abs().mean()
        assert rel < 2e-2, (idx, float(rel))
    # the whole model once more, deterministic
    again = model(ids, pos, valid)
    assert torch.equal(again, logits)


def test_dream_forward_end_to_end_close_to_oracle(mrsa, cuda_device):
    from mrsa_b200.dream_forward import DreamConfig, DreamForward, landmark_inputs

    cfg = DreamConfig(layers=4, hidden=896, ffn=1024, q_heads=7, kv_heads=1, vocab=512, swa_window=300)
    model = DreamForward(cfg, seed=5, device=cuda_device)
    ids, pos, _ = landmark_inputs(1, 512, cfg, mask_id=cfg.vocab - 1, seed=2, device=cuda_device)
    valid = torch.ones(1, 512, dtype=torch.bool, device=cuda_device)
    logits = model(ids, pos, valid).float().cpu()
    lmk = (torch.arange(512) + 1) % cfg.chunk == 0
    x = model.embed.cpu()[ids.cpu()]
    x = torch.where(lmk[None, :, None], x + model.role.cpu(), x)
    for idx in range(cfg.layers):
        x = _oracle_layer(model, idx, x, pos.cpu(), valid.cpu())
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.rms_eps)
    ref = F.linear((model.final_norm.cpu() * xf.to(x.dtype)), model.lm_head.cpu()).float()
    cos = F.cosine_similarity(logits.flatten(), ref.flatten(), dim=0)
    assert cos > 0.999, float(cos)
