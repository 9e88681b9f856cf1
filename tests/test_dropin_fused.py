"""The fused replacement of ``KernelDreamFullHiLSAttention.forward``
(``dropin._fused_forward``) on a stand-in module that carries the reference
module's attribute names (``dream_dllm_hils/attention.py:906-920, 1313-1820``).

CPU: every configuration the fused layer does not reproduce goes to the
reference forward.  GPU: the fused path equals the oracle route layer over
the module's own projections, Q-Cal weights, RMSNorm eps, entropy-bias scale,
fusion gate and rotary embedding (non-default values for each).
"""

import pytest
import torch

from oracle import route_layer as orc

REFERENCE = "reference forward"


class RMSNormStandIn(torch.nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim))
        self.eps = eps


class RotaryStandIn(torch.nn.Module):
    """The attributes the fused layer reads from an HF rotary module."""

    def __init__(self, cfg):
        super().__init__()
        inv, af = orc.yarn_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.yarn_factor, cfg.yarn_orig_max_pos)
        self.register_buffer("inv_freq", inv)
        self.attention_scaling = af


class RouteAttentionStandIn(torch.nn.Module):
    """Attribute names of ``KernelDreamFullHiLSAttention`` (eval defaults)."""

    def __init__(self, hidden=3584, seed=0, eps=1e-5, qcal_scale=0.5):
        super().__init__()
        cfg = orc.MRSAConfig()
        g = torch.Generator().manual_seed(seed)
        self.num_heads, self.num_key_value_heads, self.head_dim = 28, 4, 128
        self.num_key_value_groups = 7
        self.hidden_size = 28 * 128
        self.chunk_size, self.topk, self.local_window = 64, 32, 256
        self.route_temperature = 1.0
        self.qcal_scale = qcal_scale

        def lin(i, o, bias):
            m = torch.nn.Linear(i, o, bias=bias)
            with torch.no_grad():
                m.weight.copy_(torch.randn(o, i, generator=g) * 0.02)
                if bias:
                    m.bias.copy_(torch.randn(o, generator=g) * 0.02)
            return m

        self.q_proj = lin(hidden, 28 * 128, True)
        self.k_proj = lin(hidden, 4 * 128, True)
        self.v_proj = lin(hidden, 4 * 128, True)
        self.o_proj = lin(28 * 128, hidden, False)
        self.qcal = torch.nn.Sequential(lin(hidden, 64, False), lin(64, 28 * 128, False))
        self.qcal_norm = RMSNormStandIn(128, eps)
        with torch.no_grad():
            self.qcal_norm.weight.copy_(1 + 0.1 * torch.randn(128, generator=g))
        self.entropy_bias_scale = torch.nn.Parameter(0.5 + torch.rand(28, generator=g))
        self.fusion_gate_offset = torch.nn.Parameter(torch.tensor(0.3))
        self.fusion_gate_scale = torch.nn.Parameter(torch.tensor(1.2))
        self.rotary_emb = RotaryStandIn(cfg)
        self.skip_inert_slots = True
        self.chunk_summary = "attn"
        self.entropy_prior = True
        self.route_query_positions = None
        self.force_remote_query_mask = None
        self.token_budget = 0

    def _key_valid_mask(self, attention_mask, bsz, seq_len, device):
        # attention.py:615-627 for the masks the fused path accepts
        if attention_mask is None:
            return torch.ones((bsz, seq_len), dtype=torch.bool, device=device)
        return attention_mask.to(device=device).bool()

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None,
                output_attentions=False, use_cache=False, cache_position=None, position_embeddings=None,
                **kwargs):
        return REFERENCE


class FakeHidden:
    """Stands for BF16 CUDA hidden states in the host-side checks."""

    def __init__(self, shape):
        self.shape = shape
        self.device = torch.device("cuda", 0)
        self.dtype = torch.bfloat16


@pytest.fixture
def fused_cls(mrsa):
    from mrsa_b200 import dropin

    class Fused(RouteAttentionStandIn):
        pass

    dropin.install_fused_forward(Fused)
    return Fused


def test_unsupported_calls_go_to_the_reference_forward(mrsa, fused_cls):
    from mrsa_b200 import dropin

    m = fused_cls(hidden=256).eval()
    h = FakeHidden((1, 1024, 256))
    pos = torch.arange(1024)[None]
    assert dropin.fused_unsupported(m, h, None, pos) == "gradient requested (the fused layer is forward-only)"
    with torch.no_grad():
        assert dropin.fused_unsupported(m, h, None, pos) is None
    mask4 = torch.ones(1, 1, 1024, 1024, dtype=torch.bool)
    cases = {
        "4-D allowed mask": dict(attention_mask=mask4),
        "explicit position_embeddings": dict(position_embeddings=(torch.ones(1), torch.ones(1))),
        "KV cache requested": dict(use_cache=True),
        "no position_ids": dict(position_ids=None),
    }
    for p in m.parameters():
        p.requires_grad_(False)
    for why, kw in cases.items():
        args = dict(attention_mask=None, position_ids=pos)
        args.update(kw)
        assert dropin.fused_unsupported(m, h, **args).startswith(why)
    for attr, value, why in [("skip_inert_slots", False, "skip_inert_slots=False"),
                             ("chunk_summary", "mean", "chunk_summary != 'attn'"),
                             ("entropy_prior", False, "entropy_prior=False"),
                             ("token_budget", 128, "token refinement"),
                             ("qcal_norm", None, "Q-Cal without RMSNorm"),
                             ("route_query_positions", torch.tensor([3]), "route_query_positions"),
                             ("_prefill_capture", True, "prefill cache capture")]:
        m2 = fused_cls(hidden=256).eval().requires_grad_(False)
        setattr(m2, attr, value)
        assert dropin.fused_unsupported(m2, h, None, pos) == why, attr
    m.train()
    assert dropin.fused_unsupported(m, h, None, pos) == "training forward"
    # a real call that is not on a CUDA device reaches the reference forward
    m.eval()
    assert m(torch.zeros(1, 64, 256), None, pos[:, :64]) == REFERENCE
    assert dropin.fused_unsupported(m, torch.zeros(1, 64, 256), None, pos[:, :64]) is not None


def test_install_keeps_and_restores_the_reference_forward(mrsa):
    from mrsa_b200 import dropin

    class Fused(RouteAttentionStandIn):
        pass

    orig = Fused.forward
    dropin.install_fused_forward(Fused)
    dropin.install_fused_forward(Fused)          # idempotent
    assert Fused.forward is dropin._fused_forward
    assert Fused._mrsa_b200_reference_forward is orig


@pytest.mark.gpu
def test_fused_forward_matches_the_oracle_layer(mrsa, fused_cls, cuda_device):
    dev, l = cuda_device, 2048
    cfg = orc.MRSAConfig(rms_eps=1e-5, qcal_scale=0.5)
    m = fused_cls(hidden=3584, seed=4, eps=cfg.rms_eps, qcal_scale=cfg.qcal_scale).eval()
    m = m.to(device=dev, dtype=torch.bfloat16)
    # the rotary module keeps fp32 frequencies (as HF rotary modules compute in fp32)
    m.rotary_emb.inv_freq = orc.yarn_inv_freq(128, cfg.rope_theta, cfg.yarn_factor,
                                              cfg.yarn_orig_max_pos)[0].to(dev)
    g = torch.Generator().manual_seed(8)
    h = torch.randn(1, l, 3584, generator=g).bfloat16().to(dev)
    mask = torch.ones(1, l, dtype=torch.bool)
    mask[0, 1500:1530] = False
    pos = orc.landmark_position_ids(1, l).to(dev)
    seen = {}
    hook = m.o_proj.register_forward_pre_hook(lambda mod, args: seen.update(attn=args[0].detach().clone()))
    try:
        with torch.no_grad():
            out, _, _ = m(h, mask.to(dev), pos)
    finally:
        hook.remove()
    assert out.shape == (1, l, 3584)
    attn = seen["attn"].view(1, l, 28, 128)
    with torch.no_grad():
        q = m.q_proj(h).view(1, l, 28, 128)
        k = m.k_proj(h).view(1, l, 4, 128)
        v = m.v_proj(h).view(1, l, 4, 128)
    layer = m._mrsa_b200_layer
    st = layer.forward(q.contiguous(), k.contiguous(), v.contiguous(), h, pos, mask.to(dev), stages=True)
    assert torch.equal(st["out"], attn), "fused forward differs from its staged layer"
    inp = {"q_pre": q.cpu(), "k_pre": k.cpu(), "v": v.cpu(), "hidden": h.cpu(),
           "w_in": m.qcal[0].weight.detach().cpu(), "w_out": m.qcal[1].weight.detach().cpu(),
           "norm_weight": m.qcal_norm.weight.detach().float().cpu(),
           "entropy_bias_scale": m.entropy_bias_scale.detach().float().cpu(),
           "gate_offset": float(m.fusion_gate_offset), "gate_scale": float(m.fusion_gate_scale),
           "position_ids": pos.cpu(), "key_valid": mask}
    sl = slice(1024, 1280)
    ref = orc.route_layer_forward(inp, cfg, query_slice=sl)
    viol, exact = orc.topk_set_agreement(ref["route_key"], st["indices"][:, sl].cpu(), ref["indices"], 32)
    assert viol == 0 and exact >= 0.9, (viol, exact)
    own = orc.route_layer_forward(inp, cfg, query_slice=sl, indices=st["indices"][:, sl].cpu())
    got, want = attn[:, sl].float().cpu(), own["out"].float()
    d = (got - want).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() / want.abs().mean().item() <= 1e-3
    # o_proj of the fused path is the module's own
    with torch.no_grad():
        torch.testing.assert_close(out, m.o_proj(attn.reshape(1, l, 3584)), atol=0, rtol=0)
