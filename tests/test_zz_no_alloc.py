"""GPU: the route-layer entry point that allocates nothing.

Hosts that cannot call cudaMalloc (a plugin inside a framework that owns all
device memory, a server with a fixed pool) use
``mrsa_route_layer_forward_noalloc``, which runs the layer in a scratch area
built into the library instead of a caller workspace.  Its output must equal
that of ``mrsa_route_layer_forward`` with a caller workspace, on consecutive
calls that reuse the shared scratch with different inputs.  This file is
collected last so a run that stops at the first failure has run everything
else first.
"""

import ctypes as C

import pytest
import torch

from oracle import route_layer as orc

pytestmark = pytest.mark.gpu


def _case(mrsa, dev, seed, l=512, hidden=256):
    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(1, l, cfg, hidden=hidden, seed=seed)
    layer = mrsa.RouteLayer(inp["w_in"].to(dev), inp["w_out"].to(dev))
    args = [inp[n].to(dev).contiguous() for n in ("q_pre", "k_pre", "v", "hidden", "position_ids")]
    valid = inp["key_valid"].to(dev).contiguous()
    return layer, args, valid


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(mrsa, cuda_device):
    lib = mrsa._lib.load()
    stream = C.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    for seed in (11, 12):                       # two calls in a row share the scratch
        layer, args, valid = _case(mrsa, cuda_device, seed)
        ref = layer(*args, valid)               # caller-workspace entry point
        out = torch.full_like(ref, float("nan"))
        a = layer._args(*args, valid, out)
        assert lib.mrsa_route_layer_workspace_size(C.byref(a)) <= 32 * 1024 * 1024
        rc = lib.mrsa_route_layer_forward_noalloc(C.byref(a), stream)
        assert rc == 0, lib.mrsa_strerror(rc)
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        assert torch.isfinite(out).all()
        assert d.max().item() <= 2e-2
        assert d.mean().item() / ref.float().abs().mean().item() <= 1e-3
        assert torch.equal(out, ref)            # same kernels, same order: identical bits


def test_noalloc_rejects_problems_larger_than_its_scratch(mrsa, cuda_device):
    lib = mrsa._lib.load()
    a = mrsa._lib.RouteLayerArgs()
    a.batch, a.seq_len, a.q_heads, a.kv_heads, a.head_dim = 1, 16384, 28, 4, 128
    a.hidden_size, a.rank, a.topk, a.local_window = 3584, 64, 32, 256
    assert lib.mrsa_route_layer_workspace_size(C.byref(a)) > 32 * 1024 * 1024
    # rejected from the sizes alone, before any pointer is looked at or any launch
    assert lib.mrsa_route_layer_forward_noalloc(C.byref(a), None) == mrsa._lib.ERR_WORKSPACE
    assert lib.mrsa_route_layer_forward_noalloc(None, None) == mrsa._lib.ERR_NULL
