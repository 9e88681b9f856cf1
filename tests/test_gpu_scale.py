"""GPU parity at the benchmarked sizes and on the sharded path.

* The fused route layer at configs[1] (L=16384, 256 chunks) and at the
  chunk count of configs[4] on one GPU (L=131072, 2048 chunks), on three
  256-row slices (start, middle, end) against the CPU oracle: no routing
  difference where the key gap exceeds 1e-3, attention outputs within
  max-abs 2e-2 / mean-rel 1e-3 on the kernel's own selection.
* The sharded route and SWA layers (``shard.py``) for ranks of a simulated
  N=8 / N=4 run in one process: every stage runs as that rank would run it
  (halo buffer, ``q_offset``, routing over all chunks, gathered K/V), with
  the other ranks' contributions computed by the same kernels beforehand.
  Their rows must be bit-equal to the same rows of the single-GPU layer.
"""

import pytest
import torch

from oracle import route_layer as orc

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-3


def close_bf16(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all()
    d = (got - ref).abs()
    rel = d.mean().item() / max(ref.abs().mean().item(), 1e-30)
    assert d.max().item() <= max_abs and rel <= mean_rel, (d.max().item(), rel)


def _check_slices(mrsa, dev, l, seed, slices, min_exact):
    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(1, l, cfg, hidden=3584, seed=seed)
    layer = mrsa.RouteLayer(inp["w_in"].to(dev), inp["w_out"].to(dev))
    args = [inp[n].to(dev) for n in ("q_pre", "k_pre", "v", "hidden", "position_ids")]
    kv = inp["key_valid"].to(dev)
    fused = layer.forward(*args, kv)
    st = layer.forward(*args, kv, stages=True)
    assert torch.equal(fused, st["out"]), "fused C-ABI layer differs from the staged ops"
    del fused
    rows = torch.zeros(l, dtype=torch.bool)
    for sl in slices:
        rows[sl] = True
    rows[cfg.chunk - 1::cfg.chunk] = True
    shared = orc.route_layer_shared(inp, cfg, rows=rows)
    # the stages every row shares: landmark routing queries, landmarks, entropy
    rq = torch.arange(cfg.chunk - 1, l, cfg.chunk)
    close_bf16(st["route_q"][:, rq.to(dev)], shared["route_q"][:, rq], max_abs=6.5e-2, mean_rel=2e-3)
    close_bf16(st["lmk"], shared["lmk"], max_abs=2e-2, mean_rel=2e-3)
    torch.testing.assert_close(st["entropy"].cpu(), shared["entropy"], atol=2e-3, rtol=1e-3)
    for sl in slices:
        ref = orc.route_layer_rows(inp, shared, cfg, sl)
        close_bf16(st["local_out"][:, sl], ref["local_out"])
        torch.testing.assert_close(st["local_lse"][:, sl].cpu(), ref["local_lse"], atol=5e-4, rtol=1e-5)
        viol, exact = orc.topk_set_agreement(ref["route_key"], st["indices"][:, sl].cpu(), ref["indices"], cfg.topk)
        assert viol == 0, (sl, viol)
        assert exact >= min_exact, (sl, exact)
        own = orc.route_layer_rows(inp, shared, cfg, sl, indices=st["indices"][:, sl].cpu())
        close_bf16(st["remote_weights"][:, sl], own["remote_weights"], max_abs=2e-2, mean_rel=2e-3)
        close_bf16(st["local_weight"][:, sl], own["local_weight"], max_abs=2e-2, mean_rel=2e-3)
        close_bf16(st["remote_out"][:, sl], own["remote_out"])
        close_bf16(st["out"][:, sl], own["out"])


def test_route_layer_configs1_l16384_three_slices(mrsa, cuda_device):
    """the bench workload (256 chunks)."""
    l = 16384
    _check_slices(mrsa, cuda_device, l, 0, [slice(0, 256), slice(8064, 8320), slice(l - 256, l)], 0.9)


def test_route_layer_l131072_2048_chunks_three_slices(mrsa, cuda_device):
    """configs[4]'s sequence on one GPU: 2048 chunks, where the selected
    kernel's items carry one or two owners and routing selects with the
    64-chunks-per-lane kernel."""
    l = 131072
    _check_slices(mrsa, cuda_device, l, 1, [slice(0, 256), slice(65536, 65792), slice(l - 256, l)], 0.8)


# ---------------------------------------------------------------- sharded path
class LocalExchange:
    """The transfers of one rank of a simulated world, served from the whole
    sequence's K/V, validity and chunk summaries computed beforehand (what
    the other ranks would send).  The rank's own contributions must equal
    those rows bit for bit."""

    def __init__(self, rank, world, full):
        self.rank, self.world, self.full = rank, world, full
        self.bulk = None

    def halo(self, bufs, ls, h):
        r = self.rank
        left = h if r > 0 else 0
        start = r * ls - left
        for t, src in zip(bufs, (self.full["k"], self.full["v"], self.full["kv"])):
            rows = t.shape[1]
            own = t[:, left:left + ls]
            assert torch.equal(own, src[:, r * ls:(r + 1) * ls]), "own rows differ from the precomputed ones"
            t.copy_(src[:, start:start + rows])
        return _Done()

    def gather(self, out, inp, bulk=False):
        key = (out.dtype, tuple(out.shape[1:]))
        src = self.full["by_shape"][key]
        assert torch.equal(inp.reshape(out.shape[1:]), src[self.rank]), key
        out.copy_(src)
        return _Done()


class _Done:
    def wait(self):
        return None


def _sharded_case(mrsa, dev, world, ls, seed):
    from mrsa_b200.shard import KernelOps

    l = world * ls
    g = torch.Generator(device=dev).manual_seed(seed)
    q = (torch.randn(1, l, 28, 128, device=dev, generator=g) / 128 ** 0.5).bfloat16()
    k = (torch.randn(1, l, 4, 128, device=dev, generator=g) / 128 ** 0.5).bfloat16()
    v = (torch.randn(1, l, 4, 128, device=dev, generator=g) / 128 ** 0.5).bfloat16()
    h = torch.randn(1, l, 3584, device=dev, generator=g).bfloat16()
    w_in = (torch.randn(64, 3584, device=dev, generator=g) * 0.02).bfloat16()
    w_out = (torch.randn(28 * 128, 64, device=dev, generator=g) * 0.02).bfloat16()
    i = torch.arange(l, device=dev)
    pos = (i - i // 64).view(1, l).contiguous()
    valid = torch.ones(1, l, dtype=torch.bool, device=dev)
    valid[0, ls + 100:ls + 140] = False                 # ragged validity near a shard edge
    layer = mrsa.RouteLayer(w_in, w_out)
    ops = KernelOps(layer)
    # what every rank contributes to the exchanges
    cs = ls // 64
    k_all = torch.empty(1, l, 4, 128, dtype=torch.bfloat16, device=dev)
    lmk = torch.empty(world, cs, 4, 7, 128, dtype=torch.bfloat16, device=dev)
    prior = torch.empty(world, cs, 4, 7, dtype=torch.float32, device=dev)
    ok = torch.empty(world, cs, dtype=torch.uint8, device=dev)
    ent = torch.empty(1, cs, 4, 7, dtype=torch.float32, device=dev)
    for r in range(world):
        sl = slice(r * ls, (r + 1) * ls)
        qr = ops.rope(q[:, sl], k[:, sl], pos[:, sl], k_all[:, sl])
        rq = ops.qcal(h[:, sl], qr, pos[:, sl], torch.empty_like(qr))
        ops.pool(rq, k_all[:, sl], valid[:, sl], lmk[r].view(1, cs, 4, 7, 128), prior[r].view(1, cs, 4, 7),
                 ok[r].view(1, cs), ent)
    v16 = mrsa.to_f16(v)
    full = {"k": k_all, "v": v16, "kv": valid,
            "by_shape": {(torch.bfloat16, (ls, 4, 128)): k_all.view(world, ls, 4, 128),
                         (torch.float16, (ls, 4, 128)): v16.view(world, ls, 4, 128),
                         (torch.bool, (ls,)): valid.view(world, ls),
                         (torch.bfloat16, (cs, 4, 7, 128)): lmk,
                         (torch.float32, (cs, 4, 7)): prior,
                         (torch.uint8, (cs,)): ok}}
    ref = layer(q, k, v, h, pos, valid)
    return layer, (q, k, v, h, pos, valid), full, ref


@pytest.mark.parametrize("world,ls,ranks", [(8, 2048, (0, 3, 7)), (8, 16384, (0, 4, 7))])
def test_sharded_route_layer_rows_equal_the_single_gpu_layer(mrsa, cuda_device, world, ls, ranks):
    from mrsa_b200.shard import ShardedRouteLayer

    layer, (q, k, v, h, pos, valid), full, ref = _sharded_case(mrsa, cuda_device, world, ls, 5)
    for r in ranks:
        sl = slice(r * ls, (r + 1) * ls)
        shard = ShardedRouteLayer(layer, exchange=LocalExchange(r, world, full))
        out = shard(q[:, sl], k[:, sl], v[:, sl], h[:, sl], pos[:, sl], valid[:, sl])
        torch.cuda.synchronize()
        assert torch.equal(out, ref[:, sl]), (r, (out.float() - ref[:, sl].float()).abs().max().item())


def test_sharded_swa_layer_rows_equal_the_single_gpu_window(mrsa, cuda_device):
    """SWA layer sharded over a simulated N=4, batch 2, 1280-row halo."""
    from mrsa_b200.shard import ShardedSWALayer

    dev, world, ls, b = cuda_device, 4, 2048, 2
    l = world * ls
    g = torch.Generator(device=dev).manual_seed(9)
    q = (torch.randn(b, l, 28, 128, device=dev, generator=g) / 128 ** 0.5).bfloat16()
    k = (torch.randn(b, l, 4, 128, device=dev, generator=g) / 128 ** 0.5).bfloat16()
    v = (torch.randn(b, l, 4, 128, device=dev, generator=g) / 128 ** 0.5).bfloat16()
    i = torch.arange(l, device=dev)
    pos = (i - i // 64).expand(b, l).contiguous()
    valid = torch.ones(b, l, dtype=torch.bool, device=dev)
    valid[1, 3 * ls - 50:3 * ls + 30] = False
    inv, af = mrsa.yarn_inv_freq(128, 1.0e6, 8.0, 2048)
    qr, kr = mrsa.yarn_rope_qk(q, k, pos, inv.to(dev), af)
    v16 = mrsa.to_f16(v)
    ref, ref_lse = mrsa.window_attention(qr, kr, v16, valid, 1280, skip_inert=False, chunk=64)
    full = {"k": kr, "v": v16, "kv": valid, "by_shape": {}}
    for r in range(world):
        sl = slice(r * ls, (r + 1) * ls)
        swa = ShardedSWALayer(1280, exchange=LocalExchange(r, world, full))
        out, lse = swa(q[:, sl], k[:, sl], v[:, sl], pos[:, sl], valid[:, sl], return_lse=True)
        torch.cuda.synchronize()
        assert torch.equal(out, ref[:, sl]), r
        assert torch.equal(lse, ref_lse[:, sl]), r


def test_no_device_side_wait_gave_up_at_scale(mrsa, cuda_device):
    torch.cuda.synchronize()
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0
