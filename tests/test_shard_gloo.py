"""The sequence-sharded route and SWA layers' host plan on CPU (gloo).

Each rank runs ``ShardedRouteLayer.forward`` / ``ShardedSWALayer.forward`` on
its share of the tokens with the compute stages supplied by the CPU oracle;
the exchange (halo send/receive to the neighbours, the all-gathers on two
communicators, rank order, async handles), the shard offsets, halo buffers,
global position ids and the per-shard landmark pool are the product's own
code.  Three ranks, so a middle rank with two neighbours is covered.  Every
rank's output rows must equal the single-process oracle layer restricted to
those rows.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import route_layer as orc

L_TOTAL, HIDDEN, SEED, WORLD = 1152, 256, 3, 3      # 384 rows (6 chunks) per rank >= the 320-row halo
SWA_WINDOW, SWA_BATCH = 300, 2


def _same(got, ref):
    """Equal up to the summation order of the oracle's blocked fp32 window
    (the halo buffer blocks the keys differently from the whole sequence):
    bf16 results at most one ulp apart."""
    d = (got.float() - ref.float()).abs()
    return bool((d <= ref.float().abs() * 2.0 ** -7 + 2.0 ** -20).all())


class OracleOps:
    """Stage ops of ``ShardedRouteLayer`` evaluated by the CPU oracle."""

    launches_per_step = 0
    v_dtype = torch.bfloat16

    def __init__(self, inp, cfg):
        self.inp, self.cfg = inp, cfg
        self.inv_freq, self.af = orc.yarn_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.yarn_factor,
                                                   cfg.yarn_orig_max_pos)

    def attention_v(self, v, out=None):
        return v if out is None else out.copy_(v)

    def _cs(self, pos):
        return orc.rope_cos_sin(pos, self.inv_freq, self.af)

    def rope(self, q_pre, k_pre, position_ids, k_out):
        cos, sin = self._cs(position_ids)
        k_out.copy_(orc.apply_rope(k_pre, cos, sin, self.cfg.rope_precision))
        return orc.apply_rope(q_pre, cos, sin, self.cfg.rope_precision)

    def qcal(self, hidden, q, position_ids, out):
        cos, sin = self._cs(position_ids)
        out.copy_(orc.qcal_route_query(hidden, q, self.inp["w_in"], self.inp["w_out"], self.inp["norm_weight"],
                                       cos, sin, eps=self.cfg.rms_eps, precision=self.cfg.rope_precision))
        return out

    def pool(self, route_q, k_local, kv_local, lmk_out, prior_out, ok_out, ent_out):
        c = self.cfg.chunk
        b, ls, hq, d = route_q.shape
        hkv = k_local.shape[2]
        g, cs = hq // hkv, ls // c
        mu = route_q[:, c - 1::c].reshape(b, cs, hkv, g, d)
        lmk, ent = orc.chunk_pool(mu, k_local.reshape(b, cs, c, hkv, d), kv_local.reshape(b, cs, c))
        lmk_out.copy_(lmk)
        ent_out.copy_(ent)
        prior_out.copy_(ent * self.inp["entropy_bias_scale"].float().view(1, 1, hkv, g))
        real = (torch.arange(ls) + 1) % c != 0
        ok_out.copy_((kv_local.bool() & real[None]).view(b, cs, c).any(-1).to(ok_out.dtype))

    def local(self, q, k_halo, v_halo, valid_halo, q_offset, window=None, skip_inert=True, need_lse=True):
        # the oracle's window over the rank's halo buffer (which starts on a chunk boundary)
        b, ls = q.shape[:2]
        qf = torch.zeros(b, k_halo.shape[1], *q.shape[2:], dtype=q.dtype)
        qf[:, q_offset:q_offset + ls] = q
        w = self.cfg.local_window if window is None else window
        return orc._local_rows(qf, k_halo, v_halo, valid_halo.bool(), w, self.cfg.chunk, skip_inert,
                               slice(q_offset, q_offset + ls))

    def route(self, route_q, lmk_all, local_lse, prior_all, ok_all, q_offset):
        # the drop rule of remote_drop_mask from the gathered chunk validity
        b, ls, hq, _ = route_q.shape
        hkv, c = lmk_all.shape[2], lmk_all.shape[1]
        ch, w = self.cfg.chunk, self.cfg.local_window
        pos = torch.arange(q_offset, q_offset + ls)
        lo = (pos - w).clamp_min(0) // ch
        hi = (pos + w).clamp_max(c * ch - 1) // ch
        cid = torch.arange(c)
        local = (cid[None, :] >= lo[:, None]) & (cid[None, :] <= hi[:, None])
        drop = (local[None] | (ok_all == 0)[:, None, :]).to(torch.int32)
        idx, scores = orc.route_topk_blocked(route_q, lmk_all, local_lse.view(b, -1, hkv, hq // hkv), prior_all,
                                             drop, self.cfg.topk)
        rw, lw = orc.route_weights_affine(scores, idx, prior_all, local_lse, temperature=self.cfg.route_temperature,
                                          gate_offset=self.inp["gate_offset"], gate_scale=self.inp["gate_scale"])
        return idx, rw, lw

    def selected(self, q, k_all, v_all, rw, idx, valid_all, local_out, local_w, out):
        remote = orc.selected_attention(q, k_all, v_all, rw, idx, valid_all.bool(), self.cfg.chunk)
        return orc.fuse_outputs(remote, local_out, local_w)


def _worker(rank, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        import __graft_entry__

        __graft_entry__.load_package()
        from mrsa_b200.shard import ShardedRouteLayer

        cfg = orc.MRSAConfig()
        inp = orc.make_route_layer_inputs(1, L_TOTAL, cfg, hidden=HIDDEN, seed=SEED)
        ls = L_TOTAL // WORLD
        sl = slice(rank * ls, (rank + 1) * ls)
        layer = ShardedRouteLayer(ops=OracleOps(inp, cfg))
        assert (layer.rank, layer.world) == (rank, WORLD)
        out = layer(inp["q_pre"][:, sl], inp["k_pre"][:, sl], inp["v"][:, sl], inp["hidden"][:, sl],
                    inp["position_ids"][:, sl], inp["key_valid"][:, sl])
        ref = orc.route_layer_forward(inp, cfg, keep=False, query_slice=sl)["out"]
        results[rank] = (_same(out, ref), (out.float() - ref.float()).abs().max().item())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(600)
def test_sharded_plan_matches_single_process_oracle():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=540)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(results)
    assert sorted(res) == list(range(WORLD))
    for rank, (equal, diff) in res.items():
        assert equal, (rank, diff)



def _worker_swa(rank, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        import __graft_entry__

        __graft_entry__.load_package()
        from mrsa_b200.shard import ShardedSWALayer

        cfg = orc.MRSAConfig()
        inp = orc.make_route_layer_inputs(SWA_BATCH, L_TOTAL, cfg, hidden=64, seed=SEED + 1)
        inp["key_valid"][1, 700:760] = False           # ragged validity in the second sequence
        ls = L_TOTAL // WORLD
        sl = slice(rank * ls, (rank + 1) * ls)
        layer = ShardedSWALayer(window=SWA_WINDOW, ops=OracleOps(inp, cfg))
        out, lse = layer(inp["q_pre"][:, sl], inp["k_pre"][:, sl], inp["v"][:, sl], inp["position_ids"][:, sl],
                         inp["key_valid"][:, sl], return_lse=True)
        ref = orc.swa_layer_forward(inp, cfg, window=SWA_WINDOW)
        results[rank] = (_same(out, ref["out"][:, sl]) and
                         torch.allclose(lse, ref["lse"][:, sl], atol=1e-5, rtol=1e-6),
                         (out.float() - ref["out"][:, sl].float()).abs().max().item())
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_sharded_swa_halo_matches_single_process_oracle():
    """The SWA layer's halo exchange (window 300 -> 320 rows each side), batch 2."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker_swa, args=(r, port, results)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=540)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(results)
    assert sorted(res) == list(range(WORLD))
    for rank, (equal, diff) in res.items():
        assert equal, (rank, diff)


def _worker_lost_peer(rank, port, results):
    """Rank 1 joins the group and leaves before the layer's first exchange;
    rank 0 must get an error from that exchange (no hang) and report it."""
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=20))
    if rank == 1:
        results[rank] = "left"
        return                      # the peer is lost between steps, with nothing in flight
    import __graft_entry__

    __graft_entry__.load_package()
    from mrsa_b200.shard import ShardedRouteLayer

    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(1, L_TOTAL, cfg, hidden=HIDDEN, seed=SEED)
    sl = slice(0, L_TOTAL // 2)
    layer = ShardedRouteLayer(ops=OracleOps(inp, cfg))
    try:
        layer(inp["q_pre"][:, sl], inp["k_pre"][:, sl], inp["v"][:, sl], inp["hidden"][:, sl],
              inp["position_ids"][:, sl], inp["key_valid"][:, sl])
        results[rank] = "no error"
    except Exception as exc:  # the backend's error type differs between versions
        results[rank] = f"error: {type(exc).__name__}"


@pytest.mark.timeout(300)
def test_lost_rank_ends_the_exchange_with_an_error():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker_lost_peer, args=(r, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
        alive = [p.is_alive() for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        res = dict(results)
    assert not any(alive), "a rank did not finish: the lost peer was not detected"
    assert res.get(1) == "left"
    assert str(res.get(0, "")).startswith("error"), res
