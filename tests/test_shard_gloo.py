"""The sequence-sharded route layer's host plan on CPU, world size 2 (gloo).

Each rank runs ``ShardedRouteLayer.forward`` on its half of the tokens with
the compute stages supplied by the CPU oracle; the exchange (``gather_rows``,
rank order, async handles), the shard offsets, global position ids and the
per-shard landmark pool are the product's own code.  Every rank's output rows
must equal the single-process oracle layer restricted to those rows.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import route_layer as orc

L_TOTAL, HIDDEN, SEED, WORLD = 1024, 256, 3, 2


class OracleOps:
    """Stage ops of ``ShardedRouteLayer`` evaluated by the CPU oracle."""

    launches_per_step = 0

    def __init__(self, inp, cfg):
        self.inp, self.cfg = inp, cfg
        self.inv_freq, self.af = orc.yarn_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.yarn_factor,
                                                   cfg.yarn_orig_max_pos)

    def attention_v(self, v):
        return v

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
        ok_out.fill_(1)

    def local(self, q, k_all, v_all, valid_all, q_offset):
        b, ls = q.shape[:2]
        qf = torch.zeros(b, k_all.shape[1], *q.shape[2:], dtype=q.dtype)
        qf[:, q_offset:q_offset + ls] = q
        return orc._local_rows(qf, k_all, v_all, valid_all.bool(), self.cfg.local_window, self.cfg.chunk, True,
                               slice(q_offset, q_offset + ls))

    def route(self, route_q, lmk_all, local_lse, prior_all, ok_all, valid_all, q_offset):
        b, ls, hq, _ = route_q.shape
        hkv = lmk_all.shape[2]
        drop = orc.remote_drop_mask(valid_all.bool(), self.cfg.local_window, self.cfg.chunk)[:, q_offset:q_offset + ls]
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
        results[rank] = (torch.equal(out, ref), (out.float() - ref.float()).abs().max().item())
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


def _worker_lost_peer(rank, port, results):
    """Rank 1 joins the group and leaves before the layer's first exchange;
    rank 0 must get an error from that exchange (no hang) and report it."""
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=20))
    if rank == 1:
        results[rank] = "left"
        return                      # the peer is lost between steps, with nothing in flight
    import __graft_entry__

    __graft_entry__.load_package()
    from mrsa_b200.shard import ShardedRouteLayer

    cfg = orc.MRSAConfig()
    inp = orc.make_route_layer_inputs(1, L_TOTAL, cfg, hidden=HIDDEN, seed=SEED)
    sl = slice(0, L_TOTAL // WORLD)
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
        procs = [ctx.Process(target=_worker_lost_peer, args=(r, port, results)) for r in range(WORLD)]
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
