"""Sequence-sharded route layer over the GPUs of one node.

Rank ``r`` of ``N`` owns the contiguous tokens ``[r*L/N, (r+1)*L/N)`` (whole
64-token chunks).  Queries are independent once K, V, the chunk summaries
(landmarks + entropy prior) and chunk validity are globally visible, so one
exchange step per layer suffices:

1. RoPE on the local q/k (cos/sin from global position ids);
2. all-gather K, V and key validity (NCCL over NVLink) -- issued
   asynchronously, it runs while this rank computes its Q-Cal routing
   queries and landmark pool;
3. all-gather the landmarks, prior and chunk validity (small);
4. local window attention, routing over all C chunks and selected-chunk
   attention for the local queries, reading only local HBM.

The reference never shards a sequence (it splits layers across two GPUs for
memory at 128k, ``scripts/from_dense16k/eval_jingneng_official_ruler.py:99``).
The collectives are ``torch.distributed`` NCCL all-gathers; every rank issues
the same collectives in the same order.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .layer import RouteLayer
from .local_attention import window_attention
from .rope_fp32 import yarn_rope_qk
from .routing import route_topk_fused
from .selected_attention import selected_attention


class ShardedRouteLayer:
    """Route layer whose query rows are sharded across ``group``.

    ``layer`` carries the (replicated) weights.  ``forward`` takes this rank's
    slice of q/k/v/h/position_ids/key_valid (``B == 1``) and returns this
    rank's output rows."""

    launches_per_step = 6   # rope, qcal, pool, local, route, selected (own kernels)

    def __init__(self, layer: RouteLayer, group=None):
        self.layer = layer
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._bufs = {}

    def _buf(self, name, shape, dtype, device):
        t = self._bufs.get(name)
        if t is None or t.shape != torch.Size(shape) or t.device != device:
            t = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = t
        return t

    def forward(self, q_pre, k_pre, v, hidden, position_ids, key_valid=None, out=None):
        lay, c = self.layer, self.layer.cfg
        b, ls, hq, d = q_pre.shape
        if b != 1:
            raise ValueError("the sharded route layer takes batch 1 (one long sequence)")
        if ls % c.chunk:
            raise ValueError(f"per-rank length {ls} must be a multiple of {c.chunk}")
        hkv, g = k_pre.shape[2], hq // k_pre.shape[2]
        n, r = self.world, self.rank
        L, cs = ls * n, ls // c.chunk
        C = cs * n
        dev = q_pre.device
        st = _lib.stream_of(q_pre)
        if key_valid is None:
            key_valid = torch.ones(b, ls, dtype=torch.bool, device=dev)
        kv_local = key_valid.to(torch.bool).contiguous()

        # 1. RoPE straight into this rank's slot of the gathered K buffer
        k_full = self._buf("k", (n, ls, hkv, d), torch.bfloat16, dev)
        v_full = self._buf("v", (n, ls, hkv, d), torch.bfloat16, dev)
        kv_full = self._buf("kv", (n, ls), torch.bool, dev)
        q, _ = yarn_rope_qk(q_pre, k_pre, position_ids, lay.inv_freq, lay.attention_factor,
                            out_k=k_full[r].view(1, ls, hkv, d))
        # 2. K/V/validity all-gather, overlapped with Q-Cal + pool below
        h_k = dist.all_gather_into_tensor(k_full, k_full[r], group=self.group, async_op=True)
        h_v = dist.all_gather_into_tensor(v_full, v.reshape(ls, hkv, d).contiguous(),
                                          group=self.group, async_op=True)
        h_m = dist.all_gather_into_tensor(kv_full, kv_local.reshape(ls), group=self.group,
                                          async_op=True)

        route_q = self._buf("route_q", (1, ls, hq, d), torch.bfloat16, dev)
        _lib.call("mrsa_qcal_route_query", _lib.ptr(hidden), _lib.ptr(q), _lib.ptr(lay.w_in),
                  _lib.ptr(lay.w_out), _lib.ptr(lay.norm_weight), float(c.rms_eps),
                  float(c.qcal_scale), _lib.ptr(position_ids), _lib.ptr(lay.inv_freq),
                  float(lay.attention_factor), _lib.ptr(route_q), 1, ls, hidden.shape[-1],
                  lay.w_in.shape[0], hq, d, st)
        lmk_full = self._buf("lmk", (n, cs, hkv, g, d), torch.bfloat16, dev)
        prior_full = self._buf("prior", (n, cs, hkv, g), torch.float32, dev)
        ok_full = self._buf("ok", (n, cs), torch.uint8, dev)
        ent = self._buf("ent", (1, cs, hkv, g), torch.float32, dev)
        mu = route_q[:, c.chunk - 1:]
        _lib.call("mrsa_chunk_pool", _lib.ptr(mu), ls * hq * d, c.chunk * hq * d,
                  _lib.ptr(k_full[r]), _lib.ptr(kv_local), d ** -0.5, _lib.ptr(lay.bias_scale),
                  _lib.ptr(lmk_full[r]), _lib.ptr(ent), _lib.ptr(prior_full[r]),
                  _lib.ptr(ok_full[r]), 1, cs, hkv, g, d, st)
        # 3. chunk summaries
        h_l = dist.all_gather_into_tensor(lmk_full, lmk_full[r], group=self.group, async_op=True)
        h_p = dist.all_gather_into_tensor(prior_full, prior_full[r], group=self.group, async_op=True)
        h_o = dist.all_gather_into_tensor(ok_full, ok_full[r], group=self.group, async_op=True)
        for h in (h_k, h_v, h_m):
            h.wait()
        # 4. local queries over the global K/V
        k_all = k_full.view(1, L, hkv, d)
        v_all = v_full.view(1, L, hkv, d)
        valid_all = kv_full.view(1, L)
        local_out, local_lse = window_attention(q, k_all, v_all, valid_all,
                                                c.local_window + c.chunk - 1, skip_inert=True,
                                                chunk=c.chunk, q_offset=r * ls)
        for h in (h_l, h_p, h_o):
            h.wait()
        idx, _, rw, lw = route_topk_fused(route_q, lmk_full.view(1, C, hkv, g, d), local_lse,
                                          prior_full.view(1, C, hkv, g), ok_full.view(1, C),
                                          c.topk, c.local_window, q_offset=r * ls,
                                          temperature=c.route_temperature,
                                          gate_scale=lay.gate_scale, gate_offset=lay.gate_offset)
        return selected_attention(q, k_all, v_all, rw, idx, valid_all, chunk=c.chunk,
                                  local_out=local_out, local_weight=lw, out=out)

    __call__ = forward
