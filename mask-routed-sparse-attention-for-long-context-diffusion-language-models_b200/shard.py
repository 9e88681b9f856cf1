"""Sequence-sharded route layer over the GPUs of one node.

Rank ``r`` of ``N`` owns the contiguous tokens ``[r*L/N, (r+1)*L/N)`` (whole
64-token chunks).  Queries are independent once K, V, the chunk summaries
(landmarks + entropy prior) and chunk validity are globally visible, so one
exchange step per layer suffices:

1. RoPE on the local q/k (cos/sin from global position ids);
2. all-gather K, V (in fp16, the form both attention kernels take) and key
   validity (NCCL over NVLink) -- issued
   asynchronously, it runs while this rank computes its Q-Cal routing
   queries and landmark pool;
3. all-gather the landmarks, prior and chunk validity (small);
4. local window attention, routing over all C chunks and selected-chunk
   attention for the local queries, reading only local HBM.

The reference never shards a sequence (it splits layers across two GPUs for
memory at 128k, ``scripts/from_dense16k/eval_jingneng_official_ruler.py:99``).
The collectives are ``torch.distributed`` all-gathers; every rank issues the
same collectives in the same order.  The six compute stages go through an
ops object (``KernelOps``: the B200 kernels); the exchange plan itself is
backend-neutral, so it also runs on CPU process groups.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .layer import RouteLayer
from .local_attention import window_attention
from .rope_fp32 import yarn_rope_qk
from .routing import route_topk_fused
from .selected_attention import selected_attention, to_f16


def gather_rows(out: torch.Tensor, inp: torch.Tensor, group=None, async_op: bool = False):
    """All-gather ``inp`` (this rank's rows) into ``out`` (``[world, *inp.shape]``,
    rank order).  One ``all_gather_into_tensor`` on NCCL; the list form
    elsewhere (gloo splits a stacked output differently)."""
    inp = inp.reshape(out.shape[1:])
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(out, inp, group=group, async_op=async_op)
    return dist.all_gather(list(out.unbind(0)), inp.contiguous(), group=group, async_op=async_op)


class KernelOps:
    """The compute stages of a sharded route layer on the B200 kernels."""

    launches_per_step = 8   # rope, V to fp16, qcal, pool, local, route keys + selection, selected

    def __init__(self, layer: RouteLayer):
        self.layer = layer
        self.cfg = layer.cfg

    def attention_v(self, v):
        """V as the attention kernels take it: fp16 (P then travels as one fp16 tile)."""
        return to_f16(v)

    def rope(self, q_pre, k_pre, position_ids, k_out):
        lay = self.layer
        q, _ = yarn_rope_qk(q_pre, k_pre, position_ids, lay.inv_freq, lay.attention_factor, out_k=k_out)
        return q

    def qcal(self, hidden, q, position_ids, out):
        lay, c = self.layer, self.cfg
        _, ls, hq, d = q.shape
        _lib.call("mrsa_qcal_route_query", _lib.ptr(hidden), _lib.ptr(q), _lib.ptr(lay.w_in),
                  _lib.ptr(lay.w_out), _lib.ptr(lay.norm_weight), float(c.rms_eps),
                  float(c.qcal_scale), _lib.ptr(position_ids), _lib.ptr(lay.inv_freq),
                  float(lay.attention_factor), _lib.ptr(out), 1, ls, hidden.shape[-1],
                  lay.w_in.shape[0], hq, d, _lib.stream_of(q))
        return out

    def pool(self, route_q, k_local, kv_local, lmk_out, prior_out, ok_out, ent_out):
        lay, c = self.layer, self.cfg
        _, ls, hq, d = route_q.shape
        cs, hkv, g = lmk_out.shape[1], lmk_out.shape[2], lmk_out.shape[3]
        mu = route_q[:, c.chunk - 1:]
        _lib.call("mrsa_chunk_pool", _lib.ptr(mu), ls * hq * d, c.chunk * hq * d,
                  _lib.ptr(k_local), _lib.ptr(kv_local), d ** -0.5, _lib.ptr(lay.bias_scale),
                  _lib.ptr(lmk_out), _lib.ptr(ent_out), _lib.ptr(prior_out),
                  _lib.ptr(ok_out), 1, cs, hkv, g, d, _lib.stream_of(route_q))

    def local(self, q, k_all, v_all, valid_all, q_offset):
        c = self.cfg
        return window_attention(q, k_all, v_all, valid_all, c.local_window + c.chunk - 1,
                                skip_inert=True, chunk=c.chunk, q_offset=q_offset)

    def route(self, route_q, lmk_all, local_lse, prior_all, ok_all, valid_all, q_offset):
        lay, c = self.layer, self.cfg
        idx, _, rw, lw = route_topk_fused(route_q, lmk_all, local_lse, prior_all, ok_all, c.topk,
                                          c.local_window, q_offset=q_offset,
                                          temperature=c.route_temperature,
                                          gate_scale=lay.gate_scale, gate_offset=lay.gate_offset)
        return idx, rw, lw

    def selected(self, q, k_all, v_all, rw, idx, valid_all, local_out, local_w, out):
        return selected_attention(q, k_all, v_all, rw, idx, valid_all, chunk=self.cfg.chunk,
                                  local_out=local_out, local_weight=local_w, out=out)


class ShardedRouteLayer:
    """Route layer whose query rows are sharded across ``group``.

    ``layer`` carries the (replicated) weights; ``ops`` (default: the B200
    kernels over ``layer``) computes the stages.  ``forward`` takes this
    rank's slice of q/k/v/h/position_ids/key_valid (``B == 1``) and returns
    this rank's output rows."""

    launches_per_step = KernelOps.launches_per_step

    def __init__(self, layer: RouteLayer | None = None, group=None, ops=None):
        if ops is None:
            ops = KernelOps(layer)
        self.ops = ops
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
        ops, c = self.ops, self.ops.cfg
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
        if key_valid is None:
            key_valid = torch.ones(b, ls, dtype=torch.bool, device=dev)
        kv_local = key_valid.to(torch.bool).contiguous()

        # 1. RoPE straight into this rank's slot of the gathered K buffer
        k_full = self._buf("k", (n, ls, hkv, d), torch.bfloat16, dev)
        v_att = ops.attention_v(v)           # gathered in the form the attention stages take
        v_full = self._buf("v", (n, ls, hkv, d), v_att.dtype, dev)
        kv_full = self._buf("kv", (n, ls), torch.bool, dev)
        q = ops.rope(q_pre, k_pre, position_ids, k_full[r].view(1, ls, hkv, d))
        # 2. K/V/validity all-gather, overlapped with Q-Cal + pool below
        h_k = gather_rows(k_full, k_full[r], self.group, async_op=True)
        h_v = gather_rows(v_full, v_att, self.group, async_op=True)
        h_m = gather_rows(kv_full, kv_local, self.group, async_op=True)

        route_q = ops.qcal(hidden, q, position_ids, self._buf("route_q", (1, ls, hq, d), torch.bfloat16, dev))
        lmk_full = self._buf("lmk", (n, cs, hkv, g, d), torch.bfloat16, dev)
        prior_full = self._buf("prior", (n, cs, hkv, g), torch.float32, dev)
        ok_full = self._buf("ok", (n, cs), torch.uint8, dev)
        ent = self._buf("ent", (1, cs, hkv, g), torch.float32, dev)
        ops.pool(route_q, k_full[r].view(1, ls, hkv, d), kv_local, lmk_full[r].view(1, cs, hkv, g, d),
                 prior_full[r].view(1, cs, hkv, g), ok_full[r].view(1, cs), ent)
        # 3. chunk summaries
        h_l = gather_rows(lmk_full, lmk_full[r], self.group, async_op=True)
        h_p = gather_rows(prior_full, prior_full[r], self.group, async_op=True)
        h_o = gather_rows(ok_full, ok_full[r], self.group, async_op=True)
        for h in (h_k, h_v, h_m):
            h.wait()
        # 4. local queries over the global K/V
        k_all = k_full.view(1, L, hkv, d)
        v_all = v_full.view(1, L, hkv, d)
        valid_all = kv_full.view(1, L)
        local_out, local_lse = ops.local(q, k_all, v_all, valid_all, r * ls)
        for h in (h_l, h_p, h_o):
            h.wait()
        idx, rw, lw = ops.route(route_q, lmk_full.view(1, C, hkv, g, d), local_lse,
                                prior_full.view(1, C, hkv, g), ok_full.view(1, C), valid_all, r * ls)
        return ops.selected(q, k_all, v_all, rw, idx, valid_all, local_out, lw, out)

    __call__ = forward
