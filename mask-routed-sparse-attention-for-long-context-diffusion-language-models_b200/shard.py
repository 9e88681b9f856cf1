"""Sequence-sharded route layer and SWA layer over the GPUs of one node.

Rank ``r`` of ``N`` owns the contiguous tokens ``[r*L/N, (r+1)*L/N)`` (whole
64-token chunks).  Queries are independent once the keys they read are
visible, so each layer needs one exchange step, laid out so that the big
transfer hides behind compute:

* **Halo** (point-to-point to the two neighbours): the first and last ``H``
  rows of this rank's K, V and key validity, ``H`` = the attention window
  rounded up to whole chunks (320 rows for the route layer's 256 + 63
  window, 1280 for the SWA layer).  The local window attention then reads
  ``[left halo | own rows | right halo]`` and needs nothing else.
* **Chunk summaries** (all-gather, small): landmark keys, entropy prior and
  chunk validity of every chunk -- routing scores all C chunks.
* **K/V** (all-gather, 235 MB received per rank at N=8, route layer only):
  the selected chunks can lie anywhere in the sequence.  It runs on its own
  communicator and is posted after the summaries, so neither Q-Cal nor the
  two small exchanges share the GPU with it, and only selected-chunk
  attention waits for it.

Route-layer order on the compute stream: RoPE (K straight into the halo
buffer) and V to fp16; post the halo; Q-Cal and the landmark pool of this
rank's chunks; post the summary all-gather, then the K/V all-gather; wait
for the halo, local window attention; wait for the summaries, routing over
all C chunks; wait for K/V, selected-chunk attention with the fused local
merge.
Every kernel reads only local HBM.  The SWA layer (21 of the 28 layers,
``dream_dllm_hils/attention.py:1168-1220``) is RoPE, the halo exchange and
the window attention.

The reference never shards a sequence (it splits layers across two GPUs for
memory at 128k, ``scripts/from_dense16k/eval_jingneng_official_ruler.py:99``).
Every rank issues the same collectives in the same order.  The compute
stages go through an ops object (``KernelOps``: the B200 kernels) and the
transfers through an exchange object (``GroupExchange``: ``torch.distributed``
over NCCL or gloo), so the same plan runs on CPU process groups with other
stages, and in one process over precomputed neighbours' data.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _lib
from .layer import RouteLayer
from .local_attention import window_attention
from .rope_fp32 import yarn_inv_freq, yarn_rope_qk
from .routing import route_topk_fused
from .selected_attention import selected_attention, to_f16


def halo_rows(window: int, chunk: int) -> int:
    """Rows of the neighbours' K/V a window attention of effective window
    ``window`` reads: the window rounded up to whole chunks (the halo buffer
    then starts on a chunk boundary, which keeps landmark slots at
    positions ``63 mod 64``)."""
    return int(math.ceil(window / chunk)) * chunk


def gather_rows(out: torch.Tensor, inp: torch.Tensor, group=None, async_op: bool = False):
    """All-gather ``inp`` (this rank's rows) into ``out`` (``[world, *inp.shape]``,
    rank order).  One ``all_gather_into_tensor`` on NCCL; the list form
    elsewhere (gloo splits a stacked output differently)."""
    inp = inp.reshape(out.shape[1:])
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(out, inp, group=group, async_op=async_op)
    return dist.all_gather(list(out.unbind(0)), inp.contiguous(), group=group, async_op=async_op)


class _Done:
    """Handle of a transfer that has already completed."""

    def wait(self):
        return None


class _Many:
    def __init__(self, works):
        self.works = [w for w in works if w is not None]

    def wait(self):
        for w in self.works:
            w.wait()


class GroupExchange:
    """The transfers of the sharded layers over a ``torch.distributed`` group.

    ``bulk`` (optional) is a second group over the same ranks -- its own
    communicator -- for the K/V all-gather, so the halo and the chunk
    summaries never queue behind it; without it every transfer shares
    ``group``.  Create it once (``dist.new_group``, every rank) before the
    first forward."""

    def __init__(self, group=None, bulk=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.bulk = bulk

    def align(self):
        """Barrier over the group (every rank), so a timed forward starts on all
        ranks together and the exchange waits inside it measure transfers, not
        how far one rank's host ran ahead of another's."""
        dist.barrier(group=self.group)

    def halo(self, bufs, ls: int, h: int):
        """Post the halo exchange of the tensors ``bufs`` (each
        ``[B, rows, ...]``: this rank's ``ls`` rows after an ``h``-row left
        halo when this rank has a left neighbour, and an ``h``-row right halo
        after them when it has a right one).  Returns a handle whose
        ``wait()`` makes the halo rows valid."""
        r, n = self.rank, self.world
        left = h if r > 0 else 0
        ops, keep, copies = [], [], []

        def send(src, peer):
            s = src.contiguous()
            keep.append(s)
            ops.append(dist.P2POp(dist.isend, s, peer, self.group))

        def recv_into(dst, peer):
            if dst.is_contiguous():
                ops.append(dist.P2POp(dist.irecv, dst, peer, self.group))
            else:                                # batch > 1: receive into a staging copy
                tmp = torch.empty(dst.shape, dtype=dst.dtype, device=dst.device)
                ops.append(dist.P2POp(dist.irecv, tmp, peer, self.group))
                copies.append((dst, tmp))

        for t in bufs:
            if r > 0:
                send(t[:, left:left + h], self._peer(r - 1))
                recv_into(t[:, :h], self._peer(r - 1))
            if r < n - 1:
                send(t[:, left + ls - h:left + ls], self._peer(r + 1))
                recv_into(t[:, left + ls:], self._peer(r + 1))
        if not ops:
            return _Done()
        return _HaloHandle(dist.batch_isend_irecv(ops), keep, copies)

    def _peer(self, r):
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def gather(self, out, inp, bulk: bool = False):
        """Post an all-gather of ``inp`` into ``out`` (``[world, ...]``)."""
        return gather_rows(out, inp, self.bulk if (bulk and self.bulk is not None) else self.group,
                           async_op=True)


class _HaloHandle:
    def __init__(self, works, keep, recv_tmp):
        self.works, self.keep, self.recv_tmp = works, keep, recv_tmp

    def wait(self):
        for w in self.works:
            w.wait()
        for dst, tmp in self.recv_tmp:
            dst.copy_(tmp)
        self.keep = self.recv_tmp = None


class KernelOps:
    """The compute stages of the sharded layers on the B200 kernels."""

    launches_per_step = 8   # rope, V to fp16, qcal, pool, local, route keys + selection, selected
    v_dtype = torch.float16  # the attention kernels' V: fp16, so P travels as one fp16 tile

    def __init__(self, layer: RouteLayer):
        self.layer = layer
        self.cfg = layer.cfg

    def attention_v(self, v, out=None):
        """V as the attention kernels take it: fp16 (P then travels as one fp16 tile)."""
        return to_f16(v, out=out)

    def rope(self, q_pre, k_pre, position_ids, k_out):
        lay = self.layer
        q, _ = yarn_rope_qk(q_pre, k_pre, position_ids, lay.inv_freq, lay.attention_factor, out_k=k_out)
        return q

    def qcal(self, hidden, q, position_ids, out):
        lay, c = self.layer, self.cfg
        b, ls, hq, d = q.shape
        _lib.call("mrsa_qcal_route_query", _lib.ptr(hidden), _lib.ptr(q), _lib.ptr(lay.w_in),
                  _lib.ptr(lay.w_out), _lib.ptr(lay.norm_weight), float(c.rms_eps),
                  float(c.qcal_scale), _lib.ptr(position_ids), _lib.ptr(lay.inv_freq),
                  float(lay.attention_factor), _lib.ptr(out), b, ls, hidden.shape[-1],
                  lay.w_in.shape[0], hq, d, _lib.stream_of(q))
        return out

    def pool(self, route_q, k_local, kv_local, lmk_out, prior_out, ok_out, ent_out):
        lay, c = self.layer, self.cfg
        b, ls, hq, d = route_q.shape
        cs, hkv, g = lmk_out.shape[1], lmk_out.shape[2], lmk_out.shape[3]
        mu = route_q[:, c.chunk - 1:]
        _lib.call("mrsa_chunk_pool", _lib.ptr(mu), ls * hq * d, c.chunk * hq * d,
                  _lib.ptr(k_local), _lib.ptr(kv_local), d ** -0.5, _lib.ptr(lay.bias_scale),
                  _lib.ptr(lmk_out), _lib.ptr(ent_out), _lib.ptr(prior_out),
                  _lib.ptr(ok_out), b, cs, hkv, g, d, _lib.stream_of(route_q))

    def local(self, q, k_halo, v_halo, valid_halo, q_offset, window=None, skip_inert=True, need_lse=True):
        c = self.cfg
        w = c.local_window + c.chunk - 1 if window is None else window
        return window_attention(q, k_halo, v_halo, valid_halo, w, skip_inert=skip_inert, chunk=c.chunk,
                                q_offset=q_offset, need_lse=need_lse)

    def route(self, route_q, lmk_all, local_lse, prior_all, ok_all, q_offset):
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
    kernels over ``layer``) computes the stages and ``exchange`` (default:
    :class:`GroupExchange` over ``group``) moves the data.  ``forward``
    takes this rank's slice of q/k/v/h/position_ids/key_valid (``B == 1``)
    and returns this rank's output rows."""

    launches_per_step = KernelOps.launches_per_step
    STAGES = ("rope", "qcal", "pool", "halo_wait", "local_attention", "summaries_wait", "route",
              "kv_wait", "selected_attention")

    def __init__(self, layer: RouteLayer | None = None, group=None, ops=None, exchange=None, bulk_group=None):
        if ops is None:
            ops = KernelOps(layer)
        self.ops = ops
        self.exchange = exchange if exchange is not None else GroupExchange(group, bulk_group)
        self.world = self.exchange.world
        self.rank = self.exchange.rank
        self._bufs = {}

    def _buf(self, name, shape, dtype, device):
        t = self._bufs.get(name)
        if t is None or t.shape != torch.Size(shape) or t.dtype != dtype or t.device != device:
            t = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = t
        return t

    def forward(self, q_pre, k_pre, v, hidden, position_ids, key_valid=None, out=None, events=None):
        ops, c, ex = self.ops, self.ops.cfg, self.exchange
        mark = (lambda name: events[name].record()) if events is not None else (lambda name: None)
        b, ls, hq, d = q_pre.shape
        if b != 1:
            raise ValueError("the sharded route layer takes batch 1 (one long sequence)")
        if ls % c.chunk:
            raise ValueError(f"per-rank length {ls} must be a multiple of {c.chunk}")
        n, r = self.world, self.rank
        h = halo_rows(c.local_window + c.chunk - 1, c.chunk)
        if n > 1 and ls < h:
            raise ValueError(f"per-rank length {ls} is shorter than the {h}-row halo")
        hkv, g = k_pre.shape[2], hq // k_pre.shape[2]
        L, cs = ls * n, ls // c.chunk
        C = cs * n
        dev = q_pre.device
        if key_valid is None:
            key_valid = torch.ones(b, ls, dtype=torch.bool, device=dev)
        left = h if r > 0 else 0
        rows = left + ls + (h if r < n - 1 else 0)

        # 1. RoPE with K straight into the halo buffer; V in the attention kernels' dtype
        mark("start")
        k_h = self._buf("k_halo", (1, rows, hkv, d), torch.bfloat16, dev)
        v_h = self._buf("v_halo", (1, rows, hkv, d), ops.v_dtype, dev)
        m_h = self._buf("kv_halo", (1, rows), torch.bool, dev)
        k_own, v_own, m_own = k_h[:, left:left + ls], v_h[:, left:left + ls], m_h[:, left:left + ls]
        q = ops.rope(q_pre, k_pre, position_ids, k_own)
        ops.attention_v(v, out=v_own)
        m_own.copy_(key_valid.to(torch.bool))
        mark("rope")
        # 2. post the halo exchange (small; the local window needs it first)
        h_halo = ex.halo((k_h, v_h, m_h), ls, h)
        # 3. Q-Cal and the landmark pool of this rank's chunks, then the summaries
        route_q = ops.qcal(hidden, q, position_ids, self._buf("route_q", (1, ls, hq, d), torch.bfloat16, dev))
        mark("qcal")
        lmk_full = self._buf("lmk", (n, cs, hkv, g, d), torch.bfloat16, dev)
        prior_full = self._buf("prior", (n, cs, hkv, g), torch.float32, dev)
        ok_full = self._buf("ok", (n, cs), torch.uint8, dev)
        ent = self._buf("ent", (1, cs, hkv, g), torch.float32, dev)
        ops.pool(route_q, k_own, m_own, lmk_full[r].view(1, cs, hkv, g, d),
                 prior_full[r].view(1, cs, hkv, g), ok_full[r].view(1, cs), ent)
        mark("pool")
        h_sum = _Many([ex.gather(lmk_full, lmk_full[r]), ex.gather(prior_full, prior_full[r]),
                       ex.gather(ok_full, ok_full[r])])
        # the K/V all-gather (own communicator) goes out after the summaries, so
        # neither Q-Cal nor the summaries' gather shares the GPU with it; local
        # attention and routing (which need no remote K/V) hide it
        k_full = self._buf("k", (n, ls, hkv, d), torch.bfloat16, dev)
        v_full = self._buf("v", (n, ls, hkv, d), ops.v_dtype, dev)
        m_full = self._buf("kv", (n, ls), torch.bool, dev)
        h_kv = _Many([ex.gather(k_full, k_own, bulk=True), ex.gather(v_full, v_own, bulk=True),
                      ex.gather(m_full, m_own, bulk=True)])
        # 4. local window attention over [left halo | own rows | right halo]
        h_halo.wait()
        mark("halo_wait")
        local_out, local_lse = ops.local(q, k_h, v_h, m_h, left)
        mark("local_attention")
        # 5. routing over all C chunks
        h_sum.wait()
        mark("summaries_wait")
        idx, rw, lw = ops.route(route_q, lmk_full.view(1, C, hkv, g, d), local_lse,
                                prior_full.view(1, C, hkv, g), ok_full.view(1, C), r * ls)
        mark("route")
        # 6. selected chunks anywhere in the sequence, fused with the local branch
        h_kv.wait()
        mark("kv_wait")
        res = ops.selected(q, k_full.view(1, L, hkv, d), v_full.view(1, L, hkv, d), rw, idx,
                           m_full.view(1, L), local_out, lw, out)
        mark("selected_attention")
        return res

    __call__ = forward

    def stage_times(self, *args, reps: int = 5):
        """Average device milliseconds of each stage of this rank's forward
        (CUDA events on the current stream; the ``*_wait`` entries are the
        time the stream stalled on a transfer)."""
        names = ("start",) + self.STAGES
        tot = {n: 0.0 for n in self.STAGES}
        align = getattr(self.exchange, "align", None)
        for it in range(reps + 1):
            ev = {n: torch.cuda.Event(enable_timing=True) for n in names}
            if align is not None:
                align()
            self.forward(*args, events=ev)
            torch.cuda.synchronize()
            if it == 0:
                continue
            for a, bn in zip(names[:-1], names[1:]):
                tot[bn] += ev[a].elapsed_time(ev[bn])
        return {n: v / reps for n, v in tot.items()}


class ShardedSWALayer:
    """Bidirectional sliding-window (SWA) layer whose rows are sharded across
    ``group``: RoPE on this rank's rows, a ``window``-row halo of K and V from
    each neighbour, window attention over ``[left | own | right]``
    (``dream_dllm_hils/attention.py:1168-1220``: window 1280, landmarks as
    ordinary keys).  Any batch size; inputs are this rank's ``[B, L/N, ...]``
    rows."""

    def __init__(self, window: int = 1280, group=None, exchange=None, cfg=None, ops=None):
        from .layer import RouteLayerConfig

        self.cfg = cfg or RouteLayerConfig()
        self.window = int(window)
        self.exchange = exchange if exchange is not None else GroupExchange(group)
        self.world, self.rank = self.exchange.world, self.exchange.rank
        c = self.cfg
        inv, af = yarn_inv_freq(c.head_dim, c.rope_theta, c.yarn_factor, c.yarn_orig_max_pos)
        self.inv_freq, self.attention_factor = inv, af
        self.ops = ops
        self._bufs = {}

    def _buf(self, name, shape, dtype, device):
        t = self._bufs.get(name)
        if t is None or t.shape != torch.Size(shape) or t.dtype != dtype or t.device != device:
            t = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = t
        return t

    def forward(self, q_pre, k_pre, v, position_ids, key_valid=None, return_lse: bool = False):
        c, ex = self.cfg, self.exchange
        b, ls, hq, d = q_pre.shape
        hkv = k_pre.shape[2]
        n, r = self.world, self.rank
        h = halo_rows(self.window, c.chunk)
        if ls % c.chunk:
            raise ValueError(f"per-rank length {ls} must be a multiple of {c.chunk}")
        if n > 1 and ls < h:
            raise ValueError(f"per-rank length {ls} is shorter than the {h}-row halo")
        dev = q_pre.device
        if key_valid is None:
            key_valid = torch.ones(b, ls, dtype=torch.bool, device=dev)
        left = h if r > 0 else 0
        rows = left + ls + (h if r < n - 1 else 0)
        k_h = self._buf("k", (b, rows, hkv, d), torch.bfloat16, dev)
        m_h = self._buf("m", (b, rows), torch.bool, dev)
        k_own, m_own = k_h[:, left:left + ls], m_h[:, left:left + ls]
        v_dtype = self.ops.v_dtype if self.ops is not None else torch.float16
        v_h = self._buf("v", (b, rows, hkv, d), v_dtype, dev)
        if self.ops is not None:                 # stage ops supplied by the caller (CPU tests)
            q = self.ops.rope(q_pre, k_pre, position_ids, k_own)
            v_h[:, left:left + ls].copy_(self.ops.attention_v(v))
        else:
            inv = self.inv_freq.to(dev)
            q, k_r = yarn_rope_qk(q_pre, k_pre, position_ids, inv, self.attention_factor)
            k_own.copy_(k_r)
            v_h[:, left:left + ls].copy_(to_f16(v))
        m_own.copy_(key_valid.to(torch.bool))
        ex.halo((k_h, v_h, m_h), ls, h).wait()
        if self.ops is not None:
            out, lse = self.ops.local(q, k_h, v_h, m_h, left, window=self.window, skip_inert=False,
                                      need_lse=return_lse)
        else:
            out, lse = window_attention(q, k_h, v_h, m_h, self.window, skip_inert=False, chunk=c.chunk,
                                        q_offset=left, need_lse=return_lse)
        return (out, lse) if return_lse else out

    __call__ = forward
