"""Fast-dLLM cached decode step on the B200 kernels.

``cached_route_layer_step`` is ``dream_dllm_hils/fastdllm_attention.py:70-382
cached_attention_forward`` for the HiLS route layer, and
``cached_swa_layer_step`` its sliding-window branch (``:227-244``): partial
query rows at physical cache positions, the K/V cache updated at the owned
positions, landmark summaries refreshed for the affected chunks, and the
attention output (the input of ``o_proj``) for the query rows.  Every step
runs on this package's kernels:

* RoPE of the partial q / k (``mrsa_rope`` from position ids);
* the local branch at arbitrary cache positions (``mrsa_local_attention_positions``);
* Q-Cal of the partial rows (``mrsa_qcal_route_query``);
* the landmark refresh of the affected chunks (``mrsa_chunk_pool`` with the
  prior fused: ``entropy * entropy_bias_scale``);
* the drop mask rows of the query positions (``mrsa_remote_drop_mask_positions``);
* routing with the route weights fused (``mrsa_route_topk``; the cached path
  normalises remote and local with one softmax: ``_route_weights_torch``
  with no gate, temperature 1, or ``route_weights`` for top-k < 32 -- the
  same function);
* selected attention with the local branch merged in its epilogue
  (``mrsa_selected_attention``, bf16 V: the cache's V is not converted).

``LayerKVCache`` mirrors ``dream_dllm_hils/fastdllm_cache.py:10-127``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .layer import RouteLayer
from .local_attention import positions_window_attention
from .rope_fp32 import yarn_inv_freq, yarn_rope_qk
from .routing import _route
from .selected_attention import selected_attention


@dataclass
class LayerKVCache:
    """One layer's Fast-dLLM cache (``dream_dllm_hils/fastdllm_cache.py:10``):
    RoPE'd keys and values ``[1, L, 4, D]``, key validity ``[1, L]`` bool and,
    for route layers, landmark keys ``[1, C, 4, 7, D]`` and prior bias
    ``[1, C, 4, 7]`` fp32."""

    key: torch.Tensor
    value: torch.Tensor
    key_valid: torch.Tensor
    landmark_keys: torch.Tensor | None = None
    prior_bias: torch.Tensor | None = None

    def __post_init__(self) -> None:
        # mirrors dream_dllm_hils/fastdllm_cache.py:20-95
        if self.key.ndim != 4 or self.value.shape != self.key.shape:
            raise ValueError("key and value must have identical [B,L,Hkv,D] shape")
        if self.key.shape[0] != 1:
            raise ValueError("Fast-dLLM cache currently requires batch size one")
        if self.key.dtype != self.value.dtype:
            raise ValueError("key and value dtype must match")
        if self.key.device != self.value.device:
            raise ValueError("key and value device must match")
        if self.key_valid.shape != self.key.shape[:2]:
            raise ValueError("key_valid shape must match the cache batch and sequence")
        if self.key_valid.dtype != torch.bool:
            raise ValueError("key_valid must be boolean")
        if (self.landmark_keys is None) != (self.prior_bias is None):
            raise ValueError("landmark_keys and prior_bias must be provided together")
        if self.landmark_keys is not None:
            b, _, hkv, dim = self.key.shape
            if self.landmark_keys.ndim != 5 or self.landmark_keys.shape[0] != b or \
                    self.landmark_keys.shape[2] != hkv or self.landmark_keys.shape[4] != dim:
                raise ValueError("landmark_keys must have shape [B,C,Hkv,G,D]")
            if self.prior_bias.shape != self.landmark_keys.shape[:-1]:
                raise ValueError(f"prior_bias must have shape {tuple(self.landmark_keys.shape[:-1])}, "
                                 f"got {tuple(self.prior_bias.shape)}")
            if self.landmark_keys.dtype != self.key.dtype:
                raise ValueError("landmark_keys and K/V dtype must match")

    @property
    def physical_length(self) -> int:
        return int(self.key.shape[1])

    def replace(self, positions: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
        """Overwrite K/V at ``positions`` (``fastdllm_cache.py:100-127``)."""
        positions = positions.to(device=self.key.device, dtype=torch.long)
        if positions.ndim != 1:
            raise ValueError("cache update positions must be one-dimensional")
        if torch.unique(positions).numel() != positions.numel():
            raise ValueError("cache update positions must be unique")
        if bool(((positions < 0) | (positions >= self.physical_length)).any()):
            raise ValueError("cache update positions must be in range")
        expected = (self.key.shape[0], positions.numel(), self.key.shape[2], self.key.shape[3])
        if key.shape != expected or value.shape != expected:
            raise ValueError(f"replacement K/V shape must be {expected}, got "
                             f"{tuple(key.shape)} and {tuple(value.shape)}")
        if key.dtype != self.key.dtype or value.dtype != self.value.dtype:
            raise ValueError("replacement K/V dtype must match the cache")
        self.key.index_copy_(1, positions, key)
        self.value.index_copy_(1, positions, value)


@dataclass(frozen=True)
class CachedAttentionStats:
    """``fastdllm_attention.py:27-31``."""

    updated_positions: torch.Tensor
    refreshed_chunks: torch.Tensor
    routing_calls: int


class _Checks:
    """The validation of a cached step, read back from the GPU once.

    The reference checks its position tensors one condition at a time, each
    with a host read (``fastdllm_attention.py:34-65``, ``fastdllm_cache.py:100-127``):
    about ten synchronisations per layer step.  Here each condition that needs
    the tensors' values is a 0-dim bool on the device, the conditions known on
    the host are plain bools, and ``settle()`` reads every pending device
    condition in one transfer and raises the first failure in the order the
    reference checks them: same exception, same message."""

    def __init__(self):
        self.items = []

    def dev(self, ok: torch.Tensor, msg: str, exc=ValueError) -> None:
        self.items.append((ok, msg, exc))

    def host(self, ok: bool, msg: str, exc=ValueError) -> None:
        """A host-side condition; a failure settles at once (later conditions
        may not even be computable), after any earlier pending failure."""
        self.items.append((bool(ok), msg, exc))
        if not ok:
            self.settle()

    def settle(self) -> None:
        pending = [ok for ok, _, _ in self.items if torch.is_tensor(ok)]
        values = iter(torch.stack(pending).cpu().tolist()) if pending else iter(())
        items, self.items = self.items, []
        for ok, msg, exc in items:
            if not (next(values) if torch.is_tensor(ok) else ok):
                raise exc(msg)


def _positions(p, name, upper, device, ck: _Checks):
    # mirrors fastdllm_attention.py:34-49
    p = p.to(device=device, dtype=torch.long)
    ck.host(p.ndim == 1, f"{name} must be one-dimensional")
    srt = torch.sort(p).values
    ck.dev(~(srt[1:] == srt[:-1]).any(), f"{name} must be unique")
    ck.dev(~((p < 0) | (p >= upper)).any(), f"{name} must be in range")
    return p


def _rows_for(query_positions, owned, ck: _Checks):
    # mirrors fastdllm_attention.py:52-65
    if owned.numel() == 0:
        return owned
    n = query_positions.numel()
    if n == 0:
        ck.host(False, "all owned positions must also be query positions")
    rows = torch.searchsorted(query_positions, owned)
    safe = rows.clamp(max=max(n - 1, 0))
    ck.dev(~(rows >= n).any() & (query_positions.index_select(0, safe) == owned).all(),
           "all owned positions must also be query positions")
    return safe


def _prepare(q_pre, k_pre, v, position_ids, query_positions, kv_update_positions, cache, inv_freq, af):
    ck = _Checks()
    ck.host(q_pre.ndim == 4 and q_pre.shape[0] == 1, "cached attention requires partial queries [1,M,Hq,D]")
    m = q_pre.shape[1]
    dev = q_pre.device
    qp = _positions(query_positions, "query_positions", cache.physical_length, dev, ck)
    ck.host(qp.numel() == m, "query position count must match partial hidden length")
    if m > 1:
        ck.dev(~(qp[1:] <= qp[:-1]).any(), "query_positions must be sorted")
    up = _positions(kv_update_positions, "kv_update_positions", cache.physical_length, dev, ck)
    rows = _rows_for(qp, up, ck)
    ck.host(position_ids.shape == (1, m), f"position_ids must have shape {(1, m)}")
    ck.settle()
    pos = position_ids.to(device=dev, dtype=torch.long).contiguous()
    q, k = yarn_rope_qk(q_pre.contiguous(), k_pre.contiguous(), pos, inv_freq, af)
    kr, vr = k.index_select(1, rows), v.to(cache.value.dtype).index_select(1, rows)
    # LayerKVCache.replace's remaining checks (fastdllm_cache.py:100-127); its
    # unique / in-range conditions are the kv_update_positions ones above
    expected = (cache.key.shape[0], up.numel(), cache.key.shape[2], cache.key.shape[3])
    if kr.shape != expected or vr.shape != expected:
        raise ValueError(f"replacement K/V shape must be {expected}, got "
                         f"{tuple(kr.shape)} and {tuple(vr.shape)}")
    if kr.dtype != cache.key.dtype or vr.dtype != cache.value.dtype:
        raise ValueError("replacement K/V dtype must match the cache")
    cache.key.index_copy_(1, up, kr)
    cache.value.index_copy_(1, up, vr)
    return q, qp, up, pos


@torch.inference_mode()
def cached_route_layer_step(layer: RouteLayer, q_pre, k_pre, v, hidden, position_ids, query_positions,
                            kv_update_positions, affected_chunks, cache: LayerKVCache, *, stages: bool = False):
    """One Fast-dLLM step of a route layer on ``M`` partial rows.

    ``q_pre [1,M,Hq,D]``, ``k_pre``/``v [1,M,Hkv,D]`` (bf16, before RoPE, as
    the module's projections give them), ``hidden [1,M,H]`` (Q-Cal input),
    ``position_ids [1,M]`` (RoPE positions of the rows), ``query_positions``
    ``[M]`` (sorted cache positions), ``kv_update_positions`` (the rows whose
    K/V enter the cache; a subset of ``query_positions``),
    ``affected_chunks`` (chunks whose landmark summary is recomputed; their
    landmark slot must be a query position).  Returns ``(attn [1,M,Hq,D]
    bf16, stats)``, with ``stages=True`` also a dict of the intermediates;
    ``cache`` is updated in place."""
    c = layer.cfg
    if cache.landmark_keys is None or cache.prior_bias is None:
        raise ValueError("HiLS layer cache is missing landmark summaries")
    q, qp, up, pos = _prepare(q_pre, k_pre, v, position_ids, query_positions, kv_update_positions, cache,
                              layer.inv_freq, layer.attention_factor)
    dev = q.device
    _, m, hq, d = q.shape
    hkv = cache.key.shape[2]
    g = hq // hkv
    chunk = c.chunk
    n_chunks = cache.physical_length // chunk
    ck = _Checks()
    aff = _positions(affected_chunks, "affected_chunks", n_chunks, dev, ck)
    lrows = _rows_for(qp, aff * chunk + (chunk - 1), ck) if aff.numel() else aff
    ck.settle()
    kv = cache.key_valid.contiguous()
    # local branch at the rows' cache positions (fastdllm_attention.py:214-224)
    # (the rows' positions were checked above: unique and inside the cache)
    if c.local_window < 0 or chunk <= 0 or cache.physical_length % chunk:
        raise ValueError(f"invalid window/chunk layout: L={cache.physical_length}, W={c.local_window}, S={chunk}")
    local_o, local_lse = positions_window_attention(q, cache.key, cache.value, kv, qp, c.local_window, chunk,
                                                    skip_inert_slots=True)
    # Q-Cal of the partial rows (:252)
    route_q = torch.empty_like(q)
    h = hidden.to(torch.bfloat16).contiguous()
    _lib.call("mrsa_qcal_route_query", _lib.ptr(h), _lib.ptr(q), _lib.ptr(layer.w_in), _lib.ptr(layer.w_out),
              _lib.ptr(layer.norm_weight), float(c.rms_eps), float(c.qcal_scale), _lib.ptr(pos),
              _lib.ptr(layer.inv_freq), float(layer.attention_factor), _lib.ptr(route_q), 1, m, h.shape[-1],
              layer.w_in.shape[0], hq, d, _lib.stream_of(q))
    # landmark refresh of the affected chunks (:254-312)
    if aff.numel():
        mu = route_q.index_select(1, lrows).contiguous()                       # [1, A, Hq, D]
        span = (aff[:, None] * chunk + torch.arange(chunk, device=dev)[None]).reshape(-1)
        keys = cache.key.index_select(1, span).contiguous()                  # [1, A*chunk, Hkv, D]
        valid = kv.index_select(1, span).contiguous()
        na = aff.numel()
        lmk = torch.empty(1, na, hkv, g, d, dtype=cache.landmark_keys.dtype, device=dev)
        ent = torch.empty(1, na, hkv, g, dtype=torch.float32, device=dev)
        prior = torch.empty_like(ent)
        _lib.call("mrsa_chunk_pool", _lib.ptr(mu), na * hq * d, hq * d, _lib.ptr(keys), _lib.ptr(valid),
                  float(d) ** -0.5, _lib.ptr(layer.bias_scale), _lib.ptr(lmk), _lib.ptr(ent), _lib.ptr(prior),
                  None, 1, na, hkv, g, d, _lib.stream_of(q))
        cache.landmark_keys.index_copy_(1, aff, lmk)
        cache.prior_bias.index_copy_(1, aff, prior.to(cache.prior_bias.dtype))
    # drop mask rows of the query positions (:279-283)
    drop = torch.empty(1, m, n_chunks, dtype=torch.int32, device=dev)
    _lib.call("mrsa_remote_drop_mask_positions", _lib.ptr(kv), _lib.ptr(qp), _lib.ptr(drop), 1,
              cache.physical_length, m, c.local_window, chunk, _lib.stream_of(q))
    # routing + route weights, one softmax over remote and local (:284-310)
    lmk_all = cache.landmark_keys.reshape(1, n_chunks, hq, d)
    idx, _, rw, lw = _route(route_q.view(1, m, hkv, g, d), lmk_all, local_lse, c.topk, drop,
                            cache.prior_bias.contiguous(), torch.bfloat16,
                            weights=(_lib.WEIGHTS_SOFTMAX, 1.0, 1.0, 0.0))
    # selected attention, local branch merged (:347-361)
    out = selected_attention(q, cache.key, cache.value, rw, idx, kv, chunk=chunk, local_out=local_o,
                             local_weight=lw)
    stats = CachedAttentionStats(updated_positions=up.clone(), refreshed_chunks=aff.clone(), routing_calls=1)
    if stages:
        return out, stats, {"q": q, "route_q": route_q, "local_out": local_o, "local_lse": local_lse,
                            "drop": drop, "indices": idx, "remote_weights": rw, "local_weight": lw}
    return out, stats


@torch.inference_mode()
def cached_swa_layer_step(q_pre, k_pre, v, position_ids, query_positions, kv_update_positions,
                          cache: LayerKVCache, *, window: int = 1280, chunk: int = 64, inv_freq=None,
                          attention_factor=None):
    """The sliding-window branch of the cached step
    (``fastdllm_attention.py:214-244``): RoPE, cache update, local rows."""
    dev = q_pre.device
    if inv_freq is None:
        inv, af = yarn_inv_freq(q_pre.shape[-1], 1.0e6, 8.0, 2048)
        inv_freq, attention_factor = inv.to(dev), af
    q, qp, up, _ = _prepare(q_pre, k_pre, v, position_ids, query_positions, kv_update_positions, cache,
                            inv_freq, attention_factor)
    if window < 0 or chunk <= 0 or cache.physical_length % chunk:
        raise ValueError(f"invalid window/chunk layout: L={cache.physical_length}, W={window}, S={chunk}")
    out, _ = positions_window_attention(q, cache.key, cache.value, cache.key_valid.contiguous(), qp, window, chunk,
                                        skip_inert_slots=False)
    return out, CachedAttentionStats(updated_positions=up.clone(), refreshed_chunks=up.new_empty(0),
                                     routing_calls=0)
