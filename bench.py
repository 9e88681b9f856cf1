"""MRSA route-layer forward benchmark (headline metric: route-layer fwd tokens/s, bf16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N=1 runs configs[1]: B=1, L=16384 (256 chunks), 28/4 heads, d=128, Q-Cal
hidden 3584 / rank 64, top-32 of 64-token chunks + local radius 256, YaRN-8
fp32 RoPE, seeded N(0,1) activations (N(0,1)/sqrt(128) for q/k/v).  N>1
(torchrun) shards one sequence of L = 16384*N tokens into contiguous query
blocks of 16384 per GPU (N=8: configs[4], L=131072), i.e. weak scaling in
query rows: a halo exchange with the neighbours, an all-gather of the chunk
summaries and an all-gather of K/V on its own communicator, hidden behind
the local window attention and routing.  A step is one route-layer forward
from the projected q/k/v/h to the o_proj input.  Inputs (q 117 MB + h 117 MB
+ k/v 33 MB per 16k tokens) are larger than L2 (126 MB).  Every arm draws
the same inputs from seeded CPU generators (:func:`make_inputs`).

``--impl reference`` times the reference's PyTorch path restated on the CPU
(``oracle/``; the reference is Python and its checkout is not on the GPU
host) with all host threads, on rank 0 only: every timed step computes a
disjoint share of the layer's query rows (the whole layer at N=1), the
stages all rows share inside the first step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L_PER_GPU = 16384
HQ, HKV, D, HIDDEN, RANK, TOPK, CHUNK, WLOC = 28, 4, 128, 3584, 64, 32, 64, 256
METRIC = "MRSA route-layer fwd tokens/s (bf16)"
# this repository's kernels per forward: RoPE, V to fp16, local window, Q-Cal,
# landmark pool, routing keys, top-K selection, selected attention
LAUNCHES_PER_STEP = 8


def algorithmic(l_local: int, l_total: int):
    """Algorithmic FLOPs of one route-layer forward over ``l_local`` query rows
    with ``l_total`` keys: selected 4*L*Hq*K*S*D (S = 64 slots, the masked
    landmark column included), local 4*Hq*D per (query, key) pair within
    256 + 63, routing 2*L*Hq*C*D per pass, Q-Cal 2*L*(hidden*rank + rank*Hq*D)."""
    c = l_total // CHUNK
    f_sel = l_local * HQ * TOPK * CHUNK * D * 4
    w = WLOC + CHUNK - 1
    band = l_local * (2 * w + 1) - (w * (w + 1) if l_local == l_total else 0)
    f_loc = HQ * D * 4 * band
    f_route = l_local * HQ * c * D * 2
    f_qcal = l_local * (HIDDEN * RANK * 2 + RANK * HQ * D * 2)
    return {"selected_attention": f_sel, "local_attention": f_loc, "route": 2 * f_route,
            "qcal": f_qcal, "route_one_pass": f_route}


def stage_bytes(l: int):
    """Compulsory HBM bytes of the memory-bound stages."""
    c = l // CHUNK
    return {"rope": l * (HQ + HKV) * D * 2 * 2,
            "pool": l * HKV * D * 2 + c * HQ * D * 2 * 2 + c * HQ * 8,
            "qcal": l * HIDDEN * 2 + 2 * l * HQ * D * 2}


# DRAM bytes (read + write) of one launch of the dominant kernel, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum) of this bench's own
# single-GPU workload; kept under profiles/ with the command that produced it.
# Keyed by (kernel, query rows per GPU, total keys); other workloads report null.
MEASURED_TRAFFIC = {("selected_attention", 16384, 16384): 331471360 + 99500288}


def selected_items(indices: torch.Tensor, chunks: int, qb: int = 32, own: int = 8):
    """Work items of the selected-attention kernel for these chunk lists: per
    block of ``qb`` queries and KV head, one item per (chunk, up to ``own``
    owner queries).  Returns (items, owner-chunk pairs)."""
    b, l, hkv, k = indices.shape
    nb = (l + qb - 1) // qb
    idx = torch.full((b, nb * qb, hkv, k), -1, dtype=torch.int64, device=indices.device)
    idx[:, :l] = indices.long()
    idx = idx.view(b, nb, qb, hkv, k).permute(0, 1, 3, 2, 4).reshape(b * nb * hkv, qb * k)
    # owner count per (block, head, chunk): each query counts a chunk once
    keyed = torch.where(idx >= 0, idx, torch.full_like(idx, chunks))
    hist = torch.zeros(idx.shape[0], chunks + 1, dtype=torch.int32, device=idx.device)
    qid = torch.arange(qb, device=idx.device).repeat_interleave(k).expand_as(idx)
    flat = keyed * qb + qid                              # (chunk, query) pairs, deduplicated per row
    flat = torch.sort(flat, dim=1).values
    first = torch.ones_like(flat, dtype=torch.bool)
    first[:, 1:] = flat[:, 1:] != flat[:, :-1]
    hist.scatter_add_(1, flat // qb, first.to(torch.int32))
    hist = hist[:, :chunks]
    items = int(((hist + own - 1) // own).sum().item())
    return items, int(hist.sum().item())


def gather_peak_gbs(lib, k, v, q, owners: int, items_per_cta: int, reps: int = 5):
    """Measured L2 -> shared-memory ceiling of the selected kernel's loads:
    ``mrsa_probe_tile_gather`` on the kernel's own K, V and query operands
    (L2-resident), one CTA per SM loading K+V tiles and ``owners`` query boxes
    per item and computing nothing.  GB/s, CUDA events on this stream."""
    dev = k.device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    stream = torch.cuda.current_stream(dev)
    b, lk, hkv, d = k.shape
    q_rows = q.numel() // d

    def launch():
        rc = lib.mrsa_probe_tile_gather(k.data_ptr(), v.data_ptr(), q.data_ptr(), b * lk, hkv, q_rows, owners,
                                        items_per_cta, status.data_ptr(), stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"mrsa_probe_tile_gather: {lib.mrsa_strerror(rc).decode()}")

    for _ in range(2):
        launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if int(status.item()) != 0:
        raise RuntimeError("tile-gather probe gave up on a bounded wait")
    moved = sms * items_per_cta * (32768 + 2048 * owners) * reps
    return moved / (e0.elapsed_time(e1) * 1e-3) / 1e9


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(l_local: int, rank: int, seed: int = 0):
    """Seeded synthetic inputs of rank ``rank``'s rows, on the host (bf16).

    A CPU generator seeded ``seed + rank`` draws, in this order, h
    ``[1,l,3584]`` ~ N(0,1), q ``[1,l,28,128]``, k and v ``[1,l,4,128]`` ~
    N(0,1)/sqrt(128) (the distributions of configs[0]); a second generator
    seeded 7 draws the weights every rank shares: Q-Cal W_in ``[64,3584]``,
    W_out ``[3584,64]`` and the landmark role offset ``[3584]`` ~ N(0,0.02),
    the offset added to h at landmark slots (63 mod 64).  Position ids follow
    the landmark layout (slot i -> i - i//64); every key is valid."""
    g = torch.Generator().manual_seed(seed + rank)
    h = torch.randn(1, l_local, HIDDEN, generator=g)
    q = torch.randn(1, l_local, HQ, D, generator=g).div_(math.sqrt(D)).bfloat16()
    k = torch.randn(1, l_local, HKV, D, generator=g).div_(math.sqrt(D)).bfloat16()
    v = torch.randn(1, l_local, HKV, D, generator=g).div_(math.sqrt(D)).bfloat16()
    gw = torch.Generator().manual_seed(7)
    w_in = (torch.randn(RANK, HIDDEN, generator=gw) * 0.02).bfloat16()
    w_out = (torch.randn(HQ * D, RANK, generator=gw) * 0.02).bfloat16()
    role = torch.randn(HIDDEN, generator=gw) * 0.02
    i = torch.arange(rank * l_local, (rank + 1) * l_local)
    h[0, (i + 1) % CHUNK == 0] += role                        # landmark role offset
    h = h.bfloat16()
    pos = (i - i // CHUNK).view(1, -1).contiguous()
    valid = torch.ones(1, l_local, dtype=torch.bool)
    return {"q_pre": q, "k_pre": k, "v": v, "hidden": h, "position_ids": pos, "key_valid": valid,
            "w_in": w_in, "w_out": w_out}


def bench_config(l_total: int, lq: int, world: int):
    """The ``config`` object of both arms' JSON lines."""
    return {"workload": (f"route-layer fwd B=1 L={l_total} (query blocks of {lq} per GPU) "
                         "28/4 heads d=128 top-32x64 + local-256, Q-Cal 3584->64, YaRN-8"),
            "global_batch": 1, "seq_len": l_total, "parallelism": f"seq{world}",
            "l2": "inputs larger than L2 (267 MB per 16k tokens)"}


def _oracle_inputs(parts, orc):
    """The oracle's input dict for the whole sequence from the ranks' parts."""
    def cat(name):
        return torch.cat([p[name] for p in parts], dim=1)

    return {"q_pre": cat("q_pre"), "k_pre": cat("k_pre"), "v": cat("v"), "hidden": cat("hidden"),
            "position_ids": cat("position_ids"), "key_valid": cat("key_valid"),
            "w_in": parts[0]["w_in"], "w_out": parts[0]["w_out"],
            "norm_weight": torch.ones(D), "entropy_bias_scale": torch.ones(HQ),
            "gate_offset": 0.0, "gate_scale": 1.0}


def cpu_layer_sample(inp, shares, orc):
    """The oracle route layer on the query-row ``shares`` (a list of slices,
    one per step): the stages every row shares (RoPE of K, Q-Cal of the
    landmark and sampled rows, landmark pool, prior) inside the first step,
    then each share's rows.  Returns the seconds of each step."""
    cfg = orc.MRSAConfig()
    l = inp["q_pre"].shape[1]
    rows = torch.zeros(l, dtype=torch.bool)
    for sl in shares:
        rows[sl] = True
    rows[CHUNK - 1::CHUNK] = True
    times, shared = [], None
    for sl in shares:
        t0 = time.perf_counter()
        if shared is None:
            shared = orc.route_layer_shared(inp, cfg, rows=rows)
        orc.route_layer_rows(inp, shared, cfg, sl, keep=False)
        times.append(time.perf_counter() - t0)
    return times


def _cpu_model():
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in out.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return None


def _shares(l_total: int, n_queries: int, steps: int):
    """``steps`` disjoint query-row slices spread evenly over the sequence,
    ``n_queries`` rows in all (with ``n_queries == l_total``: the whole
    sequence, the remainder rows spread one each over the first slices)."""
    if n_queries >= l_total:
        bounds = [l_total * s // steps for s in range(steps + 1)]
        return [slice(bounds[s], bounds[s + 1]) for s in range(steps)]
    per = max(1, n_queries // steps)
    stride = l_total // steps
    return [slice(s * stride, s * stride + per) for s in range(steps)]


def run_reference(args, world, rank):
    """Reference arm: the oracle port on the host cores, rank 0 only.

    Each timed step computes a disjoint share of the route layer's query rows
    on the GPU arm's inputs: at N=1 the shares cover every row, so the timed
    region computes the whole layer once; at N>1 (L = 16384 N) they cover
    16384 rows spread over the sequence, which bounds the run."""
    if rank != 0:
        return
    from oracle import route_layer as orc

    lq = args.seq_per_gpu
    l_total = lq * world
    torch.set_num_threads(os.cpu_count() or 1)
    inp = _oracle_inputs([make_inputs(lq, r) for r in range(world)], orc)
    n_q = l_total if world == 1 else min(l_total, L_PER_GPU)
    for i in range(max(1, args.warmup)):                 # warm-up: small shares
        cpu_layer_sample(inp, [slice(i * 64, i * 64 + 32)], orc)
    shares = _shares(l_total, n_q, args.steps)
    times = cpu_layer_sample(inp, shares, orc)
    total = sum(times)
    rows = sum(sl.stop - sl.start for sl in shares)
    value = rows / total
    cores = torch.get_num_threads()
    sample = (f"oracle route layer at L={l_total}: {args.steps} timed steps of ~{rows // args.steps} disjoint "
              f"query rows ({rows} rows{', the whole layer' if rows == l_total else ''}); the stages all rows "
              "share (K RoPE, landmark Q-Cal, pool, prior) inside the first step")
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": bench_config(l_total, lq, world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample, "cpu_count": os.cpu_count(), "cpu_model": _cpu_model()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if world == 1:
        # fp32 storage, B=1, L=4096, the whole layer, median of 3 after one warm-up
        cfg = orc.MRSAConfig()
        inp0 = orc.make_route_layer_inputs(1, 4096, cfg, hidden=HIDDEN, seed=0, dtype=torch.float32)
        runs = []
        for _ in range(4):
            t0 = time.perf_counter()
            orc.route_layer_forward(inp0, cfg, keep=False)
            runs.append(time.perf_counter() - t0)
        med = statistics.median(runs[1:])
        line["configs0"] = {"workload": "route-layer fwd, fp32 storage, B=1 L=4096 28/4 heads d=128 (oracle port)",
                            "value": 4096 / med, "unit": "tokens/s", "ms_per_forward": 1e3 * med,
                            "runs_s": runs[1:], "threads": cores, "cpu_count": os.cpu_count(),
                            "cpu_model": _cpu_model()}
    print(json.dumps(line), flush=True)


def _flex_pairs(l: int, window: int, chunk: int) -> int:
    """Visible (query, key) pairs of the causal chunk-expanded window with the
    landmark slots masked (training layout, Lq = Lk = l)."""
    i = torch.arange(l, dtype=torch.int64)
    start = torch.div(i - window + 1, chunk, rounding_mode="floor").mul(chunk).clamp(min=0)
    # landmarks (j+1) % chunk == 0 in [start, i]: floor((i+1)/chunk) - floor(start/chunk)
    lmk = torch.div(i + 1, chunk, rounding_mode="floor") - torch.div(start, chunk, rounding_mode="floor")
    return int((i - start + 1 - lmk).sum())


def run_ops(args):
    """``--op``: one JSON line per off-path op at Dream shapes (one GPU), timed
    with CUDA events after warm-up; inputs are regenerated per op."""
    import __graft_entry__

    mrsa = __graft_entry__.load_package()
    mrsa.load_library()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, tflops, peak_kind = load_peaks()
    g = torch.Generator(device=dev).manual_seed(11)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).bfloat16()

    def timed(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    def emit(op, workload, ms, unit_count, unit, bound, work, l2_note, launches=1):
        if bound == "tensor":
            ach = work / (ms * 1e-3) / 1e12
            roof = {"bound": "tensor", "achieved": ach, "peak": tflops, "unit": "TFLOP/s",
                    "frac": ach / tflops, "traffic": None, "peak_kind": f"{peak_kind} bf16 burst"}
        else:
            ach = work / (ms * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                    "traffic": None, "peak_kind": f"{peak_kind} HBM copy"}
        print(json.dumps({"op": op, "metric": f"{op} {unit}/s", "value": unit_count / (ms * 1e-3),
                          "unit": f"{unit}/s", "ms_per_call": ms, "higher_is_better": True,
                          "dtype": "bf16", "data": "synthetic", "n_gpus": 1,
                          "config": {"workload": workload, "l2": l2_note}, "roofline": roof,
                          "gpu_launches_per_call": launches}), flush=True)

    ops = (["swa", "flex", "cached_local", "token_scores", "dsa", "selected_keep"] if args.op == "all"
           else [args.op])
    L = L_PER_GPU
    if "swa" in ops:
        # one bidirectional SWA-1280 layer, B=4, L=16384 (RoPE + window attention)
        bsz, w = 4, 1280
        qp, kp = rnd(bsz, L, HQ, D, scale=D ** -0.5), rnd(bsz, L, HKV, D, scale=D ** -0.5)
        v = rnd(bsz, L, HKV, D, scale=D ** -0.5)
        i = torch.arange(L, device=dev)
        pos = (i - i // CHUNK).expand(bsz, L).contiguous()
        valid = torch.ones(bsz, L, dtype=torch.bool, device=dev)
        inv, af = mrsa.yarn_inv_freq(D, 1.0e6, 8.0, 2048)
        inv = inv.to(dev)

        def swa():
            q, k = mrsa.yarn_rope_qk(qp, kp, pos, inv, af)
            return mrsa.window_attention(q, k, mrsa.to_f16(v), valid, w, skip_inert=False, chunk=CHUNK,
                                         need_lse=False)

        ms = timed(swa, args.steps)
        pairs = L * (2 * w + 1) - w * (w + 1)
        emit("swa", f"SWA layer fwd B={bsz} L={L} 28/4 heads d=128 radius {w} (RoPE + window, fp16 V)",
             ms, bsz * L, "tokens", "tensor", bsz * HQ * D * 4 * pairs, "inputs larger than L2", launches=3)
        ops = [o for o in ops if o != "swa"]
    if "coherent" in ops:
        # Diagnostic, not a configs[] workload: the route layer at configs[1]'s
        # shape with q, k and h sharing a component that varies slowly along the
        # sequence, so neighbouring queries route to overlapping chunks (as real
        # text does) and each gathered K/V tile serves more owner rows of a
        # query block.
        for mix in (0.0, 0.5, 0.8):
            inp = {n: t.to(dev) for n, t in make_inputs(L, 0).items()}
            if mix > 0:
                gsm = torch.Generator(device=dev).manual_seed(21)
                anchors = torch.randn(L // 256 + 2, HQ, D, device=dev, generator=gsm)
                pos = torch.arange(L, device=dev, dtype=torch.float32) / 256
                i0 = pos.floor().long()
                fr = (pos - i0)[:, None, None]
                smooth = (anchors[i0] * (1 - fr) + anchors[i0 + 1] * fr)[None] / math.sqrt(D)
                qf = inp["q_pre"].float() * (1 - mix) + smooth * mix
                inp["q_pre"] = qf.bfloat16()
                kf = inp["k_pre"].float()
                kf = kf * (1 - mix) + mix * smooth.view(1, L, HKV, HQ // HKV, D).mean(3)
                inp["k_pre"] = kf.bfloat16()
                # the Q-Cal term of the routing query comes from h: h shares a
                # slowly varying component too, or that term stays random
                h_anchor = torch.randn(L // 256 + 2, HIDDEN, device=dev, generator=gsm)
                hs = h_anchor[i0] * (1 - fr[:, :, 0]) + h_anchor[i0 + 1] * fr[:, :, 0]
                inp["hidden"] = (inp["hidden"].float() * (1 - mix) + hs[None] * mix).bfloat16()
            layer = mrsa.RouteLayer(inp["w_in"], inp["w_out"], check_errors=False)
            args = [inp[n] for n in ("q_pre", "k_pre", "v", "hidden", "position_ids")]
            st = layer.stage_times(*args, inp["key_valid"], reps=5)
            idx = layer.forward(*args, inp["key_valid"], stages=True)["indices"]
            items, pairs = selected_items(idx, L // CHUNK)
            ms = st["selected_attention"]
            emit("coherent", f"diagnostic (not a configs[] workload): route layer L={L}, q, k and h mixed "
                 f"{mix:.1f} with a component varying over 256 tokens; selected attention {items} work items, "
                 f"{pairs / items:.2f} owner queries per item", ms, L, "tokens", "tensor",
                 L * HQ * TOPK * CHUNK * D * 4, "inputs larger than L2")
        ops = [o for o in ops if o != "coherent"]
    if "gemm" in ops:
        # Not a configs[] workload: the dense layers of configs[3] (Dream-shaped
        # forward, B=1, L=32768) on the tcgen05 GEMM, torch's cuBLAS GEMM timed
        # beside it for reference.
        from mrsa_b200 import dense

        m = 32768
        x = rnd(m, 3584)
        for name, n, k, mode in (("qkv_proj", 4608, 3584, "plain"), ("o_proj", 3584, 3584, "residual"),
                                 ("gate_up_swiglu", 2 * 18944, 3584, "swiglu"), ("down_proj", 3584, 18944, "residual"),
                                 ("lm_head", 152064, 3584, "plain")):
            a = x if k == 3584 else rnd(m, k)
            w = rnd(n, k, scale=0.02)
            if mode == "plain":
                fn = lambda: dense.linear(a, w)
            elif mode == "residual":
                r = rnd(m, n)
                fn = lambda: dense.linear_residual(a, w, r)
            else:
                fn = lambda: dense.swiglu(a, w)
            reps = max(2, args.steps // (4 if n > 100000 else 1))
            ms = timed(fn, reps)
            ms_ref = timed(lambda: torch.matmul(a, w.t()), reps)
            emit("gemm", f"{name}: M={m} N={n} K={k} bf16 (epilogue {mode}); torch cuBLAS matmul of the same "
                 f"shape {ms_ref:.3f} ms ({2 * m * n * k / ms_ref / 1e9:.0f} TFLOP/s)", ms, m, "rows", "tensor",
                 2 * m * n * k, "operands larger than L2")
        ops = [o for o in ops if o != "gemm"]
    if "backward" in ops:
        # Not a configs[] workload: the backward kernels at configs[1]'s route
        # layer (L=16384, the layer's own routing), gradients of random cotangents.
        inp = {n: t.to(dev) for n, t in make_inputs(L, 0).items()}
        layer = mrsa.RouteLayer(inp["w_in"], inp["w_out"], check_errors=False)
        args5 = [inp[n] for n in ("q_pre", "k_pre", "v", "hidden", "position_ids")]
        st = layer.forward(*args5, inp["key_valid"], stages=True)
        q, k, v = st["q"], st["k"], inp["v"]
        idx, w = st["indices"], st["remote_weights"]
        go = rnd(1, L, HQ, D)
        valid = inp["key_valid"]
        ms = timed(lambda: mrsa.selected_attention_backward(q, k, v, w, idx, go, valid), args.steps)
        f_sel = L * HQ * TOPK * CHUNK * D * 4
        emit("selected_backward", f"selected-attention backward (dQ, dK, dV, dW) at route-layer L={L}, "
             "28/4 heads, top-32x64, the layer's own routing; work = 2.5 x the forward's FLOPs "
             "(S recomputed, dP, dQ, dK, dV)", ms, L, "tokens", "tensor", 2.5 * f_sel, "inputs larger than L2",
             launches=7)
        lmk = st["lmk"]
        gs = rnd(1, L, HQ, TOPK)
        ms = timed(lambda: mrsa.route_scores_backward(st["route_q"], lmk, idx, gs), args.steps)
        emit("route_scores_backward", f"routing-score backward (dq gather + d_landmarks over the inverted "
             f"index) at L={L}", ms, L, "tokens", "hbm",
             L * HQ * D * (2 + 4) + L * HQ * TOPK * 2 * 2 + L * HQ * D * 2 * TOPK / 8, "inputs larger than L2",
             launches=6)
        c = L // CHUNK
        mu = st["route_q"][:, CHUNK - 1::CHUNK].reshape(1, c, HKV, HQ // HKV, D).contiguous()
        kc = k.view(1, c, CHUNK, HKV, D)
        gl = rnd(1, c, HKV, HQ // HKV, D)
        ge = torch.randn(1, c, HKV, HQ // HKV, device=dev)
        ms = timed(lambda: mrsa.chunk_pool_backward(mu, kc, valid.view(1, c, CHUNK), gl, ge), args.steps)
        emit("pool_backward", f"landmark-pool backward at L={L}", ms, L, "tokens", "hbm", L * HKV * D * 2 * 2,
             "K fits L2 (16.8 MB)", launches=1)
        # the local window's backward (route layer: effective window 319, landmark keys zeroed)
        kv_b = valid
        lo, llse = mrsa.window_attention(q, k, v, kv_b, WLOC + CHUNK - 1, skip_inert=True, chunk=CHUNK)
        gl_lse = torch.randn(1, L, HQ, device=dev)
        ms = timed(lambda: mrsa.window_attention_backward(q, k, v, kv_b, lo, llse, go, gl_lse, window=WLOC + CHUNK - 1,
                                                          skip_inert=True), args.steps)
        pairs_loc = sum(min(L - 1, i + WLOC + CHUNK - 1) - max(0, i - WLOC - CHUNK + 1) + 1 for i in range(L))
        emit("local_backward", f"local-window backward (dQ, dK, dV with the LSE gradient) at route-layer L={L}, "
             "window 319; work = 2.5 x the forward's band FLOPs", ms, L, "tokens", "tensor",
             2.5 * HQ * D * 4 * pairs_loc, "inputs larger than L2", launches=3)
        from mrsa_b200.route_weights import route_weights_backward
        from mrsa_b200 import _lib as mlib

        grw, glw = rnd(1, L, HQ, TOPK), rnd(1, L, HQ)
        ms = timed(lambda: route_weights_backward(st["scores"], idx, st["prior_bias"], st["local_lse"], grw, glw,
                                                  mode=mlib.WEIGHTS_AFFINE), args.steps)
        emit("route_weights_backward", f"route-weights backward (affine gate) at L={L}", ms, L, "tokens", "hbm",
             L * HQ * TOPK * (2 + 2 + 4) + L * HKV * TOPK * 4 + L * HQ * 12, "inputs larger than L2", launches=1)
        ops = [o for o in ops if o != "backward"]
    if "train" in ops:
        # Not a configs[] workload: one training step of configs[1]'s route layer
        # (L=16384, top-32) through the drop-ins under autograd -- RoPE, the local
        # window, Q-Cal (torch, as the reference module computes it), landmark
        # pool, routing, affine-gate route weights, selected attention and the
        # fusion, forward and backward -- with a random output cotangent.
        inp = {n: t.to(dev) for n, t in make_inputs(L, 0).items()}
        inv, af = mrsa.yarn_inv_freq(D, 1.0e6, 8.0, 2048)
        freqs = inp["position_ids"].float()[..., None] * inv.to(dev).float()
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos() * af, emb.sin() * af
        vd = inp["key_valid"]
        gout = rnd(1, L, HQ, D)
        names = ("q_pre", "k_pre", "v", "hidden", "w_in", "w_out")
        leaves = {n: inp[n].clone().requires_grad_() for n in names}
        gate_off, gate_sc = torch.tensor(0.3, device=dev), torch.tensor(1.2, device=dev)
        nc = L // CHUNK

        def train_step():
            for t_ in leaves.values():
                t_.grad = None
            q = mrsa.single_tensor_rope_autograd(leaves["q_pre"], cos, sin)
            k = mrsa.single_tensor_rope_autograd(leaves["k_pre"], cos, sin)
            lo, lse = mrsa.bidir_local_attention(q, k, leaves["v"], vd, WLOC, CHUNK, skip_inert_slots=True)
            t_ = leaves["hidden"] @ leaves["w_in"].t()
            delta = (t_ @ leaves["w_out"].t()).view(1, L, HQ, D)
            comb = (mrsa.single_tensor_rope_autograd(q, cos, -sin).float() + delta.float()).bfloat16()
            cf = comb.float()
            normed = (cf * torch.rsqrt(cf.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16()
            route_q = mrsa.single_tensor_rope_autograd(normed, cos, sin)
            mu = route_q[:, CHUNK - 1::CHUNK].reshape(1, nc, HKV, HQ // HKV, D)
            lmk, ent = mrsa.chunk_attn_pool_gqa(mu, k.view(1, nc, CHUNK, HKV, D), vd.view(1, nc, CHUNK))
            drop = mrsa.remote_drop_mask(vd, WLOC, CHUNK)
            idx, sc = mrsa.route_topk_g7(route_q, lmk, lse.view(1, L, HKV, HQ // HKV), ent, drop, TOPK, CHUNK, WLOC)
            rw, lw = mrsa.route_weights_torch(sc, idx, ent, lse, temperature=1.0, gate_offset=gate_off,
                                              gate_scale=gate_sc)
            remote = mrsa.HiLS_block_M_head(q, k, leaves["v"], rw, idx, key_valid=vd)
            out = mrsa.fuse_hils_outputs(remote, lo, lw)
            out.backward(gout)

        ms = timed(train_step, max(3, args.steps))
        f_sel = L * HQ * TOPK * CHUNK * D * 4
        pairs_loc = sum(min(L - 1, i + WLOC + CHUNK - 1) - max(0, i - WLOC - CHUNK + 1) + 1 for i in range(L))
        f_loc = HQ * D * 4 * pairs_loc
        emit("train", f"route-layer training step (forward + backward through the drop-ins under autograd) at "
             f"L={L}, 28/4 heads, top-32x64 + local-256; work = 3.5 x (selected + local forward FLOPs)",
             ms, L, "tokens", "tensor", 3.5 * (f_sel + f_loc), "inputs larger than L2", launches=None)
        ops = [o for o in ops if o != "train"]
    if "dream" in ops:
        # the whole Dream-shaped forward, B=1, L=32768, random weights
        from mrsa_b200.dream_forward import DreamConfig, DreamForward, landmark_inputs, model_parameters

        cfg = DreamConfig()
        model = DreamForward(cfg, seed=0, device=dev)
        lseq = 32768
        ids, pos, _ = landmark_inputs(1, lseq, cfg, mask_id=cfg.vocab - 1, device=dev)
        valid = torch.ones(1, lseq, dtype=torch.bool, device=dev)
        ms = timed(lambda: model(ids, pos, valid), max(1, args.steps))
        emit("dream", f"Dream-7B-shaped forward B=1 L={lseq}: 28 layers (7 route, 21 SWA-1280), hidden 3584, "
             f"FFN 18944, vocab 152064, {model_parameters(cfg) / 1e9:.2f} B random N(0,0.02) parameters, "
             "logits out", ms, lseq, "tokens", "tensor", lseq * model.flops_per_token(lseq),
             "weights 15 GB and activations larger than L2",
             # this repository's kernels per layer: 2 RMSNorm + 3 projection GEMMs + o_proj + SwiGLU +
             # down_proj, and the attention (8 per route layer; RoPE + V to fp16 + window per SWA
             # layer); the final RMSNorm and lm_head
             launches=28 * 8 + 7 * LAUNCHES_PER_STEP + 21 * 3 + 2)
        ops = [o for o in ops if o != "dream"]
    if "decode" in ops:
        # The Fast-dLLM cached decode step of one route layer
        # (dream_dllm_hils/fastdllm_attention.py:70-382) on a cache of configs[1]'s
        # length: one 32-row decode block in mid-sequence plus the landmark slot
        # of each chunk it touches; RoPE and cache update of the block, the local
        # branch at cache positions, Q-Cal, landmark refresh of the touched chunks,
        # drop-mask rows, routing over all chunks, selected attention with the
        # local merge.  The step validates its positions on the host as the
        # reference does, so its time includes those synchronisations.
        from mrsa_b200.fastdllm import LayerKVCache, cached_route_layer_step

        c = L // CHUNK
        gh = torch.Generator().manual_seed(5)
        w_in = (torch.randn(RANK, HIDDEN, generator=gh) * 0.02).bfloat16().to(dev)
        w_out = (torch.randn(HQ * D, RANK, generator=gh) * 0.02).bfloat16().to(dev)
        layer = mrsa.RouteLayer(w_in, w_out)
        cache = LayerKVCache(rnd(1, L, HKV, D, scale=D ** -0.5), rnd(1, L, HKV, D, scale=D ** -0.5),
                             torch.ones(1, L, dtype=torch.bool, device=dev),
                             rnd(1, c, HKV, HQ // HKV, D, scale=D ** -0.5),
                             torch.zeros(1, c, HKV, HQ // HKV, device=dev))
        blk = torch.arange(L // 2 + 16, L // 2 + 48, device=dev)
        aff = torch.unique(blk // CHUNK)
        qp = torch.unique(torch.cat([blk, aff * CHUNK + CHUNK - 1]))
        m = qp.numel()
        qpre, kpre = rnd(1, m, HQ, D, scale=D ** -0.5), rnd(1, m, HKV, D, scale=D ** -0.5)
        vnew, hid = rnd(1, m, HKV, D, scale=D ** -0.5), rnd(1, m, HIDDEN)
        pos = (qp - qp // CHUNK).view(1, -1)

        def decode():
            return cached_route_layer_step(layer, qpre, kpre, vnew, hid, pos, qp, blk, aff, cache)

        ms = timed(decode, args.steps)
        wf = WLOC + CHUNK - 1
        # compulsory bytes: the selected chunks' K and V, the local window's K and
        # V, every landmark key (routing scores all chunks), the rows' h, q and output
        work = (m * HKV * TOPK * CHUNK * D * 2 * 2 + m * HKV * (2 * wf + 1) * D * 2 * 2 + c * HQ * D * 2
                + m * (HIDDEN + 2 * HQ * D) * 2)
        emit("decode", f"Fast-dLLM cached route-layer step: {m} rows ({blk.numel()}-row block + "
             f"{aff.numel()} landmark slot(s)) against a {L}-token cache, 28/4 heads top-32x64 + local-256",
             ms, m, "rows", "hbm", work, "decode-sized; cache K/V (33 MB) and landmarks stay in L2 across calls",
             launches=8)
        ops = [o for o in ops if o != "decode"]
    for op in ops:
        if op == "flex":
            w = 1280
            q, k, v = rnd(1, L, HQ, D, scale=D ** -0.5), rnd(1, L, HKV, D, scale=D ** -0.5), rnd(1, L, HKV, D)
            ms = timed(lambda: mrsa.flex_attn_tl(q, k, v, w, CHUNK), args.steps)
            emit(op, f"flex_attn_tl fwd B=1 L={L} 28/4 heads d=128 window {w} chunk 64, landmarks masked",
                 ms, L, "tokens", "tensor", HQ * D * 4 * _flex_pairs(L, w, CHUNK),
                 "inputs (q 117 MB + k/v 33 MB) near L2 size; no flush")
        elif op == "cached_local":
            nq = 32
            q = rnd(1, nq, HQ, D, scale=D ** -0.5)
            k, v = rnd(1, L, HKV, D, scale=D ** -0.5), rnd(1, L, HKV, D)
            valid = torch.ones(1, L, dtype=torch.bool, device=dev)
            pos = torch.arange(L // 2, L // 2 + nq, device=dev)
            ms = timed(lambda: mrsa.cached_local_attention(q, k, v, valid, pos, WLOC, CHUNK,
                                                           skip_inert_slots=True), args.steps)
            wf = WLOC + CHUNK - 1
            emit(op, f"cached_local_attention: {nq} decode rows against a {L}-token cache, window {WLOC}+63",
                 ms, nq, "rows", "tensor", HQ * D * 4 * nq * (2 * wf + 1),
                 "decode-sized; the window's K/V stay in L2 across calls")
        elif op == "token_scores":
            k_sel = TOPK
            q, k = rnd(1, L, HQ, D, scale=D ** -0.5), rnd(1, L, HKV, D)
            idx = torch.argsort(torch.rand(1, L, HKV, L // CHUNK, device=dev, generator=g), dim=-1)[..., :k_sel]
            idx = idx.sort(dim=-1).values.to(torch.int32).contiguous()
            valid = torch.ones(1, L, dtype=torch.bool, device=dev)
            ms = timed(lambda: mrsa.candidate_token_scores_gqa(q, k, idx, valid, CHUNK), args.steps)
            out_bytes = L * HKV * k_sel * CHUNK * 4
            emit(op, f"candidate_token_scores_gqa Lq=Lk={L} 28/4 heads K={k_sel} chunk 64 (fp32 scores out)",
                 ms, L, "tokens", "hbm", L * HQ * D * 2 + out_bytes + idx.numel() * 4,
                 f"output {out_bytes >> 20} MB larger than L2")
        elif op == "dsa":
            lq, topk = 4096, 2560
            q = rnd(1, lq, HQ, D, scale=D ** -0.5)
            k, v = rnd(1, L, HKV, D), rnd(1, L, HKV, D)
            idx = torch.randint(0, L, (1, lq, topk), device=dev, generator=g)
            valid = torch.ones(1, lq, topk, dtype=torch.bool, device=dev)
            ms = timed(lambda: mrsa.selected_token_attention_tilelang(q, k, v, idx, valid), args.steps)
            emit(op, f"selected_token_attention_tilelang Lq={lq} Lk={L} 28/4 heads top-{topk} tokens",
                 ms, lq, "tokens", "hbm", lq * HKV * topk * 2 * D * 2,
                 "work = K and V rows gathered per (query, KV head), mostly L2 hits (k/v 33 MB)")
        elif op == "selected_keep":
            q, k, v = rnd(1, L, HQ, D, scale=D ** -0.5), rnd(1, L, HKV, D, scale=D ** -0.5), rnd(1, L, HKV, D)
            c = L // CHUNK
            idx = torch.argsort(torch.rand(1, L, HKV, c, device=dev, generator=g), dim=-1)[..., :TOPK]
            idx = idx.sort(dim=-1).values.to(torch.int32).contiguous()
            w = torch.softmax(torch.randn(1, L, HQ, TOPK, device=dev, generator=g), -1).bfloat16()
            keep = torch.rand(1, L, HKV, TOPK, CHUNK, device=dev, generator=g) > 0.4
            valid = torch.ones(1, L, dtype=torch.bool, device=dev)
            v16 = mrsa.to_f16(v)
            ms = timed(lambda: mrsa.selected_attention(q, k, v16, w, idx, valid, token_keep=keep), args.steps)
            emit(op, f"selected attention with token_keep (60 % kept) L={L} 28/4 heads top-32x64, fp16 V, "
                 "random sorted chunk lists", ms, L, "tokens", "tensor", L * HQ * TOPK * CHUNK * D * 4,
                 "inputs larger than L2")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seq-per-gpu", type=int, default=L_PER_GPU)
    ap.add_argument("--profile", type=int, default=0, metavar="N",
                    help="run N untimed fused layer forwards at the bench workload and exit "
                         "(the target of the ncu captures summarised under profiles/)")
    ap.add_argument("--op", default=None,
                    choices=["flex", "cached_local", "token_scores", "dsa", "selected_keep", "swa", "dream", "coherent",
                             "decode",
                             "backward", "gemm", "train",
                             "all"],
                    help="time one off-path op (or all) instead of the route layer; one JSON line each")
    args = ap.parse_args()
    if args.op:
        return run_ops(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import __graft_entry__

    mrsa = __graft_entry__.load_package()
    mrsa.load_library()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    lq = args.seq_per_gpu
    l_total = lq * world
    host_inp = make_inputs(lq, rank)
    inp = {n: t.to(dev) for n, t in host_inp.items()}
    # device errors (fp16 range of V, bounded waits) are read once after the timed region
    layer = mrsa.RouteLayer(inp["w_in"], inp["w_out"], check_errors=False)
    if world > 1:
        import datetime

        from mrsa_b200.shard import ShardedRouteLayer

        bulk = dist.new_group(list(range(world)), timeout=datetime.timedelta(seconds=120))
        runner = ShardedRouteLayer(layer, bulk_group=bulk)
    else:
        runner = layer
    names = ("q_pre", "k_pre", "v", "hidden", "position_ids", "key_valid")
    x = [inp[n] for n in names]
    out = torch.empty_like(inp["q_pre"])

    def step():
        runner(*x, out=out)

    if args.profile:
        for _ in range(args.profile):
            step()
        torch.cuda.synchronize()
        print(json.dumps({"profile_forwards": args.profile, "seq_per_gpu": lq,
                          "device_error_flags": mrsa._lib.load().mrsa_device_error_flags(1)}))
        return
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    clk = ClockSampler(local) if rank == 0 else None
    if clk:
        clk.start()
        time.sleep(0.3)
    # every rank enters the timed region together (after rank 0's sampler is up)
    if dist:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = clk.stop() if clk else None
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    ms_step = ms / args.steps
    value = l_total / (ms_step / 1e3)

    # ---- e2e through the public API with pinned host buffers ---------------
    # Pipelined as a serving loop would run it: step i's inputs go up on one
    # copy stream while step i-1 computes, and its output comes back on a
    # second copy stream while step i+1 computes (two buffer slots, events
    # keep a slot's inputs until its compute has read them and its output until
    # it has been read back).  Every step's own copies are inside the timed
    # region: it starts before the first upload and ends after the last readback.
    host = [t.cpu().pin_memory() for t in x]
    dev_in = [[torch.empty_like(t) for t in x] for _ in range(2)]
    dev_out = [torch.empty_like(out) for _ in range(2)]
    host_out = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = host_out[0].numel() * host_out[0].element_size()
    s_up, s_comp, s_down = (torch.cuda.Stream(dev) for _ in range(3))
    up_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    down_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        sl = i & 1
        with torch.cuda.stream(s_up):
            if i >= 2:
                s_up.wait_event(comp_done[sl])        # step i-2 has read these inputs
            for d_, h_ in zip(dev_in[sl], host):
                d_.copy_(h_, non_blocking=True)
            up_done[sl].record(s_up)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(up_done[sl])
            if i >= 2:
                s_comp.wait_event(down_done[sl])      # step i-2's output has been read back
            runner(*dev_in[sl], out=dev_out[sl])
            comp_done[sl].record(s_comp)
        with torch.cuda.stream(s_down):
            s_down.wait_event(comp_done[sl])
            host_out[sl].copy_(dev_out[sl], non_blocking=True)
            down_done[sl].record(s_down)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2 = max(3, args.steps // 2)
    e0.record(s_up)
    for i in range(e2):
        e2e_step(i)
    e1.record(s_down)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = t.item()
    e2e_value = l_total / (ms_e2e / e2 / 1e3)

    # ---- per-kernel times, roofline of the dominant kernel -----------------
    hbm, tflops, peak_kind = load_peaks()
    if world == 1:
        stages = layer.stage_times(*x[:5], x[5], reps=5)
    else:
        stages = runner.stage_times(*x, reps=5)
    kernel_stages = {n: v for n, v in stages.items() if not n.endswith("_wait")}
    dom = max(kernel_stages, key=kernel_stages.get)
    dom_ms = stages[dom]
    if dist:                                  # the slowest rank's time for the dominant kernel
        t = torch.tensor([dom_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dom_ms = t.item()
    flops = algorithmic(lq, l_total)
    byts = stage_bytes(lq)
    if dom in ("selected_attention", "local_attention", "route"):
        ach = flops[dom] / (dom_ms * 1e-3) / 1e12
        roof = {"kernel": dom, "bound": "tensor", "achieved": ach, "peak": tflops,
                "unit": "TFLOP/s", "frac": ach / tflops,
                "traffic": MEASURED_TRAFFIC.get((dom, lq, l_total)),
                "traffic_unit": "bytes per launch (ncu DRAM read + write)",
                "peak_kind": f"{peak_kind} bf16 burst"}
    else:
        ach = byts[dom] / (dom_ms * 1e-3) / 1e9
        roof = {"kernel": dom, "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                "frac": ach / hbm, "traffic": None, "peak_kind": f"{peak_kind} HBM copy"}
    if dom == "selected_attention":
        # the gather bound beside the tensor one: the K and V tiles (32 KB) of
        # every work item and each owner's query rows (2 KB) go through L2
        if world == 1:
            idx = layer.forward(*x[:5], x[5], stages=True)["indices"]
        else:
            idx = None
        if idx is not None:
            items, pairs = selected_items(idx, l_total // CHUNK)
            gbytes = items * 32768 + pairs * 2048
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            owners = max(1, round(pairs / items))
            peak_g = gather_peak_gbs(mrsa._lib.load(), x[1], x[2], x[0], owners, -(-items // sms))
            ach_g = gbytes / (dom_ms * 1e-3) / 1e9
            roof["gather"] = {"bound": "l2", "bytes_per_launch": gbytes, "achieved": ach_g, "unit": "GB/s",
                              "peak": peak_g, "frac": ach_g / peak_g, "items": items,
                              "owners_per_item": pairs / items,
                              "peak_kind": (f"measured in this run: mrsa_probe_tile_gather, the kernel's K/V tile "
                                            f"and {owners} query boxes per item from L2, nothing computed")}
    waits = None
    if dist:
        # time each rank's compute stream stalled on a transfer, max over ranks
        w = torch.tensor([stages.get(n, 0.0) for n in ("halo_wait", "summaries_wait", "kv_wait")], device=dev)
        dist.all_reduce(w, op=dist.ReduceOp.MAX)
        waits = dict(zip(("halo_wait_ms", "summaries_wait_ms", "kv_wait_ms"), w.tolist()))

    # ---- device error flags of everything above (fp16 range of V, bounded waits)
    flags = int(mrsa._lib.load().mrsa_device_error_flags(1))

    # ---- N>1: this rank's rows against the single-GPU layer on the whole sequence
    parity = None
    if dist:
        from mrsa_b200.shard import gather_rows

        full = []
        for t in x:
            buf = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=dev)
            gather_rows(buf, t.contiguous())
            full.append(buf.transpose(0, 1).reshape(1, world * t.shape[1], *t.shape[2:]).contiguous())
        ref = layer(*full)
        mine = runner(*x)
        ok = torch.tensor([1.0 if torch.equal(mine, ref[:, rank * lq:(rank + 1) * lq]) else 0.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        parity = {"ok": bool(ok.item() == 1.0),
                  "check": ("every rank's output rows bit-equal to the same rows of the single-GPU fused "
                            f"layer run on the whole L={l_total} sequence (gathered inputs)")}
        del full, ref, mine

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic",
                "config": bench_config(l_total, lq, world),
                "roofline": roof, "stage_ms": stages,
                "gpu_launches": args.steps * LAUNCHES_PER_STEP,
                "clocks": clocks,
                "device_error_flags": flags,
                "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                        "d2h_bytes_per_step": d2h * world, "steps": e2,
                        "pipelining": "step i's upload and readback overlap the compute of steps i-1 and i+1"}}
        if waits is not None:
            line["exchange_wait_ms"] = waits
        if parity is not None:
            line["parity"] = parity
        if world == 1 and not args.no_cpu_baseline:
            from oracle import route_layer as orc

            torch.set_num_threads(os.cpu_count() or 1)
            shares = _shares(l_total, min(l_total, 4096), 4)
            t_cpu = cpu_layer_sample(_oracle_inputs([host_inp], orc), shares, orc)
            n_rows = sum(sl.stop - sl.start for sl in shares)
            line["cpu_baseline"] = {
                "value": n_rows / sum(t_cpu), "unit": "tokens/s", "cores": torch.get_num_threads(),
                "kind": "port",
                "sample": (f"oracle route layer on this run's inputs (L={l_total}): {n_rows} query rows in "
                           f"{len(shares)} slices spread over the sequence plus the stages all rows share, "
                           f"{sum(t_cpu):.1f} s")}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
