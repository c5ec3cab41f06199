"""Benchmark of the INT4-KV decode hot path (Llama-3.1-8B decode, B16, S4096, per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Llama-3.1-8B single-layer decode, B=16, 32 q heads, 8 KV heads,
d=128, context S=4096, INT4 group size 32, bf16 q/K/V, K channels scaled by
log-uniform [0.5, 8] factors, seeded synthetic data.  A step = quantize-append
of the new K/V token + fused decode attention over the S-token INT4 cache,
for one layer, in ONE launch (kv4_append_attention: the attention kernel
quantizes the new row itself).  The timed loop replays a CUDA graph holding
one step per layer (a model's per-token decode graph).  Steps rotate over
layer caches of >= 2.4 GB in total, so every step reads its cache from HBM,
not L2 (126 MB).

With N ranks the KV heads of the one problem are split over the ranks
(rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and their q heads): strong
scaling, no collective on the data path.  `value` = algorithmic bytes of the
whole problem per step / max-over-ranks device time (GB/s).  `e2e` = the same
metric through the public Python API with pinned host q/k/v copied in and the
output copied out every step.  Rank 0 at N=1 also reports the other
workloads (batch-1 long context, the 70B one-KV-head-per-GPU shape) and the
reference's microbenchmark sweeps (B=1, S=512..32K; G=32/64/128) next to the
reference's own Triton kernel.  `--impl reference` times the reference's CPU
formulation (oracle/torch_ref.py) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "kv-cache-triton_b200"))
sys.path.insert(0, ROOT)

# workloads: Llama-3.1-8B decode at batch 16 (default), batch-1 long context
WORKLOADS = {
    "config2": dict(B=16, HQ=32, HKV=8, S=4096),
    "long16k": dict(B=1, HQ=32, HKV=8, S=16384),
    "long64k": dict(B=1, HQ=32, HKV=8, S=65536),
    "long128k": dict(B=1, HQ=32, HKV=8, S=131072),
    # Llama-3.1-70B decode layer (8 GPUs: one KV head and its 8 q heads each)
    "config4": dict(B=32, HQ=64, HKV=8, S=16384),
}
B, HQ, HKV, S, D, G = 16, 32, 8, 4096, 128, 32
LAYERS = 32
METRIC = "INT4-KV decode attention HBM GB/s (Llama-3.1-8B shape, B16, S4096, G32)"


HQ_L, HKV_L = HQ, HKV  # this rank's share of the heads (KV-head sharding)


def attn_bytes(ss=2, qs=2, hq=None, hkv=None):
    """Algorithmic bytes of one decode-attention launch: packed K/V + scales
    over the S-token cache, q read, output written (whole problem unless
    hq/hkv name a share)."""
    hq = HQ if hq is None else hq
    hkv = HKV if hkv is None else hkv
    return 2 * B * hkv * S * (D // 2 + (D // G) * ss) + 2 * B * hq * D * qs


def append_bytes(ss=2, xs=2, hkv=None):
    hkv = HKV if hkv is None else hkv
    return 2 * B * hkv * (D * xs + D // 2 + (D // G) * ss)


def step_bytes(hq=None, hkv=None):
    return attn_bytes(hq=hq, hkv=hkv) + append_bytes(hkv=hkv)


def local_step_bytes():
    return step_bytes(HQ_L, HKV_L)


def set_workload(name, ws=1):
    global B, HQ, HKV, S, LAYERS, METRIC, HQ_L, HKV_L
    w = WORKLOADS[name]
    B, HQ, HKV, S = w["B"], w["HQ"], w["HKV"], w["S"]
    if HKV % ws:
        raise SystemExit(f"{HKV} KV heads do not split over {ws} ranks")
    HQ_L, HKV_L = HQ // ws, HKV // ws
    # enough layer caches to keep ~2.4 GB resident per GPU (>> the 126 MB L2)
    LAYERS = max(2, min(32, -(-2_400_000_000 // attn_bytes(hq=HQ_L, hkv=HKV_L))))
    shape = "Llama-3.1-70B shape" if name == "config4" else "Llama-3.1-8B shape"
    METRIC = f"INT4-KV decode attention HBM GB/s ({shape}, B{B}, S{S}, G{G})"


def workload_config(args, ws):
    """The ``config`` object, identical for both arms of a run."""
    model = "llama3.1-70b" if args.workload == "config4" else "llama3.1-8b"
    return {"workload": f"{args.workload}: {model} single-layer decode step: append 1 token "
                        "+ INT4 decode attention",
            "batch": B, "q_heads": HQ, "kv_heads": HKV, "seq_len": S, "d_head": D,
            "group_size": G,
            "parallelism": (f"kv-head shard x{ws}: {HKV // ws} KV heads and {HQ // ws} q heads "
                            "per rank, no collective") if ws > 1 else "single",
            "l2": "inputs larger than L2: steps rotate over layer caches of >= 2.4 GB per GPU",
            "bytes_per_step": step_bytes()}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, index: int):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    _NAMES = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
              0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self._NAMES.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                break
            time.sleep(0.002)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def build_caches(dev, seed=0, hq=None, hkv=None, layers=None):
    """Layer caches of this rank's heads (full-length INT4 K/V) plus q and the
    new token's K/V per layer."""
    from kvint4.cache import Int4KVStore
    hq = HQ_L if hq is None else hq
    hkv = HKV_L if hkv is None else hkv
    layers = LAYERS if layers is None else layers
    g = torch.Generator(device=dev).manual_seed(seed)
    store = Int4KVStore(G, capacity=S)
    fac = torch.exp(torch.empty(D, device=dev).uniform_(math.log(0.5), math.log(8.0),
                                                        generator=g))
    for layer in range(layers):
        for b0 in range(0, B, 8):  # in batch chunks: bounded bf16 staging
            b1 = min(B, b0 + 8)
            k = (torch.randn(b1 - b0, hkv, S, D, device=dev, generator=g) * fac).to(torch.bfloat16)
            v = torch.randn(b1 - b0, hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
            if b0 == 0:
                store.append(torch.empty(B, hkv, 0, D, device=dev, dtype=torch.bfloat16),
                             torch.empty(B, hkv, 0, D, device=dev, dtype=torch.bfloat16), layer)
            st = store.layer(layer)
            from kvint4 import ops
            ops.append_kv(k, v, st.k_packed_buf[b0:b1], st.k_scales_buf[b0:b1],
                          st.v_packed_buf[b0:b1], st.v_scales_buf[b0:b1], 0, G)
            del k, v
        store.layer(layer).seq_len = S
    q = torch.randn(layers, B, hq, 1, D, device=dev, generator=g).to(torch.bfloat16)
    kn = (torch.randn(layers, B, hkv, 1, D, device=dev, generator=g) * fac).to(torch.bfloat16)
    vn = torch.randn(layers, B, hkv, 1, D, device=dev, generator=g).to(torch.bfloat16)
    return store, q, kn, vn


def run_ours(args, ws, rank, local):
    from kvint4 import ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    store, q, kn, vn = build_caches(dev, seed=rank)
    out = torch.empty(B, HQ_L, 1, D, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev)

    def append_op(l):
        layer = store.layer(l)
        ops.append_kv(kn[l], vn[l], layer.k_packed_buf, layer.k_scales_buf, layer.v_packed_buf,
                      layer.v_scales_buf, S - 1, G)  # the new token is row S-1: context stays S

    def attn_op(l):
        kp, ks, vp, vs = store.layer(l).views()
        ops.attention_into(q[l], kp, ks, vp, vs, out, G, False)

    def step_op(l, early=True):  # the product's decode step: append fused into the attention
        # launch, started early behind the previous layer's step (the cache
        # layer's own decode loop does the same: kv4_attn_opts.early_start)
        kp, ks, vp, vs = store.layer(l).views()
        ops.append_attention_into(q[l], kn[l], vn[l], kp, ks, vp, vs, out, G, False,
                                  early_start=early)

    for l in range(LAYERS):
        store.layer(l).seq_len = S
    p = ops.plan(q[0], *store.layer(0).views(), out, G, False)
    # eager warm-up (caches occupancy queries / smem attributes), then CUDA
    # graphs so the timed loops are device-bound, not host-bound: one graph
    # per layer for the step, and, for comparison, one per layer for the
    # unfused pair (append kernel + attention kernel)
    for l in range(LAYERS):
        step_op(l)
        append_op(l)
        attn_op(l)
    torch.cuda.synchronize()
    # The timed region replays a per-token decode graph: one step per layer
    # for `span` consecutive layers, where span is the largest divisor of
    # --steps up to LAYERS, so that exactly --steps steps run as whole graph
    # replays (a model's per-token graph), whatever --steps is.
    span = max(k for k in range(1, min(LAYERS, args.steps) + 1) if args.steps % k == 0)
    g_all, g_all_pair = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_all):
        for l in range(span):
            step_op(l)
    with torch.cuda.graph(g_all_pair):
        for l in range(span):
            append_op(l)
            attn_op(l)
    g_all_plain = torch.cuda.CUDAGraph()  # fused steps in plain stream order
    with torch.cuda.graph(g_all_plain):
        for l in range(span):
            step_op(l, early=False)
    reps = args.steps // span

    for _ in range(max(1, -(-args.warmup // span))):
        g_all.replay()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        _hold(st)
        t0.record(st)
        for _ in range(reps):
            g_all.replay()
        t1.record(st)
        torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)

    # the same steps unfused (append kernel + attention kernel), for comparison
    for _ in range(max(1, -(-args.warmup // span))):
        g_all_pair.replay()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _hold(st)
    p0.record(st)
    for _ in range(reps):
        g_all_pair.replay()
    p1.record(st)
    torch.cuda.synchronize()
    pair_ms = p0.elapsed_time(p1)
    for _ in range(max(1, -(-args.warmup // span))):
        g_all_plain.replay()
    torch.cuda.synchronize()
    _hold(st)
    p0.record(st)
    for _ in range(reps):
        g_all_plain.replay()
    p1.record(st)
    torch.cuda.synchronize()
    plain_ms = p0.elapsed_time(p1)
    gpu_ref = None
    if not args.no_gpu_reference and ws == 1:
        gpu_ref = triton_reference_leg(store, q, span, reps, args.warmup, st)

    # ---- e2e: public API, pinned host buffers in and out every step ----
    # each step's q, k, v packed in one pinned host row: one copy in per step
    nq, nk = B * HQ_L * D, B * HKV_L * D
    hin = torch.randn(args.steps, nq + 2 * nk).to(torch.bfloat16).pin_memory()
    hout = torch.empty(args.steps, B, HQ_L, 1, D, dtype=torch.bfloat16).pin_memory()
    from models.llama3.kv_cache import QuantizedKVCache
    caches = []
    for l in range(LAYERS):
        c = QuantizedKVCache(group_size=G)
        c._store._layers[0] = store.layer(l)
        caches.append(c)
    din = torch.empty(nq + 2 * nk, dtype=torch.bfloat16, device=dev)
    dq = din[:nq].view(B, HQ_L, 1, D)
    dk = din[nq:nq + nk].view(B, HKV_L, 1, D)
    dv = din[nq + nk:].view(B, HKV_L, 1, D)
    do = torch.empty(B, HQ_L, 1, D, dtype=torch.bfloat16, device=dev)

    def e2e_step(i):
        c = caches[i % LAYERS]
        c._store.layer(0).seq_len = S - 1
        din.copy_(hin[i % args.steps], non_blocking=True)
        o = c.append_attend(dq, dk, dv, 0, do, n_q_heads=HQ_L, n_kv_heads=HKV_L)
        hout[i % args.steps].copy_(o, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    # max over ranks
    t = torch.tensor([ms, e2e_ms, pair_ms, plain_ms], device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.barrier()
    ms, e2e_ms, pair_ms, plain_ms = (float(x) for x in t.tolist())
    # the timed region holds only the fused kernel, one launch per step: its
    # average launch duration is the region's time / launches
    attn_avg_ms = ms / (args.steps * int(p.kernels))
    pair_avg_ms = pair_ms / args.steps
    if rank != 0:
        return None
    peak, peak_kind = _peaks()
    per_step_ms = ms / args.steps
    value = step_bytes() * args.steps / (ms * 1e-3) / 1e9  # whole problem / max-rank time
    achieved = local_step_bytes() / (attn_avg_ms * 1e-3) / 1e9  # per GPU
    h2d = (B * HQ_L * D + 2 * B * HKV_L * D) * 2
    d2h = B * HQ_L * D * 2
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_step_ms, 5),
        "us_per_step": round(per_step_ms * 1e3, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 q/out, int4 KV codes, bf16 scales, fp32 accumulate",
        "data": "synthetic (seeded N(0,1), K channels x log-uniform[0.5,8])",
        "config": workload_config(args, ws),
        "gpu_launches": args.steps * int(p.kernels),
        "e2e": {"value": round(step_bytes() * args.steps / (e2e_ms * 1e-3) / 1e9, 1),
                "unit": "GB/s", "us_per_step": round(e2e_ms * 1e3 / args.steps, 2),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "kv4_attn_fast",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "kernel_us": round(attn_avg_ms * 1e3, 2),
                     "unfused_append_plus_attention_us": round(pair_avg_ms * 1e3, 2),
                     "plain_stream_order_us": round(plain_ms * 1e3 / args.steps, 2),
                     # DRAM bytes come from an ncu capture, not from this run
                     "traffic": None},
        "clocks": clk.summary(),
        "plan": {"path": int(p.path), "ctas": int(p.ctas), "tiles_per_cta": int(p.tiles_per_cta),
                 "kernels_per_attention": int(p.kernels)},
    }
    if gpu_ref is not None:
        line["gpu_reference"] = gpu_ref
    if ws == 1 and not args.no_extra:
        line["workloads"] = extra_workloads(dev, with_reference=not args.no_gpu_reference)
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    return line


class workload_dims:
    """Temporarily switch the module's problem dimensions (extra workloads)."""

    def __init__(self, **kw):
        self.kw = kw

    def __enter__(self):
        g = globals()
        self.saved = {k: g[k] for k in ("B", "HQ", "HKV", "S", "G", "HQ_L", "HKV_L", "LAYERS")}
        g.update(self.kw)
        g["HQ_L"], g["HKV_L"] = g["HQ"], g["HKV"]
        if "LAYERS" not in self.kw:
            g["LAYERS"] = max(2, min(32, -(-2_400_000_000 // attn_bytes())))
        return self

    def __exit__(self, *a):
        globals().update(self.saved)


def _hold(st=None):
    """Keep the stream busy for about 1 ms (a device-side spin) before a timed
    region starts, so that the region's first event and the launches behind
    it are all queued before the GPU reaches them: the region then measures
    device time only, not the host's launch latency or a thread switch."""
    torch.cuda._sleep(2_000_000)


def _graph_time_us(step, span, reps, st):
    """Device time per step of `reps` replays of a graph of `span` steps."""
    for l in range(span):
        step(l)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for l in range(span):
            step(l)
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _hold(st)
    t0.record(st)
    for _ in range(reps):
        graph.replay()
    t1.record(st)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) * 1e3 / (span * reps)


def extra_workloads(dev, with_reference=True):
    """The other workloads (fused append + attention steps, one graph per
    token over >= 2.4 GB of layer caches) and the reference's microbenchmark
    sweeps (attention alone, B=1, 32/8 heads, d=128) beside the reference's
    own Triton kernel on the same caches."""
    from kvint4 import ops
    peak, _ = _peaks()
    st = torch.cuda.current_stream(dev)
    ref_fn = None
    if with_reference:
        try:
            from oracle import triton_ref
            ref_fn = triton_ref.llama3_attention().attention_forward_quant_gqa
        except Exception:
            ref_fn = None
    res = {}
    for name, dims in (("long16k", dict(B=1, HQ=32, HKV=8, S=16384)),
                       ("long64k", dict(B=1, HQ=32, HKV=8, S=65536)),
                       ("long128k", dict(B=1, HQ=32, HKV=8, S=131072)),
                       ("llama70b_one_kv_head_per_gpu", dict(B=32, HQ=8, HKV=1, S=16384))):
        with workload_dims(**dims):
            store, q, kn, vn = build_caches(dev)
            out = torch.empty(B, HQ, 1, D, dtype=torch.bfloat16, device=dev)

            def step(l):
                kp, ks, vp, vs = store.layer(l).views()
                ops.append_attention_into(q[l], kn[l], vn[l], kp, ks, vp, vs, out, G, False,
                                          early_start=True)

            with ClockSampler(dev.index or 0) as clk:
                us = _graph_time_us(step, LAYERS, max(2, 64 // LAYERS), st)
            gbs = step_bytes() / (us * 1e-6) / 1e9
            res[name] = {"B": B, "q_heads": HQ, "kv_heads": HKV, "seq_len": S, "group_size": G,
                         "us_per_step": round(us, 2), "GB/s": round(gbs, 1),
                         "frac": round(gbs / peak, 4), "layers": LAYERS,
                         "clocks": clk.summary()}
            del store, q, kn, vn
            torch.cuda.empty_cache()
    sweeps = []
    points = [(s_, 32) for s_ in (512, 1024, 2048, 4096, 8192, 16384, 32768)]
    points += [(4096, 64), (4096, 128)]
    for s_, g_ in points:
        with workload_dims(B=1, HQ=32, HKV=8, S=s_, G=g_, LAYERS=None):
            globals()["LAYERS"] = max(2, min(64, -(-256_000_000 // attn_bytes())))
            store, q, _, _ = build_caches(dev)
            out = torch.empty(B, HQ, 1, D, dtype=torch.bfloat16, device=dev)

            def attn(l):
                kp, ks, vp, vs = store.layer(l).views()
                ops.attention_into(q[l], kp, ks, vp, vs, out, G, False, early_start=True)

            us = _graph_time_us(attn, LAYERS, max(2, 128 // LAYERS), st)
            row = {"seq_len": S, "group_size": G, "layer_copies": LAYERS,
                   "l2_resident": LAYERS * attn_bytes() < 126e6,
                   "ours_us": round(us, 2),
                   "ours_GB/s": round(attn_bytes() / (us * 1e-6) / 1e9, 1)}
            if ref_fn is not None:
                try:
                    def ref(l):
                        kp, ks, vp, vs = store.layer(l).views()
                        ref_fn(q[l], kp, ks, vp, vs, n_q_heads=HQ, n_kv_heads=HKV, group_size=G)

                    rus = _graph_time_us(ref, LAYERS, max(2, 32 // LAYERS), st)
                    row["reference_triton_us"] = round(rus, 2)
                    row["speedup_vs_reference"] = round(rus / us, 1)
                except Exception as e:  # noqa: BLE001
                    row["reference_triton"] = f"unavailable: {type(e).__name__}"
            sweeps.append(row)
            del store, q
            torch.cuda.empty_cache()
    res["sweep_b1_32q_8kv_d128"] = sweeps
    res["prefill_b1_32q_8kv_d128"] = prefill_workloads(dev, ref_fn)
    return res


def _bf16_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def prefill_workloads(dev, ref_fn=None):
    """Causal prefill attention over the packed cache (one layer, B=1, 32/8
    heads, d=128, G=32, sq = sk): the tensor-core kernel
    (``kv4_prefill_attention``) beside the dequantize + flash-attention route
    and the reference's Triton kernel.  FLOPs counted as 4 * Hq * d * (number
    of visible (query, key) pairs)."""
    from kvint4 import frontend, ops
    st = torch.cuda.current_stream(dev)
    peak, kind = _bf16_peak()
    rows = []
    for s_ in (2048, 8192, 16384):
        with workload_dims(B=1, HQ=32, HKV=8, S=s_, G=32, LAYERS=2):
            store, _, _, _ = build_caches(dev)
            g = torch.Generator(device=dev).manual_seed(5)
            q = torch.randn(LAYERS, B, HQ, S, D, device=dev, generator=g).to(torch.bfloat16)
            out = torch.empty(B, HQ, S, D, dtype=torch.bfloat16, device=dev)
            pairs = B * S * (S + 1) // 2
            flops = 4.0 * HQ * D * pairs

            def ours(l):
                ops.prefill_attention_into(q[l], *store.layer(l).views(), out, G, True)

            def sdpa(l):
                frontend._prefill_sdpa(q[l], *store.layer(l).views(), G, True, out)

            us = _graph_time_us(ours, LAYERS, 4, st)
            row = {"seq_len": S, "ours_us": round(us, 1),
                   "ours_TFLOP/s": round(flops / (us * 1e-6) / 1e12, 1),
                   "frac_of_bf16_peak": round(flops / (us * 1e-6) / 1e12 / peak, 3),
                   "peak_kind": kind}
            try:
                dus = _graph_time_us(sdpa, LAYERS, 4, st)
                row["dequant_sdpa_us"] = round(dus, 1)
                row["speedup_vs_dequant_sdpa"] = round(dus / us, 2)
            except Exception as e:  # noqa: BLE001
                row["dequant_sdpa"] = f"unavailable: {type(e).__name__}"
            if ref_fn is not None:
                try:
                    def ref(l):
                        ref_fn(q[l], *store.layer(l).views(), n_q_heads=HQ, n_kv_heads=HKV,
                               group_size=G, is_causal=True)

                    rus = _graph_time_us(ref, LAYERS, 2, st)
                    row["reference_triton_us"] = round(rus, 1)
                    row["speedup_vs_reference"] = round(rus / us, 2)
                except Exception as e:  # noqa: BLE001
                    row["reference_triton"] = f"unavailable: {type(e).__name__}"
            rows.append(row)
            del store, q, out
            torch.cuda.empty_cache()
    return rows


def triton_reference_leg(store, q, span, reps, warmup, st):
    """Device time of the reference's own fused decode kernel
    (``kernels/llama3/attention_quant.py:24-286`` of johnchmura/kv-cache-triton,
    Triton, unmodified, staged in oracle/_ref) on the same caches, q and
    layer rotation as the timed region above, captured in a CUDA graph the
    same way.  A baseline leg: it reports, it is not the product."""
    try:
        from oracle import triton_ref
        fn = triton_ref.llama3_attention().attention_forward_quant_gqa
    except Exception as e:  # Triton missing, or the files were not staged
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    try:
        def call(l):
            kp, ks, vp, vs = store.layer(l).views()
            return fn(q[l], kp, ks, vp, vs, n_q_heads=HQ, n_kv_heads=HKV, group_size=G)

        for l in range(span):
            call(l)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for l in range(span):
                call(l)
        for _ in range(max(1, -(-warmup // span))):
            graph.replay()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _hold(st)
        t0.record(st)
        for _ in range(reps):
            graph.replay()
        t1.record(st)
        torch.cuda.synchronize()
        us = t0.elapsed_time(t1) * 1e3 / (span * reps)
        import triton
        return {"kernel": "_attention_fwd_quant_gqa_kernel (reference, Triton "
                          f"{triton.__version__}, sm_100)",
                "us_per_step": round(us, 2),
                "value": round(attn_bytes() / (us * 1e-6) / 1e9, 1), "unit": "GB/s",
                "note": "attention only (the reference appends with separate quantize + "
                        "torch.cat launches, not timed here)"}
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}


def _cpu_ref_problem():
    """The full workload (all B sequences, S-1 cached tokens + the new one) on
    host tensors, quantized with the reference's torch path."""
    from oracle import torch_ref
    g = torch.Generator().manual_seed(0)
    fac = torch.exp(torch.empty(D).uniform_(math.log(0.5), math.log(8.0), generator=g))
    k = (torch.randn(B, HKV, S - 1, D, generator=g) * fac).to(torch.bfloat16)
    v = torch.randn(B, HKV, S - 1, D, generator=g).to(torch.bfloat16)
    kp, ks = torch_ref.quantize_int4(k, G)
    vp, vs = torch_ref.quantize_int4(v, G)
    base = {"kp": kp, "ks": ks, "vp": vp, "vs": vs}
    q = torch.randn(B, HQ, 1, D, generator=g).to(torch.bfloat16)
    kn = (torch.randn(B, HKV, 1, D, generator=g) * fac).to(torch.bfloat16)
    vn = torch.randn(B, HKV, 1, D, generator=g).to(torch.bfloat16)
    return lambda: torch_ref.decode_step(dict(base), q, kn, vn, HQ, HKV, G)


_CPU_SAMPLE = ("one decode step of the full workload (B={B}, S={S}) per step through the "
               "reference's torch CPU route: quantize (half-even) + torch.cat append + "
               "dequantize to bf16 + repeat_kv + SDPA in bf16; no extrapolation")


def cpu_baseline(budget_s: float = 15.0):
    """The reference's CPU formulation of the same step, all host threads,
    for about ``budget_s`` seconds (at least 2 steps)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step = _cpu_ref_problem()
    step()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if (el > budget_s and n >= 2) or n >= 200:
            break
    step_s = el / n
    return {"value": round(step_bytes() / step_s / 1e9, 3), "unit": "GB/s",
            "us_per_step": round(step_s * 1e6, 1), "cores": threads, "kind": "port",
            "sample": f"{n} steps; " + _CPU_SAMPLE.format(B=B, S=S)}


def run_reference(args, ws, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    step = _cpu_ref_problem()
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    step_s = el / args.steps
    value = step_bytes() / step_s / 1e9
    sample = _CPU_SAMPLE.format(B=B, S=S)
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 3), "us_per_step": round(step_s * 1e6, 1),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference",
        "config": workload_config(args, ws),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_seq_shard(args, ws, rank, local):
    """Config 3 across ranks: rank r holds tokens shard_range(S, ws, r) of
    every layer's batch-1 cache; a step is the partial attention over the
    local tokens, an NCCL all-gather of (o, lse) and the log-sum-exp combine
    (kvint4/shard.py).  Total work is fixed as ws grows (strong scaling)."""
    import torch.distributed as dist

    from kvint4 import ops, shard
    from kvint4.cache import Int4KVStore
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:  # a short timeout: a rank that stops answering ends the run with an error
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    lo, hi = shard.shard_range(S, ws, rank)
    n = hi - lo
    layers = max(2, min(32, -(-2_400_000_000 // max(1, attn_bytes() // ws))))
    g = torch.Generator(device=dev).manual_seed(rank)
    store = Int4KVStore(G, capacity=n)
    for layer in range(layers):
        k = torch.randn(B, HKV, n, D, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(B, HKV, n, D, device=dev, generator=g).to(torch.bfloat16)
        store.append(k, v, layer)
        del k, v
    q = torch.randn(layers, B, HQ, 1, D, device=dev,
                    generator=torch.Generator(device=dev).manual_seed(123)).to(torch.bfloat16)
    out = torch.empty(B, HQ, 1, D, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev)

    # ranks exchange partials over peer memory (kv4_lse_exchange): two
    # launches per step, no collective library, so the step sits in a graph
    xchg = (shard.PeerExchange(rows=B * HQ, d=D, device=dev)
            if ws > 1 and args.seq_transport == "peer" else None)

    def step(l):
        kp, ks, vp, vs = store.layer(l).views()
        if ws == 1:
            ops.attention_into(q[l], kp, ks, vp, vs, out, G, False)
        else:
            shard.seq_sharded_attention(q[l], kp, ks, vp, vs, k_offset=lo, sk_total=S,
                                        group_size=G, out=out, exchange=xchg)

    for l in range(layers):
        step(l)
    torch.cuda.synchronize()
    # NCCL all-gathers run eagerly (a capture that failed on one rank only
    # would leave the ranks' collective sequences mismatched); the peer
    # exchange and the single-GPU step replay from a CUDA graph.
    graph = None
    if ws == 1 or xchg is not None:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for l in range(layers):
                step(l)
        graph.replay()
        torch.cuda.synchronize()

    def run_steps(k):
        if graph is not None:
            for _ in range(k // layers):
                graph.replay()
            for i in range(k % layers):
                step(i)
        else:
            for i in range(k):
                step(i % layers)

    run_steps(args.warmup)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start = torch.zeros(1, device=dev)
    with ClockSampler(local) as clk:
        _hold(st)
        if ws > 1:
            # a device-side start line: the ranks' GPUs leave this all-reduce
            # together, so host launch skew between ranks does not show up
            # as waiting inside the first exchange of the timed region
            dist.all_reduce(start, async_op=True).wait()
        t0.record(st)
        run_steps(args.steps)
        t1.record(st)
        torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
    if ws > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    if ws > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    peak, peak_kind = _peaks()
    value = attn_bytes() * args.steps / (ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "us_per_step": round(ms * 1e3 / args.steps, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 q/out, int4 KV codes, bf16 scales, fp32 accumulate",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": f"{args.workload}: batch-1 decode attention, sequence sharded",
                   "batch": B, "q_heads": HQ, "kv_heads": HKV, "seq_len": S, "d_head": D,
                   "group_size": G, "tokens_per_rank": n,
                   "parallelism": f"sequence shard x{ws}: partial attention + " + (
                       "peer-memory exchange and LSE merge in one kernel (NVLink)"
                       if xchg is not None else "NCCL all-gather of (o, lse) + LSE combine"),
                   "graph": graph is not None,
                   "l2": f"steps rotate over {layers} layer caches per rank"},
        "roofline": {"bound": "hbm", "achieved_per_gpu": round(value / ws, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(value / ws / peak, 4),
                     "peak_source": peak_kind},
        "clocks": clk.summary(),
        "gpu_launches": args.steps * (1 if ws == 1 else 2),  # partial + exchange/combine
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the other workloads and the sweeps (rank 0, N=1)")
    ap.add_argument("--no-gpu-reference", action="store_true",
                    help="skip timing the reference's Triton kernel on the same caches")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--shard", choices=["batch", "seq"], default="batch",
                    help="seq: config-3 sequence sharding over the ranks (strong scaling)")
    ap.add_argument("--seq-transport", choices=["peer", "allgather"], default="peer",
                    help="--shard seq: partials over peer memory (one kernel) or NCCL")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2",
                    help="config2 = 8B decode at batch 16 (the headline); long* = batch-1 long context; "
                         "config4 = 70B shape, one KV head per GPU")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    ws, rank, local = _dist()
    set_workload(args.workload, 1 if (args.impl == "reference" or args.shard == "seq") else ws)
    if args.impl == "reference":
        line = run_reference(args, ws, rank)
    else:
        line = (run_seq_shard(args, ws, rank, local) if args.shard == "seq"
                else run_ours(args, ws, rank, local))
    if line is not None:
        print(json.dumps(line), flush=True)
    if ws > 1 and args.impl == "ours" and args.shard != "seq":
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
