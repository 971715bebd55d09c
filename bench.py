"""Benchmark of the IMI KV-cache path on B200.

Workload (Llama-3-8B attention geometry, synthetic): 32 layers, 32 query / 8 KV
heads, head_dim 128, bf16, batch 1, 131072-token context.  Keys per layer and
head come from a 64-component Gaussian mixture (std 0.3) with RoPE
(theta 500000); values N(0, 1).  IMI with subspace_parts=2 (adaptive k = 90),
retrieval_budget 0.1, k-means settings of the reference's Llama config
(max_iters 20, early stop min iter 20, tol / rel tol 5e-4), decode-time cell
assignment on (batch 16, threshold 16, 512 delta tokens).

A step is one decode step through all layers: per layer the new token is
appended (``decode_update_kv_cache``) and attention runs through
``imi_decode_attn`` (cell scoring, selection, gather attention).  The metric is
microseconds per layer per step (lower is better).  ``value`` runs with the
step inputs resident in HBM; ``e2e`` runs the same API with the inputs in
pinned host memory, copied in every step, and every layer's attention output
copied back.  The working set per step (about 1.7 GB of K/V rows) is larger
than L2, so no explicit flush is needed.

Under torchrun (N > 1) the KV heads are sharded over the ranks (no collective
on the data path); the reported time is the max over ranks.

``--impl reference`` times the reference's own CPU code for the path on the
host cores: the index build (imi::kmeans_execute + reorganize_from_kmeans,
compiled from the reference sources into oracle/_ref) and the decode selection
(the C port in oracle/ of the scorer, the top-k + token budget rule and the
batch_access page truncation, with torch fp32 attention), on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "sparse_decode_us_per_layer_step@128K"
UNIT = "us/layer/step"
CFG = dict(model="Llama-3-8B-geometry", layers=32, q_heads=32, kv_heads=8, head_dim=128, context=131072,
           subspace_parts=2, retrieval_budget=0.1, static_start=32, static_end=64, buffer_cluster_num=32,
           max_new_length=257, theta=500000.0, components=64)
KMEANS = {"max_iters": 20, "tol": 0.0005, "early_stop_min_iter": 20, "early_stop_rel_tol": 0.0005}
# DRAM bytes per attention launch at this geometry, from one ncu capture of
# `python bench.py --layers 2 --steps 2 --warmup 3 --no-cpu-baseline` with
# --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
# -k regex:imi_attn_kernel -s 4 -c 3 (each launch is one full layer).
ATTN_TRAFFIC_BYTES = 50_290_518
ASYNC = {"enabled": True, "batch": 16, "threshold": 16, "delta_tokens": 512}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the burst figure (the build's kernels are timed as
    one short burst per layer)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops)"
    return 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.proc = None
        self.index = index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap,utilization.gpu",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        rows = []
        for ln in getattr(self, "lines", []):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), parts[2:6], float(parts[6])))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        loaded = [r for r in rows if r[3] > 0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ----------------------------------------------------------------------------
# our implementation
# ----------------------------------------------------------------------------
def make_inputs(layers, heads_local, head0, G, ctx, steps, dev, seed=0):
    """Per-layer prefill K/V generator and per-step decode inputs (device)."""
    from adaptiveimi_b200.synthetic import mixture_keys, rope

    D = CFG["head_dim"]
    kvh = CFG["kv_heads"]

    def layer_kv(l):
        k, means = mixture_keys(kvh, ctx, D, CFG["components"], seed + 1000 * l, CFG["theta"], device=dev)
        g = torch.Generator(device=dev).manual_seed(seed + 1000 * l + 7)
        v = torch.randn(kvh, ctx, D, generator=g, device=dev)
        sl = slice(head0, head0 + heads_local)
        return k[sl].to(torch.bfloat16), v[sl].to(torch.bfloat16), means[sl]

    return layer_kv


def decode_inputs(means_per_layer, G, ctx, steps, dev, seed=0):
    """q [steps, L, 1, 1, H, D], k/v [steps, L, 1, 1, kv, D] (bf16, device)."""
    from adaptiveimi_b200.synthetic import rope

    L = len(means_per_layer)
    kvh, D = means_per_layer[0].shape[0], means_per_layer[0].shape[2]
    g = torch.Generator(device=dev).manual_seed(seed + 99)
    qs, ks, vs = [], [], []
    for l in range(L):
        m = means_per_layer[l]
        C = m.shape[1]
        comp = torch.randint(0, C, (steps, kvh, G + 1), generator=g, device=dev)
        x = torch.gather(m.unsqueeze(0).expand(steps, -1, -1, -1), 2,
                         comp[..., None].expand(-1, -1, -1, D)) + 0.3 * torch.randn(steps, kvh, G + 1, D,
                                                                                   generator=g, device=dev)
        pos = torch.arange(ctx, ctx + steps, device=dev)
        x = rope(x.permute(1, 2, 0, 3), pos, CFG["theta"]).permute(2, 0, 1, 3)  # [steps, kv, G+1, D]
        qs.append(x[:, :, :G].reshape(steps, 1, 1, kvh * G, D))
        ks.append(x[:, :, G].reshape(steps, 1, 1, kvh, D))
        vs.append(torch.randn(steps, 1, 1, kvh, D, generator=g, device=dev))
    st = lambda a: torch.stack(a, 1).to(torch.bfloat16).contiguous()  # noqa: E731
    return st(qs), st(ks), st(vs)


def run_ours(args):
    from adaptiveimi_b200.attn import imi_decode_attn
    from adaptiveimi_b200.cache import adpimi_cache
    from adaptiveimi_b200.sharding import max_over_ranks, shard_kv_heads

    ws, rank, local = dist_env()
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", init_method="env://")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L, ctx, kvh, G = args.layers, args.context, CFG["kv_heads"], CFG["q_heads"] // CFG["kv_heads"]
    head0, hl = shard_kv_heads(kvh, ws, rank)
    steps_total = args.steps + args.warmup
    cache = adpimi_cache(
        valid_start=[0], layer_num=L, batch_size=1, max_length=ctx + CFG["max_new_length"], num_key_value_heads=hl,
        num_heads=hl * G, head_dim=CFG["head_dim"], dtype=torch.bfloat16,
        layer_mapping={str(i): f"cuda:{local}" for i in range(L)}, max_new_length=CFG["max_new_length"],
        input_length=ctx, static_pattern_start=CFG["static_start"], static_pattern_end=CFG["static_end"],
        core=os.cpu_count() or 1, pages_per_cluster=2, retrieval_budget=CFG["retrieval_budget"], cache_ratio=0.05,
        buffer_cluster_num=CFG["buffer_cluster_num"], prefill_bsz=1, num_gpus=1, model_size=8,
        subspace_parts=CFG["subspace_parts"],
        # the build is timed on the prefill stream here (its side-stream overlap
        # with the prefill is measured by --workload prefill_overlap)
        runtime_config={"kmeans": KMEANS, "async_update": ASYNC, "pipeline": {"async_build": False}})
    # ---- prefill: device index build of every layer (timed for the build metric)
    layer_kv = make_inputs(L, hl, head0, G, ctx, steps_total, dev)
    means = []
    build_ms = 0.0
    for l in range(L):
        k, v, m = layer_kv(l)
        means.append(m)
        ks = k.transpose(0, 1).unsqueeze(0)  # [1, ctx, kv, D] strided view (model layout)
        vs = v.transpose(0, 1).unsqueeze(0)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        cache.prefill_update_kv_cache(None, ks, vs, l, 0)
        e1.record()
        torch.cuda.synchronize()
        build_ms += e0.elapsed_time(e1)
        del k, v, ks, vs
    torch.cuda.empty_cache()
    cache.prepare_cache()
    n_mid = cache.list_stride
    n_active = [int(cache.index[l].n_active.max()) for l in range(L)]
    qd, kd, vd = decode_inputs(means, G, ctx, steps_total, dev)

    def step(t, q_src, k_src, v_src, out_sink=None):
        outs = []
        for l in range(L):
            cache.decode_update_kv_cache(k_src[l], v_src[l], l)
            outs.append(imi_decode_attn(q_src[l], None, None, l, cache))
        if out_sink is not None:  # the step's result: every layer's output, one read-back
            out_sink.copy_(torch.stack(outs), non_blocking=True)

    # ---- warmup (device inputs)
    for t in range(args.warmup):
        step(t, qd[t], kd[t], vd[t])
    torch.cuda.synchronize()
    # ---- timed region: device-resident inputs
    cache.row_count_log = torch.zeros((args.steps * L, hl), dtype=torch.int32, device=dev)
    cache._log_pos = 0
    cache.attn_event_log = None  # the roofline pass below times the attention kernel alone
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        h0 = time.perf_counter()
        for t in range(args.steps):
            step(args.warmup + t, qd[args.warmup + t], kd[args.warmup + t], vd[args.warmup + t])
        host_s = time.perf_counter() - h0
        e1.record()
        torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    dev_ms = e0.elapsed_time(e1)
    rows_timed = cache.row_count_log.to(torch.int64).sum().item()
    cache.row_count_log = None
    cache.attn_event_log = None
    attn = attention_kernel_pass(cache, qd[args.warmup + args.steps - 1], L, hl, G, dev)
    # ---- e2e: pinned host inputs copied in, outputs copied out, every step
    # (the cache has capacity for warmup + steps appended tokens; e2e reuses the
    # last `e2e_steps` positions after a reset of the appended-token counter)
    e2e_steps = min(args.steps, 8)
    e2e_warm = min(2, max(0, args.steps - e2e_steps))  # untimed, through the same pinned-copy path
    e2e_total = e2e_warm + e2e_steps
    qh = qd[:e2e_total].cpu().pin_memory()
    kh = kd[:e2e_total].cpu().pin_memory()
    vh = vd[:e2e_total].cpu().pin_memory()
    outs_h = torch.empty((e2e_total, L, 1, 1, hl * G, CFG["head_dim"]), dtype=torch.bfloat16).pin_memory()
    qb, kb, vb = torch.empty_like(qd[0]), torch.empty_like(kd[0]), torch.empty_like(vd[0])
    cache.static_pattern_total -= e2e_total  # re-use appended positions (same shapes, same work)
    cache.context -= e2e_total
    for t in range(e2e_steps, e2e_total):  # the warm-up steps (their own inputs)
        qb.copy_(qh[t], non_blocking=True)
        kb.copy_(kh[t], non_blocking=True)
        vb.copy_(vh[t], non_blocking=True)
        step(t, qb, kb, vb, out_sink=outs_h[t])
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for t in range(e2e_steps):
        qb.copy_(qh[t], non_blocking=True)
        kb.copy_(kh[t], non_blocking=True)
        vb.copy_(vh[t], non_blocking=True)
        step(t, qb, kb, vb, out_sink=outs_h[t])
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    # ---- max over ranks
    dev_ms, e2e_ms, attn_avg_us, build_ms_max = max_over_ranks([dev_ms, e2e_ms, attn["avg_us"], build_ms], dev)
    if rank != 0:
        if ws > 1:
            torch.distributed.destroy_process_group()
        return None
    us_per_layer_step = dev_ms * 1e3 / (args.steps * L)
    e2e_us = e2e_ms * 1e3 / (e2e_steps * L)
    hbm, src = peaks()
    achieved = attn["algo_bytes"] / (attn_avg_us * 1e-6) / 1e9 if attn_avg_us > 0 else 0.0
    roofline = {"kernel": "imi_attn_kernel (gather attention with in-kernel split merge)", "bound": "hbm",
                "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                "peak_source": src + " (MEASURED_PEAKS.json hbm_gbs)", "traffic": ATTN_TRAFFIC_BYTES,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, mean of 3 launches of "
                                  "the same kernel on the same geometry",
                "algorithmic_bytes_per_launch": int(attn["algo_bytes"]), "avg_launch_us": round(attn_avg_us, 3),
                "launches_timed": attn["launches"], "rows_per_launch": attn["rows_per_launch"]}
    keys_built = L * kvh * n_mid
    # algorithmic k-means flops of the whole build, from each index's own iteration counts
    build_flops = 0
    for l in range(L):
        idx = cache.index[l]
        its = idx.iters_run.cpu().tolist()  # [heads, S]
        S_ = len(idx.ks)
        for row in its:
            for s_, it in enumerate(row):
                build_flops += (int(it) + 1) * 2 * n_mid * int(idx.ks[s_]) * (CFG["head_dim"] // S_)
    build_flops *= ws  # every rank builds an equal share of the KV heads
    tpk, tpk_src = tensor_peak()
    res = {
        "metric": METRIC, "value": round(us_per_layer_step, 3), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (Gaussian-mixture keys + RoPE, N(0,1) values; seeded)",
        "config": {"workload": "BASELINE configs[1]: Llama-3-8B geometry, 128K context, 32 layers, IMI S=2, "
                               "budget 0.1, async cell assignment on", "context": ctx, "layers": L,
                   "kv_heads": kvh, "q_heads": CFG["q_heads"], "head_dim": 128, "global_batch": 1,
                   "parallelism": f"kv-head shard x{ws}" if ws > 1 else "single GPU",
                   "l2": "working set per step > L2 (no flush needed)",
                   "n_slots": cache.n_centroids, "nprobe": cache.nprobe, "budget_tokens": cache.max_retrieval_tokens,
                   "max_active_cells": max(n_active), "splits": cache.splits},
        "e2e": {"value": round(e2e_us, 3), "unit": UNIT, "h2d_bytes_per_step": int(L * (qh[0, 0].numel() +
                                                                                        2 * kh[0, 0].numel()) * 2),
                "d2h_bytes_per_step": int(L * outs_h[0, 0].numel() * 2), "steps": e2e_steps},
        "roofline": roofline,
        "build": {"metric": "IMI build Mkeys/s", "value": round(keys_built / (build_ms_max * 1e-3) / 1e6, 3),
                  "unit": "Mkeys/s", "build_ms_total": round(build_ms_max, 2), "keys": keys_built,
                  "kmeans": KMEANS,
                  "roofline": {"bound": "tensor", "achieved": round(build_flops / (build_ms_max * 1e-3) / 1e12, 2),
                               "peak": tpk, "unit": "TFLOP/s",
                               "frac": round(build_flops / (build_ms_max * 1e-3) / 1e12 / tpk, 4),
                               "peak_source": tpk_src, "flops": build_flops,
                               "flops_formula": "sum over (head, subspace) of (iters_run + 1) * 2 * n * k * D/S "
                                                "(Lloyd distance passes plus the k-means++ pass), whole build time"}},
        "gpu_launches": None,
        "host_launch_us_per_layer_step": round(host_s * 1e6 / (args.steps * L), 2),
        "clocks": clk.summary(),
    }
    # our kernels per layer-step: select (which also does the append) +
    # attention (which also merges its splits); every ASYNC["batch"] steps a
    # layer instead launches the append and the two assignment kernels before
    # them (+3), and at its next visit the centroid publish (+1)
    res["gpu_launches"] = int(args.steps * L * 2 + (args.steps // ASYNC["batch"]) * L * 4)
    if ws == 1 and not args.no_cpu_baseline:
        try:
            res["cpu_baseline"] = cpu_baseline(args, sample_layers=1, sample_steps=2)
        except Exception as exc:  # reported, not fatal
            res["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    if ws > 1:
        torch.distributed.destroy_process_group()
    return res


def attention_kernel_pass(cache, q_last, L, hl, G, dev, repeats=6):
    """Live CUDA-event timing of the attention kernel alone (imi_sparse_attention:
    gather attention with the in-kernel split merge) on every layer's row list
    of the last decode step: sweeps of the 32 layers launched back to back (as
    in the decode pipeline), one event pair per sweep, so each launch streams
    its rows from HBM (the layers' rows together exceed L2).

    Algorithmic bytes per launch = rows * (256 B key + 256 B value + 4 B row
    index) + q and out (bf16) + the split partials written and read back."""
    from adaptiveimi_b200 import ops

    bg = hl
    rows, rcs = [], []
    for l in range(L):
        r = torch.empty((bg, cache.execution_stride), dtype=torch.int32, device=dev)
        rc = torch.empty((bg,), dtype=torch.int32, device=dev)
        q = q_last[l].reshape(bg, G, 128).contiguous()
        ops.select_cells(q=q, index=cache.index[l], nprobe=cache.nprobe, max_tokens=cache.max_retrieval_tokens,
                         buffer_pages=cache.buffer_size, page_size=8, padding_id=cache.padding_cluster_id,
                         static_len=cache.static_pattern_total, exec_capacity=cache.execution_stride,
                         sel_cells=torch.empty((bg, cache.nprobe), dtype=torch.int32, device=dev),
                         sel_count=torch.empty((bg,), dtype=torch.int32, device=dev), row_index=r, row_count=rc)
        rows.append((q, r))
        rcs.append(rc)
    out = torch.empty((bg, G, 128), dtype=torch.bfloat16, device=dev)
    part_o = torch.empty((bg, cache.splits, G, 128), dtype=torch.float32, device=dev)
    part_ml = torch.empty((bg, cache.splits, G, 2), dtype=torch.float32, device=dev)
    counters = torch.zeros((bg,), dtype=torch.int32, device=dev)
    # one descriptor per layer, built once: the timed loop is C-ABI calls only,
    # so launches queue back to back and the events bracket kernel time
    import ctypes
    from adaptiveimi_b200 import _lib
    L_ = _lib.load()
    descs = []
    for l in range(L):
        q, r = rows[l]
        d = _lib.AttnDesc()
        d.bg, d.G, d.splits, d.exec_capacity = bg, G, cache.splits, cache.execution_stride
        d.scale = 1.0 / math.sqrt(128)
        d.q, d.row_index, d.row_count = q.data_ptr(), r.data_ptr(), rcs[l].data_ptr()
        d.list_keys, d.list_values = cache.index[l].list_keys.data_ptr(), cache.index[l].list_values.data_ptr()
        d.list_rows = cache.index[l].list_keys.shape[1]
        d.static_keys, d.static_values = cache.steady_zone_keys[l].data_ptr(), cache.steady_zone_values[l].data_ptr()
        d.static_rows = cache.static_capacity
        d.part_o, d.part_ml, d.out, d.counters = part_o.data_ptr(), part_ml.data_ptr(), out.data_ptr(), \
            counters.data_ptr()
        descs.append(d)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    # one event pair per sweep over the L layers: events between launches
    # would break the programmatic-launch overlap the decode pipeline has
    evs = []
    torch.cuda.synchronize()
    for rep in range(repeats + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for l in range(L):
            _lib.check(L_.imi_sparse_attention(ctypes.byref(descs[l]), stream), "imi_sparse_attention")
        b.record()
        if rep > 0:  # the first sweep is warmup
            evs.append((a, b))
    torch.cuda.synchronize()
    times = [a.elapsed_time(b) * 1e3 / L for a, b in evs]
    total_rows = sum(int(rc.to(torch.int64).sum()) for rc in rcs)
    rows_per_launch = total_rows / L
    algo = rows_per_launch * (512 + 4) + bg * G * 128 * 2 * 2 + bg * cache.splits * G * (128 + 2) * 4 * 2
    return {"avg_us": sum(times) / len(times), "algo_bytes": algo, "launches": len(times) * L,
            "rows_per_launch": rows_per_launch}


# ----------------------------------------------------------------------------
# reference CPU path (bounded sample)
# ----------------------------------------------------------------------------
def _ref_modules():
    ref_dir = ROOT / "oracle" / "_ref"
    if not any(ref_dir.glob("imi_ref*.so")):
        return None
    sys.path.insert(0, str(ref_dir))
    import AdpIMI_Index  # noqa: E402
    import imi_ref  # noqa: E402
    return imi_ref, AdpIMI_Index


def cpu_baseline(args, sample_layers=1, sample_steps=2, build_heads=2, sample_warmup=1):
    """The reference's CPU path on a bounded sample: build of `build_heads` heads
    of one 128K layer with every host thread, and `sample_steps` timed decode
    steps of `sample_layers` layers (8 KV heads) after `sample_warmup` untimed
    ones."""
    import numpy as np

    from adaptiveimi_b200.sizing import RetrievalSizes, adaptive_k
    from adaptiveimi_b200.synthetic import mixture_keys
    from oracle import oracle as O

    mods = _ref_modules()
    kind = "reference" if mods is not None else "port"
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ctx = args.context
    D = 128
    kvh, G = CFG["kv_heads"], CFG["q_heads"] // CFG["kv_heads"]
    k, means = mixture_keys(kvh, ctx, D, CFG["components"], 0, CFG["theta"])
    g = torch.Generator().manual_seed(7)
    v = torch.randn(kvh, ctx, D, generator=g)
    k, v = k.to(torch.bfloat16), v.to(torch.bfloat16)
    mid_k = k[:, 32:ctx - 64].contiguous()
    mid_v = v[:, 32:ctx - 64].contiguous()
    n = mid_k.shape[1]
    ks = adaptive_k(n, 2)
    # ---- build sample
    t0 = time.perf_counter()
    if mods is not None:
        r = mods[0].build(mid_k[:build_heads].contiguous(), mid_v[:build_heads].contiguous(), 2, list(ks),
                          KMEANS["max_iters"], KMEANS["tol"], KMEANS["early_stop_min_iter"],
                          KMEANS["early_stop_rel_tol"], cores)
    else:
        kb, vb = O.bf16_bits(mid_k), O.bf16_bits(mid_v)
        for h in range(build_heads):
            O.build_head(kb[h], vb[h], 2, ks, KMEANS["max_iters"], KMEANS["tol"], KMEANS["early_stop_min_iter"],
                         KMEANS["early_stop_rel_tol"])
    build_s = time.perf_counter() - t0
    build_mkeys = build_heads * n / build_s / 1e6
    # ---- decode sample: the index of `build_heads` heads tiled over the 8 KV
    # groups (the selection and gather work per group does not depend on which
    # head's index it scans), queried with the mixture queries the GPU arm uses.
    #  * scorer: the C port of compute_impl.cu:62-103 (the reference scores on
    #    the GPU; its CPU fallback is a torch einsum with other rounding);
    #  * top-k + token budget: the reference's torch calls (retrieval.py:295-303);
    #  * page truncation: the reference's own AdpIMI_Index.batch_access (C++,
    #    oracle/_ref), cold cache;
    #  * gather + attention: torch fp32 on the host cores (the reference's
    #    weighted_flash_decoding is an absent GPU package).
    from oracle.ref_index import PageTruncation, reference_select, rows_of

    sizes = RetrievalSizes.from_capacity(n, 2, CFG["retrieval_budget"], CFG["buffer_cluster_num"], 96 + 256)
    if mods is None:
        raise RuntimeError("decode CPU baseline needs the reference build (oracle/_ref)")
    ns = sizes.n_centroids
    sizes_t = torch.zeros((kvh, ns), dtype=torch.int32)
    offs_t = torch.zeros((kvh, ns + 1), dtype=torch.int32)
    cents = np.zeros((kvh, ns, D), np.float32)
    mask = np.ones((kvh, ns), np.uint8)
    lk = [None] * kvh
    lv = [None] * kvh
    for h in range(kvh):
        src = h % build_heads
        c = int(r["cluster_counts"][src])
        sizes_t[h, :c] = r["cluster_sizes"][src, :c]
        offs_t[h, :c + 1] = r["cluster_offsets"][src, :c + 1]
        offs_t[h, c + 1:] = offs_t[h, c]
        cents[h, :c] = r["centroids"][src, :c].numpy()
        mask[h, :c] = 0
        lk[h] = r["list_keys"][src]
        lv[h] = r["list_values"][src]
    trunc = PageTruncation(mods[1], sizes_t, offs_t, sizes.nprobe, sizes.buffer_size, threads=min(cores, 8))
    steps_total = sample_steps * sample_layers
    warm_total = sample_warmup * sample_layers
    qs, _, _ = decode_inputs([means], G, ctx, warm_total + steps_total, "cpu", seed=0)
    for t in range(warm_total + steps_total):
        if t == warm_total:
            t0 = time.perf_counter()
        q = qs[t, 0, 0, 0].reshape(kvh, G, D)
        qb = O.bf16_bits(q)
        sims = torch.from_numpy(np.stack([O.scores(qb[h], cents[h], mask[h]) for h in range(kvh)]))
        sel = reference_select(sims, sizes_t, sizes.nprobe, sizes.max_retrieval_tokens, sizes.padding_cluster_id)
        runs = trunc.access(sel)
        for h in range(kvh):
            ridx = torch.from_numpy(rows_of(runs[h]))
            kr = lk[h][ridx].float()
            vr = lv[h][ridx].float()
            s_ = (q[h].float() @ kr.T) / math.sqrt(D)
            torch.softmax(s_, -1) @ vr
    dec_s = time.perf_counter() - t0
    us = dec_s * 1e6 / steps_total
    return {"value": round(us, 1), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"decode: {sample_steps} step(s) x {sample_layers} layer(s) after {sample_warmup} untimed, "
                      f"8 KV heads, {ctx}-token context, "
                      f"mixture queries; scorer = C port of compute_impl.cu, top-k/budget = the reference's torch "
                      f"calls, page truncation = the reference's AdpIMI_Index.batch_access (C++), gather + "
                      f"attention = torch fp32",
            "build": {"value": round(build_mkeys, 4), "unit": "Mkeys/s", "seconds": round(build_s, 2),
                      "kind": kind, "cores": cores,
                      "sample": f"the reference's own kmeans_execute + reorganize_from_kmeans (oracle/_ref): "
                                f"{build_heads} heads x {n} keys, k={ks[0]}x{ks[1]}, {KMEANS['max_iters']} iters"}}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return None
    warm = max(0, min(args.warmup, 5))      # a decode step of the sample is ~30 ms on the host cores
    steps = max(1, min(args.steps, 20))
    cb = cpu_baseline(args, sample_layers=1, sample_steps=steps, sample_warmup=warm)
    res = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": ws,
        "steps": steps, "warmup": warm, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (same generator)",
        "config": {"workload": "BASELINE configs[1] (bounded CPU sample)", "context": args.context},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "build": cb["build"],
    }
    return res


# ----------------------------------------------------------------------------
# 1M context, sequence-sharded over the ranks
# ----------------------------------------------------------------------------
METRIC_1M = "sparse_decode_us_per_layer_step@1M"


def run_1m(args):
    """Every rank holds one contiguous shard of the 1M-token middle of every
    layer, builds its IMI, and each decode step runs, per layer: local
    selection under the global rules, an exchange of the candidate records
    (imi_peer_allgather over NVLink peer memory), the global merge, attention over this shard's rows (rank 0 also
    the steady zone, which receives the step's appended token), an exchange
    of the (o, m, l) partials and the log-sum-exp combine.  Each
    timed step (all layers) is replayed from a CUDA graph captured before the
    timed region, so the host's per-layer calls are not what is measured."""
    import torch.distributed as dist

    from adaptiveimi_b200 import seqshard
    from adaptiveimi_b200.sharding import max_over_ranks
    from adaptiveimi_b200.synthetic import rope

    ws, rank, local = dist_env()
    if ws > 1:
        dist.init_process_group("nccl", init_method="env://")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L, kvh, G, D = args.layers, CFG["kv_heads"], CFG["q_heads"] // CFG["kv_heads"], CFG["head_dim"]
    ctx = args.context
    static0 = CFG["static_start"] + CFG["static_end"]
    n = ctx - static0
    budget = 0.05
    try:
        plan = seqshard.plan_shards(n, ws, CFG["subspace_parts"], budget, CFG["buffer_cluster_num"])
    except ValueError as e:
        if rank == 0:
            print(json.dumps({"metric": METRIC_1M, "unavailable": f"{ctx} tokens over {ws} shard(s): {e}"}),
                  flush=True)
        return None
    steps_total = args.warmup + args.steps
    cap = static0 + steps_total + 1
    th, C = CFG["theta"], CFG["components"]
    shards, zk, zv, qs, nk, nv = [], [], [], [], [], []
    t0 = time.perf_counter()
    for l in range(L):
        means = torch.randn(kvh, C, D, generator=torch.Generator(device=dev).manual_seed(1000 * l), device=dev)

        def mix(count, positions, seed):
            g = torch.Generator(device=dev).manual_seed(seed)
            comp = torch.randint(0, C, (kvh, count), generator=g, device=dev)
            x = torch.gather(means, 1, comp[..., None].expand(-1, -1, D)) + \
                0.3 * torch.randn(kvh, count, D, generator=g, device=dev)
            return rope(x, positions, th), torch.randn(kvh, count, D, generator=g, device=dev)

        a0, ln = plan.starts[rank], plan.lengths[rank]
        k, v = mix(ln, torch.arange(CFG["static_start"] + a0, CFG["static_start"] + a0 + ln, device=dev),
                   1000 * l + 17 + rank)
        s = seqshard.SeqShard(plan, rank, kvh, G, cap, dev)
        s.build(k.to(torch.bfloat16).contiguous(), v.to(torch.bfloat16).contiguous(), **KMEANS)
        if ws > 1 and not s.enable_peer_exchange():
            raise SystemExit("peer-memory exchange unavailable for this geometry")
        shards.append(s)
        del k, v
        zpos = torch.cat([torch.arange(0, CFG["static_start"], device=dev),
                          torch.arange(ctx - CFG["static_end"], ctx, device=dev)])
        zkk, zvv = mix(static0, zpos, 1000 * l + 5)
        zk.append(torch.zeros((kvh, cap, D), dtype=torch.bfloat16, device=dev))
        zv.append(torch.zeros((kvh, cap, D), dtype=torch.bfloat16, device=dev))
        zk[-1][:, :static0] = zkk.to(torch.bfloat16)
        zv[-1][:, :static0] = zvv.to(torch.bfloat16)
        qq, _ = mix(steps_total * (G + 1), torch.arange(ctx, ctx + steps_total, device=dev).repeat_interleave(G + 1),
                    1000 * l + 9)
        qq = qq.reshape(kvh, steps_total, G + 1, D).permute(1, 0, 2, 3).to(torch.bfloat16).contiguous()
        qs.append(qq[:, :, :G].contiguous())                # [steps, kv, G, D]
        nk.append(qq[:, :, G].contiguous())                 # [steps, kv, D]: the appended key
        nv.append(torch.randn(steps_total, kvh, D, device=dev).to(torch.bfloat16))
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0

    from adaptiveimi_b200 import ops

    def step(t):
        for l in range(L):
            if rank == 0:  # decode append into the steady zone (imi_decode_append)
                ops.decode_append(new_keys=nk[l][t], new_values=nv[l][t], zone_keys=zk[l], zone_values=zv[l],
                                  pos=static0 + t)
            seqshard.decode_step([shards[l]], qs[l][t], zk[l], zv[l], static0 + t + 1)

    for t in range(args.warmup):
        step(t)
    torch.cuda.synchronize()
    graphs = []
    for t in range(args.warmup, steps_total):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(t)
        graphs.append(g)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for g in graphs:
            g.replay()
        e1.record()
        torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        for s in shards:
            s.check_exchange()
    ms, build_s = max_over_ranks([ms, build_s], dev)
    if rank != 0:
        return None
    us = ms * 1000.0 / (args.steps * L)
    return {
        "metric": METRIC_1M, "value": round(us, 3), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (Gaussian-mixture keys + RoPE, N(0,1) values; seeded per layer and shard)",
        "config": {"workload": f"BASELINE configs[2]: {ctx} tokens sequence-sharded {ws}-way, per-shard IMI S=2, "
                               f"global budget {budget}, {L} layers, one append per step",
                   "context": ctx, "layers": L, "kv_heads": kvh, "q_heads": CFG["q_heads"], "shards": ws,
                   "nprobe": plan.nprobe, "budget_tokens": plan.max_tokens, "slots_per_shard": list(plan.n_slots),
                   "parallelism": f"sequence shards x{ws}, candidates and partials exchanged over NVLink peer memory "
                                  "(imi_peer_allgather)",
                   "timing": "CUDA-graph replay of each whole step, device events, max over ranks"},
        "build_s_max": round(build_s, 3),
        "clocks": clk.summary(),
    }


# ----------------------------------------------------------------------------
# Qwen2.5-7B geometry, batch 8 with ragged contexts, S=4
# ----------------------------------------------------------------------------
METRIC_QWEN = "sparse_decode_us_per_layer_step@qwen7b_b8"
CFG3 = dict(layers=28, q_heads=28, kv_heads=4, head_dim=128, theta=1e6, components=128, batch=8, ctx_lo=32768,
            ctx_hi=131072, ctx_seed=1, subspace_parts=4, retrieval_budget=0.05, buffer_cluster_num=32,
            static_start=32, static_end=64)
# the reference's Qwen2.5-7B k-means settings (config/Qwen2.5-7B-Instruct.json); async update off there
KMEANS3 = {"max_iters": 15, "tol": 0.0005, "early_stop_min_iter": 15, "early_stop_rel_tol": 0.0005}


def run_qwen7b(args):
    """8 sequences, contexts U[32768, 131072] (seed 1),
    Qwen2.5-7B attention geometry (28 layers, 28 query / 4 KV heads), keys from a
    128-component mixture with RoPE theta 1e6, IMI S=4, budget ratio 0.05
    without a fixed token budget (top-nprobe cells; see RetrievalSizes).  The
    reference's cache is batch-1 (cache_hub/adaptive_imi/cache.py:83-84), so
    each sequence has its own cache, as a batch-8 server running the reference
    would.  Each decode step (every layer, every sequence: append + select +
    attention) is replayed from a CUDA graph captured before the timed region;
    the value is device time per layer per step for the whole batch."""
    from adaptiveimi_b200.attn import imi_decode_attn
    from adaptiveimi_b200.cache import adpimi_cache
    from adaptiveimi_b200.synthetic import mixture_keys

    ws, rank, local = dist_env()
    if rank != 0:
        return None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    c = CFG3
    L, kvh, G, D, B = c["layers"], c["kv_heads"], c["q_heads"] // c["kv_heads"], c["head_dim"], c["batch"]
    g = torch.Generator().manual_seed(c["ctx_seed"])
    ctxs = [int(x) for x in torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (B,), generator=g)]
    steps_total = args.warmup + args.steps
    caches, means = [], []
    keys_built, build_ms = 0, 0.0
    for b, ctx in enumerate(ctxs):
        cache = adpimi_cache(
            valid_start=[0], layer_num=L, batch_size=1, max_length=ctx + steps_total + 2, num_key_value_heads=kvh,
            num_heads=kvh * G, head_dim=D, dtype=torch.bfloat16, layer_mapping={str(i): f"cuda:{local}" for i in range(L)},
            max_new_length=steps_total + 2, input_length=ctx, static_pattern_start=c["static_start"],
            static_pattern_end=c["static_end"], core=os.cpu_count() or 1, pages_per_cluster=2,
            retrieval_budget=c["retrieval_budget"], cache_ratio=0.05, buffer_cluster_num=c["buffer_cluster_num"],
            prefill_bsz=1, num_gpus=1, model_size=7, subspace_parts=c["subspace_parts"],
            runtime_config={"kmeans": KMEANS3, "retrieval": {"fixed_budget": False}, "pipeline": {"async_build": False}})
        mb = []
        for l in range(L):
            k, m = mixture_keys(kvh, ctx, D, c["components"], 7919 * b + 1000 * l, c["theta"], device=dev)
            gv = torch.Generator(device=dev).manual_seed(7919 * b + 1000 * l + 7)
            v = torch.randn(kvh, ctx, D, generator=gv, device=dev)
            ks = k.to(torch.bfloat16).transpose(0, 1).unsqueeze(0)
            vs = v.to(torch.bfloat16).transpose(0, 1).unsqueeze(0)
            del k, v
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            cache.prefill_update_kv_cache(None, ks, vs, l, 0)
            e1.record()
            torch.cuda.synchronize()
            build_ms += e0.elapsed_time(e1)
            keys_built += kvh * cache.list_stride
            mb.append(m)
            del ks, vs
        cache.prepare_cache()
        caches.append(cache)
        means.append(mb)
        torch.cuda.empty_cache()
    qds = [decode_inputs(means[b], G, ctxs[b], steps_total, dev, seed=b) for b in range(B)]

    def step(t):
        for l in range(L):
            for b in range(B):
                qd, kd, vd = qds[b]
                caches[b].decode_update_kv_cache(kd[t, l], vd[t, l], l)
                imi_decode_attn(qd[t, l], None, None, l, caches[b])

    for t in range(args.warmup):
        step(t)
    torch.cuda.synchronize()
    graphs = []
    for t in range(args.warmup, steps_total):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step(t)
        graphs.append(gr)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for gr in graphs:
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    us = ms * 1000.0 / (args.steps * L)
    rows = [int(cc._dec[f"cuda:{local}"]["row_count"].sum()) for cc in caches]
    return {
        "metric": METRIC_QWEN, "value": round(us, 3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (128-component Gaussian-mixture keys + RoPE theta 1e6, N(0,1) values; seeded)",
        "config": {"workload": "BASELINE configs[3]: Qwen2.5-7B geometry, batch 8 (one batch-1 cache per sequence), "
                               "ragged contexts U[32768, 131072] seed 1, IMI S=4, budget ratio 0.05 without a fixed "
                               "token budget (top-nprobe cells; not a reference mode, unpinned)",
                   "contexts": ctxs, "layers": L, "kv_heads": kvh, "q_heads": c["q_heads"], "head_dim": D,
                   "global_batch": B, "n_slots": [cc.n_centroids for cc in caches],
                   "nprobe": [cc.nprobe for cc in caches], "rows_last_layer": rows,
                   "timing": "CUDA-graph replay of each whole step (28 layers x 8 sequences), device events"},
        "build": {"metric": "IMI build Mkeys/s", "value": round(keys_built / (build_ms * 1e-3) / 1e6, 3),
                  "unit": "Mkeys/s", "build_ms_total": round(build_ms, 2), "keys": keys_built, "kmeans": KMEANS3},
        "clocks": clk.summary(),
    }


def run_prefill_overlap(args):
    """The index build next to the prefill that produces its keys.
    Per layer: a stand-in for one Llama-3-8B decoder layer's dense prefill work
    at 128K tokens (three [131072 x 4096] x [4096 x 14336] bf16 GEMMs, about
    46 TFLOP, on the prefill stream), then the layer's K/V handed to the cache,
    whose device build reads them in place.  With the build on the prefill
    stream the layers serialise; with the build on the cache's side stream
    (runtime_config pipeline.async_build) layer l's k-means runs under layer
    l+1's GEMMs.  Reports both wall times (device work, synchronised ends)."""
    from adaptiveimi_b200.cache import adpimi_cache

    ws, rank, local = dist_env()
    if rank != 0:
        return None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L, ctx, kvh, G, D = min(args.layers, 6), CFG["context"], CFG["kv_heads"], CFG["q_heads"] // CFG["kv_heads"], 128
    layer_kv = make_inputs(L, kvh, 0, G, ctx, 1, dev)
    kvs = []
    for l in range(L):
        k, v, _ = layer_kv(l)
        kvs.append((k.transpose(0, 1).unsqueeze(0), v.transpose(0, 1).unsqueeze(0)))
    x = torch.randn(ctx, 4096, device=dev, dtype=torch.bfloat16)
    w = torch.randn(4096, 14336, device=dev, dtype=torch.bfloat16) * 0.01
    y = torch.empty(ctx, 14336, device=dev, dtype=torch.bfloat16)

    def produce():
        for _ in range(3):
            torch.matmul(x, w, out=y)

    res = {}
    for mode in ("sync", "async", "sync"):
        cache = adpimi_cache(
            valid_start=[0], layer_num=L, batch_size=1, max_length=ctx + 8, num_key_value_heads=kvh,
            num_heads=kvh * G, head_dim=D, dtype=torch.bfloat16, layer_mapping={str(i): f"cuda:{local}" for i in range(L)},
            max_new_length=8, input_length=ctx, static_pattern_start=32, static_pattern_end=64, core=1,
            pages_per_cluster=2, retrieval_budget=0.1, cache_ratio=0.05, buffer_cluster_num=32, prefill_bsz=1,
            num_gpus=1, model_size=8, subspace_parts=2,
            runtime_config={"kmeans": KMEANS, "pipeline": {"async_build": mode == "async"}})
        produce()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for l in range(L):
            produce()
            cache.prefill_update_kv_cache(None, kvs[l][0], kvs[l][1], l, 0)
        cache.prepare_cache()  # waits for every layer's build
        torch.cuda.synchronize()
        res[mode] = (time.perf_counter() - t0) * 1e3
        stats = [cache.imi_pipelines[l].get_pipeline_stats() for l in range(L)]
        res[mode + "_build_ms"] = sum(st["kmeans_ms"] + st["reorganize_ms"] for st in stats)
        cache.cleanup()
        del cache
        torch.cuda.empty_cache()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for l in range(L):
        produce()
    torch.cuda.synchronize()
    produce_ms = (time.perf_counter() - t0) * 1e3
    return {"metric": "prefill_with_index_build_ms", "layers": L, "context": ctx, "unit": "ms",
            "producer_only_ms": round(produce_ms, 2), "build_on_prefill_stream_ms": round(res["sync"], 2),
            "build_on_side_stream_ms": round(res["async"], 2),
            "device_build_ms_sum": round(res["async_build_ms"], 2),
            "note": "producer = three [131072x4096]x[4096x14336] bf16 GEMMs per layer (a stand-in for a decoder "
                    "layer's dense prefill work); keys/values synthetic; the build reads them in place"}


# ----------------------------------------------------------------------------
# random-init Qwen2.5-72B, 8 GPUs, 128 greedy tokens
# ----------------------------------------------------------------------------
METRIC_E2E = "decode_tokens_per_s@qwen72b_128K"
# the reference's Qwen2.5-72B k-means settings (config/Qwen2.5-72B-Instruct.json)
KMEANS4 = {"max_iters": 5, "tol": 0.0005, "early_stop_min_iter": 5, "early_stop_rel_tol": 0.0005}


def run_qwen72b_e2e(args):
    """Tensor-parallel random-init Qwen2.5-72B (80 layers, hidden 8192, 64 query
    / 8 KV heads, head_dim 128; one KV head per GPU at 8 GPUs): a prompt of
    random token ids (vocabulary 152064), prefill with the IMI of every layer
    built at the end of its prefill, then greedy decoding through the cache
    (adaptiveimi_b200.model_e2e, the reference's inference loop).  Reports
    decode tokens/s, prefill seconds and the device build time (max over
    ranks)."""
    import torch.distributed as dist

    from adaptiveimi_b200.model_e2e import DecoderConfig, TPDecoder, generate
    from adaptiveimi_b200.sharding import max_over_ranks

    ws, rank, local = dist_env()
    if ws > 1:
        dist.init_process_group("nccl", init_method="env://")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    base = DecoderConfig.qwen25_72b()
    cfg = DecoderConfig(layers=min(args.layers, base.layers) if args.layers else base.layers)
    ctx = args.context
    new_tokens = 128
    model = TPDecoder(cfg, dev, seed=0, attention="imi")
    ids = torch.randint(0, cfg.vocab, (ctx,), generator=torch.Generator().manual_seed(0)).to(dev)
    model.make_cache(ctx, new_tokens, budget=0.1, parts=2, kmeans=KMEANS4)
    with Clocks(local) as clk:
        r = generate(model, ids, new_tokens, graphs=ws == 1 and not args.eager_decode)
    prefill_s, decode_s, build_ms = max_over_ranks([r["prefill_s"], r["decode_s"], r["build_ms"]], dev)
    if rank != 0:
        if ws > 1:
            dist.destroy_process_group()
        return None
    steps = new_tokens - 1
    res = {"metric": METRIC_E2E, "value": round(steps / decode_s, 3), "unit": "tokens/s", "n_gpus": ws,
           "steps": steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic: random-init weights, random prompt token ids (no checkpoint, no dataset)",
           "config": {"workload": "BASELINE configs[4]: Qwen2.5-72B geometry, random init, 131072-token prompt, "
                                  "128 greedy tokens, KV heads split over the GPUs, budget 0.1, S=2",
                      "layers": cfg.layers, "context": ctx, "kv_heads_per_gpu": model.kvh,
                      "parallelism": f"tensor parallel x{ws} (NCCL all-reduce after o_proj and down_proj)",
                      "decode_dense_work": "eager" if (ws > 1 or args.eager_decode) else "CUDA graphs per layer (cache calls eager)"},
           "prefill_s": round(prefill_s, 3), "decode_ms_per_token": round(decode_s * 1000 / steps, 3),
           "imi_build_ms_total": round(build_ms, 2), "tokens_head": r["tokens"][:8], "clocks": clk.summary()}
    if ws > 1:
        dist.destroy_process_group()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="default: the workload's model (32, or 80 for qwen72b_e2e)")
    ap.add_argument("--context", type=int, default=None, help="default: 131072 (128k) or 1048576 (1m)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager-decode", action="store_true",
                    help="qwen72b_e2e on one GPU: run the decode layers' dense work eagerly instead of as "
                         "CUDA graphs (multi-GPU runs are always eager)")
    ap.add_argument("--workload", default="128k", choices=["128k", "1m", "qwen7b", "prefill_overlap", "qwen72b_e2e"],
                    help="1m: BASELINE configs[2], the 1M context sequence-sharded over the ranks; "
                         "qwen7b: BASELINE configs[3], batch 8 with ragged contexts, S=4")
    args = ap.parse_args()
    if args.layers is None:
        args.layers = 80 if args.workload == "qwen72b_e2e" else CFG["layers"]
    if args.context is None:
        args.context = 1_048_576 if args.workload == "1m" else CFG["context"]
    if args.workload == "1m":
        if args.impl == "reference":
            ws, rank, _ = dist_env()
            if rank == 0:
                print(json.dumps({"impl": "reference", "metric": METRIC_1M,
                                  "unavailable": "the reference's CPU decode path at 1M context is not sampled"}),
                      flush=True)
            return
        if args.warmup < 3:
            args.warmup = 3
        res = run_1m(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.workload == "qwen72b_e2e":
        if args.impl == "reference":
            ws, rank, _ = dist_env()
            if rank == 0:
                print(json.dumps({"impl": "reference", "metric": METRIC_E2E,
                                  "unavailable": "the reference's model loop needs HF checkpoints and its CPU page "
                                                 "cache; not run"}), flush=True)
            return
        res = run_qwen72b_e2e(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.workload == "prefill_overlap":
        res = run_prefill_overlap(args) if args.impl == "ours" else None
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.workload == "qwen7b":
        if args.impl == "reference":
            ws, rank, _ = dist_env()
            if rank == 0:
                print(json.dumps({"impl": "reference", "metric": METRIC_QWEN,
                                  "unavailable": "the reference's CPU decode path for config 3 is not sampled"}),
                      flush=True)
            return
        args.warmup = max(args.warmup, 3)
        args.steps = min(args.steps, 16)
        res = run_qwen7b(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.steps + args.warmup + 8 > CFG["max_new_length"] - 1:
        raise SystemExit("steps + warmup exceed the decode capacity (256 tokens)")
    res = run_reference(args) if args.impl == "reference" else run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
