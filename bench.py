"""Benchmark of the packed-INT2 MLA cache path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (BASELINE.json metric "INT2 MLA decode-attn tok/s @B64,16K ctx; writer GB/s
vs HBM peak"): one *step* is one decode step of DeepSeek-V2-Lite's 27 MLA layers for
64 requests at 16384 tokens of context: per layer, the fused writer stores the 64 new
latents (tcgen05 rotation + INT2 codec + k_pe + s4r16 ring), then packed decode
attention reads the INT2 cache.  ``value`` = whole-job tokens/s (N x 64 tokens per step)
with everything resident in HBM (the step replayed from a CUDA graph); ``e2e`` = the
same step through the public plugin API (``try_fast_decode_store``,
``packed_mla_decode_gf_fwd``) with the per-step queries / new latents copied from
pinned host memory and the outputs copied back, inside the timed region.  The
``writer`` object reports the config-1 prefill writer (27 layers x 8 x 16384 rows).

Data are seeded synthetic tensors with the benchmark distributions (no dataset or
checkpoint).  Multi-GPU (torchrun): every rank serves its own 64 requests (request
sharding, weak scaling, no data-path collective); time is the max over ranks.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "INT2 MLA decode-attn tok/s @B64,16K ctx; writer GB/s vs HBM peak"
LAYERS, HEADS, D, DR = 27, 16, 512, 64
SINK, RECENT = 4, 16
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
REF_SAMPLE_REQS = 2  # requests per step of the reference arm (one layer each)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def decode_bytes(batch, ctx, heads=HEADS, d=D, dr=DR, window=SINK + RECENT):
    """Algorithmic HBM bytes of one decode launch (one layer)."""
    per_int2 = d // 4 + (d // 128) * 8 + dr * 2  # 288 B: codes + (scale, zero) + k_pe
    per_win = d * 2 + dr * 2 + 8  # BF16 ring row + k_pe + slot/ring maps
    win = min(window, ctx)
    return batch * ((ctx - win) * per_int2 + win * per_win) + batch * heads * ((d + dr) * 2 + d * 2)


def writer_bytes(rows, d=D, dr=DR):
    """Algorithmic HBM bytes of one writer launch: c_kv + k_pe + slot in, codes + params + k_pe out."""
    return rows * ((2 * d + 2 * dr + 8) + (d // 4 + (d // 128) * 8 + 2 * dr))


def read_traffic():
    """Per-launch DRAM bytes (read + write) of the decode call as one ncu capture measured
    them, with the capture it came from: ``profiles/decode_traffic.json`` holds the figure
    and the command next to the markdown summary of the same capture.  (None, None) when
    the file is absent: no stale constant is reported."""
    f = ROOT / "profiles" / "decode_traffic.json"
    if not f.exists():
        return None, None
    j = json.loads(f.read_text())
    return float(j["traffic_bytes_per_launch"]), j.get("source")


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    def __init__(self, dev: torch.device):
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        self.index = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        self.proc = None
        self.out = None

    def __enter__(self):
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.2)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in Path(self.out.name).read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9:
                    rows.append(f)
        finally:
            os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------


def build_state(dev, batch, ctx, seed):
    from mla_kv_quant_b200 import ops, synth
    from mla_kv_quant_b200.pool import PackedLatentPool

    rot = {i: synth.rotation(D, 1000 + i) for i in range(LAYERS)}
    params = synth.layer_params(LAYERS, seed=2)
    pages = (ctx + 63) // 64
    pt, num_slots = synth.page_table(batch, ctx, seed=4 + seed, device=dev)
    pool = PackedLatentPool(num_slots, LAYERS, D, DR, max_reqs=batch, sink=SINK, recent=RECENT, device=dev,
                            rotations=rot, quantizer_params=params)
    return pool, pt, pages


def fill_cache(pool, pt, batch, ctx, dev, seed):
    fill_cache_layers(pool, pt, batch, ctx, dev, seed, LAYERS)


def fill_cache_layers(pool, pt, batch, ctx, dev, seed, layers):
    """Prefill every layer: 8 requests x ctx rows per writer launch (config-1 shape)."""
    from mla_kv_quant_b200 import ops, synth

    scale = synth.channel_scale(D, 77, dev)
    chunk = 8
    pos = torch.arange(ctx, device=dev)
    for li in range(layers):
        rt = pool.write_rotation_t(li)
        codec = pool.codec(li)
        view = pool.layer_view(li)
        for b0 in range(0, batch, chunk):
            bs = list(range(b0, min(batch, b0 + chunk)))
            n = len(bs) * ctx
            x = synth.latents(n, D, seed + 131 * li + b0, dev, scale=scale)
            pe = synth.normal_bf16((n, DR), seed + 7 * li + b0 + 1, dev)
            slots = torch.cat([pt[b, pos // 64].long() * 64 + pos % 64 for b in bs])
            seq = torch.full((n,), ctx, dtype=torch.int32, device=dev)
            req = torch.cat([torch.full((ctx,), b, dtype=torch.int64, device=dev) for b in bs])
            p = pos.repeat(len(bs)).to(torch.int32)
            ops.fused_write(x, pe, slots, rt, codec, view, seq_lens=seq, req_idx=req, positions=p)
    torch.cuda.synchronize()


def time_writer(pool, dev, ctx, warmup, iters):
    """Config 1: 27 layers x (8 x ctx) prefill rows through the fused writer."""
    from mla_kv_quant_b200 import ops, synth

    n = 8 * ctx
    x = synth.latents(n, D, 5, dev)
    pe = synth.normal_bf16((n, DR), 6, dev)
    slots = torch.arange(64, 64 + n, device=dev, dtype=torch.int64)
    pos = torch.arange(ctx, device=dev, dtype=torch.int32).repeat(8)
    seq = torch.full((n,), ctx, dtype=torch.int32, device=dev)
    req = torch.arange(8, device=dev).repeat_interleave(ctx)
    views = [pool.layer_view(li) for li in range(LAYERS)]
    rts = [pool.write_rotation_t(li) for li in range(LAYERS)]
    codecs = [pool.codec(li) for li in range(LAYERS)]

    def run():
        for li in range(LAYERS):
            ops.fused_write(x, pe, slots, rts[li], codecs[li], views[li], seq_lens=seq, req_idx=req, positions=pos)

    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        run()
    e.record()
    torch.cuda.synchronize()
    per_launch_s = s.elapsed_time(e) / 1e3 / (iters * LAYERS)
    return n, per_launch_s


def run_ours(args, rank, world, dev):
    from mla_kv_quant_b200 import ops, synth
    from mla_kv_quant_b200.mla_fused_writer import try_fast_decode_store
    from mla_kv_quant_b200.mla_packed_decode import packed_mla_decode_gf_fwd

    batch, ctx = args.batch, args.ctx
    hbm, tf_burst, tf_sus, peak_kind = peaks()
    pool, pt, pages = build_state(dev, batch, ctx, seed=rank)
    fill_cache(pool, pt, batch, ctx, dev, seed=100 * rank)
    splits = args.splits or ops.default_num_splits(batch, ctx)
    sm_scale = 1.0 / math.sqrt(192.0)

    # per-step inputs: queries per layer and one new latent row per request per layer
    q = synth.normal_bf16((LAYERS, batch, HEADS, D + DR), 11 + rank, dev)
    new_ckv = synth.latents(LAYERS * batch, D, 12 + rank, dev).view(LAYERS, batch, D)
    new_pe = synth.normal_bf16((LAYERS, batch, DR), 13 + rank, dev)
    out = torch.empty(LAYERS, batch, HEADS, D, dtype=torch.bfloat16, device=dev)
    seq = torch.full((batch,), ctx, dtype=torch.int32, device=dev)
    req = torch.arange(batch, device=dev, dtype=torch.int64)
    last = ctx - 1
    loc = (pt[:, last // 64].long() * 64 + last % 64).contiguous()
    part_o = torch.empty(batch, HEADS, splits + 1, D, device=dev)
    part_lse = torch.empty(batch, HEADS, splits + 1, device=dev)
    views = [pool.layer_view(li) for li in range(LAYERS)]
    rts = [pool.write_rotation_t(li) for li in range(LAYERS)]
    codecs = [pool.codec(li) for li in range(LAYERS)]
    dec_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(LAYERS)]

    def step(timed_events=False):
        for li in range(LAYERS):
            ops.fused_write(new_ckv[li], new_pe[li], loc, rts[li], codecs[li], views[li], seq_lens=seq, req_idx=req)
            if timed_events:
                dec_ev[li][0].record()
            ops.packed_decode(q[li], views[li], pt, seq, sm_scale, splits, part_o, part_lse, out[li])
            if timed_events:
                dec_ev[li][1].record()

    # decode-kernel roofline: events around each decode launch (eager, same stream)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dec_times = []
    for _ in range(max(3, args.steps // 10)):
        step(timed_events=True)
        torch.cuda.synchronize()
        dec_times += [a.elapsed_time(b) / 1e3 for a, b in dec_ev]
    dec_s = statistics.mean(dec_times)

    # value: the step replayed from a CUDA graph
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        torch.cuda.nvtx.range_push("timed")  # `ncu --nvtx --nvtx-include timed/` captures exactly this
        s.record()
        for _ in range(args.steps):
            graph.replay()
        e.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    if world > 1:
        torch.distributed.barrier()
    step_s = s.elapsed_time(e) / 1e3 / args.steps
    step_s = max_over_ranks(step_s, world, dev)
    clocks = clk.summary()
    del graph

    # e2e: public API, host buffers, copies inside the timed region
    pool.set_window_meta(True, seq, req)
    pool._rolaq_fused_decode_write = True
    h_q = q.cpu().pin_memory()
    h_ckv = new_ckv.cpu().pin_memory()
    h_pe = new_pe.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    # Double-buffered device inputs: layer l+1's inputs go up on an H2D stream while layer l
    # runs, layer l's output comes down on a D2H stream; events order the three streams.
    d_q = [torch.empty_like(q[0]) for _ in range(2)]
    d_ckv = [torch.empty_like(new_ckv[0]) for _ in range(2)]
    d_pe = [torch.empty_like(new_pe[0]) for _ in range(2)]
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(LAYERS)]
    ev_done = [torch.cuda.Event() for _ in range(LAYERS)]

    def e2e_step():
        main = torch.cuda.current_stream(dev)  # the capture stream when captured into a graph
        up.wait_stream(main)  # the previous step's layers are done with the input buffers

        def h2d(li):
            bi = li & 1
            with torch.cuda.stream(up):
                if li >= 2:
                    up.wait_event(ev_done[li - 2])  # layer li-2 has read buffer bi
                d_ckv[bi].copy_(h_ckv[li], non_blocking=True)
                d_pe[bi].copy_(h_pe[li], non_blocking=True)
                d_q[bi].copy_(h_q[li], non_blocking=True)
                ev_in[li].record(up)

        h2d(0)
        for li in range(LAYERS):
            if li + 1 < LAYERS:
                h2d(li + 1)
            bi = li & 1
            main.wait_event(ev_in[li])
            if not try_fast_decode_store(pool, li, loc, d_ckv[bi], d_pe[bi]):
                raise RuntimeError("fused decode writer declined a decode step")
            packed_mla_decode_gf_fwd(d_q[bi], pool, li, pt, seq, sm_scale, splits, attn_logits=part_o,
                                     attn_lse=part_lse, out=out[li])
            ev_done[li].record(main)
            with torch.cuda.stream(down):
                down.wait_event(ev_done[li])
                h_out[li].copy_(out[li], non_blocking=True)
        main.wait_stream(up)
        main.wait_stream(down)  # every output is on the host before the step ends

    for _ in range(args.warmup):
        e2e_step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s.record()
    for _ in range(args.steps):
        e2e_step()
    e.record()
    torch.cuda.synchronize()
    e2e_eager_s = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world, dev)
    # The same step (copies, public calls, every output read back) captured into a CUDA
    # graph, as a serving engine captures its decode step: the plugin calls allocate nothing
    # and never synchronise with the host, so they capture; the replay removes the per-launch
    # gaps of 81 eager launches.
    e2e_graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(e2e_graph):
        e2e_step()
    for _ in range(args.warmup):
        e2e_graph.replay()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s.record()
    for _ in range(args.steps):
        e2e_graph.replay()
    e.record()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world, dev)
    del e2e_graph
    h2d = LAYERS * (q[0].numel() * 2 + new_ckv[0].numel() * 2 + new_pe[0].numel() * 2)
    d2h = LAYERS * out[0].numel() * 2

    # e2e of the absorbed layer: the same step starting from q_nope / q_pe and ending at the
    # projected output (rolaq_sglang.patch:205-248): per layer absorb_query (q_nope W_kc' and
    # the q_pe concat), the fused writer, the packed decode, project_output (o W_vc'); inputs
    # copied up and the projected outputs copied down inside the timed region, graph-replayed.
    e2e_abs = e2e_absorbed(args, world, dev, pool, pt, seq, req, loc, splits, sm_scale, new_ckv, new_pe, part_o,
                           part_lse)

    # writer leg (config 1), rank-local
    wrows, w_s = time_writer(pool, dev, ctx, warmup=2, iters=max(3, min(10, args.steps // 20)))
    w_bytes = writer_bytes(wrows)
    w_flops = 2.0 * wrows * D * D

    dbytes = decode_bytes(batch, ctx)
    achieved = dbytes / dec_s / 1e9
    traffic, traffic_src = read_traffic()
    res = {
        "metric": METRIC,
        "value": world * batch / step_s,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_s * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; latents N(0,1) x lognormal(0,0.5) channel scale, 8 outlier channels x10)",
        "config": {
            "workload": f"decode step: {LAYERS} MLA layers (DeepSeek-V2-Lite shape) x batch {batch} x ctx {ctx}, "
                        "fused decode write + packed INT2 decode attention per layer",
            "batch_per_gpu": batch, "global_batch": batch * world, "ctx": ctx, "layers": LAYERS, "heads": HEADS,
            "kv_lora_rank": D, "rope_dim": DR, "window": "s4r16", "page": 64, "num_splits": splits,
            "l2": "no flush: per-step working set %.1f GB >> 126 MB L2" % (LAYERS * dbytes / 1e9),
            "parallelism": f"dp{world} (request-sharded, no collective)",
        },
        "e2e": {"value": world * batch / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_s * 1e3,
                "path": "try_fast_decode_store + packed_mla_decode_gf_fwd per layer, pinned host buffers, copies "
                        "overlapped with the layers on two copy streams, the whole step (copies included) replayed "
                        "from a CUDA graph as a serving engine captures its decode step",
                "eager": {"value": world * batch / e2e_eager_s, "unit": "tok/s", "ms_per_step": e2e_eager_s * 1e3,
                          "path": "the same calls and copies launched eagerly every step"},
                "absorbed": e2e_abs},
        "roofline": {"kernel": "rolaq decode call, one layer (window_split_kernel, decode_tc_kernel and "
                               "merge_splits_kernel when the INT2 grid is one wave, else decode_tc_kernel and "
                               "merge_window_kernel)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": traffic, "traffic_source": traffic_src,
                     "algorithmic_bytes_per_launch": dbytes, "launch_us": dec_s * 1e6},
        "writer": {"rows_per_launch": wrows, "launch_us": w_s * 1e6, "gbs": w_bytes / w_s / 1e9,
                   "hbm_frac": (w_bytes / w_s / 1e9) / hbm, "tflops": w_flops / w_s / 1e12,
                   "tensor_frac": (w_flops / w_s / 1e12) / tf_burst,
                   "tensor_frac_sustained": (w_flops / w_s / 1e12) / tf_sus,
                   "roofline_frac": max(w_bytes / (hbm * 1e9), w_flops / (tf_burst * 1e12)) / w_s,
                   "bound": "tensor" if w_flops / (tf_burst * 1e12) > w_bytes / (hbm * 1e9) else "hbm",
                   "note": "roofline_frac = max(bytes/HBM peak, flops/bf16 peak) / time, of " + peak_kind},
        "clocks": clocks,
        # per layer: the fused writer, then window_split + decode_tc + merge_splits (one-wave INT2
        # grid) or decode_tc + merge_window
        "gpu_launches": args.steps * LAYERS * (4 if batch * splits < 148 else 3),
        "gpus_active": world,
    }
    return res


# Configs 3a / 3b: decode plus writer on 1 x B200.  MiniCPM3-4B's
# softmax scale is 1/sqrt(qk_nope_head_dim + qk_rope_head_dim) with the model's published
# head dims 64 + 32 (the checkpoint is not in this container: a stated parameter).
EXTRA_CONFIGS = {
    "3a_minicpm3_4b": dict(layers=62, heads=40, d=256, dr=32, batch=128, ctx=8192, sm_scale=1.0 / math.sqrt(96.0)),
    "3b_moonlight_16b_a3b": dict(layers=27, heads=16, d=512, dr=64, batch=128, ctx=8192,
                                 sm_scale=1.0 / math.sqrt(192.0)),
}


def decode_step_config(dev, layers, heads, d, dr, batch, ctx, sm_scale, steps, warmup, world=1, seed=0):
    """One decode step of ``layers`` MLA layers for ``batch`` requests at ``ctx`` tokens (per
    layer: the fused writer stores the new latents, then the packed decode reads the INT2
    cache), replayed from a CUDA graph; plus the decode launch alone (CUDA events around
    each launch, eager) for the roofline.  The cache is filled through the same fused
    writer (8 requests x ctx rows per launch)."""
    from mla_kv_quant_b200 import ops, synth
    from mla_kv_quant_b200.pool import PackedLatentPool

    rot = {i: synth.rotation(d, 1000 + i) for i in range(layers)}
    params = synth.layer_params(layers, seed=2)
    pt, num_slots = synth.page_table(batch, ctx, seed=4 + seed, device=dev)
    pool = PackedLatentPool(num_slots, layers, d, dr, max_reqs=batch, sink=SINK, recent=RECENT, device=dev,
                            rotations=rot, quantizer_params=params)
    scale = synth.channel_scale(d, 77, dev)
    pos = torch.arange(ctx, device=dev)
    for li in range(layers):
        rt, codec, view = pool.write_rotation_t(li), pool.codec(li), pool.layer_view(li)
        for b0 in range(0, batch, 8):
            bs = list(range(b0, min(batch, b0 + 8)))
            n = len(bs) * ctx
            x = synth.latents(n, d, seed + 131 * li + b0, dev, scale=scale)
            pe = synth.normal_bf16((n, dr), seed + 7 * li + b0 + 1, dev)
            slots = torch.cat([pt[b, pos // 64].long() * 64 + pos % 64 for b in bs])
            req = torch.tensor(bs, device=dev).repeat_interleave(ctx)
            ops.fused_write(x, pe, slots, rt, codec, view, seq_lens=torch.full((n,), ctx, dtype=torch.int32,
                                                                               device=dev),
                            req_idx=req, positions=pos.repeat(len(bs)).to(torch.int32))
            del x, pe, slots, req
    torch.cuda.synchronize()
    splits = ops.default_num_splits(batch, ctx, latent_dim=d, rope_dim=dr, heads=heads)
    q = synth.normal_bf16((layers, batch, heads, d + dr), 11 + seed, dev)
    new_ckv = synth.latents(layers * batch, d, 12 + seed, dev).view(layers, batch, d)
    new_pe = synth.normal_bf16((layers, batch, dr), 13 + seed, dev)
    out = torch.empty(layers, batch, heads, d, dtype=torch.bfloat16, device=dev)
    seq = torch.full((batch,), ctx, dtype=torch.int32, device=dev)
    req = torch.arange(batch, device=dev, dtype=torch.int64)
    loc = (pt[:, (ctx - 1) // 64].long() * 64 + (ctx - 1) % 64).contiguous()
    part_o = torch.empty(batch, heads, splits + 1, d, device=dev)
    part_lse = torch.empty(batch, heads, splits + 1, device=dev)
    views = [pool.layer_view(li) for li in range(layers)]
    rts = [pool.write_rotation_t(li) for li in range(layers)]
    codecs = [pool.codec(li) for li in range(layers)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(layers)]

    def step(timed=False):
        for li in range(layers):
            ops.fused_write(new_ckv[li], new_pe[li], loc, rts[li], codecs[li], views[li], seq_lens=seq, req_idx=req)
            if timed:
                ev[li][0].record()
            ops.packed_decode(q[li], views[li], pt, seq, sm_scale, splits, part_o, part_lse, out[li])
            if timed:
                ev[li][1].record()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dec = []
    for _ in range(2):
        step(timed=True)
        torch.cuda.synchronize()
        dec += [a.elapsed_time(b) / 1e3 for a, b in ev]
    dec_s = statistics.mean(dec)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        step()
    for _ in range(warmup):
        graph.replay()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(steps):
        graph.replay()
    s1.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    step_s = max_over_ranks(s0.elapsed_time(s1) / 1e3 / steps, world, dev)
    del graph
    hbm = peaks()[0]
    dbytes = decode_bytes(batch, ctx, heads=heads, d=d, dr=dr)
    res = {"tok_s": world * batch / step_s, "ms_per_step": step_s * 1e3, "steps": steps, "warmup": warmup,
           "layers": layers, "heads": heads, "kv_lora_rank": d, "rope_dim": dr, "batch_per_gpu": batch, "ctx": ctx,
           "sm_scale": sm_scale, "num_splits": splits,
           "decode_kernel": f"decode_tc_kernel<{d}, {dr}, {heads}> (tcgen05)",
           "roofline": {"bound": "hbm", "launch_us": dec_s * 1e6, "algorithmic_bytes_per_launch": dbytes,
                        "achieved": dbytes / dec_s / 1e9, "peak": hbm, "unit": "GB/s",
                        "frac": dbytes / dec_s / 1e9 / hbm}}
    del pool, q, new_ckv, new_pe, out, part_o, part_lse
    torch.cuda.empty_cache()
    return res


def run_batch4a(args, rank, world, dev):
    """Config 4(a): 512 requests x 32768 tokens of context, 27 DeepSeek-V2-Lite layers,
    sharded by request over the ranks (512 / N each, no data-path collective); one GPU
    holds all 512 (~130 GB of cache).  Strong scaling: value = 512 tokens per step / the
    step time (max over ranks)."""
    total = 512
    if total % world:
        raise SystemExit("--gpus must divide 512")
    r = decode_step_config(dev, LAYERS, HEADS, D, DR, total // world, 32768, 1.0 / math.sqrt(192.0),
                           args.steps, args.warmup, world=world, seed=rank)
    return {"mode": "batch4a", "metric": "INT2 MLA decode tok/s, B512 x 32K ctx, request-sharded", "n_gpus": world,
            "gpus_active": world, "value": r["tok_s"], "unit": "tok/s", "scaling": "strong",
            "global_batch": total, **{k: v for k, v in r.items() if k != "tok_s"}}


def e2e_absorbed(args, world, dev, pool, pt, seq, req, loc, splits, sm_scale, new_ckv, new_pe, part_o, part_lse,
                 qk_nope=128, v_head=128):
    """The decode step from the per-head q_nope / q_pe to the projected attention output:
    absorb_query -> try_fast_decode_store -> packed_mla_decode_gf_fwd -> project_output per
    layer, with seeded BF16 kv_b_proj weights in SGLang's bmm layouts."""
    from mla_kv_quant_b200 import absorbed, synth
    from mla_kv_quant_b200.mla_fused_writer import try_fast_decode_store
    from mla_kv_quant_b200.mla_packed_decode import packed_mla_decode_gf_fwd

    batch = seq.numel()
    w_kc, w_vc = [], []
    for li in range(LAYERS):
        w = (synth.normal_bf16((HEADS * (qk_nope + v_head), D), 300 + li, dev).float() * 0.05).to(torch.bfloat16)
        a, b = absorbed.split_absorbed_weights(w, HEADS, qk_nope, v_head)
        w_kc.append(a)
        w_vc.append(b)
    h_qn = synth.normal_bf16((LAYERS, batch, HEADS, qk_nope), 21, dev).cpu().pin_memory()
    h_qp = synth.normal_bf16((LAYERS, batch, HEADS, DR), 22, dev).cpu().pin_memory()
    h_ckv, h_pe = new_ckv.cpu().pin_memory(), new_pe.cpu().pin_memory()
    h_y = torch.empty(LAYERS, batch, HEADS, v_head, dtype=torch.bfloat16).pin_memory()
    # double-buffered per-layer inputs, as the plain e2e leg: layer l+1's inputs go up on a
    # copy stream while layer l runs, layer l's projected output comes down on another
    d_qn = [torch.empty(batch, HEADS, qk_nope, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    d_qp = [torch.empty(batch, HEADS, DR, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    d_ckv = [torch.empty_like(new_ckv[0]) for _ in range(2)]
    d_pe = [torch.empty_like(new_pe[0]) for _ in range(2)]
    q = torch.empty(batch, HEADS, D + DR, dtype=torch.bfloat16, device=dev)
    o = torch.empty(batch, HEADS, D, dtype=torch.bfloat16, device=dev)
    y = torch.empty(LAYERS, batch, HEADS, v_head, dtype=torch.bfloat16, device=dev)
    pool.set_window_meta(True, seq, req)
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(LAYERS)]
    ev_done = [torch.cuda.Event() for _ in range(LAYERS)]

    def step():
        main = torch.cuda.current_stream(dev)
        up.wait_stream(main)

        def h2d(li):
            bi = li & 1
            with torch.cuda.stream(up):
                if li >= 2:
                    up.wait_event(ev_done[li - 2])
                d_qn[bi].copy_(h_qn[li], non_blocking=True)
                d_qp[bi].copy_(h_qp[li], non_blocking=True)
                d_ckv[bi].copy_(h_ckv[li], non_blocking=True)
                d_pe[bi].copy_(h_pe[li], non_blocking=True)
                ev_in[li].record(up)

        h2d(0)
        for li in range(LAYERS):
            if li + 1 < LAYERS:
                h2d(li + 1)
            bi = li & 1
            main.wait_event(ev_in[li])
            absorbed.absorb_query(d_qn[bi], d_qp[bi], w_kc[li], out=q)
            if not try_fast_decode_store(pool, li, loc, d_ckv[bi], d_pe[bi]):
                raise RuntimeError("fused decode writer declined a decode step")
            packed_mla_decode_gf_fwd(q, pool, li, pt, seq, sm_scale, splits, attn_logits=part_o, attn_lse=part_lse,
                                     out=o)
            absorbed.project_output(o, w_vc[li], out=y[li])
            ev_done[li].record(main)
            with torch.cuda.stream(down):
                down.wait_event(ev_done[li])
                h_y[li].copy_(y[li], non_blocking=True)
        main.wait_stream(up)
        main.wait_stream(down)

    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(args.steps):
        graph.replay()
    s1.record()
    torch.cuda.synchronize()
    t = max_over_ranks(s0.elapsed_time(s1) / 1e3 / args.steps, world, dev)
    del graph
    h2d = (h_qn.numel() + h_qp.numel() + h_ckv.numel() + h_pe.numel()) * 2
    return {"value": world * batch / t, "unit": "tok/s", "ms_per_step": t * 1e3, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": h_y.numel() * 2,
            "path": "per layer absorb_query (q_nope W_kc' + q_pe concat, tcgen05) -> try_fast_decode_store -> "
                    "packed_mla_decode_gf_fwd -> project_output (o W_vc', tcgen05); copies in and out inside the "
                    "timed region; whole step graph-replayed"}


def max_over_ranks(x, world, dev):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------------------
# CPU baseline (the oracle port of the reference algorithm on the host cores)
# ---------------------------------------------------------------------------------------------


def cpu_decode_sample(batch_sample=2, ctx=16384, seed=0):
    """Time the oracle decode (FP32 numpy, all host threads) for `batch_sample`
    requests of one layer; return seconds per (request, layer)."""
    from oracle import codec as ocodec
    from oracle import decode as odecode
    from oracle import writer as owriter

    rng = np.random.default_rng(seed)
    pages = (ctx + 63) // 64
    pool = owriter.Pool((batch_sample * pages + 1) * 64, D, DR, batch_sample, SINK, RECENT)
    n = pool.num_slots
    pool.codes[:] = rng.integers(0, 256, size=pool.codes.shape, dtype=np.uint8)
    pool.params[..., 0] = rng.uniform(0.5, 1.5, size=pool.params.shape[:2]).astype(np.float32)
    pool.params[..., 1] = rng.uniform(0.0, 3.0, size=pool.params.shape[:2]).astype(np.float32)
    pool.rope[:] = owriter.bf16_bits(rng.standard_normal(pool.rope.shape).astype(np.float32))
    pt = (np.arange(batch_sample * pages) + 1).reshape(batch_sample, pages).astype(np.int32)
    q = owriter.bf16_bits(rng.standard_normal((batch_sample, HEADS, D + DR)).astype(np.float32))
    odecode.decode(pool, q, pt[:, :1], [64] * batch_sample, 0.07, dtype=np.float32)  # warm-up
    t0 = time.perf_counter()
    odecode.decode(pool, q, pt, [ctx] * batch_sample, 1 / math.sqrt(192), dtype=np.float32)
    dt = time.perf_counter() - t0
    del ocodec
    return dt / batch_sample


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_baseline(batch, ctx):
    per = cpu_decode_sample(2, ctx)
    step = per * batch * LAYERS
    return {"value": batch / step, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "cpu": cpu_model(),
            "sample": f"oracle.decode (numpy FP32, BLAS on all {os.cpu_count()} host threads): 2 requests x 1 layer "
                      f"x ctx {ctx}, i.e. 2/{LAYERS} of a token per request; tok/s = requests / ({LAYERS} x seconds "
                      "per request-layer)"}


def _reference_rotate_quantize():
    """The reference's own ``mla_quant.quantizer.rotate_quantize`` when the unmodified
    reference is installed in ``baseline/_ref`` (it travels with the repository copy),
    else None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "mla_quant" / "quantizer.py").exists():
        return None, None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    try:
        from mla_quant.numerics import configure_reference_numerics
        from mla_quant.quantizer import rotate_quantize
    except Exception:  # noqa: BLE001 -- an unusable install falls back to the port
        return None, None
    return rotate_quantize, configure_reference_numerics


def cpu_qdq_baseline(reps=10):
    """Config 0: the reference's PyTorch CPU quantize-dequantize (``rotate_quantize``,
    ``mla_quant/quantizer.py:102-124``) on one ``[1, 4096, 512]`` BF16 latent with an
    s4r16 mask, timed on this host at 1 thread and at all threads (median of ``reps``
    calls after 2 warm-ups).  The reference itself when ``baseline/_ref`` holds it, else
    the oracle's restatement (``oracle.quantizer``)."""
    from mla_kv_quant_b200 import synth

    n, d = 4096, 512
    lat = synth.latents(n, d, seed=0)  # BF16, configs[0] distribution
    r = synth.rotation(d, seed=1)
    t = float(torch.empty(1).uniform_(0.7, 1.0, generator=torch.Generator().manual_seed(2)))
    g = synth.signal_gain(t)
    mask = torch.zeros(n, dtype=torch.bool)
    mask[:4] = True
    mask[-16:] = True
    ref_fn, configure = _reference_rotate_quantize()
    if ref_fn is not None:
        configure()
        x3 = lat.reshape(1, n, d)
        tt, gt = torch.tensor(t, dtype=torch.float32), torch.tensor(g, dtype=torch.float32)

        def call():
            ref_fn(x3, r, 128, "oscar_lloyd", tt, gt, high_precision_mask=mask)

        kind, what = "reference", "mla_quant.quantizer.rotate_quantize from baseline/_ref (unmodified reference)"
    else:
        from oracle import quantizer as oquant

        xf, rf, mk = lat.float().numpy(), r.numpy(), mask.numpy()

        def call():
            oquant.rotate_quantize(xf, rf, t, g, mask=mk)

        kind, what = "port", "oracle.quantizer.rotate_quantize (restatement; the reference is not installed here)"
    out = {}
    prev = torch.get_num_threads()
    for label, threads in (("1_thread", 1), ("all_threads", os.cpu_count() or 1)):
        torch.set_num_threads(threads)
        for _ in range(2):
            call()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            call()
            ts.append(time.perf_counter() - t0)
        sec = statistics.median(ts)
        out[label] = {"threads": threads, "s_per_call": sec, "tok_s": n / sec,
                      "gbs": n * (2 * d + 2 * d) / sec / 1e9}
    torch.set_num_threads(prev)
    return {"config": "configs[0]: [1, 4096, 512] bf16 latent, R 512x512, s4r16 mask, group 128", "kind": kind,
            "what": what, "cpu": cpu_model(), "cores": os.cpu_count(), "reps": reps, "statistic": "median",
            "bytes_per_token": 2 * d + 2 * d, **out}


def run_reference(args, rank, world):
    """The reference arm: the path's CPU implementation on the host cores.  The reference's
    decode kernel is upstream Triton (not vendored), so the timed code is the oracle's
    restatement of its math (kind "port").  One *step* of this arm is one bounded sample of
    the benchmark workload, timed for real: ``REF_SAMPLE_REQS`` requests x 1 layer of the
    decode at the benchmark context, which is ``REF_SAMPLE_REQS / 27`` of a decode token per
    request; ``value`` = tokens/s = requests / (27 x seconds per request-layer), the same
    unit as our arm's.  ``ms_per_step`` is the measured sample time (not an extrapolation),
    so ``steps x ms_per_step`` is the real timed region."""
    if rank != 0:
        return None
    batch, ctx = args.batch, args.ctx
    reqs = REF_SAMPLE_REQS
    for _ in range(args.warmup):
        cpu_decode_sample(reqs, ctx, seed=1)
    times = []
    for i in range(args.steps):
        times.append(cpu_decode_sample(reqs, ctx, seed=2 + i) * reqs)  # seconds per sample
    step = statistics.median(times)
    val = reqs / (LAYERS * step)
    return {
        "metric": METRIC, "impl": "reference", "value": val, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decode step: {LAYERS} layers x batch {batch} x ctx {ctx}; one step of this arm = "
                               f"{reqs} requests x 1 layer of it (a bounded sample, timed as run)",
                   "batch_per_gpu": batch, "ctx": ctx, "parallelism": "host CPU, one process"},
        "cpu_baseline": {"value": val, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port", "cpu": cpu_model(),
                         "sample": f"oracle.decode (numpy FP32, BLAS on all {os.cpu_count()} host threads), "
                                   f"{reqs} requests x 1 layer x ctx {ctx} per step"},
        "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def profile_layer(args, what):
    """One layer of the benchmark shape for ncu captures (~0.3 GB on the device):
    fill the cache with the config-1 writer, then run 3 decode (or writer) launches."""
    from mla_kv_quant_b200 import ops, synth
    from mla_kv_quant_b200.pool import PackedLatentPool

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    batch, ctx = args.batch, args.ctx
    d, dr, heads, sm = (256, 32, 40, 1 / math.sqrt(96.0)) if args.shape == "minicpm3" else \
        (D, DR, HEADS, 1 / math.sqrt(192.0))
    pt, num_slots = synth.page_table(batch, ctx, seed=4, device=dev)
    pool = PackedLatentPool(num_slots, 1, d, dr, max_reqs=batch, sink=SINK, recent=RECENT, device=dev,
                            rotations={0: synth.rotation(d, 1000)}, quantizer_params=[(0.85, synth.signal_gain(0.85))])
    if d == D:
        fill_cache_layers(pool, pt, batch, ctx, dev, seed=0, layers=1)
    else:
        pos = torch.arange(ctx, device=dev)
        for b0 in range(0, batch, 8):
            bs = list(range(b0, min(batch, b0 + 8)))
            n = len(bs) * ctx
            slots = torch.cat([pt[b, pos // 64].long() * 64 + pos % 64 for b in bs])
            ops.fused_write(synth.latents(n, d, b0, dev), synth.normal_bf16((n, dr), b0 + 1, dev), slots,
                            pool.write_rotation_t(0), pool.codec(0), pool.layer_view(0),
                            seq_lens=torch.full((n,), ctx, dtype=torch.int32, device=dev),
                            req_idx=torch.tensor(bs, device=dev).repeat_interleave(ctx),
                            positions=pos.repeat(len(bs)).to(torch.int32))
        torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    times = []
    if what == "decode":
        splits = args.splits or ops.default_num_splits(batch, ctx, latent_dim=d, rope_dim=dr, heads=heads)
        q = synth.normal_bf16((batch, heads, d + dr), 3, dev)
        sl = torch.full((batch,), ctx, dtype=torch.int32, device=dev)
        po = torch.empty(batch, heads, splits + 1, d, device=dev)
        pl = torch.empty(batch, heads, splits + 1, device=dev)
        out = torch.empty(batch, heads, d, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            ev[0].record()
            ops.packed_decode(q, pool.layer_view(0), pt, sl, sm, splits, po, pl, out)
            ev[1].record()
            torch.cuda.synchronize()
            times.append(ev[0].elapsed_time(ev[1]) * 1e3)
        print(json.dumps({"mode": "decode-layer", "shape": args.shape, "us": times, "splits": splits,
                          "algorithmic_bytes": decode_bytes(batch, ctx, heads=heads, d=d, dr=dr)}))
    elif what == "absorbed":
        from mla_kv_quant_b200 import absorbed

        dn = dv = 128 if d == D else 64
        w = (synth.normal_bf16((heads * (dn + dv), d), 300, dev).float() * 0.05).to(torch.bfloat16)
        w_kc, w_vc = absorbed.split_absorbed_weights(w, heads, dn, dv)
        qn = synth.normal_bf16((batch, heads, dn), 21, dev)
        qp = synth.normal_bf16((batch, heads, dr), 22, dev)
        q = torch.empty(batch, heads, d + dr, dtype=torch.bfloat16, device=dev)
        o = synth.normal_bf16((batch, heads, d), 23, dev)
        y = torch.empty(batch, heads, dv, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            ev[0].record()
            absorbed.absorb_query(qn, qp, w_kc, out=q)
            absorbed.project_output(o, w_vc, out=y)
            ev[1].record()
            torch.cuda.synchronize()
            times.append(ev[0].elapsed_time(ev[1]) * 1e3)
        print(json.dumps({"mode": "absorbed-layer", "shape": args.shape, "us": times}))
    else:
        n = 8 * ctx
        x = synth.latents(n, D, 5, dev)
        pe = synth.normal_bf16((n, DR), 6, dev)
        slots = torch.arange(64, 64 + n, device=dev, dtype=torch.int64)
        for _ in range(3):
            ev[0].record()
            ops.fused_write(x, pe, slots, pool.write_rotation_t(0), pool.codec(0), pool.layer_view(0))
            ev[1].record()
            torch.cuda.synchronize()
            times.append(ev[0].elapsed_time(ev[1]) * 1e3)
        print(json.dumps({"mode": "writer-layer", "us": times, "rows": n, "algorithmic_bytes": writer_bytes(n),
                          "flops": 2.0 * n * D * D}))


def run_seqsplit(args, rank, world, dev):
    """Config 4b: one request of ``ctx`` tokens (131072 unless --ctx says otherwise) whose
    pages are split into contiguous page-aligned slices over the ranks.  Per layer: each
    rank decodes its slice (INT2 splits + window rows inside the slice, local LSE merge to
    FP32), one NCCL all-gather of the (o, lse) partials, the same merge kernel.  Latency is
    the max over ranks, timed with CUDA events; printed by rank 0 as one JSON line."""
    from mla_kv_quant_b200 import ops, synth
    from mla_kv_quant_b200.pool import PackedLatentPool
    from mla_kv_quant_b200.seqsplit import gather_merge, rank_token_range

    ctx = args.ctx if args.ctx != 16384 else 131072
    start, end = rank_token_range(ctx, world, rank)
    pt, num_slots = synth.page_table(1, ctx, seed=4, device=dev)
    pool = PackedLatentPool(num_slots, 1, D, DR, max_reqs=1, sink=SINK, recent=RECENT, device=dev,
                            rotations={0: synth.rotation(D, 1000)}, quantizer_params=[(0.85, synth.signal_gain(0.85))])
    view = pool.layer_view(0)
    # this rank fills (and later reads) only its own slice of the request
    n = end - start
    pos = torch.arange(start, end, device=dev)
    x = synth.latents(max(n, 1), D, 100 + rank, dev)[:n]
    pe = synth.normal_bf16((max(n, 1), DR), 200 + rank, dev)[:n]
    slots = (pt[0, pos // 64].long() * 64 + pos % 64).contiguous()
    if n > 0:
        ops.fused_write(x, pe, slots, pool.write_rotation_t(0), pool.codec(0), view,
                        seq_lens=torch.full((n,), ctx, dtype=torch.int32, device=dev),
                        req_idx=torch.zeros(n, dtype=torch.int64, device=dev), positions=pos.to(torch.int32))
    q = synth.normal_bf16((1, HEADS, D + DR), 3, dev)
    sl = torch.tensor([ctx], dtype=torch.int32, device=dev)
    rng = torch.tensor([[start, end]], dtype=torch.int32, device=dev)
    splits = args.splits or ops.default_num_splits(1, max(n, 64))
    parts = splits + 1
    part_o = torch.empty(1, HEADS, parts, D, device=dev)
    part_lse = torch.empty(1, HEADS, parts, device=dev)
    lse_loc = torch.empty(HEADS, device=dev)
    o_loc = torch.empty(HEADS, D, device=dev)
    sm = 1.0 / math.sqrt(192.0)

    def layer():  # the slice's FP32 partial and LSE, as SequenceSplitDecoder.local_partial
        ops.packed_decode(q, view, pt, sl, sm, splits, part_o, part_lse, None, token_range=rng)
        ops.merge_partials(part_o.view(HEADS, parts, D).transpose(0, 1), part_lse.view(HEADS, parts).t(),
                           out_f32=o_loc, out_lse=lse_loc)

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    kern, coll = [], []
    for it in range(args.warmup + args.steps):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev[0].record()
        layer()
        ev[1].record()
        if world > 1:
            gather_merge(o_loc, lse_loc)
        ev[2].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            kern.append(ev[0].elapsed_time(ev[1]) * 1e3)
            coll.append(ev[1].elapsed_time(ev[2]) * 1e3)
    k_us = sorted(kern)[len(kern) // 2]
    c_us = sorted(coll)[len(coll) // 2]

    # The same layer replayed from a CUDA graph, the NCCL all-gather captured with the decode
    # and the merge: no host launch gaps between them.
    def layer_and_merge():
        layer()
        if world > 1:
            gather_merge(o_loc, lse_loc)

    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        layer_and_merge()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer_and_merge()
    gl = []
    for it in range(args.warmup + args.steps):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev[0].record()
        graph.replay()
        ev[2].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            gl.append(ev[0].elapsed_time(ev[2]) * 1e3)
    reps = 50
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(reps):
        graph.replay()
    ev[2].record()
    torch.cuda.synchronize()
    gs_us = ev[0].elapsed_time(ev[2]) * 1e3 / reps
    del graph  # before the process group goes: the graph holds the NCCL call
    g_us = sorted(gl)[len(gl) // 2]

    # The same layer with the partials exchanged over NVLink peer memory (PeerExchange): the
    # slice's splits are merged and written into every rank's receive buffer by one kernel,
    # and the final merge waits for every rank's partial; eager and graph-replayed.  The
    # output is compared with the NCCL path's (max abs difference of the BF16 outputs).
    from mla_kv_quant_b200.seqsplit import PeerExchange

    if world > 1:
        ref32, _ = gather_merge(o_loc, lse_loc)
    else:
        ref32 = o_loc.clone()
    ref = ref32.to(torch.bfloat16).view(1, HEADS, D)
    xch = PeerExchange(HEADS, D, device=dev)
    out_p = torch.empty(1, HEADS, D, dtype=torch.bfloat16, device=dev)
    perr = torch.zeros(1, dtype=torch.int32, device=dev)

    def layer_peer():
        ops.packed_decode(q, view, pt, sl, sm, splits, part_o, part_lse, None, token_range=rng)
        xch.exchange(part_o, part_lse, out_bf16=out_p, err=perr)

    pl = []
    for it in range(args.warmup + args.steps):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev[0].record()
        layer_peer()
        ev[2].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            pl.append(ev[0].elapsed_time(ev[2]) * 1e3)
    peer_diff = float((out_p.float() - ref.float()).abs().max())
    with torch.cuda.stream(side):
        layer_peer()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer_peer()
    pg = []
    for it in range(args.warmup + args.steps):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev[0].record()
        graph.replay()
        ev[2].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            pg.append(ev[0].elapsed_time(ev[2]) * 1e3)
    # steady state: the graph replayed back to back, as consecutive decode steps run; the
    # exchange itself keeps the ranks in step (no host barrier between replays)
    reps = 50
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(reps):
        graph.replay()
    ev[2].record()
    torch.cuda.synchronize()
    ps_us = ev[0].elapsed_time(ev[2]) * 1e3 / reps
    del graph
    peer_err = int(perr.item())
    xch.close()
    p_us, pg_us = sorted(pl)[len(pl) // 2], sorted(pg)[len(pg) // 2]

    t = torch.tensor([k_us, c_us, k_us + c_us, g_us, p_us, pg_us, peer_diff, float(peer_err), ps_us, gs_us],
                     device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return {"mode": "seqsplit", "n_gpus": world, "batch": 1, "ctx": ctx, "tokens_per_rank": n,
            "num_splits_per_rank": splits, "us_per_layer": float(t[2]), "kernel_us": float(t[0]),
            "gather_merge_us": float(t[1]), "us_per_layer_graph": float(t[3]),
            "us_per_layer_graph_steady": float(t[9]),
            "peer": {"us_per_layer": float(t[4]), "us_per_layer_graph": float(t[5]),
                     "us_per_layer_graph_steady": float(t[8]),
                     "max_abs_diff_vs_nccl": float(t[6]), "err_bits": int(t[7]),
                     "path": "the slice's split partials (window split + INT2 kernel, no merge) + one kernel that "
                             "merges them and writes the FP32 partial into every rank's receive buffer over "
                             "NVLink (CUDA IPC) + a merge that waits for every rank's partial; no library "
                             "collective"},
            "note": "median over steps of each rank, max over ranks; kernel = the slice's split partials (INT2 "
                    "splits + window) and their FP32 merge, gather_merge = one NCCL "
                    "all-gather of the (o, lse) partials + the merge kernel (eager launches); "
                    "us_per_layer_graph = the same layer replayed from a CUDA graph after a host barrier "
                    "(includes the ranks' start skew); *_steady = 50 replays back to back / 50"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--mode", choices=["step", "decode-layer", "writer-layer", "absorbed-layer", "seqsplit", "batch4a"],
                    default="step",
                    help="step: the benchmark; *-layer: one layer, 3 launches (for ncu captures); "
                         "seqsplit: one 128K-token request split over the ranks (latency per layer); "
                         "batch4a: 512 requests x 32K sharded over the ranks")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=16384)
    ap.add_argument("--splits", type=int, default=0, help="INT2 KV splits per request (0: auto)")
    ap.add_argument("--shape", choices=["dsv2", "minicpm3"], default="dsv2",
                    help="latent / rope / heads of the *-layer modes: DeepSeek-V2-Lite 512/64/16 or "
                         "MiniCPM3-4B 256/32/40")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true", help="skip the configs 3a / 3b lines")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.mode == "seqsplit":
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        if world > 1:
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        res = run_seqsplit(args, rank, world, dev)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        if rank == 0:
            print(json.dumps(res))
        return 0
    if args.mode == "batch4a":
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        if world > 1:
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            print(f"rank {rank}/{world} on {torch.cuda.get_device_name(dev)} "
                  f"({torch.cuda.get_device_properties(dev).uuid})", file=sys.stderr)
        res = run_batch4a(args, rank, world, dev)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        if rank == 0:
            print(json.dumps(res))
        return 0
    if args.mode != "step":
        profile_layer(args, args.mode.split("-")[0])
        return 0

    if args.impl == "reference":
        if world > 1:
            # only rank 0 runs the CPU reference; the other ranks exit without work
            if rank != 0:
                return 0
        res = run_reference(args, rank, world)
        print(json.dumps(res))
        return 0

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        print(f"rank {rank}/{world} on {torch.cuda.get_device_name(dev)} "
              f"({torch.cuda.get_device_properties(dev).uuid})", file=sys.stderr)
    res = run_ours(args, rank, world, dev)
    if world == 1 and not args.no_extra_configs:
        res["configs"] = {name: decode_step_config(dev, **cfg, steps=max(3, min(args.steps, 20)), warmup=args.warmup)
                          for name, cfg in EXTRA_CONFIGS.items()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(args.batch, args.ctx)
        res["cpu_qdq_baseline"] = cpu_qdq_baseline()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
