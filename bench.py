#!/usr/bin/env python
"""Benchmark: ConvMixer-1536/20 images/s on N B200s, plus every BASELINE depthwise layer's
µs/layer and roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Headline workload: ConvMixer-1536/20 ks9 p7 GELU
inference, batch 1 per GPU (weak scaling: every GPU runs its own batch-1
replica, no collectives), fp16 NHWC, random init (weights N(0,0.02), BN gamma
1 beta 0 mean 0 var 1), synthetic N(0,1) 3x224x224 inputs.  Each depthwise
block (DW conv + GELU + BN + residual) is one kernel of this engine; the 1x1
convs and the stem are cuBLAS GEMMs followed by one engine epilogue kernel.
The forward is captured in a CUDA graph and replayed.

One JSON line (rank 0):
  value     whole-job images/s with inputs already in HBM (device-timed, max over ranks)
  e2e       the same metric through the public API with a pinned-host input
            copied in and the logits copied out inside the timed region
  roofline  the depthwise kernel on the model's layer shape (1x32x32x1536,
            k9, fused GELU+BN+residual), against the CUDA-core FMA rate
            measured in this run
  cpu_baseline  the reference's CPU path (fp32 PyTorch ConvMixer, depthwise
            via conv2d(groups=C)) timed on this host's cores, rank 0, N=1
  convmixer_768_32  BASELINE configs[0]: the same measurement for ConvMixer-768/32
  dw_configs  every depthwise layer of BASELINE configs[1..4] (RepLKNet C3-C6, the
            ConvMixer layers C1/C2, the k9 batch sweep B in {1,16,64,256}, the
            k-sweep k in {7..31} at B=64 with GELU+BN): µs/layer warm (CUDA graph
            of back-to-back launches, the reference's protocol) and cold (L2
            flushed before every launch), images/s, FMA and HBM roofline
            fractions, and (N=1) the reference's CPU path for the same layer.
            Batched configs are sharded over the ranks (strong scaling); the
            batch-1 configs run as one replica per GPU.

--impl reference times that CPU path alone (the reference's own GPU ops are
not an installable package, and its tier here is the CPU path) with the same
metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "ConvMixer-1536/20 img/s (DW-conv µs/layer & % roofline)"
DW_SHAPE = (1, 32, 32, 1536, 9)  # B, H, W, C, K of the model's depthwise layers
L2_FLUSH_BYTES = 256 << 20       # > 126 MB L2: flushed between timed iterations


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1, help="images per GPU per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    ap.add_argument("--workload", choices=["convmixer", "dw"], default="convmixer",
                    help="convmixer: the headline ConvMixer-1536/20 img/s; dw: one depthwise layer (µs/layer)")
    ap.add_argument("--shape", default="64,56,56,1024,31",
                    help="dw workload: global B,H,W,C,K (the batch is sharded over the ranks)")
    ap.add_argument("--epilogue", choices=["none", "gelu_bn", "gelu_bn_res"], default="gelu_bn",
                    help="dw workload: plain conv, the fused bias+GELU+BN-scale/shift epilogue, or that plus the "
                         "residual add of a ConvMixer block (residual = the input)")
    ap.add_argument("--accum", choices=["mixed", "f32"], default="mixed")
    ap.add_argument("--backward", action="store_true",
                    help="--workload dw: also time the layer's gradients (input and weight), warm protocol")
    ap.add_argument("--no-dw-configs", action="store_true",
                    help="convmixer workload: skip the per-layer section (dw_configs) and ConvMixer-768/32")
    ap.add_argument("--dw-configs-only", default="",
                    help="comma-separated dw_configs names to run (default: all)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi takes a moment to start: wait (bounded) for its first sample so the
        # samples that follow fall inside the timed region
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < 5.0:
            time.sleep(0.01)
        self.first = len(self.lines)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[getattr(self, "first", 0):] or self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- helpers

def valid_flops(B, H, W, C, K):
    """FLOPs of the in-image taps only (padding zeros are free work a kernel may skip)."""
    p = K // 2
    vh = sum(min(K, H + p - h) - max(0, p - h) for h in range(H))
    vw = sum(min(K, W + p - w) - max(0, p - w) for w in range(W))
    return 2.0 * B * C * vh * vw


def dw_bytes(B, H, W, C, K, epilogue=True):
    """Algorithmic HBM bytes of one layer: input and output once, weights once (+ bias/scale/shift, residual)."""
    b = 2 * (2 * B * C * H * W) + 2 * K * K * C
    if epilogue:
        b += 3 * 2 * C + 2 * B * C * H * W  # bias, scale, shift and the residual read
    return b


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def profiled_traffic():
    """DRAM bytes per launch of the DW kernel from the committed ncu summary (profiles/dw_traffic.txt):
    {name: bytes, or {"bytes": B, "source": ...}}."""
    path = os.path.join(ROOT, "profiles", "dw_traffic.txt")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# ----------------------------------------------------------------------------- CPU baseline

def cpu_convmixer_rate(seconds: float, max_images: int | None = None, name: str = "1536_20"):
    """img/s of the fp32 CPU ConvMixer (reference's CPU path) on a bounded sample."""
    import torch
    from oracle.convmixer_ref import convmixer_cpu

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = convmixer_cpu(name, seed=0)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, 3, 224, 224, generator=g)
    model(x)  # warm-up (allocator, thread pool)
    n, t0 = 0, time.perf_counter()
    while True:
        model(x)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_images and n >= max_images):
            break
    return n / el, threads, n, el


def cpu_layer_us(B, H, W, C, K, seconds: float = 5.0, epilogue: bool = False):
    """The reference's CPU path for one depthwise layer -- torch fp32 conv2d(groups=C), NCHW and
    channels_last, the faster kept (with ``epilogue``: + bias, exact GELU and the BN scale/shift, the
    sequence of benchmark_cudnn_fused_e2e.py:65-74) -- timed on this host's cores on a bounded sample
    of images and scaled to the whole batch: (µs per layer of B images, threads, images timed, layout)."""
    import torch
    import torch.nn.functional as F

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, C, H, W, generator=g)
    w = torch.randn(C, 1, K, K, generator=g) / K
    b = torch.zeros(C)
    s = torch.full((1, C, 1, 1), 1.0 / (1.0 + 1e-5) ** 0.5)
    t = torch.zeros(1, C, 1, 1)

    def layer(xi):
        if not epilogue:
            return F.conv2d(xi, w, padding=K // 2, groups=C)
        return F.gelu(F.conv2d(xi, w, b, padding=K // 2, groups=C)) * s + t

    best = None
    for layout in ("nchw", "channels_last"):
        xi = x.contiguous(memory_format=torch.channels_last) if layout == "channels_last" else x
        layer(xi)  # warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            layer(xi)
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds / 2 or n >= 10000:
                break
        per_image = el / n
        if best is None or per_image < best[0]:
            best = (per_image, n, layout)
    return best[0] * B * 1e6, threads, best[1], best[2]


# ----------------------------------------------------------------------------- our arm

# Every depthwise layer of BASELINE configs[1..4]: (name, B, H, W, C, K, epilogue, sharding).
# "replica": a batch-1 layer, one per GPU (weak scaling); "batch": the global batch is split over
# the ranks (strong scaling).  x ~ N(0,1), w ~ N(0,1/K^2); the k-sweep adds bias 0, BN scale
# 1/sqrt(1+1e-5), shift 0 and the exact GELU.
DW_CONFIGS = [
    ("C1_32x32x768_k7", 1, 32, 32, 768, 7, "none", "replica"),
    ("C2_32x32x1536_k9", 1, 32, 32, 1536, 9, "none", "replica"),
    ("C3_56x56x128_k31", 1, 56, 56, 128, 31, "none", "replica"),
    ("C4_28x28x256_k29", 1, 28, 28, 256, 29, "none", "replica"),
    ("C5_14x14x512_k27", 1, 14, 14, 512, 27, "none", "replica"),
    ("C6_7x7x1024_k13", 1, 7, 7, 1024, 13, "none", "replica"),
] + [(f"bsweep_k9_b{b}", b, 32, 32, 1536, 9, "none", "replica" if b == 1 else "batch") for b in (1, 16, 64, 256)] \
  + [(f"ksweep_k{k}_b64", 64, 56, 56, 1024, k, "gelu_bn", "batch") for k in (7, 9, 13, 17, 21, 27, 29, 31)]


def _graph_warm_us(torch, fn, stream, target_ms=30.0):
    """The reference's warm protocol (bench_custom_warm.py:17-31: back-to-back launches, inputs left
    in L2 when they fit), as a CUDA graph of `reps` launches: best of 3 replays, µs per launch."""
    with torch.cuda.stream(stream):
        fn()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        stream.synchronize()
        est_us = max(1.0, e0.elapsed_time(e1) * 1000.0)
        reps = int(max(3, min(200, target_ms * 1000.0 / est_us)))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                fn()
        g.replay()
        stream.synchronize()
        best = 1e30
        for _ in range(3):
            e0.record(stream)
            g.replay()
            e1.record(stream)
            stream.synchronize()
            best = min(best, e0.elapsed_time(e1) / reps)
    del g
    return best * 1000.0, reps


def _cold_us(torch, fn, stream, flush, n):
    """Mean µs per launch with the L2 flushed (a write larger than L2) before every launch, each
    launch bracketed by its own CUDA events (benchmark_batch_sweep.py:154-178's per-iteration events)."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    with torch.cuda.stream(stream):
        for s_, e_ in evs:
            flush.add_(1.0)
            s_.record(stream)
            fn()
            e_.record(stream)
        stream.synchronize()
    return sum(s_.elapsed_time(e_) for s_, e_ in evs) / n * 1000.0


def run_dw_configs(args, dev, stream, flush, rank, world, hfma2_tf, only=()):
    """µs/layer of every BASELINE depthwise layer on this rank's share; times are the max over ranks."""
    import torch

    import depthwise_conv_b200 as dwb
    from depthwise_conv_b200 import _lib
    from depthwise_conv_b200.shard import max_over_ranks, shard_range

    peaks = measured_peaks()
    traffic = profiled_traffic()
    out = []
    data = {}  # (B, H, W, C) -> the global input batch, generated once from a fixed seed on every rank
    do_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    cpu_cache = {}
    for name, Bg, H, W, C, K, epi, shard in DW_CONFIGS:
        if only and name not in only:
            continue
        if shard == "batch":
            lo, hi = shard_range(Bg, world, rank)
        else:
            lo, hi = 0, Bg
        B = hi - lo
        key = (Bg, H, W, C)
        if key not in data:
            data.clear()
            torch.cuda.empty_cache()
            gen = torch.Generator(device=dev).manual_seed(1234 + Bg + H + C)
            data[key] = torch.randn((Bg, H, W, C), generator=gen, device=dev, dtype=torch.float16)
        xg = data[key]
        x = xg[lo:hi].permute(0, 3, 1, 2)  # channels_last view of this rank's images
        gw = torch.Generator(device=dev).manual_seed(99 + K)
        w = (torch.randn((K, K, C), generator=gw, device=dev) / K).half()
        kw = {}
        if epi == "gelu_bn":
            kw = dict(bias=torch.zeros(C, dtype=torch.float16, device=dev),
                      scale=torch.full((C,), 1.0 / (1.0 + 1e-5) ** 0.5, dtype=torch.float16, device=dev),
                      shift=torch.zeros(C, dtype=torch.float16, device=dev), act="gelu")
        y = torch.empty_like(x)
        fn = (lambda: dwb.conv2d_nhwc_fused(x, w, out=y, **kw))  # noqa: E731
        warm = cold = 0.0
        reps = 0
        if B:
            warm, reps = _graph_warm_us(torch, fn, stream)
            cold = _cold_us(torch, fn, stream, flush, 5 if warm > 1000 else 20)
        warm = max_over_ranks(warm, dev)
        cold = max_over_ranks(cold, dev)
        images = Bg if shard == "batch" else world * Bg
        fl_gpu = valid_flops(Bg, H, W, C, K) / (world if shard == "batch" else 1)  # per GPU
        by = dw_bytes(Bg, H, W, C, K, epilogue=False) + (3 * 2 * C if epi != "none" else 0)
        by_gpu = by / (world if shard == "batch" else 1)
        ent = {"name": name, "B": Bg, "H": H, "W": W, "C": C, "K": K, "epilogue": epi,
               "parallelism": (f"batch-sharded x{world}" if shard == "batch" else f"replicas x{world}"),
               "warm_us": warm, "cold_us": cold, "warm_reps": reps,
               "images_per_s_warm": images / (warm * 1e-6) if warm else None,
               "images_per_s_cold": images / (cold * 1e-6) if cold else None,
               "valid_flops_per_gpu": fl_gpu,
               "fma_frac_warm": fl_gpu / (warm * 1e-6) / 1e12 / hfma2_tf if warm else None,
               "fma_frac_cold": fl_gpu / (cold * 1e-6) / 1e12 / hfma2_tf if cold else None,
               "hbm_bytes_per_gpu": by_gpu,
               "hbm_frac_cold": (by_gpu / (cold * 1e-6) / 1e9 / peaks["hbm_gbs"]) if cold and peaks.get("hbm_gbs")
               else None}
        if B:
            pl = _lib.plan_select(B, H, W, C, K)
            ent["kernel"] = "dw_band_kernel" if pl["band_tiles"] else "dw_stream_kernel"
            ent["plan"] = {k: pl[k] for k in ("cols_per_thread", "rows_per_thread", "tile_h", "tile_w", "ring_rows",
                                              "consumer_warps", "grid", "row_splits", "load_schedule", "band_tiles")}
        tr = traffic.get(name)
        if tr is not None:
            ent["dram_traffic"] = tr
        if do_cpu:
            ck = (H, W, C, K, epi)
            if ck not in cpu_cache:
                cpu_cache[ck] = cpu_layer_us(1, H, W, C, K, seconds=1.5, epilogue=epi != "none")
            us1, threads, n, layout = cpu_cache[ck]
            ent["cpu_baseline"] = {"us_per_layer": us1 * Bg, "cores": threads, "kind": "port",
                                   "sample": f"{n} single-image fp32 conv2d(groups=C) calls ({layout})"
                                             + (" + GELU + BN" if epi != "none" else "") + f", scaled to B={Bg}"}
        out.append(ent)
        del y, x, w
    data.clear()
    return out


def convmixer_rates(args, name, dev, stream, flush, rank, world):
    """Device-timed and end-to-end images/s of one ConvMixer at batch args.batch per GPU (max over ranks)."""
    import torch

    from depthwise_conv_b200.convmixer import convmixer, fuse_dw_blocks
    from depthwise_conv_b200.shard import max_over_ranks

    B = args.batch
    model = convmixer(name, seed=0).half().to(dev).to(memory_format=torch.channels_last)
    fuse_dw_blocks(model)
    # engine kernels per forward: one per fused DW block, pointwise epilogue and the stem epilogue
    ours_per_step = sum(1 for m in model.modules()
                        if m.__class__.__name__ in ("FusedDWBlock", "FusedPointwiseBlock", "FusedStem"))
    g = torch.Generator().manual_seed(1000 + rank)
    host_in = torch.randn(B, 3, 224, 224, generator=g).half().contiguous(memory_format=torch.channels_last)
    host_in = host_in.pin_memory()
    host_out = torch.empty(B, 1000, dtype=torch.float16).pin_memory()
    static_in = host_in.to(dev, non_blocking=False)
    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            model(static_in)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            static_out = model(static_in)
        for _ in range(args.warmup):
            graph.replay()
        stream.synchronize()

    def timed_loop(e2e: bool) -> float:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.add_(1.0)  # L2 flush, outside the timed window
                s, e = evs[i]
                s.record(stream)
                if e2e:
                    static_in.copy_(host_in, non_blocking=True)
                graph.replay()
                if e2e:
                    host_out.copy_(static_out, non_blocking=True)
                e.record(stream)
            stream.synchronize()
        return sum(s.elapsed_time(e) for s, e in evs)

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(dev)
    dev_ms = timed_loop(e2e=False)
    torch.cuda.synchronize(dev)
    e2e_ms = timed_loop(e2e=True)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    dev_ms_max = max_over_ranks(dev_ms, dev)
    e2e_ms_max = max_over_ranks(e2e_ms, dev)
    del graph
    images = B * world * args.steps
    return {"model": model, "value": images / (dev_ms_max / 1000.0), "e2e": images / (e2e_ms_max / 1000.0),
            "ms_per_step": dev_ms_max / args.steps, "e2e_ms_per_step": e2e_ms_max / args.steps,
            "h2d": host_in.numel() * host_in.element_size() * world,
            "d2h": host_out.numel() * host_out.element_size() * world,
            "launches_per_step": ours_per_step}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import depthwise_conv_b200 as dwb
    from depthwise_conv_b200 import _lib

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    torch.backends.cudnn.benchmark = True
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)

    clocks = ClockSampler(local)
    clocks.start()
    head = convmixer_rates(args, "1536_20", dev, stream, flush, rank, world)
    clk = clocks.stop()
    model = head.pop("model")

    # ---- the depthwise kernel alone on the model's layer shape (roofline) ----
    Bd, H, W, C, K = DW_SHAPE
    blk = next(m for m in model.modules() if m.__class__.__name__ == "FusedDWBlock")
    x = torch.randn(Bd, C, H, W, generator=torch.Generator().manual_seed(7)).half().to(dev)
    x = x.contiguous(memory_format=torch.channels_last)
    y = torch.empty_like(x)
    with torch.no_grad():
        dw_us, _ = _graph_warm_us(torch, lambda: dwb.conv2d_nhwc_fused(x, blk.weight, blk.bias, blk.scale, blk.shift,
                                                                       x, "gelu", out=y), stream, target_ms=2.0)
        hfma2_tf, ffma2_tf = dwb.probe_fma_peak(stream.cuda_stream)
    fl = valid_flops(Bd, H, W, C, K)
    achieved_tf = fl / (dw_us * 1e-6) / 1e12
    peaks = measured_peaks()
    traffic = profiled_traffic().get("convmixer1536_dw_layer")
    dw_gbs = dw_bytes(Bd, H, W, C, K) / (dw_us * 1e-6) / 1e9
    plan = _lib.plan_select(Bd, H, W, C, K)
    del model

    extra, dw_cfg, clk_cfg = None, None, None
    if not args.no_dw_configs:
        clocks2 = ClockSampler(local)
        clocks2.start()
        m768 = convmixer_rates(args, "768_32", dev, stream, flush, rank, world)
        del m768["model"]
        extra = m768
        only = tuple(v for v in args.dw_configs_only.split(",") if v)
        dw_cfg = run_dw_configs(args, dev, stream, flush, rank, world, hfma2_tf, only)
        clk_cfg = clocks2.stop()

    cpu = cpu768 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, threads, n, el = cpu_convmixer_rate(args.cpu_seconds)
        cpu = {"value": rate, "unit": "img/s", "cores": threads, "kind": "port",
               "sample": f"{n} images of ConvMixer-1536/20 fp32 forward on the CPU in {el:.1f} s "
                         f"(oracle/convmixer_ref.py; depthwise via torch conv2d groups=C)"}
        if extra is not None:
            rate, threads, n, el = cpu_convmixer_rate(args.cpu_seconds / 2, name="768_32")
            cpu768 = {"value": rate, "unit": "img/s", "cores": threads, "kind": "port",
                      "sample": f"{n} images of ConvMixer-768/32 fp32 forward on the CPU in {el:.1f} s"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    B = args.batch
    line = {
        "metric": METRIC, "value": head["value"], "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (depthwise: fp16x2 FMA, fp32 accumulation)",
        "data": "synthetic N(0,1) 3x224x224 images, random-init weights (no checkpoint)",
        "config": {"workload": "ConvMixer-1536/20 ks9 p7 GELU inference (BASELINE configs[1])",
                   "batch_per_gpu": B, "global_batch": B * world, "image": "3x224x224", "layout": "NHWC fp16",
                   "parallelism": f"replicas x{world} (batch-sharded, no collectives)",
                   "cuda_graph": True, "l2": "flushed (256 MB write) between timed iterations",
                   "dw_layer": {"B": Bd, "H": H, "W": W, "C": C, "K": K,
                                "epilogue": "bias+GELU+BN+residual fused",
                                "plan": {k: plan[k] for k in ("cols_per_thread", "rows_per_thread", "tile_h",
                                                              "tile_w", "ring_rows", "consumer_warps", "grid",
                                                              "row_splits", "band_tiles", "accum")}}},
        "e2e": {"value": head["e2e"], "unit": "img/s", "h2d_bytes_per_step": head["h2d"],
                "d2h_bytes_per_step": head["d2h"]},
        "dw_us_per_layer": dw_us,
        "roofline": {"bound": "fma", "achieved": achieved_tf, "peak": hfma2_tf, "unit": "TFLOP/s",
                     "frac": achieved_tf / hfma2_tf, "traffic": traffic,
                     "peak_source": "measured in this run: CUDA-core HFMA2 microbenchmark (dwb_probe_fma_peak); "
                                    "MEASURED_PEAKS.json has no CUDA-core FMA figure",
                     "kernel": ("dw_band_kernel" if plan.get("band_tiles") else "dw_stream_kernel") +
                               " on 1x32x32x1536 k9 with bias+GELU+BN+residual (the model's DW layer)",
                     "flops_per_launch": fl, "ffma2_peak": ffma2_tf,
                     "hbm": {"achieved": dw_gbs, "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                             "frac": dw_gbs / peaks["hbm_gbs"] if peaks.get("hbm_gbs") else None,
                             "bytes_per_launch": dw_bytes(Bd, H, W, C, K)}},
        "cpu_baseline": cpu,
        "gpu_launches": head["launches_per_step"] * args.steps * 2,  # two timed loops: device-resident and e2e
        "clocks": clk,
    }
    if extra is not None:
        line["convmixer_768_32"] = {
            "workload": "ConvMixer-768/32 ks7 p7 ReLU inference (BASELINE configs[0])", "unit": "img/s",
            "value": extra["value"], "ms_per_step": extra["ms_per_step"],
            "e2e": {"value": extra["e2e"], "unit": "img/s", "h2d_bytes_per_step": extra["h2d"],
                    "d2h_bytes_per_step": extra["d2h"]},
            "parallelism": f"replicas x{world}", "batch_per_gpu": B, "cpu_baseline": cpu768}
    if dw_cfg is not None:
        line["dw_configs"] = dw_cfg
        line["dw_configs_clocks"] = clk_cfg
        line["dw_configs_protocol"] = (
            "warm: CUDA graph of back-to-back launches, best of 3 replays (bench_custom_warm.py:17-31); cold: L2 "
            "flushed (256 MB write) before each launch, per-launch CUDA events, mean; times are the max over "
            "ranks; fma_frac = valid FLOPs per GPU / time / the HFMA2 peak measured in this run; inputs seeded "
            "on the device, x ~ N(0,1), w ~ N(0,1/K^2)")
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- one depthwise layer

def run_dw(args):
    """µs/layer of one depthwise layer (BASELINE configs[2..4]); the batch is sharded over the ranks."""
    import torch
    import torch.distributed as dist

    import depthwise_conv_b200 as dwb
    from depthwise_conv_b200 import _lib
    from depthwise_conv_b200.shard import max_over_ranks, shard_range

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    Bg, H, W, C, K = (int(v) for v in args.shape.split(","))
    lo, hi = shard_range(Bg, world, rank)
    B = hi - lo
    accum = _lib.ACCUM_MIXED if args.accum == "mixed" else _lib.ACCUM_F32
    gen = torch.Generator().manual_seed(0)
    # seeded per image so every GPU count sees the same data: x ~ N(0,1), w ~ N(0, 1/K^2)
    x = torch.randn(Bg, C, H, W, generator=gen)[lo:hi].half().to(dev).contiguous(memory_format=torch.channels_last)
    w = (torch.randn(K, K, C, generator=gen) / K).half().to(dev)
    epi = args.epilogue in ("gelu_bn", "gelu_bn_res")
    res = x if args.epilogue == "gelu_bn_res" else None  # a ConvMixer block adds its input
    bias = torch.zeros(C, dtype=torch.float16, device=dev) if epi else None
    scale = torch.full((C,), 1.0 / (1.0 + 1e-5) ** 0.5, dtype=torch.float16, device=dev) if epi else None
    shift = torch.zeros(C, dtype=torch.float16, device=dev) if epi else None
    act = "gelu" if epi else "none"
    y = torch.empty_like(x)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)
    layer = lambda: dwb.conv2d_nhwc_fused(x, w, bias, scale, shift, res, act, accum, out=y)  # noqa: E731
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            if B:
                layer()
        stream.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush.add_(1.0)  # L2 flush between timed iterations
            evs[i][0].record(stream)
            if B:
                layer()
            evs[i][1].record(stream)
        stream.synchronize()
    clk = clocks.stop()
    ms = sum(s.elapsed_time(e) for s, e in evs)
    # warm protocol (the reference's: back-to-back launches, inputs in L2 when they fit): a CUDA
    # graph of `reps` launches, best of 3 replays
    warm_us = None
    if B:
        reps = max(3, min(200, int(2e5 // max(1.0, ms * 1000.0 / args.steps))))
        with torch.cuda.stream(stream):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(reps):
                    layer()
            g.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            best = 1e30
            for _ in range(3):
                e0.record(stream)
                g.replay()
                e1.record(stream)
                stream.synchronize()
                best = min(best, e0.elapsed_time(e1) / reps)
        del g
        warm_us = best * 1000.0

    def warm_time(fn, reps=20):
        with torch.cuda.stream(stream):
            fn()
            stream.synchronize()
            gb = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gb, stream=stream):
                for _ in range(reps):
                    fn()
            gb.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            best = 1e30
            for _ in range(3):
                e0.record(stream)
                gb.replay()
                e1.record(stream)
                stream.synchronize()
                best = min(best, e0.elapsed_time(e1) / reps)
        del gb
        return best * 1000.0

    bwd = None
    if args.backward and B:
        dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(1)).half().to(dev).contiguous(
            memory_format=torch.channels_last)
        w_rot = torch.empty_like(w)
        dx = torch.empty_like(x)
        dw = torch.zeros((K, K, C), dtype=torch.float32, device=dev)
        s_ = lambda: stream.cuda_stream  # noqa: E731

        def bwd_input():
            _lib.call("dwb_weight_rot180", w.data_ptr(), w_rot.data_ptr(), C, K, s_())
            _lib.call("dwb_conv2d_nhwc_bwd_data", dy.data_ptr(), w_rot.data_ptr(), dx.data_ptr(), B, H, W, C, K, s_())

        def bwd_weight():
            dw.zero_()
            _lib.call("dwb_conv2d_nhwc_bwd_weight", x.data_ptr(), dy.data_ptr(), dw.data_ptr(), B, H, W, C, K, s_())

        bwd = {"input_us": warm_time(bwd_input), "weight_us": warm_time(bwd_weight)}
    if world > 1:
        dist.barrier()
    ms_max = max_over_ranks(ms, dev)
    warm_max = max_over_ranks(warm_us if warm_us is not None else 0.0, dev)
    if args.backward:
        bwd = {k: max_over_ranks(bwd[k] if bwd else 0.0, dev) for k in ("input_us", "weight_us")}
    us_layer = ms_max * 1000.0 / args.steps
    hfma2_tf, ffma2_tf = dwb.probe_fma_peak(stream.cuda_stream)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    fl = valid_flops(Bg, H, W, C, K)
    by = dw_bytes(Bg, H, W, C, K, epilogue=False) + (3 * 2 * C if epi else 0) + (2 * Bg * H * W * C if res is not None
                                                                                  else 0)
    achieved = fl / world / (us_layer * 1e-6) / 1e12  # per GPU: each rank's launch covers its batch shard
    peaks = measured_peaks()
    plan = _lib.plan_select(max(1, -(-Bg // world)), H, W, C, K, accum)
    line = {
        "metric": "DW-conv µs/layer", "value": us_layer, "unit": "us/layer", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": us_layer / 1000.0, "higher_is_better": False,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "fp16 (" + ("fp16x2 FMA chains, fp32 accumulation" if accum else "fp32 FMA") + ")",
        "data": "synthetic x ~ N(0,1), w ~ N(0,1/k^2), seeded",
        "config": {"workload": "depthwise layer", "B": Bg, "H": H, "W": W, "C": C, "K": K,
                   "epilogue": args.epilogue, "images_per_s": Bg / (us_layer * 1e-6),
                   "warm_us_per_layer": warm_max, "warm_fma_frac": (fl / world / (warm_max * 1e-6) / 1e12 / hfma2_tf)
                   if warm_max > 0 else None,
                   "backward": None if not args.backward else {
                       "input_grad_us": bwd["input_us"], "weight_grad_us": bwd["weight_us"],
                       "input_grad_fma_frac": fl / world / (bwd["input_us"] * 1e-6) / 1e12 / hfma2_tf,
                       "weight_grad_fma_frac": fl / world / (bwd["weight_us"] * 1e-6) / 1e12 / hfma2_tf,
                       "protocol": "warm, CUDA graph of 20 launches; dy ~ N(0,1); same valid FLOPs as the forward"},
                   "parallelism": f"batch-sharded x{world}, no collectives",
                   "l2": "flushed (256 MB write) between timed iterations",
                   "plan": {k: plan[k] for k in ("cols_per_thread", "rows_per_thread", "tile_h", "tile_w",
                                                 "ring_rows", "consumer_warps", "grid", "row_splits", "band_tiles",
                                                 "accum")}},
        "roofline": {"bound": "fma", "achieved": achieved, "peak": hfma2_tf, "unit": "TFLOP/s",
                     "frac": achieved / hfma2_tf, "flops_per_launch": fl / world,
                     "traffic": profiled_traffic().get(f"dw_{Bg}_{H}_{W}_{C}_{K}"),
                     "peak_source": "measured in this run: CUDA-core HFMA2 microbenchmark",
                     "hbm": {"achieved": by / world / (us_layer * 1e-6) / 1e9, "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                             "bytes_per_launch": by}},
        "gpu_launches": args.steps,  # the timed (cold) loop; the warm graph is timed separately
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        cpu_us, threads, n, layout = cpu_layer_us(Bg, H, W, C, K)
        line["cpu_baseline"] = {"value": cpu_us, "unit": "us/layer", "cores": threads, "kind": "reference",
                                "sample": f"{n} single-image fp32 conv2d(groups=C) calls ({layout}) on the host, "
                                          f"scaled to B={Bg}; epilogue not included"}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- reference arm

def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return  # the CPU reference runs once, on rank 0
    import torch
    from oracle.convmixer_ref import convmixer_cpu

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = convmixer_cpu("1536_20", seed=0)
    x = torch.randn(args.batch, 3, 224, 224, generator=torch.Generator().manual_seed(1))
    for _ in range(args.warmup):
        model(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model(x)
    el = time.perf_counter() - t0
    rate = args.batch * args.steps / el
    line = {
        "metric": METRIC, "value": rate, "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el * 1000.0 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "impl": "reference",
        "data": "synthetic N(0,1) 3x224x224 images, random-init weights (no checkpoint)",
        "config": {"workload": "ConvMixer-1536/20 ks9 p7 GELU inference (BASELINE configs[1])",
                   "batch_per_step": args.batch, "device": "host CPU",
                   "path": "PyTorch fp32 CPU, depthwise via conv2d(groups=C) (oracle/convmixer_ref.py)"},
        "cpu_baseline": {"value": rate, "unit": "img/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x {args.batch} image(s), after {args.warmup} warm-up"},
        "e2e": {"value": rate, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        args.warmup = max(args.warmup, 3)  # at least 3 untimed steps, as for the GPU arm
        run_reference(args)
    elif args.workload == "dw":
        run_dw(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
