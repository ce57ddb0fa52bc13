"""Autotuner: time the planner's candidate plans on this GPU and write the tuned-plan table.

    python -m depthwise_conv_b200.tune [--budget SECONDS] [--accum mixed|f32] [B,H,W,C,K ...]

For every problem (default: the benchmark configurations) the candidates
from ``dwb_plan_candidates`` are timed in the planner's cost order (CUDA
graph of back-to-back launches, best of 3) on a proxy batch of at most
``--proxy-batch`` images until the per-problem time budget runs out; the
fastest few are then timed on the full batch (both load schedules, both grid
modes) and the winner is written to ``csrc/dw_tuned_plans.inc``, which the
library consults before its cost model (rebuild afterwards).  ``--epilogue``
times the fused op with the epilogue a model uses; with a residual
(``gelu_bn_res``, ``relu_bn_res``: the residual is the input, a ConvMixer
block) the winner goes to ``csrc/dw_tuned_plans_res.inc``, which the library
consults first for launches whose residual is their input.  A plan only
enters a table when it beats the plan the library would use without it.
Results are also printed as JSON lines.
"""
from __future__ import annotations

import argparse
import itertools
import json
import os
import time

HERE = os.path.dirname(os.path.abspath(__file__))
TABLE = os.path.join(HERE, "csrc", "dw_tuned_plans.inc")
# plans for a ConvMixer block (residual = the input), used by launches whose residual is their input
TABLE_RES = os.path.join(HERE, "csrc", "dw_tuned_plans_res.inc")

DEFAULT_PROBLEMS = [
    (1, 32, 32, 768, 7), (1, 32, 32, 1536, 9), (1, 16, 16, 1536, 9), (1, 32, 32, 1536, 13),
    (1, 56, 56, 128, 31), (1, 28, 28, 256, 29), (1, 14, 14, 512, 27), (1, 7, 7, 1024, 13),
    (16, 32, 32, 1536, 9), (64, 32, 32, 1536, 9), (128, 32, 32, 1536, 9), (256, 32, 32, 1536, 9),
    (8, 56, 56, 1024, 7), (8, 56, 56, 1024, 31), (32, 56, 56, 1024, 9),
] + [(64, 56, 56, 1024, k) for k in (7, 9, 13, 17, 21, 27, 29, 31)]

FIELDS = ("cols_per_thread", "rows_per_thread", "tile_h", "tile_w", "ring_rows", "ring_wrows", "grid", "row_splits",
          "load_schedule", "band_tiles")


EPILOGUE = {}  # keyword arguments of the fused op while timing (set by --epilogue)


def _epilogue_args(x):
    import torch
    if not EPILOGUE:
        return {}
    C = x.shape[1]
    v = torch.full((C,), 0.5, dtype=torch.float16, device=x.device)
    kw = dict(bias=v, scale=v, shift=v, act=EPILOGUE["act"])
    if EPILOGUE.get("residual"):
        kw["residual"] = x
    return kw


def time_plan(d, x, w, y, plan, accum, reps):
    import torch
    s = torch.cuda.Stream()
    kw = _epilogue_args(x)
    with torch.cuda.stream(s):
        d.conv2d_nhwc_fused(x, w, out=y, plan=plan, accum=accum, **kw)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                d.conv2d_nhwc_fused(x, w, out=y, plan=plan, accum=accum, **kw)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 1e30
    for _ in range(3):
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) / reps * 1000.0)
    return best


def _inputs(B, H, W, C, K):
    import torch
    x = torch.randn(B, C, H, W, device="cuda").half().contiguous(memory_format=torch.channels_last)
    w = (torch.randn(K, K, C, device="cuda") / K).half()
    return x, w, torch.empty_like(x)


def _reps(B, H, W, C):
    return 3 if B * H * W * C >= (64 << 20) else (10 if B >= 16 else 50)


def tune_problem(B, H, W, C, K, accum, budget, proxy_batch=8, finalists=8):
    """Phase 1 ranks the candidates (model order, both grid modes, the model's load schedule) on
    min(B, proxy_batch) images until the budget is spent; phase 2 times the best `finalists`
    on the full batch with both load schedules and both grid modes."""
    import depthwise_conv_b200 as d
    from depthwise_conv_b200 import _lib

    # the cost model ranks within a mode far better than across the tile and band modes, so the two
    # modes' candidates are interleaved, each in model order
    allc = _lib.plan_candidates(B, H, W, C, K, accum)
    by_mode = [sorted((c for c in allc if (c["band_tiles"] > 0) == band), key=lambda c: c["model_cost"])
               for band in (False, True)]
    cands = [c for pair in itertools.zip_longest(*by_mode) for c in pair if c is not None]
    Bp = min(B, proxy_batch)
    xp, wp, yp = _inputs(Bp, H, W, C, K)
    ranked = []
    t0 = time.time()
    for c in cands:
        for grid in (-1, 0):
            plan = dict(c, grid=grid)
            try:
                ranked.append((time_plan(d, xp, wp, yp, plan, accum, _reps(Bp, H, W, C)), plan))
            except RuntimeError:
                continue
        if time.time() - t0 > budget:
            break
    del xp, wp, yp
    x, w, y = _inputs(B, H, W, C, K)
    reps = _reps(B, H, W, C)
    default = time_plan(d, x, w, y, None, accum, reps)
    best = (default, None)
    seen = set()
    for _, plan in sorted(ranked, key=lambda r: r[0]):
        key = tuple(sorted((k, v) for k, v in plan.items() if k in FIELDS))
        if key in seen:
            continue
        seen.add(key)
        if len(seen) > finalists:
            break
        for pre in (plan["load_schedule"], 1 - plan["load_schedule"]):
            if pre == 1 and accum != _lib.ACCUM_MIXED:
                continue
            cand = dict(plan, load_schedule=pre)
            try:
                us = time_plan(d, x, w, y, cand, accum, reps)
            except RuntimeError:
                continue
            if us < best[0]:
                best = (us, cand)
    return default, best


def write_table(rows, path, base=TABLE):
    """Merge ``rows`` into the committed table ``base`` (its comment header kept) and write it to ``path``."""
    lines = ["// dw_tuned_plans.inc -- plans measured fastest on B200 by depthwise_conv_b200/tune.py.",
             "// {B, H, W, C, K, accum, R, M, tile_h, tile_w, ring_rows, ring_wrows, grid(-1 persistent, 0 one tile/CTA),",
             "//  row_splits, load_schedule, band_tiles (0 = tile mode)}"]
    old = []
    if os.path.exists(base):  # start from the committed table
        head = [ln.rstrip("\n") for ln in open(base) if ln.startswith("//")]
        lines = head or lines
        for ln in open(base):
            ln = ln.strip()
            if ln.startswith("{"):
                old.append(ln)
    keep = {}
    for ln in old:
        key = tuple(int(v) for v in ln.strip("{},").split(",")[:6])
        keep[key] = ln
    for (B, H, W, C, K, accum), plan in rows:
        vals = [B, H, W, C, K, accum] + [int(plan[f]) for f in FIELDS]
        keep[(B, H, W, C, K, accum)] = "{" + ", ".join(str(v) for v in vals) + "},"
    lines += [keep[k] for k in sorted(keep)]
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("problems", nargs="*", help="B,H,W,C,K (default: the benchmark configurations)")
    ap.add_argument("--budget", type=float, default=20.0, help="seconds of candidate timing per problem")
    ap.add_argument("--accum", choices=["mixed", "f32"], default="mixed")
    ap.add_argument("--proxy-batch", type=int, default=8, help="images per timing while ranking candidates")
    ap.add_argument("--finalists", type=int, default=8, help="plans re-timed on the full batch")
    ap.add_argument("--epilogue", choices=["none", "gelu_bn", "gelu_bn_res", "relu_bn_res"], default="none",
                    help="time with the fused epilogue a model uses (bias+GELU+BN, + residual = input)")
    ap.add_argument("--no-write", action="store_true")
    ap.add_argument("--out", default=None,
                    help="where to write the merged table (default: the library's; the ConvMixer-block table for "
                         "the *_res epilogues)")
    args = ap.parse_args()
    from depthwise_conv_b200 import _lib
    accum = _lib.ACCUM_MIXED if args.accum == "mixed" else _lib.ACCUM_F32
    if args.epilogue != "none":
        EPILOGUE.update(act="relu" if args.epilogue.startswith("relu") else "gelu",
                        residual=args.epilogue.endswith("_res"))
    probs = [tuple(int(v) for v in p.split(",")) for p in args.problems] or DEFAULT_PROBLEMS
    rows = []
    for B, H, W, C, K in probs:
        default, (us, plan) = tune_problem(B, H, W, C, K, accum, args.budget, args.proxy_batch, args.finalists)
        print(json.dumps({"problem": [B, H, W, C, K], "accum": args.accum, "default_us": default, "best_us": us,
                          "plan": {f: plan[f] for f in FIELDS} if plan else None}), flush=True)
        if plan is not None:
            rows.append(((B, H, W, C, K, accum), plan))
    if not args.no_write:
        base = TABLE_RES if args.epilogue.endswith("_res") else TABLE
        out = args.out or base
        write_table(rows, out, base)
        print("wrote", out)


if __name__ == "__main__":
    main()
