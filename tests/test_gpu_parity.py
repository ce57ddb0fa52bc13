"""Parity of the sm_100a engine with the CPU oracle (GPU).

Bar (north star): max |err| <= 1e-2 and rel-L2 <= 1e-3 against the exact
result for fp16 outputs.  Every case runs through both accumulation modes:
the fp32 mode (accum=0) is also held to a much tighter bound, within 2 fp16
ulps of the correctly rounded exact value; the default mixed mode (fp16x2
FMA chains of at most 24 taps, fp32 across chains) to the bar.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from conftest import make_problem

pytestmark = pytest.mark.gpu

MAX_TOL, REL_TOL = 1e-2, 1e-3


@pytest.fixture(scope="module")
def eng():
    import depthwise_conv_b200 as d
    return d


def to_dev(a):
    """NHWC numpy fp16 -> channels_last [B,C,H,W] CUDA tensor (or 1-D / [K,K,C] as is)."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.permute(0, 3, 1, 2) if t.dim() == 4 else t


def to_host(t):
    return t.permute(0, 2, 3, 1).contiguous().cpu().numpy() if t.dim() == 4 else t.cpu().numpy()


def ulp16(v):
    """Spacing of fp16 numbers at |v| (subnormal spacing floor)."""
    a = np.abs(np.asarray(v, np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def assert_parity(O, y_dev, exact, tight=True, what="", xw=None):
    """Bar check, plus (tight) 2 fp16 ulps of the exact value.  Where an output nearly cancels, the fp32
    accumulator's own rounding dominates: with ``xw = (x, w)`` such outputs may also differ by the
    probabilistic fp32 summation bound 6 * K * 2^-24 * sum|x w| (sqrt(K^2) terms' worth of random walk)."""
    y = to_host(y_dev).astype(np.float64)
    max_err, rel = O.parity(y, exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL, f"{what}: max {max_err:.3e} rel {rel:.3e}"
    if tight:
        err = np.abs(y - exact)
        slack = 2.0 * ulp16(exact) + 1e-6
        bad = err > slack
        if bad.any() and xw is not None:
            x, w = xw
            absum, _ = O.dw_forward(np.abs(x), np.abs(w))
            bad = err > slack + 6.0 * w.shape[0] * 2.0 ** -24 * absum.astype(np.float64)
        assert not bad.any(), f"{what}: {bad.sum()} outputs beyond 2 ulp (max {err.max():.3e})"
    return max_err, rel


def run_engine(eng, x, w, bias=None, scale=None, shift=None, residual=False, act="none", accum=0):
    xd = to_dev(x)
    wd = to_dev(w)
    bd = to_dev(bias) if bias is not None else None
    sd = to_dev(scale) if scale is not None else None
    hd = to_dev(shift) if shift is not None else None
    y = eng.conv2d_nhwc_fused(xd, wd, bd, sd, hd, xd if residual else None, act, accum)
    torch.cuda.synchronize()
    return y


# ---------------------------------------------------------------- golden vectors

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "dw_cases.npz")


def _golden():
    z = np.load(GOLDEN)
    meta = json.loads(str(z["__meta__"]))
    out = []
    for m in meta:
        c = {k.split("__", 1)[1]: z[k] for k in z.files if k.startswith(m["name"] + "__")}
        c.update(m)
        out.append(c)
    return out


@pytest.mark.parametrize("accum", [0, 1])
@pytest.mark.parametrize("case", _golden(), ids=lambda c: c["name"])
def test_golden_vectors(eng, oracle_mod, case, accum):
    f16 = lambda a: np.asarray(a).view(np.float16)  # noqa: E731
    act = {0: "none", 1: "relu", 2: "gelu"}[int(case["act"])] if "act" in case else "none"
    y = run_engine(eng, f16(case["x"]), f16(case["w"]), f16(case["bias"]) if "bias" in case else None,
                   f16(case["scale"]) if "scale" in case else None, f16(case["shift"]) if "shift" in case else None,
                   "residual" in case, act, accum)
    assert_parity(oracle_mod, y, case["y"], tight=accum == 0, what=case["name"])


# ---------------------------------------------------------------- shape sweep

SWEEP = []
for _K in range(1, 32, 2):
    SWEEP.append((1, 7 + _K % 5, 9 + _K % 3, 64, _K))    # one channel block; image smaller than K for big K
    SWEEP.append((2, 23, 17, 72, _K))                    # ragged channel block (72 = 64 + 8)
SWEEP += [(1, 1, 1, 8, 7), (3, 2, 40, 16, 9), (1, 40, 2, 24, 31), (1, 61, 70, 136, 5), (2, 33, 65, 128, 15),
          (1, 100, 3, 8, 3), (1, 5, 130, 64, 11)]


@pytest.mark.parametrize("accum", [0, 1])
@pytest.mark.parametrize("B,H,W,C,K", SWEEP)
def test_shape_sweep(eng, oracle_mod, B, H, W, C, K, accum):
    x, w = make_problem(100 + K + H, B, H, W, C, K)
    exact, _ = oracle_mod.dw_forward(x, w)
    y = run_engine(eng, x, w, accum=accum)
    assert_parity(oracle_mod, y, exact, tight=accum == 0, what=f"{(B, H, W, C, K)}", xw=(x, w))


@pytest.mark.parametrize("K", [3, 7, 9, 13, 17, 21, 27, 29, 31])
def test_mixed_accumulation_within_bar(eng, oracle_mod, K):
    x, w = make_problem(7 + K, 1, 30, 33, 64, K)
    exact, _ = oracle_mod.dw_forward(x, w)
    y = run_engine(eng, x, w, accum=1)
    max_err, rel = assert_parity(oracle_mod, y, exact, tight=False, what=f"mixed K={K}")
    print(f"mixed K={K}: max {max_err:.3e} rel-L2 {rel:.3e}")


# ---------------------------------------------------------------- fused epilogue

# ---------------------------------------------------------------- row-split plans

SPLIT_SHAPES = [(1, 14, 14, 512, 27), (1, 7, 7, 1024, 13), (2, 9, 30, 72, 31), (1, 28, 28, 256, 29), (3, 5, 11, 64, 9)]


def _split_plans(B, H, W, C, K, accum):
    """The cheapest modelled candidate for every row split S > 1 the planner offers."""
    from depthwise_conv_b200 import _lib
    best = {}
    for c in sorted(_lib.plan_candidates(B, H, W, C, K, accum), key=lambda c: c["model_cost"]):
        best.setdefault(c["row_splits"], c)
    return [best[s] for s in sorted(best) if s > 1]


@pytest.mark.parametrize("accum", [0, 1])
@pytest.mark.parametrize("B,H,W,C,K", SPLIT_SHAPES)
def test_row_split_plans(eng, oracle_mod, B, H, W, C, K, accum):
    """Warps sharing a slot over every S-th kernel row, partial sums added in shared memory: one tile
    per CTA, persistent CTAs, and 3 CTAs walking every tile (the hand-off alternates phases)."""
    x, w = make_problem(200 + K, B, H, W, C, K)
    rng = np.random.default_rng(K)
    bias = (rng.standard_normal(C) * 0.2).astype(np.float16)
    scale = rng.uniform(0.5, 1.5, C).astype(np.float16)
    shift = (rng.standard_normal(C) * 0.2).astype(np.float16)
    exact, _ = oracle_mod.dw_forward(x, w, bias, scale, shift, x, "gelu")
    plans = _split_plans(B, H, W, C, K, accum)
    assert plans, "no row-split candidates"
    from depthwise_conv_b200 import _lib
    xd, wd = to_dev(x), to_dev(w)
    ran = 0
    for plan in plans:
        for grid in (0, -1, 3):
            try:
                y = eng.conv2d_nhwc_fused(xd, wd, to_dev(bias), to_dev(scale), to_dev(shift), xd, "gelu", accum,
                                          plan=dict(plan, grid=grid))
            except _lib.DwbError as e:  # host-side candidate whose real register count does not fit
                assert e.status == _lib.ERR_BAD_ARG
                continue
            torch.cuda.synchronize()
            ran += 1
            assert_parity(oracle_mod, y, exact, tight=accum == 0, xw=(x, w),
                          what=f"S={plan['row_splits']} R={plan['cols_per_thread']} tile={plan['tile_h']}x"
                               f"{plan['tile_w']} grid={grid}")
    assert ran >= 3
    assert eng.device_error() == 0


@pytest.mark.parametrize("B,H,W,C,K", [(2, 19, 33, 128, 7), (1, 21, 30, 64, 17), (2, 9, 12, 136, 31), (1, 32, 32, 192, 9)])
def test_both_load_schedules(eng, oracle_mod, B, H, W, C, K):
    """Mixed-mode variants come in two load schedules (row read up front, or per column); both agree
    with the oracle for every register-block shape the planner offers."""
    from depthwise_conv_b200 import _lib
    x, w = make_problem(300 + K, B, H, W, C, K)
    exact, _ = oracle_mod.dw_forward(x, w)
    xd, wd = to_dev(x), to_dev(w)
    seen = set()
    for c in sorted(_lib.plan_candidates(B, H, W, C, K, 1), key=lambda c: c["model_cost"]):
        key = (c["cols_per_thread"], c["rows_per_thread"])
        if key in seen:
            continue
        seen.add(key)
        outs = []
        for pre in (0, 1):
            try:
                y = eng.conv2d_nhwc_fused(xd, wd, accum=1, plan=dict(c, load_schedule=pre, grid=-1))
            except _lib.DwbError as e:  # host-side candidate whose real register count does not fit
                assert e.status == _lib.ERR_BAD_ARG
                continue
            torch.cuda.synchronize()
            assert_parity(oracle_mod, y, exact, tight=False, what=f"R={key[0]} M={key[1]} pre={pre}")
            outs.append(y)
        if len(outs) == 2:
            assert torch.equal(outs[0], outs[1])  # same arithmetic, only the load order differs
    assert len(seen) >= 4


@pytest.mark.parametrize("act", ["none", "relu", "gelu"])
@pytest.mark.parametrize("terms", ["bias", "bias_bn", "bias_bn_res", "bn_res"])
def test_fused_epilogue(eng, oracle_mod, act, terms):
    B, H, W, C, K = 2, 19, 21, 128, 9
    x, w = make_problem(31, B, H, W, C, K)
    rng = np.random.default_rng(9)
    bias = (rng.standard_normal(C) * 0.2).astype(np.float16) if "bias" in terms else None
    scale = (rng.uniform(0.5, 1.5, C)).astype(np.float16) if "bn" in terms else None
    shift = (rng.standard_normal(C) * 0.2).astype(np.float16) if "bn" in terms else None
    res = "res" in terms
    exact, _ = oracle_mod.dw_forward(x, w, bias, scale, shift, x if res else None, act)
    y = run_engine(eng, x, w, bias, scale, shift, res, act)
    assert_parity(oracle_mod, y, exact, what=f"{terms}/{act}", xw=(x, w))


def test_gelu_over_its_whole_range(eng, oracle_mod):
    """K=1 with unit weights makes the convolution the identity, so y = act(x + bias):
    the GELU is checked from deep negative to large positive arguments."""
    C, H, W = 64, 16, 16
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((1, H, W, C)) * 3.0).astype(np.float16)
    w = np.ones((1, 1, C), np.float16)
    bias = np.linspace(-8.0, 8.0, C).astype(np.float16)
    exact, _ = oracle_mod.dw_forward(x, w, bias, None, None, None, "gelu")
    for accum in (0, 1):
        y = to_host(run_engine(eng, x, w, bias, None, None, False, "gelu", accum)).astype(np.float64)
        err = np.abs(y - exact)
        assert (err <= 2.0 * ulp16(exact) + 1e-7).all(), f"GELU off by {err.max():.3e} (accum={accum})"


# ---------------------------------------------------------------- BASELINE configs

B1_CONFIGS = [  # (name, B, H, W, C, K, weight std)
    ("convmixer768_dw", 1, 32, 32, 768, 7, 0.02),
    ("convmixer1536_dw", 1, 32, 32, 1536, 9, 0.02),
    ("replknet_c3", 1, 56, 56, 128, 31, None),
    ("replknet_c4", 1, 28, 28, 256, 29, None),
    ("replknet_c5", 1, 14, 14, 512, 27, None),
    ("replknet_c6", 1, 7, 7, 1024, 13, None),
    ("bsweep_b1", 1, 32, 32, 1536, 9, 1.0 / 9),
]


@pytest.mark.parametrize("accum", [0, 1])
@pytest.mark.parametrize("name,B,H,W,C,K,ws", B1_CONFIGS, ids=[c[0] for c in B1_CONFIGS])
def test_baseline_batch1_configs_full(eng, oracle_mod, name, B, H, W, C, K, ws, accum):
    x, w = make_problem(0, B, H, W, C, K, wscale=ws)
    exact, _ = oracle_mod.dw_forward(x, w)
    y = run_engine(eng, x, w, accum=accum)
    max_err, rel = assert_parity(oracle_mod, y, exact, tight=accum == 0, what=name, xw=(x, w))
    print(f"{name} accum={accum}: max {max_err:.3e} rel-L2 {rel:.3e}")


def _sampled_check(eng, oracle_mod, B, H, W, C, K, act="none", npix=1536, seed=0, with_epi=False, accum=1):
    """Full-size problem, checked at sampled pixels (all borders of two images) and by channel sums."""
    x, w = make_problem(seed, B, H, W, C, K)
    bias = scale = shift = None
    if with_epi:
        bias = np.zeros(C, np.float16)
        scale = np.full(C, 1.0 / np.sqrt(1.0 + 1e-5), np.float16)
        shift = np.zeros(C, np.float16)
    y = to_host(run_engine(eng, x, w, bias, scale, shift, False, act, accum)).reshape(-1, C)
    rng = np.random.default_rng(seed + 1)
    border = [(b * H + h) * W + c for b in (0, B - 1) for h in range(H) for c in range(W)
              if h in (0, H - 1) or c in (0, W - 1)]
    pix = np.unique(np.concatenate([rng.integers(0, B * H * W, npix), np.array(border, np.int64)]))
    exact, _ = oracle_mod.dw_forward_pixels(x, w, pix, bias, scale, shift, None, act)
    max_err, rel = oracle_mod.parity(y[pix].astype(np.float64), exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL, f"sampled: max {max_err:.3e} rel {rel:.3e}"
    if not with_epi:
        # size-independent property: per-channel sums over whole images
        sums = oracle_mod.channel_sums(x[[0, B - 1]], w)
        yimg = y.reshape(B, H * W, C)[[0, B - 1]].astype(np.float64)
        ysum = yimg.sum(axis=1)
        # fp16 output rounding adds a random walk of H*W half-ulps per channel
        rms = np.sqrt((yimg ** 2).mean())
        tol = 8.0 * np.sqrt(H * W) * rms * 2.0 ** -11 + 1e-3
        dev = np.abs(ysum - sums).max()
        assert dev <= tol, f"channel sums off by {dev:.3e} > {tol:.3e}"


@pytest.mark.parametrize("B", [16, 64, 256])
def test_batch_sweep_sampled(eng, oracle_mod, B):
    _sampled_check(eng, oracle_mod, B, 32, 32, 1536, 9, seed=B, accum=0 if B == 64 else 1)


@pytest.mark.parametrize("K", [7, 9, 13, 17, 21, 27, 29, 31])
def test_kernel_size_sweep_sampled_with_epilogue(eng, oracle_mod, K):
    _sampled_check(eng, oracle_mod, 64, 56, 56, 1024, K, act="gelu", npix=512, seed=K, with_epi=True)


@pytest.mark.parametrize("K", [9, 31])
def test_kernel_size_sweep_channel_sums(eng, oracle_mod, K):
    _sampled_check(eng, oracle_mod, 8, 56, 56, 1024, K, npix=256, seed=50 + K)


# ---------------------------------------------------------------- memory safety

def test_output_guard_regions_untouched(eng, oracle_mod):
    B, H, W, C, K = 2, 13, 11, 72, 9
    x, w = make_problem(77, B, H, W, C, K)
    n = B * H * W * C
    guard = 4096
    buf = torch.full((n + 2 * guard,), 12345.0, dtype=torch.float16, device="cuda")
    y = buf[guard:guard + n].view(B, H, W, C).permute(0, 3, 1, 2)
    eng.conv2d_nhwc_fused(to_dev(x), to_dev(w), out=y, accum=0)
    torch.cuda.synchronize()
    assert torch.all(buf[:guard] == 12345.0) and torch.all(buf[guard + n:] == 12345.0)
    exact, _ = oracle_mod.dw_forward(x, w)
    assert_parity(oracle_mod, y, exact)


def test_residual_reads_stay_in_bounds(eng, oracle_mod):
    # NaN guards around the residual: an out-of-bounds read would poison the output
    B, H, W, C, K = 1, 9, 10, 64, 7
    x, w = make_problem(78, B, H, W, C, K)
    n = B * H * W * C
    guard = 2048
    buf = torch.full((n + 2 * guard,), float("nan"), dtype=torch.float16, device="cuda")
    buf[guard:guard + n] = torch.from_numpy(x.reshape(-1)).cuda()
    res = buf[guard:guard + n].view(B, H, W, C).permute(0, 3, 1, 2)
    y = eng.conv2d_nhwc_fused(to_dev(x), to_dev(w), residual=res, accum=0)
    torch.cuda.synchronize()
    exact, _ = oracle_mod.dw_forward(x, w, residual=x)
    assert_parity(oracle_mod, y, exact)


def test_no_device_error_recorded(eng):
    assert eng.device_error(clear=True) == 0


# ---------------------------------------------------------------- streams / edge cases

def test_runs_on_current_stream(eng, oracle_mod):
    x, w = make_problem(5, 4, 32, 32, 256, 9)
    exact, _ = oracle_mod.dw_forward(x, w)
    xd, wd = to_dev(x), to_dev(w)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y = eng.conv2d_nhwc(xd, wd)  # default (mixed) accumulation
        y2 = y * 1.0  # consumer on the same stream
    s.synchronize()
    assert_parity(oracle_mod, y2, exact, tight=False)


def test_zero_batch_is_noop(eng):
    xd = torch.empty(0, 64, 8, 8, dtype=torch.float16, device="cuda").contiguous(memory_format=torch.channels_last)
    wd = torch.zeros(7, 7, 64, dtype=torch.float16, device="cuda")
    y = eng.conv2d_nhwc(xd, wd)
    assert y.shape == xd.shape


@pytest.mark.parametrize("accum", [0, 1])
@pytest.mark.parametrize("B,H,W,C,K", [(1, 32, 32, 256, 9), (2, 13, 21, 136, 7), (1, 11, 30, 64, 13), (1, 9, 9, 72, 5)])
def test_residual_read_from_the_stage_ring(eng, oracle_mod, B, H, W, C, K, accum):
    """A ConvMixer block's residual is the convolution's input: with one tile per CTA and a ring that
    holds the whole tile, the epilogue reads it from the staged input rows.  The result must equal,
    bit for bit, the same plan reading an identical residual tensor from global memory, and the oracle."""
    from depthwise_conv_b200 import _lib
    x, w = make_problem(900 + K, B, H, W, C, K)
    rng = np.random.default_rng(K + 1)
    bias = (rng.standard_normal(C) * 0.2).astype(np.float16)
    scale = rng.uniform(0.5, 1.5, C).astype(np.float16)
    shift = (rng.standard_normal(C) * 0.2).astype(np.float16)
    exact, _ = oracle_mod.dw_forward(x, w, bias, scale, shift, x, "gelu")
    xd, wd = to_dev(x), to_dev(w)
    x_copy = xd.clone()  # same values, another tensor: the global-memory residual path
    vec = [to_dev(v) for v in (bias, scale, shift)]
    seen, ran = set(), 0
    for c in sorted(_lib.plan_candidates(B, H, W, C, K, accum), key=lambda c: c["model_cost"]):
        key = (c["cols_per_thread"], c["rows_per_thread"], c["row_splits"])
        if key in seen:
            continue
        seen.add(key)
        plan = dict(c, grid=0, ring_rows=c["tile_h"] + K - 1)
        try:
            y_ring = eng.conv2d_nhwc_fused(xd, wd, *vec, xd, "gelu", accum, plan=plan)
            y_glob = eng.conv2d_nhwc_fused(xd, wd, *vec, x_copy, "gelu", accum, plan=plan)
        except _lib.DwbError as e:  # a candidate whose full-tile ring or registers do not fit
            assert e.status == _lib.ERR_BAD_ARG
            continue
        torch.cuda.synchronize()
        assert torch.equal(y_ring, y_glob), f"R={key[0]} M={key[1]} S={key[2]}: ring residual differs"
        assert_parity(oracle_mod, y_ring, exact, tight=accum == 0, xw=(x, w),
                      what=f"R={key[0]} M={key[1]} S={key[2]} tile={c['tile_h']}x{c['tile_w']}")
        ran += 1
        if ran >= 6:
            break
    assert ran >= 2
    assert eng.device_error() == 0


BAND_SHAPES = [(3, 20, 24, 136, 9), (2, 32, 32, 256, 7), (1, 13, 30, 64, 13), (4, 9, 40, 72, 5), (2, 17, 17, 128, 17),
               (2, 5, 7, 64, 3), (1, 40, 12, 64, 1)]


@pytest.mark.parametrize("B,H,W,C,K", BAND_SHAPES)
def test_band_mode_plans(eng, oracle_mod, B, H, W, C, K):
    """Band mode (each input row staged once per band, the K x K weights resident and double-buffered
    across bands): band sizes from 1 tile to the whole image, row splits, M = 2, ragged channel blocks
    and image edges; one band per CTA, persistent CTAs, and 3 CTAs walking every band (so each CTA's
    consecutive bands change channel block and the weight buffers alternate)."""
    from depthwise_conv_b200 import _lib
    x, w = make_problem(1200 + K, B, H, W, C, K)
    rng = np.random.default_rng(K + 7)
    bias = (rng.standard_normal(C) * 0.2).astype(np.float16)
    scale = rng.uniform(0.5, 1.5, C).astype(np.float16)
    shift = (rng.standard_normal(C) * 0.2).astype(np.float16)
    exact, _ = oracle_mod.dw_forward(x, w, bias, scale, shift, x, "gelu")
    xd, wd = to_dev(x), to_dev(w)
    vec = [to_dev(v) for v in (bias, scale, shift)]
    seen, ran = set(), 0
    cands = [c for c in _lib.plan_candidates(B, H, W, C, K, 1) if c["band_tiles"] > 0]
    assert cands, "no band-mode candidates"
    for c in sorted(cands, key=lambda c: c["model_cost"]):
        key = (c["cols_per_thread"], c["rows_per_thread"], c["row_splits"], c["band_tiles"])
        if key in seen:
            continue
        seen.add(key)
        for grid in (0, -1, 3):
            try:
                y = eng.conv2d_nhwc_fused(xd, wd, *vec, xd, "gelu", 1, plan=dict(c, grid=grid))
            except _lib.DwbError as e:  # a candidate whose real register count does not fit
                assert e.status == _lib.ERR_BAD_ARG
                break
            torch.cuda.synchronize()
            assert_parity(oracle_mod, y, exact, tight=False,
                          what=f"band={key[3]} R={key[0]} M={key[1]} S={key[2]} tile={c['tile_h']}x{c['tile_w']} "
                               f"ring={c['ring_rows']} grid={grid}")
            ran += 1
        if len(seen) >= 8:
            break
    assert ran >= 3
    assert eng.device_error() == 0


def test_band_mode_matches_tile_mode_bitwise(eng):
    """Same variant, same arithmetic: a band plan and the tile plan of the same register block agree bit
    for bit (only the staging of the rows and weights differs)."""
    from depthwise_conv_b200 import _lib
    B, H, W, C, K = 4, 32, 32, 192, 9
    x, w = make_problem(77, B, H, W, C, K)
    xd, wd = to_dev(x), to_dev(w)
    cands = _lib.plan_candidates(B, H, W, C, K, 1)
    pairs = 0
    # (row split S = 1: with S > 1 the two modes may deal the kernel rows of an edge tile to the split
    # groups differently, which changes the order of the fp32 partial-sum additions)
    for c in sorted((c for c in cands if c["band_tiles"] > 0 and c["row_splits"] == 1),
                    key=lambda c: c["model_cost"])[:12]:
        twin = next((t for t in cands if t["band_tiles"] == 0 and all(
            t[f] == c[f] for f in ("cols_per_thread", "rows_per_thread", "tile_h", "tile_w", "row_splits",
                                   "load_schedule"))), None)
        if twin is None:
            continue
        try:
            yb = eng.conv2d_nhwc_fused(xd, wd, accum=1, plan=dict(c, grid=-1))
            yt = eng.conv2d_nhwc_fused(xd, wd, accum=1, plan=dict(twin, grid=-1))
        except _lib.DwbError:
            continue
        torch.cuda.synchronize()
        assert torch.equal(yb, yt)
        pairs += 1
    assert pairs >= 2


def _tuned_entries(name="dw_tuned_plans.inc"):
    """(B, H, W, C, K) of every measured plan in one of the library's tuned tables (mixed accumulation)."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "depthwise_conv_b200", "csrc",
                        name)
    out = []
    for ln in open(path):
        ln = ln.strip()
        if ln.startswith("{"):
            v = [int(t) for t in ln.strip("{},").split(",")]
            if v[5] == 1:
                out.append(tuple(v[:5]) + (tuple(v[6:]),))
    return out


@pytest.mark.parametrize("B,H,W,C,K,fields", _tuned_entries(),
                         ids=[f"{b}x{h}x{w}x{c}_k{k}" for b, h, w, c, k, _ in _tuned_entries()])
def test_every_tuned_plan(eng, oracle_mod, B, H, W, C, K, fields):
    """The tuner times plans without checking them: run each table entry's own problem (the launcher
    picks exactly that plan) against the oracle at sampled pixels and by channel sums."""
    from depthwise_conv_b200 import _lib
    plan = _lib.plan_select(B, H, W, C, K)
    names = ("cols_per_thread", "rows_per_thread", "tile_h", "tile_w", "ring_rows")
    assert tuple(plan[n] for n in names) == fields[:5], (plan, fields)
    _sampled_check(eng, oracle_mod, B, H, W, C, K, npix=256, seed=B * 7 + K)


@pytest.mark.parametrize("B,H,W,C,K,fields", _tuned_entries("dw_tuned_plans_res.inc"),
                         ids=[f"{b}x{h}x{w}x{c}_k{k}" for b, h, w, c, k, _ in _tuned_entries("dw_tuned_plans_res.inc")])
@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_every_convmixer_block_plan(eng, oracle_mod, B, H, W, C, K, fields, act):
    """The ConvMixer-block table (used when the residual is the input): each entry's problem with the full
    epilogue and residual = input, against the oracle."""
    x, w = make_problem(B * 11 + K, B, H, W, C, K)
    rng = np.random.default_rng(K)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float16)
    scale = rng.uniform(0.5, 1.5, C).astype(np.float16)
    shift = (rng.standard_normal(C) * 0.1).astype(np.float16)
    y = run_engine(eng, x, w, bias, scale, shift, True, act, 1)
    exact, _ = oracle_mod.dw_forward(x, w, bias, scale, shift, x, act)
    max_err, rel = oracle_mod.parity(to_host(y).astype(np.float64), exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL, f"max {max_err:.3e} rel {rel:.3e}"


def _random_cases(n=120, seed=2024):
    """Seeded random problems: odd K 1..31, ragged H and W (1..70), C a multiple of 8 (8..264),
    B 1..3, a random epilogue (activation, bias/scale/shift, residual) and both accumulations."""
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        K = int(rng.choice(np.arange(1, 32, 2)))
        H, W = int(rng.integers(1, 71)), int(rng.integers(1, 71))
        C = 8 * int(rng.integers(1, 34))
        B = int(rng.integers(1, 4))
        act = ["none", "relu", "gelu"][int(rng.integers(0, 3))]
        out.append((i, B, H, W, C, K, act, bool(rng.integers(0, 2)), bool(rng.integers(0, 2)), int(rng.integers(0, 2))))
    return out


@pytest.mark.parametrize("i,B,H,W,C,K,act,with_params,residual,accum", _random_cases(),
                         ids=[f"r{c[0]}_{c[1]}x{c[2]}x{c[3]}x{c[4]}_k{c[5]}" for c in _random_cases()])
def test_random_problems(eng, oracle_mod, i, B, H, W, C, K, act, with_params, residual, accum):
    """Whatever plan the launcher picks for an arbitrary shape meets the oracle's bar."""
    x, w = make_problem(7000 + i, B, H, W, C, K)
    rng = np.random.default_rng(i)
    bias = scale = shift = None
    if with_params:
        bias = (rng.standard_normal(C) * 0.2).astype(np.float16)
        scale = rng.uniform(0.5, 1.5, C).astype(np.float16)
        shift = (rng.standard_normal(C) * 0.2).astype(np.float16)
    y = run_engine(eng, x, w, bias, scale, shift, residual, act, accum)
    exact, _ = oracle_mod.dw_forward(x, w, bias, scale, shift, x if residual else None, act)
    max_err, rel = oracle_mod.parity(to_host(y).astype(np.float64), exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL, f"max {max_err:.3e} rel {rel:.3e}"
    assert eng.device_error() == 0
