"""End-to-end ConvMixer on the GPU with the engine's fused depthwise blocks.

Compared with the fp32 CPU model (the reference's CPU path) using the
reference's own end-to-end metric, rel = max|diff| / mean|ref|
(benchmark_cudnn_fused_e2e.py:167-174), and calibrated against PyTorch's own
fp16 GPU model (nn.Conv2d depthwise) on the same weights: fusing the block
into one kernel must not be less accurate than the unfused fp16 network.
The CUDA-graph replay of the whole forward must follow changing inputs
(verify_e5b_correctness.py:26-37).
"""
from __future__ import annotations

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(y, ref):
    d = (y.float().cpu() - ref.float()).abs()
    return (d.max() / (ref.float().abs().mean() + 1e-6)).item()


@pytest.mark.parametrize("name", ["1536_20", "768_32"])
def test_convmixer_fused_matches_fp32_cpu(name):
    from depthwise_conv_b200.convmixer import convmixer, fuse_dw_blocks
    from oracle.convmixer_ref import convmixer_cpu

    torch.manual_seed(0)
    x = torch.randn(2, 3, 224, 224)
    ref = convmixer_cpu(name, seed=0)(x)

    base = convmixer(name, seed=0).half().cuda().to(memory_format=torch.channels_last)
    fused = fuse_dw_blocks(copy.deepcopy(base))
    assert fused.fused_blocks == base.depth
    xd = x.half().cuda().contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        y_torch = base(xd)
        y_fused = fused(xd)
    torch.cuda.synchronize()
    rel_torch, rel_fused = _rel(y_torch, ref), _rel(y_fused, ref)
    print(f"ConvMixer-{name}: rel(max|diff|/mean|ref|) torch-fp16 {rel_torch:.4f}, engine-fused {rel_fused:.4f}")
    assert rel_fused <= max(1.5 * rel_torch, 0.01)
    # The random-init network shrinks its signal block by block (1x1 conv gain ~0.8, GELU ~0.5 near 0),
    # so the logits are ~1e-5 and their argmax is noise.  Compare early feature maps, where every
    # value is well inside the fp16 range: patch embedding + 3 blocks.
    cpu3 = convmixer_cpu(name, seed=0).trunk(x, blocks=3)
    with torch.no_grad():
        t3 = base.model[:6](xd).float().cpu()
        f3 = fused.model[:6](xd).float().cpu()
    rel_t3 = ((t3 - cpu3).norm() / cpu3.norm()).item()
    rel_f3 = ((f3 - cpu3).norm() / cpu3.norm()).item()
    print(f"ConvMixer-{name} after 3 blocks: rel-L2 torch-fp16 {rel_t3:.2e}, engine-fused {rel_f3:.2e}")
    assert rel_f3 <= max(1.5 * rel_t3, 2e-3)


def test_convmixer_cuda_graph_replay_tracks_inputs():
    from depthwise_conv_b200.convmixer import convmixer, fuse_dw_blocks

    full = fuse_dw_blocks(convmixer("1536_20", seed=0).half().cuda().to(memory_format=torch.channels_last))
    # patch embedding + 3 blocks: the random-init network's signal decays with depth, so later
    # feature maps (and the logits) can round to the same fp16 values for different images
    model = full.model[:6]
    mk = lambda: torch.randn(1, 3, 224, 224, device="cuda").half().contiguous(memory_format=torch.channels_last)  # noqa: E731
    static_in = mk()
    s = torch.cuda.Stream()
    with torch.no_grad(), torch.cuda.stream(s):
        for _ in range(3):
            model(static_in)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            static_out = model(static_in)
    outs, refs = [], []
    with torch.no_grad():
        for _ in range(4):
            xi = mk()
            static_in.copy_(xi)
            g.replay()
            torch.cuda.synchronize()
            outs.append(static_out.clone())
            refs.append(model(xi))
    for o, r in zip(outs, refs):
        assert (o - r).abs().max().item() == 0.0
    diffs = [(outs[i] - outs[i + 1]).abs().max().item() for i in range(3)]
    assert all(d > 0 for d in diffs)


def test_convmixer_compiled_reduce_overhead_replay():
    """The fused network under torch.compile(mode="reduce-overhead", fullgraph=True): the engine's
    ops trace through their fake impls without graph breaks, the compiled forward matches eager, and
    replays of the captured graph follow changing inputs (verify_e5b_correctness.py:26-37)."""
    from depthwise_conv_b200.convmixer import convmixer, fuse_dw_blocks

    full = fuse_dw_blocks(convmixer("1536_20", seed=0).half().cuda().to(memory_format=torch.channels_last))
    model = full.model[:6]  # stem + 3 blocks (see test_convmixer_cuda_graph_replay_tracks_inputs)
    compiled = torch.compile(model, mode="reduce-overhead", fullgraph=True)
    mk = lambda: torch.randn(1, 3, 224, 224, device="cuda").half().contiguous(memory_format=torch.channels_last)  # noqa: E731
    outs = []
    with torch.no_grad():
        for i in range(5):
            xi = mk()
            yc = compiled(xi).clone()
            ye = model(xi)
            torch.cuda.synchronize()
            err = ((yc.float() - ye.float()).norm() / ye.float().norm()).item()
            assert err < 1e-3, f"call {i}: compiled vs eager rel-L2 {err:.2e}"
            outs.append(yc)
    diffs = [(outs[i] - outs[i + 1]).abs().max().item() for i in range(4)]
    assert all(d > 0 for d in diffs)


def _signal_preserving_pair(name, seed=5):
    """The GPU model and the fp32 CPU model with identical weights scaled so that the signal keeps an
    O(1) size through every block: patch conv N(0, 1/(3 p^2)), DW taps N(0, 1/K^2), 1x1 convs
    N(0, g^2/C) with g = 1.15 for GELU and 1.0 for ReLU (measured on the fp32 CPU model: feature maps
    stay at std 0.5-4 through all blocks, logits at std 2-3), head N(0, 1/C), biases 0."""
    import math

    from depthwise_conv_b200.convmixer import convmixer
    from oracle.convmixer_ref import convmixer_cpu

    gpu = convmixer(name, seed=0)
    cpu = convmixer_cpu(name, seed=0)
    C, K, p, depth = cpu.dim, cpu.k, cpu.p, cpu.depth
    gain = 1.0 if cpu.act == "relu" else 1.15
    g = torch.Generator().manual_seed(seed)
    cpu.patch_w = torch.randn(C, 3, p, p, generator=g) / math.sqrt(3 * p * p)
    cpu.dw_w = [torch.randn(C, 1, K, K, generator=g) / K for _ in range(depth)]
    cpu.pw_w = [torch.randn(C, C, 1, 1, generator=g) * gain / math.sqrt(C) for _ in range(depth)]
    cpu.head_w = torch.randn(1000, C, generator=g) / math.sqrt(C)
    with torch.no_grad():
        gpu.model[0].weight.copy_(cpu.patch_w)
        for i in range(depth):
            blk = gpu.model[3 + i]
            blk[0].fn[0].weight.copy_(cpu.dw_w[i])
            blk[1].weight.copy_(cpu.pw_w[i])
        gpu.model[-1].weight.copy_(cpu.head_w)
    return gpu, cpu


@pytest.mark.parametrize("name", ["1536_20", "768_32"])
def test_convmixer_full_depth_parity(name):
    """Every block and the logits checked: with a signal-preserving init the feature maps after the
    middle and the last block and the logits are O(1), so the fused fp16 network is compared with the
    fp32 CPU model at full depth (rel-L2), against the bar of PyTorch's own fp16 GPU model."""
    from depthwise_conv_b200.convmixer import fuse_dw_blocks

    gpu, cpu = _signal_preserving_pair(name)
    base = gpu.half().cuda().to(memory_format=torch.channels_last)
    fused = fuse_dw_blocks(copy.deepcopy(base))
    assert fused.fused_blocks == base.depth
    x = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(9))
    xd = x.half().cuda().contiguous(memory_format=torch.channels_last)
    depth = base.depth
    for n in (depth // 2, depth):
        ref = cpu.trunk(x, blocks=n)
        assert 0.1 < ref.std().item() < 50.0, f"signal left the O(1) range after {n} blocks"
        with torch.no_grad():
            t = base.model[:3 + n](xd).float().cpu()
            f = fused.model[:3 + n](xd).float().cpu()
        rel_t = ((t - ref).norm() / ref.norm()).item()
        rel_f = ((f - ref).norm() / ref.norm()).item()
        print(f"ConvMixer-{name} after {n} blocks: rel-L2 torch-fp16 {rel_t:.2e}, engine-fused {rel_f:.2e}")
        assert rel_f <= max(1.5 * rel_t, 5e-3)
    ref = cpu(x)
    with torch.no_grad():
        lt = base(xd).float().cpu()
        lf = fused(xd).float().cpu()
    rel_t = ((lt - ref).norm() / ref.norm()).item()
    rel_f = ((lf - ref).norm() / ref.norm()).item()
    print(f"ConvMixer-{name} logits (std {ref.std().item():.2f}): rel-L2 torch-fp16 {rel_t:.2e}, "
          f"engine-fused {rel_f:.2e}")
    assert rel_f <= max(1.5 * rel_t, 5e-3)
    # the top classes agree wherever the fp32 margin is clear of the fp16 error
    top2 = ref.topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 0.05 * ref.std()
    assert torch.equal(lf.argmax(1)[clear], ref.argmax(1)[clear])
