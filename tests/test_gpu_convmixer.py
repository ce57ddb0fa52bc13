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
