"""Generate the golden fixtures under tests/golden/ (run where the reference is mounted).

    python tests/golden/make_golden.py /path/to/luckychen-depthwise_conv

Writes:
  * ``dw_cases.npz`` -- seeded small problems (inputs as fp16 bit patterns)
    with outputs of the reference's own correctness check,
    ``F.conv2d(groups=C)`` on the fp16-rounded inputs
    (benchmark_sensitivity.py:254-259, benchmark_triton.py:141-144), computed
    in float64; fused cases add bias -> act -> scale/shift
    (benchmark_cudnn_fused_e2e.py:65-74,125-131) and the residual
    (convmixer/convmixer.py:58-59).
  * ``op_schemas.json`` -- the schemas of every op the reference registers,
    read by importing its two op modules (depthwise_torch_ops.py:65-90,
    depthwise_replknet_nhwc_ops.py:53-66).
  * ``swap_repack.json`` -- digests of the weights/biases produced by the reference's module
    swappers (depthwise_torch_ops.py:268-340,
    depthwise_replknet_nhwc_ops.py:155-210) on small seeded models; the
    swappers' JIT kernel build is stubbed out, nothing is launched.

Nothing at test time reads the reference; the tests read these files.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, H, W, C, K, epilogue) -- edge cases the engine must handle:
# H or W < K, odd sizes, K = 1, C not a multiple of 64, single pixel.
CASES = [
    ("k3_small", 1, 5, 7, 8, 3, None),
    ("k7_cm768_slice", 2, 9, 11, 16, 7, None),
    ("k9_cm1536_slice", 1, 12, 10, 24, 9, None),
    ("k13_stage3_like", 1, 7, 7, 32, 13, None),
    ("k27_small_image", 1, 6, 5, 16, 27, None),
    ("k31_ragged", 2, 13, 17, 8, 31, None),
    ("k1_pointwise", 3, 4, 4, 8, 1, None),
    ("k5_single_pixel", 2, 1, 1, 16, 5, None),
    ("k9_tall", 1, 33, 3, 8, 9, None),
    ("k7_gelu_fused", 2, 8, 8, 16, 7, ("gelu", True)),
    ("k9_relu_fused", 1, 10, 12, 24, 9, ("relu", True)),
    ("k31_bias_only", 1, 12, 12, 8, 31, ("none", False)),
]


def _case(seed, B, H, W, C, K, epi):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, H, W, C, generator=g).half()
    w = (torch.randn(K, K, C, generator=g) / K).half()
    out = {"x": x.view(torch.int16).numpy(), "w": w.view(torch.int16).numpy()}
    xd = x.double().permute(0, 3, 1, 2)
    wd = w.double().permute(2, 0, 1).unsqueeze(1)
    y = F.conv2d(xd, wd, padding=K // 2, groups=C)
    if epi is not None:
        act, with_bn = epi
        b = (torch.randn(C, generator=g) * 0.1).half()
        out["bias"] = b.view(torch.int16).numpy()
        y = y + b.double().view(1, C, 1, 1)
        if act == "relu":
            y = torch.relu(y)
        elif act == "gelu":
            y = F.gelu(y)
        if with_bn:
            s = (torch.rand(C, generator=g) + 0.5).half()
            t = (torch.randn(C, generator=g) * 0.1).half()
            out["scale"] = s.view(torch.int16).numpy()
            out["shift"] = t.view(torch.int16).numpy()
            y = y * s.double().view(1, C, 1, 1) + t.double().view(1, C, 1, 1)
            y = y + xd  # residual
            out["residual"] = np.array(1)
        out["act"] = np.array({"none": 0, "relu": 1, "gelu": 2}[act])
    out["y"] = y.permute(0, 2, 3, 1).contiguous().numpy()
    return out


def make_cases():
    arrays = {}
    meta = []
    for i, (name, B, H, W, C, K, epi) in enumerate(CASES):
        c = _case(1000 + i, B, H, W, C, K, epi)
        for k, v in c.items():
            arrays[f"{name}__{k}"] = v
        meta.append({"name": name, "B": B, "H": H, "W": W, "C": C, "K": K})
    arrays["__meta__"] = np.array(json.dumps(meta))
    np.savez_compressed(os.path.join(HERE, "dw_cases.npz"), **arrays)


def _import_reference(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "convmixer", "kernels"))
    sys.path.insert(0, os.path.join(ref_root, "replknet", "kernels"))
    import depthwise_torch_ops as dto  # noqa: E402
    import depthwise_replknet_nhwc_ops as rno  # noqa: E402
    # Stub the JIT kernel build: only the module swappers' host logic runs here.
    dto._load_kernels = lambda: None
    rno._load_kernels = lambda: None
    return dto, rno


def make_schemas(dto, rno):
    names = ["depthwise::conv2d_32_1536_9", "depthwise::conv2d_32_1536_9_v2", "depthwise::conv2d_32_768_7",
             "depthwise::conv2d_16_1536_9", "depthwise::conv2d_32_1536_13", "replknet_dw::conv_56_128_31",
             "replknet_dw::conv_28_256_29", "replknet_dw::conv_14_512_27"]
    schemas = {}
    for n in names:
        ns, op = n.split("::")
        schemas[n] = str(getattr(getattr(torch.ops, ns), op).default._schema)
    configs = {f"{k[0]},{k[1]},{k[2]}": v for k, v in dto.CustomDepthwiseConv2d.SUPPORTED_CONFIGS.items()}
    repl = {f"{k[0]},{k[1]}": v.__name__ for k, v in rno._REPLACEMENT_MAP.items()}
    with open(os.path.join(HERE, "op_schemas.json"), "w") as f:
        json.dump({"schemas": schemas, "supported_configs": configs, "replacement_map": repl}, f, indent=1,
                  sort_keys=True)


class _Tiny(nn.Module):
    def __init__(self, C, K, bias):
        super().__init__()
        self.body = nn.Sequential(nn.Conv2d(C, C, K, groups=C, padding=K // 2, bias=bias), nn.ReLU())


# (tag, C, K, bias, swapper) for the repack fixture; weights come from a seeded
# numpy generator so the test can rebuild the same nn.Conv2d.
REPACK_CASES = [("cm_768_7", 768, 7, True, "convmixer"), ("cm_1536_9", 1536, 9, False, "convmixer"),
                ("rl_128_31", 128, 31, True, "replknet"), ("rl_512_27", 512, 27, False, "replknet")]


def repack_model(C, K, bias, seed):
    """The small model whose depthwise conv the swappers replace (shared with the test)."""
    m = _Tiny(C, K, bias)
    rng = np.random.default_rng(seed)
    with torch.no_grad():
        m.body[0].weight.copy_(torch.from_numpy(rng.standard_normal((C, 1, K, K)).astype(np.float32) * 0.05))
        if bias:
            m.body[0].bias.copy_(torch.from_numpy(rng.standard_normal(C).astype(np.float32) * 0.1))
    return m


def _digest(t):
    import hashlib
    return hashlib.sha256(t.detach().contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def make_repack(dto, rno):
    out = {}
    for i, (tag, C, K, bias, which) in enumerate(REPACK_CASES):
        m = repack_model(C, K, bias, 500 + i)
        if which == "convmixer":
            dto.replace_depthwise_convs(m, verbose=False)
        else:
            rno.replace_replknet_depthwise_nhwc(m, verbose=False)
        mod = m.body[0]
        out[tag] = {"type": type(mod).__name__, "weight_shape": list(mod.weight.shape),
                    "weight_sha256": _digest(mod.weight),
                    "bias_sha256": _digest(mod.bias) if mod.bias is not None else None,
                    "weight_head": mod.weight.detach().float().flatten()[:8].tolist()}
    with open(os.path.join(HERE, "swap_repack.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


def main():
    make_cases()
    ref_root = sys.argv[1] if len(sys.argv) > 1 else None
    if ref_root and os.path.isdir(ref_root):
        dto, rno = _import_reference(ref_root)
        make_schemas(dto, rno)
        make_repack(dto, rno)
    else:
        print("reference not given: only dw_cases.npz regenerated")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
