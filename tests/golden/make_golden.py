"""Writes the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py [--reference-root PATH]

1. ``kernels_ref.safetensors``: the reference's own kernel fixture
   (moebius-cpu ``tests/fixtures/kernels.safetensors``, produced by its
   ``tools/dump_kernel_fixtures.py`` with PyTorch, seed 1234), copied tensor
   by tensor with its names kept, so the GPU box (which has no reference
   checkout) can replay every case of the reference's ``tests/kernels.rs``.
2. ``kernels_extra.safetensors``: additional PyTorch float64 cases written by
   this script (seeded) for edges the reference fixture does not reach:
   GroupNorm with 2 channels per group, channel counts that are not multiples
   of 4, depthwise channel tails, a GN(+SiLU) prologue fused into 3×3 convs
   (plain and upsampled), LayerNorm at UNet widths, and the broadcast adds.

Layouts follow the reference converter: activations NHWC, 1×1 weights
[o, i], dense 3×3 [o, 3, 3, i], depthwise [3, 3, c].
"""
from __future__ import annotations

import argparse
import os

import numpy as np
import torch
import torch.nn.functional as F
from safetensors.numpy import load_file, save_file

HERE = os.path.dirname(os.path.abspath(__file__))


def nhwc(x):
    return x.permute(0, 2, 3, 1).contiguous()


def w3x3(w):
    return w.permute(0, 2, 3, 1).contiguous()


def wdw(w):
    return w[:, 0].permute(1, 2, 0).contiguous()


def f32(t):
    return {k: v.detach().to(torch.float32).contiguous().numpy() for k, v in t.items()}


def extra_cases() -> dict:
    g = torch.Generator().manual_seed(20261201)

    def randn(*shape, scale=1.0, shift=0.0):
        return torch.randn(*shape, generator=g, dtype=torch.float64) * scale + shift

    t = {}
    # GroupNorm(32) over 64 channels: 2 channels per group, so one 4-wide
    # channel vector spans two groups. Pre-norm add + SiLU, eps 1e-6.
    x = randn(2, 64, 4, 5, scale=2.0, shift=0.5)
    add = randn(2, 64)
    gm, bt = randn(64, scale=0.3, shift=1.0), randn(64, scale=0.3)
    y = F.silu(F.group_norm(x + add[:, :, None, None], 32, gm, bt, eps=1e-6))
    t |= {"gn64.x": nhwc(x), "gn64.add": add, "gn64.gamma": gm, "gn64.beta": bt, "gn64.y": nhwc(y)}

    # 1×1 conv with c_in = 9 (UNet conv_in width) and c_out = 4, bias + residual.
    x = randn(2, 9, 6, 7)
    w = randn(4, 9, 1, 1, scale=0.3)
    b = randn(4)
    r = randn(2, 4, 6, 7)
    t |= {"c1o.x": nhwc(x), "c1o.w": w[:, :, 0, 0], "c1o.b": b, "c1o.r": nhwc(r),
          "c1o.y": nhwc(F.conv2d(x, w, b) + r)}

    # GN(+SiLU) prologue fused into a 3×3 same conv, plain and upsampled
    # (padding stays zero, not f(0)): the forward_prologue contract.
    x = randn(2, 40, 7, 9, scale=3.0, shift=0.7)
    gm, bt = randn(40, scale=0.5, shift=1.0), randn(40)
    w = randn(24, 40, 3, 3, scale=0.05)
    b = torch.arange(24, dtype=torch.float64) * 0.01
    a = F.silu(F.group_norm(x, 8, gm, bt, eps=1e-6))
    t |= {"pro.x": nhwc(x), "pro.gamma": gm, "pro.beta": bt, "pro.w": w3x3(w), "pro.b": b,
          "pro.y": nhwc(F.conv2d(a, w, b, padding=1)),
          "pro.yup": nhwc(F.conv2d(F.interpolate(a, scale_factor=2.0, mode="nearest"), w, b, padding=1))}

    # 3×3 convs with c_in = 4 (VAE decoder conv_in) and c_out = 3 (conv_out).
    x = randn(1, 4, 10, 12)
    w = randn(3, 4, 3, 3, scale=0.2)
    b = randn(3)
    t |= {"c3n.x": nhwc(x), "c3n.w": w3x3(w), "c3n.b": b, "c3n.y": nhwc(F.conv2d(x, w, b, padding=1))}

    # Depthwise channel tails: 70 channels plain, 140 → 70 GLU·SiLU.
    for name, c, glu in [("dw70", 70, False), ("dw140", 140, True)]:
        x = randn(1, c, 4, 9)
        w = randn(c, 1, 3, 3, scale=0.3)
        b = randn(c, scale=0.1)
        y = F.conv2d(x, w, b, padding=1, groups=c)
        if glu:
            v, gate = y.chunk(2, dim=1)
            y = v * F.silu(gate)
        t |= {f"{name}.x": nhwc(x), f"{name}.w": wdw(w), f"{name}.b": b, f"{name}.y": nhwc(y)}

    # LayerNorm over 320 channels (UNet level 0 width).
    x = randn(2, 37, 320, scale=2.0, shift=-0.5)
    gm, bt = randn(320), randn(320)
    t |= {"ln320.x": x, "ln320.gamma": gm, "ln320.beta": bt,
          "ln320.y": F.layer_norm(x, (320,), gm, bt, eps=1e-5)}

    # Broadcast adds: (x + bias[c]) + temb[n, c]; residual add; SiLU.
    x = randn(2, 5, 6, 12)
    b = randn(12)
    te = randn(2, 12)
    r = randn(2, 5, 6, 12)
    t |= {"bt.x": x, "bt.bias": b, "bt.temb": te, "bt.y": (x + b) + te[:, None, None, :],
          "bt.r": r, "bt.sum": x + r, "bt.silu": F.silu(x)}
    return f32(t)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default="/root/reference")
    args = ap.parse_args()
    src = os.path.join(args.reference_root, "tests", "fixtures", "kernels.safetensors")
    ref = load_file(src)
    save_file({k: np.ascontiguousarray(v) for k, v in ref.items()}, os.path.join(HERE, "kernels_ref.safetensors"),
              metadata={"format": "moebius-cpu-fixture/1",
                        "source": "moebius-cpu tests/fixtures/kernels.safetensors (copied tensor by tensor)"})
    extra = extra_cases()
    save_file(extra, os.path.join(HERE, "kernels_extra.safetensors"),
              metadata={"format": "moebius-b200-fixture/1", "generator": "tests/golden/make_golden.py",
                        "torch": torch.__version__, "seed": "20261201"})
    print(f"wrote {len(ref)} reference tensors and {len(extra)} extra tensors")


if __name__ == "__main__":
    main()
