"""Writes the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py --reference-root PATH   (or MOEBIUS_REFERENCE_ROOT=PATH)

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

3. ``imaging_ref.safetensors``: the reference's Pillow blur fixture
   (``tests/fixtures/blur.safetensors``, Pillow 10.4 per its generator) and its
   upstream compensated-paste fixture (``tests/fixtures/compensate.safetensors``,
   names prefixed ``comp.``), copied, plus cases written here with the installed
   Pillow: two model-size masks of random filled ellipses covering 10-40 % (the
   BASELINE mask distribution) blurred with ``GaussianBlur(3)`` as upstream
   ``_post_process`` does, and four Lanczos3 resizes (``lz*``; upstream resizes
   the crop window with ``Image.LANCZOS``).
4. ``weights_manifest.json``: every tensor of the converted UNet and VAE
   (name -> shape), derived from the reference's ``docs/weights-manifest.txt``
   with the converter's transformations (BatchNorms folded into new ``.bias``
   tensors, layouts of ``tools/convert_weights.py``).

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


def ellipse_mask(rng, side=512, lo=0.10, hi=0.40):
    """Union of random filled ellipses until the covered fraction lies in [lo, hi]."""
    yy, xx = np.mgrid[:side, :side]
    while True:
        m = np.zeros((side, side), bool)
        target = rng.uniform(lo, hi)
        while m.mean() < target:
            cy, cx = rng.uniform(0, side, 2)
            ry, rx = rng.uniform(side * 0.05, side * 0.3, 2)
            th = rng.uniform(0, np.pi)
            dy, dx = yy - cy, xx - cx
            u = (dx * np.cos(th) + dy * np.sin(th)) / rx
            v = (-dx * np.sin(th) + dy * np.cos(th)) / ry
            m |= u * u + v * v <= 1.0
        if lo <= m.mean() <= hi:
            return (m * 255).astype(np.uint8)


def imaging_cases(reference_root):
    from PIL import Image, ImageFilter
    import PIL
    t = {k: np.ascontiguousarray(v) for k, v in
         load_file(os.path.join(reference_root, "tests", "fixtures", "blur.safetensors")).items()}
    rng = np.random.default_rng(512)
    for k in ("e1", "e2"):
        m = ellipse_mask(rng)
        blurred = np.asarray(Image.fromarray(m).convert("RGB").filter(ImageFilter.GaussianBlur(radius=3)))[:, :, 0]
        t[f"{k}.mask"] = m
        t[f"{k}.blurred"] = np.ascontiguousarray(blurred, np.uint8)
    # The reference's upstream paste_compensate fixture (tests/fixtures/compensate.safetensors).
    comp = load_file(os.path.join(reference_root, "tests", "fixtures", "compensate.safetensors"))
    for k, v in comp.items():
        t[f"comp.{k}"] = np.ascontiguousarray(v)
    # Lanczos3 resizes with Pillow (Image.LANCZOS, the filter upstream resizes the crop window
    # with): RGB down and up, a mask channel, and a model-size result back to a small window.
    rng = np.random.default_rng(7)
    for k, (src, dst, ch) in {"lz1": (300, 128, 3), "lz2": (96, 128, 3), "lz3": (77, 64, 1),
                              "lz4": (128, 45, 3)}.items():
        a = rng.integers(0, 256, (src, src, ch), dtype=np.uint8)
        img = Image.fromarray(a[..., 0] if ch == 1 else a)
        t[f"{k}.src"] = a
        out = np.asarray(img.resize((dst, dst), Image.LANCZOS))
        t[f"{k}.dst"] = np.ascontiguousarray(out.reshape(dst, dst, ch))
    return t, PIL.__version__


def converted_manifest(reference_root):
    """name -> shape of the converted weights (tools/convert_weights.py transformations)."""
    import ast
    bn_targets = {"bn1": "conv_dw", "bn2": "conv_pw", "norm_q": "to_q", "norm_v": "to_v"}
    out, cur = {}, None
    for line in open(os.path.join(reference_root, "docs", "weights-manifest.txt")):
        line = line.rstrip("\n")
        if not line or line.startswith("#"):
            continue
        if line.startswith("["):
            cur = line.strip("[]")
            out[cur] = {}
            continue
        name, shape = line.split("\t")
        shape = ast.literal_eval(shape)
        mod, _, leaf = name.rpartition(".")
        parent, _, bn = mod.rpartition(".")
        if bn in bn_targets:
            if leaf == "weight":
                out[cur][f"{parent}.{bn_targets[bn]}.bias"] = [shape[0]]
            continue
        if leaf == "rel_pos_emb":
            shape = shape[:3]
        elif leaf == "weight" and len(shape) == 5:
            shape = [shape[0], shape[3] * shape[4]]
        elif leaf == "weight" and len(shape) == 4:
            o, i, kh, kw = shape
            shape = [o, i] if (kh, kw) == (1, 1) else ([3, 3, o] if i == 1 else [o, 3, 3, i])
        out[cur][name] = list(shape)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=os.environ.get("MOEBIUS_REFERENCE_ROOT"),
                    help="a moebius-cpu checkout (default: $MOEBIUS_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference_root:
        ap.error("give --reference-root or set MOEBIUS_REFERENCE_ROOT to a moebius-cpu checkout")
    src = os.path.join(args.reference_root, "tests", "fixtures", "kernels.safetensors")
    ref = load_file(src)
    save_file({k: np.ascontiguousarray(v) for k, v in ref.items()}, os.path.join(HERE, "kernels_ref.safetensors"),
              metadata={"format": "moebius-cpu-fixture/1",
                        "source": "moebius-cpu tests/fixtures/kernels.safetensors (copied tensor by tensor)"})
    extra = extra_cases()
    save_file(extra, os.path.join(HERE, "kernels_extra.safetensors"),
              metadata={"format": "moebius-b200-fixture/1", "generator": "tests/golden/make_golden.py",
                        "torch": torch.__version__, "seed": "20261201"})
    img, pil_version = imaging_cases(args.reference_root)
    save_file(img, os.path.join(HERE, "imaging_ref.safetensors"),
              metadata={"format": "moebius-b200-fixture/1", "generator": "tests/golden/make_golden.py",
                        "source": "moebius-cpu tests/fixtures/blur.safetensors (a, b, c) and "
                                  "compensate.safetensors (comp.*); e1, e2, lz* from Pillow " + pil_version})
    import json
    with open(os.path.join(HERE, "weights_manifest.json"), "w") as f:
        json.dump(converted_manifest(args.reference_root), f, indent=0, sort_keys=True)
    print(f"wrote {len(ref)} reference tensors, {len(extra)} extra tensors, {len(img)} imaging tensors")


if __name__ == "__main__":
    main()
