"""Seeded random-init weights in the reference converter's format.

No checkpoint is available offline, so the engine is exercised on random
weights of the shipped architecture (BASELINE configs 4 and 5), written as
``unet.safetensors`` / ``vae.safetensors`` exactly as the reference's
``tools/convert_weights.py`` lays them out: upstream names, BatchNorms folded
(``conv_dw.bias``, ``conv_pw.bias``, ``to_q.bias``, ``to_v.bias``), 1x1 weights
[o, i], dense 3x3 [o, 3, 3, i], depthwise [3, 3, c], ``pos_conv.weight``
[k, 225], ``rel_pos_emb`` [N, 10, k]; GEMM weights f16 (``f16=True``) or f32,
everything else f32; VAE metadata ``scaling_factor = 0.13025``.

``unet_shapes`` / ``vae_shapes`` take the level widths and latent size so that
tests can build scaled-down networks of the same structure.

Init: GEMM and conv weights N(0, 1/fan_in) (std 1/sqrt(fan_in)), biases
N(0, 0.01), norm gamma N(1, 0.02) and beta N(0, 0.02), depthwise N(0, 1/9),
the self-lambda position filter N(0, 1/(225 k)), the cross-lambda position
table N(0, 1/k), the token embedding N(0, 1).
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

UNET_WIDTHS = (320, 640, 1280)
UNET_LATENT = 64
VAE_WIDTHS = (128, 256, 512, 512)
HEADS = 8
TOKENS = 10
EHS_DIM = 768
ENCODER_HID = 3072
NUM_EMBEDDINGS = 20
TAPS = 225
SCALING_FACTOR = "0.13025"

# kinds: gemm (f16 when requested), vec, dw (depthwise), pos (self-λ filter), table (cross-λ), emb
_GEMM, _VEC, _NORM_W, _NORM_B, _DW, _POS, _TABLE, _EMB = range(8)


def unet_shapes(widths=UNET_WIDTHS, latent=UNET_LATENT) -> dict:
    """name -> (shape, kind) for the converted UNet (src/unet/*, src/unet/load.rs)."""
    s = {}
    d = "diff_model"
    ch0 = widths[0]
    te = 4 * ch0

    def conv1(name, ci, co, bias=True):
        s[f"{name}.weight"] = ((co, ci), _GEMM)
        if bias:
            s[f"{name}.bias"] = ((co,), _VEC)

    def conv3(name, ci, co):
        s[f"{name}.weight"] = ((co, 3, 3, ci), _GEMM)
        s[f"{name}.bias"] = ((co,), _VEC)

    def norm(name, c):
        s[f"{name}.weight"] = ((c,), _NORM_W)
        s[f"{name}.bias"] = ((c,), _NORM_B)

    def dw(name, c):
        s[f"{name}.weight"] = ((3, 3, c), _DW)
        s[f"{name}.bias"] = ((c,), _VEC)

    def dwconv(name, ci, co):
        dw(f"{name}.conv_dw", ci)
        conv1(f"{name}.conv_pw", ci, co)

    def resnet(name, ci, co):
        norm(f"{name}.norm1", ci)
        dwconv(f"{name}.conv1", ci, co)
        conv1(f"{name}.time_emb_proj", te, co)
        norm(f"{name}.norm2", co)
        dwconv(f"{name}.conv2", co, co)
        if ci != co:
            conv1(f"{name}.conv_shortcut", ci, co)

    def transformer(name, c, hw):
        k = c // HEADS
        hidden = c * 5 // 2
        b = f"{name}.transformer_blocks.0"
        norm(f"{name}.norm", c)
        conv1(f"{name}.proj_in", c, c)
        for i in (1, 2, 3):
            norm(f"{b}.norm{i}", c)
        conv1(f"{b}.attn1.to_q", c, c)
        conv1(f"{b}.attn1.to_k", c, k, bias=False)
        conv1(f"{b}.attn1.to_v", c, k)
        s[f"{b}.attn1.pos_conv.weight"] = ((k, TAPS), _POS)
        s[f"{b}.attn1.pos_conv.bias"] = ((k,), _VEC)
        conv1(f"{b}.attn2.to_q", c, c)
        s[f"{b}.attn2.to_k.weight"] = ((k, EHS_DIM), _GEMM)
        s[f"{b}.attn2.to_v.weight"] = ((k, EHS_DIM), _GEMM)
        s[f"{b}.attn2.to_v.bias"] = ((k,), _VEC)
        s[f"{b}.attn2.rel_pos_emb"] = ((hw, TOKENS, k), _TABLE)
        conv1(f"{b}.ff.inverted_conv.conv", c, 2 * hidden)
        dw(f"{b}.ff.depth_conv.conv", 2 * hidden)
        conv1(f"{b}.ff.point_conv.conv", hidden, c, bias=False)
        conv1(f"{name}.proj_out", c, c)

    s["embedding_layer.weight"] = ((NUM_EMBEDDINGS, ENCODER_HID), _EMB)
    conv1(f"{d}.encoder_hid_proj", ENCODER_HID, EHS_DIM)
    conv1(f"{d}.time_embedding.linear_1", ch0, te)
    conv1(f"{d}.time_embedding.linear_2", te, te)
    dwconv(f"{d}.conv_in", 9, ch0)
    c_prev = ch0
    skips = [ch0]
    for i, c in enumerate(widths):
        hw = (latent >> i) ** 2
        for j in range(2):
            resnet(f"{d}.down_blocks.{i}.resnets.{j}", c_prev if j == 0 else c, c)
            transformer(f"{d}.down_blocks.{i}.attentions.{j}", c, hw)
            skips.append(c)
        if i + 1 < len(widths):
            conv3(f"{d}.down_blocks.{i}.downsamplers.0.conv", c, c)
            skips.append(c)
        c_prev = c
    h_c = widths[-1]
    for i, c in enumerate(reversed(widths)):
        lvl = len(widths) - 1 - i
        hw = (latent >> lvl) ** 2
        for j in range(3):
            skip_c = skips.pop()
            resnet(f"{d}.up_blocks.{i}.resnets.{j}", h_c + skip_c, c)
            transformer(f"{d}.up_blocks.{i}.attentions.{j}", c, hw)
            h_c = c
        if i + 1 < len(widths):
            conv3(f"{d}.up_blocks.{i}.upsamplers.0.conv", c, c)
    assert not skips
    norm(f"{d}.conv_norm_out", ch0)
    dwconv(f"{d}.conv_out", ch0, 4)
    return s


def vae_shapes(widths=VAE_WIDTHS) -> dict:
    """name -> (shape, kind) for the converted VAE (src/vae/*)."""
    s = {}

    def conv1(name, ci, co):
        s[f"{name}.weight"] = ((co, ci), _GEMM)
        s[f"{name}.bias"] = ((co,), _VEC)

    def conv3(name, ci, co):
        s[f"{name}.weight"] = ((co, 3, 3, ci), _GEMM)
        s[f"{name}.bias"] = ((co,), _VEC)

    def norm(name, c):
        s[f"{name}.weight"] = ((c,), _NORM_W)
        s[f"{name}.bias"] = ((c,), _NORM_B)

    def resnet(name, ci, co):
        norm(f"{name}.norm1", ci)
        conv3(f"{name}.conv1", ci, co)
        norm(f"{name}.norm2", co)
        conv3(f"{name}.conv2", co, co)
        if ci != co:
            conv1(f"{name}.conv_shortcut", ci, co)

    def mid(name, c):
        resnet(f"{name}.resnets.0", c, c)
        norm(f"{name}.attentions.0.group_norm", c)
        for p in ("to_q", "to_k", "to_v", "to_out.0"):
            conv1(f"{name}.attentions.0.{p}", c, c)
        resnet(f"{name}.resnets.1", c, c)

    top = widths[-1]
    conv3("encoder.conv_in", 3, widths[0])
    c_prev = widths[0]
    for i, c in enumerate(widths):
        for j in range(2):
            resnet(f"encoder.down_blocks.{i}.resnets.{j}", c_prev if j == 0 else c, c)
        if i + 1 < len(widths):
            conv3(f"encoder.down_blocks.{i}.downsamplers.0.conv", c, c)
        c_prev = c
    mid("encoder.mid_block", top)
    norm("encoder.conv_norm_out", top)
    conv3("encoder.conv_out", top, 8)
    conv1("quant_conv", 8, 8)
    conv1("post_quant_conv", 4, 4)
    conv3("decoder.conv_in", 4, top)
    mid("decoder.mid_block", top)
    c_prev = top
    for i, c in enumerate(reversed(widths)):
        for j in range(3):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", c_prev if j == 0 else c, c)
        if i + 1 < len(widths):
            conv3(f"decoder.up_blocks.{i}.upsamplers.0.conv", c, c)
        c_prev = c
    norm("decoder.conv_norm_out", widths[0])
    conv3("decoder.conv_out", widths[0], 3)
    return s


def random_weights(shapes: dict, seed: int = 0, f16: bool = True) -> dict:
    """Seeded tensors for `shapes`; GEMM weights f16 when `f16` (the shipped storage), else f32."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(shapes):
        shape, kind = shapes[name]
        if kind == _GEMM:
            fan_in = int(np.prod(shape[1:]))
            w = rng.normal(0.0, 1.0 / np.sqrt(fan_in), shape).astype(np.float32)
            out[name] = w.astype(np.float16) if f16 else w
        elif kind == _NORM_W:
            out[name] = rng.normal(1.0, 0.02, shape).astype(np.float32)
        elif kind == _NORM_B:
            out[name] = rng.normal(0.0, 0.02, shape).astype(np.float32)
        elif kind == _DW:
            out[name] = rng.normal(0.0, 1.0 / 3.0, shape).astype(np.float32)
        elif kind == _POS:
            out[name] = rng.normal(0.0, 1.0 / np.sqrt(TAPS * shape[0]), shape).astype(np.float32)
        elif kind == _TABLE:
            out[name] = rng.normal(0.0, 1.0 / np.sqrt(shape[2]), shape).astype(np.float32)
        elif kind == _EMB:
            out[name] = rng.normal(0.0, 1.0, shape).astype(np.float32)
        else:
            out[name] = rng.normal(0.0, 0.01, shape).astype(np.float32)
    return out


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Minimal safetensors writer (8-byte little-endian header length, JSON header, raw data)."""
    header = {}
    offset = 0
    blobs = []
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        dt = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16"}[a.dtype]
        b = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [offset, offset + len(b)]}
        blobs.append(b)
        offset += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str) -> tuple[dict, dict]:
    """(tensors as numpy arrays, metadata) of a file written by `write_safetensors`."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    meta = header.pop("__metadata__", {})
    out = {}
    for name, t in header.items():
        dt = {"F32": np.float32, "F16": np.float16}[t["dtype"]]
        a, b = t["data_offsets"]
        out[name] = np.frombuffer(data[a:b], dtype=dt).reshape(t["shape"]).copy()
    return out, meta


def write_weights_dir(path: str, seed: int = 0, f16: bool = True, unet_widths=UNET_WIDTHS, latent=UNET_LATENT,
                      vae_widths=VAE_WIDTHS) -> str:
    """Writes unet.safetensors and vae.safetensors (converter format) under `path`."""
    os.makedirs(path, exist_ok=True)
    dtype = "f16" if f16 else "f32"
    write_safetensors(os.path.join(path, "unet.safetensors"),
                      random_weights(unet_shapes(unet_widths, latent), seed, f16),
                      {"format": "moebius-cpu/1", "dtype": dtype})
    write_safetensors(os.path.join(path, "vae.safetensors"), random_weights(vae_shapes(vae_widths), seed + 1, f16),
                      {"format": "moebius-cpu/1", "dtype": dtype, "scaling_factor": SCALING_FACTOR})
    return path


def ellipse_masks(rng, n: int, side: int = 512, lo: float = 0.10, hi: float = 0.40) -> np.ndarray:
    """n binary masks [n, side, side] (0 / 255): unions of random filled ellipses covering a
    fraction in [lo, hi] of the image (BASELINE config 5's mask distribution)."""
    yy, xx = np.mgrid[:side, :side].astype(np.float32)
    out = np.zeros((n, side, side), np.uint8)
    for i in range(n):
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
                out[i] = m * 255
                break
    return out
