"""TEST INFRASTRUCTURE ONLY: the moebius-cpu VAE (encoder and decoder)
composed from the oracle kernels (reference src/vae/encoder.rs:173-230,
src/vae/decoder.rs:74-99, src/vae/mod.rs:174-293): the CPU counterpart of the
library's VAE, for parity tests and the CPU baseline. Stride-1 3×3 convs run
the oracle's Winograd path and stride-2 ones its im2col path, as the reference
does; GroupNorm+SiLU is applied as the convs' prologue, as the reference does.
Weights are a dict of numpy arrays in the converter's layout (f16 widened).
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

VAE_BLOCK_OUT = (128, 256, 512, 512)
UP_LAYERS = 3
EPS = 1e-6
GROUPS = 32
SCALING_FACTOR = 0.13025


def _affine(w, name, x):
    return O.group_norm_affine(x, GROUPS, EPS, w[f"{name}.weight"], w[f"{name}.bias"])


def _conv3(w, name, x, **kw):
    return O.conv3x3(x, np.ascontiguousarray(w[f"{name}.weight"], np.float32), w[f"{name}.bias"], **kw)


def _conv1(w, name, x, residual=None):
    return O.conv1x1(x, np.ascontiguousarray(w[f"{name}.weight"], np.float32), w[f"{name}.bias"], residual)


def resnet(w, name, x):
    """src/vae/mod.rs:197-211."""
    s, t = _affine(w, f"{name}.norm1", x)
    h = _conv3(w, f"{name}.conv1", x, prologue=(s, t, True))
    s, t = _affine(w, f"{name}.norm2", h)
    out = _conv3(w, f"{name}.conv2", h, prologue=(s, t, True))
    if f"{name}.conv_shortcut.weight" in w:
        return _conv1(w, f"{name}.conv_shortcut", x, residual=out)
    return O.add(out, x)


def mid_attention(w, name, x):
    """src/vae/mod.rs:240-270 (bands of query rows do not change the values)."""
    n, h, ww, c = x.shape
    hw = h * ww
    t = O.group_norm(x, GROUPS, EPS, w[f"{name}.group_norm.weight"], w[f"{name}.group_norm.bias"])
    q, k, v = (_conv1(w, f"{name}.{p}", t) for p in ("to_q", "to_k", "to_v"))
    o = np.empty_like(t)
    for b in range(n):
        qb, kb, vb = (a[b].reshape(hw, c) for a in (q, k, v))
        scores = O.softmax_rows(O.gemm_nt(qb, kb), 1.0 / np.sqrt(c))
        o[b] = O.gemm_nt(scores, np.ascontiguousarray(vb.T)).reshape(h, ww, c)
    return _conv1(w, f"{name}.to_out.0", o, residual=x)


def decode(w, latents):
    """latents: scaled [n, h, w, 4] → (dec(latents / 0.13025) + 1) / 2, [n, 8h, 8w, 3]."""
    z = (np.asarray(latents, np.float32) / np.float32(SCALING_FACTOR)).astype(np.float32)
    cur = _conv1(w, "post_quant_conv", z)
    cur = _conv3(w, "decoder.conv_in", cur)
    cur = resnet(w, "decoder.mid_block.resnets.0", cur)
    cur = mid_attention(w, "decoder.mid_block.attentions.0", cur)
    cur = resnet(w, "decoder.mid_block.resnets.1", cur)
    for i in range(len(VAE_BLOCK_OUT)):
        for j in range(UP_LAYERS):
            cur = resnet(w, f"decoder.up_blocks.{i}.resnets.{j}", cur)
        if i + 1 < len(VAE_BLOCK_OUT):
            cur = _conv3(w, f"decoder.up_blocks.{i}.upsamplers.0.conv", cur, upsample2x=True)
    s, t = _affine(w, "decoder.conv_norm_out", cur)
    out = _conv3(w, "decoder.conv_out", cur, prologue=(s, t, True))
    return ((out + np.float32(1.0)) * np.float32(0.5)).astype(np.float32)


def encode(w, images, noise):
    """images [b, h, w, 3] in [-1, 1], noise [b, h/8, w/8, 4] -> scaled latents (encoder.rs:173-230)."""
    cur = _conv3(w, "encoder.conv_in", np.asarray(images, np.float32))
    for i in range(4):
        for j in range(2):
            cur = resnet(w, f"encoder.down_blocks.{i}.resnets.{j}", cur)
        if i < 3:
            cur = _conv3(w, f"encoder.down_blocks.{i}.downsamplers.0.conv", cur, stride=2, pad=(0, 0, 1, 1))
    cur = resnet(w, "encoder.mid_block.resnets.0", cur)
    cur = mid_attention(w, "encoder.mid_block.attentions.0", cur)
    cur = resnet(w, "encoder.mid_block.resnets.1", cur)
    s, t = _affine(w, "encoder.conv_norm_out", cur)
    mom = _conv3(w, "encoder.conv_out", cur, prologue=(s, t, True))
    moments = _conv1(w, "quant_conv", mom)
    return O.vae_sample(moments, noise)
