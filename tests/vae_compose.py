"""TEST HELPER: the moebius-cpu VAE decoder composed in Python from the
kernel ABI (include/moebius_cuda.h) entry points, to test how those kernels
compose (GroupNorm prologues, the tensor-core GEMMs and the flushed softmax of
the mid attention) independently of the engine's C++ decoder (eng_vae.cpp),
which the engine tests check against the oracle. Structure and names follow the reference's
src/vae/decoder.rs and src/vae/mod.rs (diffusers AutoencoderKL, SDXL-VAE:
block_out (128, 256, 512, 512), 3 resnets per up level, one single-head
attention in the mid block, GroupNorm(32) eps 1e-6):

    z = latents / 0.13025                         (decoder.rs:81)
    post_quant_conv 1×1 → conv_in 3×3 → mid (resnet, attention, resnet)
    → up levels (512, 512, 256, 128): 3 resnets + nearest-2× upsample conv
      on the first three                            (decoder.rs:84-94)
    → GN + SiLU fused into conv_out 3×3 (128 → 3)   (decoder.rs:95)
    → (x + 1) / 2                                    (decoder.rs:97)

Weights are a dict of numpy arrays in the reference converter's layouts
(1×1 [o, i], 3×3 [o, 3, 3, i]) under diffusers' names;
``random_decoder_weights`` makes a seeded random-init set (no checkpoint is
available offline).
"""
from __future__ import annotations

import numpy as np

from conftest import load_package

_mbx = load_package()
Context, DeviceTensor, Param = _mbx.Context, _mbx.DeviceTensor, _mbx.Param
conv1x1, conv3x3, group_norm, group_norm_affine = _mbx.conv1x1, _mbx.conv3x3, _mbx.group_norm, _mbx.group_norm_affine
check, lib = _mbx.abi.check, _mbx.abi.lib

VAE_BLOCK_OUT = (128, 256, 512, 512)
LATENT_CHANNELS = 4
IMAGE_CHANNELS = 3
UP_LAYERS = 3
VAE_EPS = 1e-6
GROUPS = 32
SCALING_FACTOR = 0.13025
SOFTMAX_FLUSH = -40.0  # probabilities below e^-40 are zero (src/vae/mod.rs:273-275)


def decoder_weight_shapes() -> dict:
    """Every decoder tensor (converted layout) by name."""
    shapes = {}

    def conv3(name, ci, co):
        shapes[f"{name}.weight"] = (co, 3, 3, ci)
        shapes[f"{name}.bias"] = (co,)

    def conv1(name, ci, co):
        shapes[f"{name}.weight"] = (co, ci)
        shapes[f"{name}.bias"] = (co,)

    def norm(name, c):
        shapes[f"{name}.weight"] = (c,)
        shapes[f"{name}.bias"] = (c,)

    def resnet(name, ci, co):
        norm(f"{name}.norm1", ci)
        conv3(f"{name}.conv1", ci, co)
        norm(f"{name}.norm2", co)
        conv3(f"{name}.conv2", co, co)
        if ci != co:
            conv1(f"{name}.conv_shortcut", ci, co)

    ch = VAE_BLOCK_OUT
    top = ch[-1]
    conv1("post_quant_conv", LATENT_CHANNELS, LATENT_CHANNELS)
    conv3("decoder.conv_in", LATENT_CHANNELS, top)
    resnet("decoder.mid_block.resnets.0", top, top)
    norm("decoder.mid_block.attentions.0.group_norm", top)
    for p in ("to_q", "to_k", "to_v", "to_out.0"):
        conv1(f"decoder.mid_block.attentions.0.{p}", top, top)
    resnet("decoder.mid_block.resnets.1", top, top)
    c_prev = top
    for i, c in enumerate(reversed(ch)):
        for j in range(UP_LAYERS):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", c_prev if j == 0 else c, c)
        if i + 1 < len(ch):
            conv3(f"decoder.up_blocks.{i}.upsamplers.0.conv", c, c)
        c_prev = c
    norm("decoder.conv_norm_out", ch[0])
    conv3("decoder.conv_out", ch[0], IMAGE_CHANNELS)
    return shapes


def random_decoder_weights(seed: int = 0, f16: bool = True) -> dict:
    """Seeded random init: conv weights N(0, 1/√fan_in) (rounded to f16 when `f16`,
    as the shipped VAE is), biases N(0, 0.01), norm γ N(1, 0.02), β N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in decoder_weight_shapes().items():
        if name.endswith(".weight") and len(shape) > 1:
            fan_in = int(np.prod(shape[1:]))
            w = rng.normal(0.0, 1.0 / np.sqrt(fan_in), shape).astype(np.float32)
            out[name] = w.astype(np.float16).astype(np.float32) if f16 else w
        elif ".norm" in name or "group_norm" in name or "conv_norm_out" in name:
            out[name] = (rng.normal(1.0, 0.02, shape) if name.endswith("weight")
                         else rng.normal(0.0, 0.02, shape)).astype(np.float32)
        else:
            out[name] = rng.normal(0.0, 0.01, shape).astype(np.float32)
    return out


class _Loader:
    def __init__(self, ctx: Context, w: dict, dtype: str):
        self.ctx, self.w, self.dtype = ctx, w, dtype
        self.params = []

    def param(self, name):
        p = Param(self.ctx, self.w[f"{name}.weight"], self.dtype)
        self.params.append(p)
        return p

    def vec(self, name):
        return self.ctx.upload(self.w[name])


class GroupNorm:
    def __init__(self, ld: _Loader, name: str):
        self.gamma, self.beta = ld.vec(f"{name}.weight"), ld.vec(f"{name}.bias")

    def affine(self, x: DeviceTensor):
        return group_norm_affine(x, GROUPS, VAE_EPS, self.gamma, self.beta)


class Conv:
    def __init__(self, ld: _Loader, name: str):
        self.weight, self.bias = ld.param(name), ld.vec(f"{name}.bias")


class Resnet:
    """diffusers ResnetBlock2D without time embedding (src/vae/mod.rs:174-211):
    h = conv1(SiLU(GN1(x))); h = conv2(SiLU(GN2(h))); h + (conv_shortcut(x) | x).
    Both GroupNorms are fused into the convs' A-operand gather; the residual (or
    the shortcut output) is fused into the last conv's epilogue."""

    def __init__(self, ld: _Loader, name: str, c_in: int, c_out: int):
        self.norm1, self.conv1 = GroupNorm(ld, f"{name}.norm1"), Conv(ld, f"{name}.conv1")
        self.norm2, self.conv2 = GroupNorm(ld, f"{name}.norm2"), Conv(ld, f"{name}.conv2")
        self.shortcut = Conv(ld, f"{name}.conv_shortcut") if c_in != c_out else None

    def forward(self, x: DeviceTensor) -> DeviceTensor:
        s1, t1 = self.norm1.affine(x)
        h = conv3x3(x, self.conv1.weight, self.conv1.bias, prologue=(s1, t1, True))
        s2, t2 = self.norm2.affine(h)
        if self.shortcut is None:
            return conv3x3(h, self.conv2.weight, self.conv2.bias, prologue=(s2, t2, True), residual=x)
        o = conv3x3(h, self.conv2.weight, self.conv2.bias, prologue=(s2, t2, True))
        return conv1x1(x, self.shortcut.weight, self.shortcut.bias, residual=o)


class MidAttention:
    """Single-head self-attention over all pixels (src/vae/mod.rs:213-270):
    to_out(softmax(q·kᵀ/√c)·v) + x with q, k, v = 1×1 convs of GN(x)."""

    def __init__(self, ld: _Loader, name: str, c: int):
        self.c = c
        self.norm = GroupNorm(ld, f"{name}.group_norm")
        self.to_q, self.to_k = Conv(ld, f"{name}.to_q"), Conv(ld, f"{name}.to_k")
        self.to_v, self.to_out = Conv(ld, f"{name}.to_v"), Conv(ld, f"{name}.to_out.0")

    def forward(self, x: DeviceTensor) -> DeviceTensor:
        ctx = x.ctx
        n, h, w, c = x.shape
        hw = h * w
        t = group_norm(x, GROUPS, VAE_EPS, self.norm.gamma, self.norm.beta)
        q = conv1x1(t, self.to_q.weight, self.to_q.bias)
        k = conv1x1(t, self.to_k.weight, self.to_k.bias)
        v = conv1x1(t, self.to_v.weight, self.to_v.bias)
        o = t  # the GN output is dead: reuse its buffer for the attention output
        scores = ctx.empty((hw, hw))
        L = lib()
        for b in range(n):
            off = b * hw * c * 4
            check(L.mbx_gemm(ctx.handle, scores.vp, _at(q, off), hw, c, _at(k, off), hw, 0, None, None))
            check(L.mbx_softmax_rows(ctx.handle, scores.vp, hw, hw, 1.0 / np.sqrt(c), SOFTMAX_FLUSH))
            check(L.mbx_gemm(ctx.handle, _at(o, off), scores.vp, hw, hw, _at(v, off), c, 1, None, None))
        return conv1x1(o, self.to_out.weight, self.to_out.bias, residual=x)


def _at(t: DeviceTensor, byte_offset: int):
    import ctypes
    return ctypes.c_void_p(t.ptr + byte_offset)


class Decoder:
    """VAE decoder (src/vae/decoder.rs:32-99). `wdtype` is the conv weights'
    storage precision: 'f16' (the shipped VAE; 2×TF32 products) or 'f32' (3×TF32)."""

    def __init__(self, ctx: Context, weights: dict, wdtype: str = "f16"):
        ld = _Loader(ctx, weights, wdtype)
        self._loader = ld
        ch = VAE_BLOCK_OUT
        top = ch[-1]
        self.post_quant_conv = Conv(ld, "post_quant_conv")
        self.conv_in = Conv(ld, "decoder.conv_in")
        self.mid = (Resnet(ld, "decoder.mid_block.resnets.0", top, top),
                    MidAttention(ld, "decoder.mid_block.attentions.0", top),
                    Resnet(ld, "decoder.mid_block.resnets.1", top, top))
        self.up = []
        c_prev = top
        for i, c in enumerate(reversed(ch)):
            resnets = [Resnet(ld, f"decoder.up_blocks.{i}.resnets.{j}", c_prev if j == 0 else c, c)
                       for j in range(UP_LAYERS)]
            ups = Conv(ld, f"decoder.up_blocks.{i}.upsamplers.0.conv") if i + 1 < len(ch) else None
            self.up.append((resnets, ups))
            c_prev = c
        self.norm_out = GroupNorm(ld, "decoder.conv_norm_out")
        self.conv_out = Conv(ld, "decoder.conv_out")

    def decode(self, latents: DeviceTensor) -> DeviceTensor:
        """latents: scaled [n, h, w, 4] → RGB (x + 1) / 2, unclamped, [n, 8h, 8w, 3]."""
        ctx = latents.ctx
        L = lib()
        z = ctx.empty(latents.shape)
        check(L.mbx_scale_add(ctx.handle, latents.vp, latents.size, 1.0 / SCALING_FACTOR, 0.0, z.vp))
        cur = conv1x1(z, self.post_quant_conv.weight, self.post_quant_conv.bias)
        cur = conv3x3(cur, self.conv_in.weight, self.conv_in.bias)
        r0, attn, r1 = self.mid
        cur = r1.forward(attn.forward(r0.forward(cur)))
        for resnets, ups in self.up:
            for r in resnets:
                cur = r.forward(cur)
            if ups is not None:
                cur = conv3x3(cur, ups.weight, ups.bias, upsample2x=True)
        s, t = self.norm_out.affine(cur)
        out = conv3x3(cur, self.conv_out.weight, self.conv_out.bias, prologue=(s, t, True))
        check(L.mbx_scale_add(ctx.handle, out.vp, out.size, 0.5, 0.5, out.vp))
        return out

    def close(self):
        for p in self._loader.params:
            p.close()
