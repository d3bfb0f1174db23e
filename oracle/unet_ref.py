"""TEST INFRASTRUCTURE ONLY: the Moebius student UNet composed from the oracle
kernels, following the reference op by op (src/unet/mod.rs:200-301,
blocks.rs:46-112, transformer.rs:319-357, lambda.rs:107-294, embed.rs:20-90).
Weights are a dict of numpy arrays in the converter's layout (f16 GEMM
weights are widened to f32, as Param::view does). Shape-driven: the level
widths and the latent side come from the weights.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

GROUPS = 32
RESNET_EPS = 1e-5
TRANSFORMER_GN_EPS = 1e-6
LAYER_NORM_EPS = 1e-5
HEADS = 8
TOKENS = 10
D = "diff_model"


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _conv1(w, name, x, residual=None, bias=True):
    return O.conv1x1(x, _f32(w[f"{name}.weight"]), w[f"{name}.bias"] if bias else None, residual)


def widths(w):
    return tuple(int(w[f"{D}.down_blocks.{i}.resnets.0.conv1.conv_pw.weight"].shape[0]) for i in range(3))


def latent_side(w):
    hw = w[f"{D}.down_blocks.0.attentions.0.transformer_blocks.0.attn2.rel_pos_emb"].shape[0]
    return int(round(np.sqrt(hw)))


def dwconv(w, name, x):
    """DwConv2d::forward, src/unet/blocks.rs:46-53."""
    mid = O.depthwise3x3(x, w[f"{name}.conv_dw.weight"], w[f"{name}.conv_dw.bias"], "relu")
    c_out = w[f"{name}.conv_pw.weight"].shape[0]
    return _conv1(w, f"{name}.conv_pw", mid, residual=x if x.shape[-1] == c_out else None)


def dwresnet(w, name, x, temb):
    """DwResnet::forward, src/unet/blocks.rs:84-112; temb [n, 1280] raw."""
    n = x.shape[0]
    a = O.group_norm(x, GROUPS, RESNET_EPS, w[f"{name}.norm1.weight"], w[f"{name}.norm1.bias"], silu=True)
    b = dwconv(w, f"{name}.conv1", a)
    t = O.silu(temb)
    tp = _conv1(w, f"{name}.time_emb_proj", t.reshape(n, 1, 1, -1)).reshape(n, -1)
    a = O.group_norm(b, GROUPS, RESNET_EPS, w[f"{name}.norm2.weight"], w[f"{name}.norm2.bias"], add=tp, silu=True)
    out = dwconv(w, f"{name}.conv2", a)
    if f"{name}.conv_shortcut.weight" in w:
        return O.add(out, _conv1(w, f"{name}.conv_shortcut", x))
    return O.add(out, x)


def self_lambda(w, name, x):
    """SelfLambda::forward, src/unet/lambda.rs:107-151 (bands of rows do not change the values)."""
    n, hh, ww, c = x.shape
    k = c // HEADS
    hw = hh * ww
    q = _conv1(w, f"{name}.to_q", x)
    kt = _conv1(w, f"{name}.to_k", x, bias=False)
    vt = _conv1(w, f"{name}.to_v", x)
    w_aug = np.concatenate([_f32(w[f"{name}.pos_conv.weight"]), _f32(w[f"{name}.pos_conv.bias"])[:, None]], axis=1)
    w_aug_t = np.ascontiguousarray(w_aug.T)  # [226, k]
    out = np.empty_like(q)
    for b in range(n):
        lam = O.softmax_lambda(kt[b].reshape(hw, k), vt[b].reshape(hw, k))
        qi = np.ascontiguousarray(q[b].reshape(hw * HEADS, k))
        o = O.gemm_nt(qi, np.ascontiguousarray(lam.T))
        a = O.gemm_nt(qi, w_aug_t)
        O.tap_filter(a, vt[b].reshape(hw, k), o, hh, ww)
        out[b] = o.reshape(hh, ww, c)
    return out


def cross_constants(w, name, ehs):
    """CrossLambda::load, src/unet/lambda.rs:203-249: per branch (λc [k, k], V [10, k])."""
    wk, wv = _f32(w[f"{name}.to_k.weight"]), _f32(w[f"{name}.to_v.weight"])
    bv = _f32(w[f"{name}.to_v.bias"])
    consts = []
    for br in range(2):
        keys = O.gemm_nt(ehs[br], wk)
        v = (O.gemm_nt(ehs[br], wv) + bv[None, :]).astype(np.float32)
        consts.append((O.softmax_lambda(keys, v), v))
    return consts


def cross_lambda(w, name, x, branches, consts):
    """CrossLambda::forward, src/unet/lambda.rs:252-273."""
    n, hh, ww, c = x.shape
    k = c // HEADS
    hw = hh * ww
    q = _conv1(w, f"{name}.to_q", x)
    e = _f32(w[f"{name}.rel_pos_emb"])
    assert e.shape[0] == hw, "CrossLambda input size does not match the position table"
    out = np.empty_like(q)
    for b, br in enumerate(branches):
        lam, v = consts[br]
        qi = np.ascontiguousarray(q[b].reshape(hw * HEADS, k))
        o = O.gemm_nt(qi, np.ascontiguousarray(lam.T))
        O.position_term(q[b].reshape(hw, c), e, v, o)
        out[b] = o.reshape(hh, ww, c)
    return out


def mix_transformer(w, name, x, branches, ehs):
    """MixTransformer::forward, src/unet/transformer.rs:319-357."""
    b = f"{name}.transformer_blocks.0"
    t = O.group_norm(x, GROUPS, TRANSFORMER_GN_EPS, w[f"{name}.norm.weight"], w[f"{name}.norm.bias"])
    h = _conv1(w, f"{name}.proj_in", t)
    t = O.layer_norm(h, w[f"{b}.norm1.weight"], w[f"{b}.norm1.bias"], LAYER_NORM_EPS)
    h = O.add(h, self_lambda(w, f"{b}.attn1", t))
    t = O.layer_norm(h, w[f"{b}.norm2.weight"], w[f"{b}.norm2.bias"], LAYER_NORM_EPS)
    h = O.add(h, cross_lambda(w, f"{b}.attn2", t, branches, cross_constants(w, f"{b}.attn2", ehs)))
    t = O.layer_norm(h, w[f"{b}.norm3.weight"], w[f"{b}.norm3.bias"], LAYER_NORM_EPS)
    a = O.silu(_conv1(w, f"{b}.ff.inverted_conv.conv", t))
    g = O.depthwise3x3(a, w[f"{b}.ff.depth_conv.conv.weight"], w[f"{b}.ff.depth_conv.conv.bias"], "glu_silu")
    u = _conv1(w, f"{b}.ff.point_conv.conv", g, residual=h, bias=False)
    return _conv1(w, f"{name}.proj_out", u, residual=x)


def conditioning(w):
    """embed::conditioning, src/unet/embed.rs:79-90: [uncond, cond] hidden states [2, 10, 768]."""
    table = _f32(w["embedding_layer.weight"])
    rows = np.concatenate([table[TOKENS:], table[:TOKENS]])[None, None]
    return _conv1(w, f"{D}.encoder_hid_proj", rows).reshape(2, TOKENS, -1)


def time_embedding(w, t, n):
    """TimeEmbedding::forward, src/unet/embed.rs:32-60: raw [n, 4·ch0]."""
    dim = w[f"{D}.time_embedding.linear_1.weight"].shape[1]
    sin = O.timestep_sinusoid(t, dim)[None, None, None]
    a = O.silu(_conv1(w, f"{D}.time_embedding.linear_1", sin))
    b = _conv1(w, f"{D}.time_embedding.linear_2", a).reshape(-1)
    return np.tile(b, (n, 1))


def forward(w, x, t, branches, ehs=None):
    """UNet::forward with the batch already tiled: x [len(branches), L, L, 9] -> ε [.., 4]."""
    ehs = conditioning(w) if ehs is None else ehs
    n = x.shape[0]
    temb = time_embedding(w, t, n)
    h = dwconv(w, f"{D}.conv_in", _f32(x))
    skips = [h]
    for i in range(3):
        for j in range(2):
            a = dwresnet(w, f"{D}.down_blocks.{i}.resnets.{j}", skips[-1], temb)
            skips.append(mix_transformer(w, f"{D}.down_blocks.{i}.attentions.{j}", a, branches, ehs))
        if i < 2:
            skips.append(O.conv3x3(skips[-1], _f32(w[f"{D}.down_blocks.{i}.downsamplers.0.conv.weight"]),
                                   w[f"{D}.down_blocks.{i}.downsamplers.0.conv.bias"], stride=2))
    h = skips[-1].copy()
    for i in range(3):
        for j in range(3):
            skip = skips.pop()
            cat = O.concat_channels(h, skip)
            a = dwresnet(w, f"{D}.up_blocks.{i}.resnets.{j}", cat, temb)
            h = mix_transformer(w, f"{D}.up_blocks.{i}.attentions.{j}", a, branches, ehs)
        if i < 2:
            h = O.conv3x3(h, _f32(w[f"{D}.up_blocks.{i}.upsamplers.0.conv.weight"]),
                          w[f"{D}.up_blocks.{i}.upsamplers.0.conv.bias"], upsample2x=True)
    assert not skips
    a = O.group_norm(h, GROUPS, RESNET_EPS, w[f"{D}.conv_norm_out.weight"], w[f"{D}.conv_norm_out.bias"], silu=True)
    return dwconv(w, f"{D}.conv_out", a)
