"""TEST INFRASTRUCTURE ONLY: numpy restatement of the reference's imaging
steps for model-size (used-whole) windows: to_model (src/imaging/resize.rs:27-57),
to_u8 (src/imaging/blend.rs:20-24), Pillow's GaussianBlur (blend.rs:26-100)
and the feathered paste (blend.rs:153-215, Paste::Feather).
"""
from __future__ import annotations

import numpy as np


def to_model(img_u8, mask_u8):
    """8-bit RGB(A) [h, w, ch] + mask [h, w] -> (rgb f32 in [-1, 1] [h, w, 3], binary mask u8 0/255)."""
    rgb = (img_u8[..., :3].astype(np.float64) / 255.0 * 2.0 - 1.0).astype(np.float32)
    binary = np.where(mask_u8 >= 128, 255, 0).astype(np.uint8)
    return rgb, binary


def to_u8(v):
    """(clamp(v, 0, 1) · 255) truncated, in f32 (NaN -> 0)."""
    v = np.nan_to_num(np.asarray(v, np.float32), nan=0.0)
    return (np.clip(v, np.float32(0), np.float32(1)) * np.float32(255)).astype(np.uint8)


def gaussian_box_radius(sigma: float, passes: int) -> np.float32:
    """Pillow's _gaussian_blur_radius in f32 with f64 sqrt / floor (blend.rs:26-39)."""
    f = np.float32
    sigma2 = f(sigma) * f(sigma) / f(passes)
    big_l = f(np.sqrt(12.0 * np.float64(sigma2) + 1.0))
    l = f(np.floor((np.float64(big_l) - 1.0) / 2.0))
    a = (f(2) * l + f(1)) * (l * (l + f(1)) - f(3) * sigma2)
    a = a / (f(6) * (sigma2 - (l + f(1)) * (l + f(1))))
    return f(l + a)


def _box_rows(buf, fr, passes):
    """`passes` fractional box passes over every row (blend.rs:41-77), vectorised over rows."""
    radius = int(fr)
    ww = np.uint64(int(np.float32(1 << 24) / (fr * np.float32(2) + np.float32(1))))
    fw = np.uint64(((1 << 24) - (radius * 2 + 1) * int(ww)) // 2)
    n = buf.shape[1]
    out = buf
    for _ in range(passes):
        pad = np.pad(out.astype(np.uint64), ((0, 0), (radius + 1, radius + 1)), mode="edge")
        cs = np.concatenate([np.zeros((pad.shape[0], 1), np.uint64), np.cumsum(pad, axis=1, dtype=np.uint64)], axis=1)
        x = np.arange(n)
        acc = cs[:, x + 2 * radius + 2] - cs[:, x + 1]          # Σ at(x−r .. x+r)
        far = pad[:, x] + pad[:, x + 2 * radius + 2]             # at(x−r−1) + at(x+r+1)
        out = ((acc * ww + far * fw + np.uint64(1 << 23)) >> np.uint64(24)).astype(np.uint8)
    return out


def pil_gaussian_blur(mask_u8, radius: float = 3.0):
    """PIL GaussianBlur(radius) of a single-channel 8-bit image [h, w]: 3 passes per axis, rows first."""
    m = np.asarray(mask_u8, np.uint8)
    if radius <= 0 or m.size == 0:
        return m.copy()
    fr = gaussian_box_radius(radius, 3)
    t = _box_rows(m, fr, 3)
    return np.ascontiguousarray(_box_rows(np.ascontiguousarray(t.T), fr, 3).T)


def feather_paste(img_u8, mask_u8, result_u8):
    """Paste::Feather over the whole image (a model-size window is the source rectangle):
    out = res·m + (1 − m)·src in f64 with m = blur(mask ≥ 128)/255, truncated."""
    binary = np.where(mask_u8 >= 128, 255, 0).astype(np.uint8)
    m = pil_gaussian_blur(binary, 3.0).astype(np.float64)[..., None] / 255.0
    out = img_u8.copy()
    res = result_u8.astype(np.float64) / 255.0
    orig = img_u8[..., :3].astype(np.float64) / 255.0
    blended = (res * m + (1.0 - m) * orig) * 255.0
    out[..., :3] = np.clip(blended, 0, 255).astype(np.uint8)
    return out
