"""TEST INFRASTRUCTURE ONLY: numpy restatement of the reference's imaging
steps: to_model (src/imaging/resize.rs:27-57), to_u8 (src/imaging/blend.rs:20-24),
Pillow's GaussianBlur (blend.rs:26-100), the feathered paste of a model-size
window (blend.rs:153-215, Paste::Feather), and for other image sizes the mask
dilation and bbox (src/imaging/mod.rs:38-89), the square crop window
(src/imaging/crop.rs:30-62), Lanczos3 resampling in Pillow's formulation
(resize.rs:16-67) and every paste mode with its source rectangle and
mean-colour compensation (blend.rs:104-215).
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


# ------------------------------------------------------------------ crop window and resampling

def dilate(mask_u8, k: int):
    """Binarised (>= 128 -> 255) mask dilated by a k x k square with anchor k // 2, out-of-range
    pixels ignored (src/imaging/mod.rs:61-89, cv2.dilate semantics)."""
    cur = np.where(np.asarray(mask_u8) >= 128, 255, 0).astype(np.uint8)
    if k <= 1:
        return cur
    h, w = cur.shape
    before, after = k // 2, k - 1 - k // 2
    tmp = np.zeros_like(cur)
    for x in range(w):
        tmp[:, x] = cur[:, max(0, x - before):min(w - 1, x + after) + 1].max(axis=1)
    out = np.zeros_like(cur)
    for y in range(h):
        out[y] = tmp[max(0, y - before):min(h - 1, y + after) + 1].max(axis=0)
    return out


def bbox(mask_u8):
    """(x, y, w, h) of the pixels >= 128, None when there are none (src/imaging/mod.rs:38-53)."""
    ys, xs = np.nonzero(np.asarray(mask_u8) >= 128)
    if ys.size == 0:
        return None
    return int(xs.min()), int(ys.min()), int(xs.max() - xs.min() + 1), int(ys.max() - ys.min() + 1)


def _place(start, length, side, extent):
    """Window start on one axis (src/imaging/crop.rs:55-62): centred on the mask and shifted
    inside the image when it fits, else centred on the image."""
    if side <= extent:
        centred = (2 * start + length) // 2 - side // 2
        return min(max(centred, 0), extent - side)
    return -((side - extent) // 2)


def crop_plan(box, width, height, model_side=512):
    """Square window (x, y, side) around the mask bbox (src/imaging/crop.rs:30-41)."""
    bx, by, bw, bh = box
    long = max(bw, bh)
    img_long = max(width, height)
    side = min(max(long + 2 * (long // 2), min(model_side, img_long)), img_long)
    return _place(bx, bw, side, width), _place(by, bh, side, height), side


def source_rect(plan, width, height):
    """The part of the window inside the image, (x, y, w, h) (src/imaging/crop.rs:44-51)."""
    x, y, side = plan
    x0, y0 = max(x, 0), max(y, 0)
    x1, y1 = min(x + side, width), min(y + side, height)
    return x0, y0, x1 - x0, y1 - y0


LANCZOS_BITS = 22  # Pillow's PRECISION_BITS for 8-bit images


def _lanczos(x: float) -> float:
    def sinc(v):
        if v == 0.0:
            return 1.0
        v = v * np.pi
        return float(np.sin(v)) / v
    return sinc(x) * sinc(x / 3.0) if -3.0 <= x < 3.0 else 0.0


def lanczos_table(in_size: int, out_size: int):
    """Pillow's Lanczos3 convolution coefficients for in_size -> out_size samples (its
    precompute_coeffs / normalize_coeffs_8bpc, the formulation fast_image_resize follows):
    bounds [out, 2] = (first input, count), coefficients [out, ksize] in 22-bit fixed point."""
    scale = in_size / out_size
    fscale = max(scale, 1.0)
    support = 3.0 * fscale
    ksize = int(np.ceil(support)) * 2 + 1
    ss = 1.0 / fscale
    bounds = np.zeros((out_size, 2), np.int64)
    kk = np.zeros((out_size, ksize), np.int64)
    for xx in range(out_size):
        center = (xx + 0.5) * scale
        xmin = max(int(center - support + 0.5), 0)
        xmax = min(int(center + support + 0.5), in_size) - xmin
        ws = [_lanczos((x + xmin - center + 0.5) * ss) for x in range(xmax)]
        ww = 0.0
        for v in ws:
            ww += v
        for x, v in enumerate(ws):
            if ww != 0.0:
                v = v / ww
            kk[xx, x] = int(-0.5 + v * (1 << LANCZOS_BITS)) if v < 0 else int(0.5 + v * (1 << LANCZOS_BITS))
        bounds[xx] = (xmin, xmax)
    return bounds, kk


def _resample_rows(img, out_size):
    """One Lanczos pass along axis 1 of [h, w, c] u8: rounding bias, 22-bit fixed point, clip to 8 bit."""
    bounds, kk = lanczos_table(img.shape[1], out_size)
    src = img.astype(np.int64)
    out = np.empty((img.shape[0], out_size, img.shape[2]), np.uint8)
    for xx in range(out_size):
        first, count = bounds[xx]
        acc = (1 << (LANCZOS_BITS - 1)) + np.tensordot(src[:, first:first + count, :], kk[xx, :count], axes=([1], [0]))
        out[:, xx, :] = np.clip(acc >> LANCZOS_BITS, 0, 255)
    return out


def resize_u8(img, out_size):
    """Lanczos3 resize of a square [s, s, c] (or [s, s]) u8 image to out_size², horizontal pass
    first; a same-size request is a copy (src/imaging/resize.rs:16-25)."""
    a = np.asarray(img, np.uint8)
    flat = a.ndim == 2
    if flat:
        a = a[..., None]
    if a.shape[0] != out_size:
        a = _resample_rows(a, out_size)
        a = np.ascontiguousarray(_resample_rows(np.ascontiguousarray(a.transpose(1, 0, 2)), out_size).transpose(1, 0, 2))
    return a[..., 0].copy() if flat else a.copy()


def window_to_model(img_u8, mask_u8, plan, model_side=512):
    """Square window -> model-size 8-bit RGB and binary mask (src/imaging/resize.rs:27-57): the
    window is read with edge replication past the image, the mask with zeros; both are Lanczos3
    resized and the mask is re-thresholded at 128. Returns (rgb u8 [S, S, 3], bin u8 [S, S])."""
    x, y, side = plan
    h, w = mask_u8.shape
    ys = np.arange(y, y + side)
    xs = np.arange(x, x + side)
    yc, xc = np.clip(ys, 0, h - 1), np.clip(xs, 0, w - 1)
    rgb = img_u8[yc][:, xc, :3]
    inside = ((ys >= 0) & (ys < h))[:, None] & ((xs >= 0) & (xs < w))[None, :]
    binary = np.where(inside & (mask_u8[yc][:, xc] >= 128), 255, 0).astype(np.uint8)
    rgb = resize_u8(rgb, model_side)
    binary = resize_u8(binary, model_side)
    return rgb, np.where(binary >= 128, 255, 0).astype(np.uint8)


def model_to_window(decoded, side):
    """Model output in [0, 1] [S, S, 3] -> 8-bit window side² (to_u8, then Lanczos3; resize.rs:61-67)."""
    return resize_u8(to_u8(decoded), side)


PASTE_NONE, PASTE_FEATHER, PASTE_FEATHER_COMPENSATE = 1, 2, 3
BLUR_MARGIN = 16
COMPENSATE_FAC = 1.1
RING_OFF = 10


def _ring_delta(setm, src, res):
    """Per-channel mean(src) − mean(res) over the ring around the mask bbox (blend.rs:116-151);
    None when the mask or the ring is empty."""
    h, w = setm.shape
    ys, xs = np.nonzero(setm)
    if ys.size == 0:
        return None
    r0, r1, c0, c1 = ys.min(), ys.max(), xs.min(), xs.max()
    hh, hw = (r1 - r0 + 1 + RING_OFF) // 2, (c1 - c0 + 1 + RING_OFF) // 2
    cr, cc = (r0 + r1) // 2, (c0 + c1) // 2
    y0, y1 = max(cr - hh, 0), min(cr + hh, h - 1)
    x0, x1 = max(cc - hw, 0), min(cc + hw, w - 1)
    ring = ~setm[y0:y1 + 1, x0:x1 + 1]
    n = int(ring.sum())
    if n == 0:
        return None
    s_src = src[y0:y1 + 1, x0:x1 + 1, :3][ring].astype(np.uint64).sum(axis=0)
    s_res = res[y0:y1 + 1, x0:x1 + 1, :3][ring].astype(np.uint64).sum(axis=0)
    return [float(s_src[c]) / n - float(s_res[c]) / n for c in range(3)]


def paste(img_u8, mask_u8, result_u8, plan, mode=PASTE_FEATHER):
    """Writes the window-size result back into (a copy of) the image (src/imaging/blend.rs:153-215).
    Returns (image, (x, y, w, h) written)."""
    h, w = mask_u8.shape
    out = img_u8.copy()
    sx, sy, sw, sh = source_rect(plan, w, h)
    if sw == 0 or sh == 0:
        return out, (0, 0, 0, 0)
    ox, oy = sx - plan[0], sy - plan[1]
    res = result_u8[oy:oy + sh, ox:ox + sw]
    if mode == PASTE_NONE:
        out[sy:sy + sh, sx:sx + sw, :3] = res
        return out, (sx, sy, sw, sh)
    comp = mode == PASTE_FEATHER_COMPENSATE
    lo = 129 if comp else 128
    rx0, ry0 = max(sx - BLUR_MARGIN, 0), max(sy - BLUR_MARGIN, 0)
    rx1, ry1 = min(sx + sw + BLUR_MARGIN, w), min(sy + sh + BLUR_MARGIN, h)
    region = np.where(mask_u8[ry0:ry1, rx0:rx1] >= lo, 255, 0).astype(np.uint8)
    blurred = pil_gaussian_blur(region, 3.0)
    src = img_u8[sy:sy + sh, sx:sx + sw, :3]
    shift = None
    if comp:
        setm = region[sy - ry0:sy - ry0 + sh, sx - rx0:sx - rx0 + sw] != 0
        d = _ring_delta(setm, src, res)
        if d is not None:
            shift = np.array([COMPENSATE_FAC * v / 255.0 for v in d], np.float64)
    m = blurred[sy - ry0:sy - ry0 + sh, sx - rx0:sx - rx0 + sw].astype(np.float64)[..., None] / 255.0
    r = res.astype(np.float64) / 255.0
    if shift is not None:
        r = r + shift
    o = r * m + (1.0 - m) * (src.astype(np.float64) / 255.0)
    if shift is not None:
        o = np.clip(o, 0.0, 1.0)
    out[sy:sy + sh, sx:sx + sw, :3] = np.clip(np.nan_to_num(o * 255.0, nan=0.0), 0, 255).astype(np.uint8)
    return out, (sx, sy, sw, sh)
