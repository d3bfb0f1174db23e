"""GPU parity of the any-size imaging kernels and the DPM-Solver++(2M) step
(include/moebius_cuda.h) with the CPU oracle, all bit-exact: mask dilation and
bbox (src/imaging/mod.rs:38-89), window -> model Lanczos3 with edge replication
(src/imaging/resize.rs:27-57), model -> window (resize.rs:61-67), every paste
mode with its source rectangle, blur margin and compensation ring
(src/imaging/blend.rs:104-215), and Dpm2M::step (src/scheduler.rs:107-152).
Regions are passed with their image origin, as the engine passes them."""
import ctypes

import numpy as np
import pytest
from conftest import load_golden

pytestmark = pytest.mark.gpu

MODEL = 128  # model side of the scaled networks; any side works


def _ellipses(rng, h, w, k=3):
    yy, xx = np.mgrid[:h, :w]
    m = np.zeros((h, w), bool)
    for _ in range(k):
        cy, cx = rng.uniform(0, h), rng.uniform(0, w)
        ry, rx = rng.uniform(2, max(3, h / 4)), rng.uniform(2, max(3, w / 4))
        m |= ((yy - cy) / ry) ** 2 + ((xx - cx) / rx) ** 2 <= 1
    return (m * 255).astype(np.uint8)


@pytest.mark.parametrize("k", [0, 1, 2, 3, 7])
def test_mask_dilate_and_bbox(mbx, ctx, k):
    from oracle import imaging_ref
    rng = np.random.default_rng(k)
    n, h, w, stride = 3, 37, 53, 64
    masks = np.zeros((n, h, stride), np.uint8)
    masks[0, :, :w] = _ellipses(rng, h, w)
    masks[1, :, :w] = rng.integers(0, 256, (h, w), dtype=np.uint8) * (rng.random((h, w)) < 0.01)
    masks[2, :, w:] = 255  # beyond the row width: must be ignored
    md, out, scratch = ctx.upload(masks, np.uint8), ctx.empty((n, h, w), np.uint8), ctx.empty((n, h, w), np.uint8)
    mbx.check(mbx.abi.lib().mbx_mask_dilate(ctx.handle, md.vp, n, h, w, stride, k, scratch.vp, out.vp))
    got = out.numpy()
    for i in range(n):
        want = imaging_ref.dilate(masks[i, :, :w], k)
        assert np.array_equal(got[i], want), i
    box = ctx.empty((n, 4), np.int32)
    od = ctx.upload(got, np.uint8)
    mbx.check(mbx.abi.lib().mbx_mask_bbox(ctx.handle, od.vp, n, h, w, w, box.vp))
    b = box.numpy()
    for i in range(n):
        want = imaging_ref.bbox(got[i])
        if want is None:
            assert b[i, 2] == -1
        else:
            x, y, bw, bh = want
            assert tuple(b[i]) == (x, y, x + bw - 1, y + bh - 1)


# (image w, h, channels, bbox-generating seed) -> geometry through crop_plan.
WINDOW_CASES = [
    (300, 200, 3, 0),    # window = image long side, padded rows, downscale 300 -> 128
    (700, 500, 4, 1),    # window inside the image, RGBA
    (90, 60, 3, 2),      # smaller than the model: upscale with padding
    (128, 128, 3, 3),    # model size: a copy
    (1500, 400, 3, 4),   # wide image, large window
]


def _region(plan, w, h, margin=16):
    from oracle import imaging_ref
    sx, sy, sw, sh = imaging_ref.source_rect(plan, w, h)
    x0, y0 = max(sx - margin, 0), max(sy - margin, 0)
    x1, y1 = min(sx + sw + margin, w), min(sy + sh + margin, h)
    return x0, y0, x1 - x0, y1 - y0


@pytest.mark.parametrize("w,h,ch,seed", WINDOW_CASES)
def test_window_to_model_matches_oracle(mbx, ctx, w, h, ch, seed):
    from oracle import imaging_ref
    rng = np.random.default_rng(seed)
    img = rng.integers(0, 256, (h, w, ch), dtype=np.uint8)
    mask = _ellipses(rng, h, w, 2)
    box = imaging_ref.bbox(mask)
    plan = imaging_ref.crop_plan(box, w, h, MODEL)
    want_rgb, want_bin = imaging_ref.window_to_model(img, mask, plan, MODEL)
    rx, ry, rw, rh = _region(plan, w, h)
    stride = rw * ch + 12  # padded rows
    reg = np.zeros((rh, stride), np.uint8)
    reg[:, :rw * ch] = img[ry:ry + rh, rx:rx + rw].reshape(rh, rw * ch)
    mreg = np.ascontiguousarray(mask[ry:ry + rh, rx:rx + rw])
    rd, md = ctx.upload(reg, np.uint8), ctx.upload(mreg, np.uint8)
    rgb, binary = ctx.empty((MODEL, MODEL, 3), np.uint8), ctx.empty((MODEL, MODEL), np.uint8)
    mbx.check(mbx.abi.lib().mbx_window_to_model(ctx.handle, rd.vp, stride, ch, md.vp, rw, rx, ry, rw, rh, w, h,
                                                plan[0], plan[1], plan[2], MODEL, rgb.vp, binary.vp))
    assert np.array_equal(rgb.numpy(), want_rgb)
    assert np.array_equal(binary.numpy(), want_bin)


def test_window_to_model_rejects_a_region_that_misses_the_window(mbx, ctx):
    rd, md = ctx.empty((10, 30), np.uint8), ctx.empty((10, 10), np.uint8)
    out, b = ctx.empty((MODEL, MODEL, 3), np.uint8), ctx.empty((MODEL, MODEL), np.uint8)
    with pytest.raises(mbx.MbxError) as e:
        mbx.check(mbx.abi.lib().mbx_window_to_model(ctx.handle, rd.vp, 30, 3, md.vp, 10, 0, 0, 10, 10, 100, 100,
                                                    0, 0, 100, MODEL, out.vp, b.vp))
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("side", [45, 300, MODEL])
def test_model_to_window_matches_oracle(mbx, ctx, side):
    from oracle import imaging_ref
    rng = np.random.default_rng(side)
    n = 2
    dec = (rng.random((n, MODEL, MODEL, 3)) * 1.3 - 0.15).astype(np.float32)
    dec[0, 0, 0, 0] = np.nan
    dd, out = ctx.upload(dec), ctx.empty((n, side, side, 3), np.uint8)
    mbx.check(mbx.abi.lib().mbx_model_to_window(ctx.handle, dd.vp, n, MODEL, side, out.vp))
    got = out.numpy()
    for i in range(n):
        assert np.array_equal(got[i], imaging_ref.model_to_window(dec[i], side)), i


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("w,h,ch,seed", WINDOW_CASES)
def test_paste_matches_oracle(mbx, ctx, mode, w, h, ch, seed):
    from oracle import imaging_ref
    rng = np.random.default_rng(100 + seed)
    img = rng.integers(0, 256, (h, w, ch), dtype=np.uint8)
    mask = _ellipses(rng, h, w, 2)
    mask[rng.random((h, w)) < 0.02] = 128  # threshold edge: Feather >= 128, compensation > 128
    plan = imaging_ref.crop_plan(imaging_ref.bbox(mask), w, h, MODEL)
    result = rng.integers(0, 256, (plan[2], plan[2], 3), dtype=np.uint8)
    want, rect = imaging_ref.paste(img, mask, result, plan, mode)
    rx, ry, rw, rh = _region(plan, w, h)
    reg = np.ascontiguousarray(img[ry:ry + rh, rx:rx + rw])
    mstride = rw + 5
    mreg = np.zeros((rh, mstride), np.uint8)
    mreg[:, :rw] = mask[ry:ry + rh, rx:rx + rw]
    rd, md, resd = ctx.upload(reg, np.uint8), ctx.upload(mreg, np.uint8), ctx.upload(result, np.uint8)
    mbx.check(mbx.abi.lib().mbx_paste(ctx.handle, rd.vp, 1, rw * ch, ch, md.vp, mstride, rx, ry, rw, rh, w, h,
                                      plan[0], plan[1], plan[2], resd.vp, mode, None))
    got = img.copy()
    got[ry:ry + rh, rx:rx + rw] = rd.numpy()
    assert np.array_equal(got, want)
    sx, sy, sw, sh = rect
    outside = np.ones((h, w), bool)
    outside[sy:sy + sh, sx:sx + sw] = False
    assert np.array_equal(got[outside], img[outside]), "only the source rectangle is written"


def test_compensated_paste_fixture_through_the_library(mbx, ctx):
    g = load_golden("imaging_ref.safetensors")
    for k, (w, h) in (("a", (96, 80)), ("b", (48, 40)), ("c", (48, 40))):
        t = lambda name: np.ascontiguousarray(g[f"comp.{k}.{name}"].astype(np.uint8))
        side = max(w, h)
        padded = np.zeros((side, side, 3), np.uint8)
        padded[:h, :w] = t("result")
        rd, md, resd = ctx.upload(t("image"), np.uint8), ctx.upload(t("mask"), np.uint8), ctx.upload(padded, np.uint8)
        mbx.check(mbx.abi.lib().mbx_paste(ctx.handle, rd.vp, 1, w * 3, 3, md.vp, w, 0, 0, w, h, w, h, 0, 0, side,
                                          resd.vp, 3, None))
        assert np.array_equal(rd.numpy(), t("out")), k


def test_batched_paste_skips_inactive_items(mbx, ctx):
    from oracle import imaging_ref
    rng = np.random.default_rng(77)
    n, s = 3, 64
    img = rng.integers(0, 256, (n, s, s, 4), dtype=np.uint8)
    masks = np.stack([_ellipses(rng, s, s) for _ in range(n)])
    res = rng.integers(0, 256, (n, s, s, 3), dtype=np.uint8)
    active = np.array([1, 0, 1], np.int32)
    for mode in (1, 2, 3):
        imd, md, rd, ad = (ctx.upload(img, np.uint8), ctx.upload(masks, np.uint8), ctx.upload(res, np.uint8),
                           ctx.upload(active, np.int32))
        mbx.check(mbx.abi.lib().mbx_paste(ctx.handle, imd.vp, n, s * 4, 4, md.vp, s, 0, 0, s, s, s, s, 0, 0, s,
                                          rd.vp, mode, ad.vp))
        got = imd.numpy()
        for i in range(n):
            want = imaging_ref.paste(img[i], masks[i], res[i], (0, 0, s), mode)[0] if active[i] else img[i]
            assert np.array_equal(got[i], want), (mode, i)
        assert np.array_equal(got[..., 3], img[..., 3]), "alpha is preserved"


@pytest.mark.parametrize("copies", [1, 2])
def test_cfg_dpm_step_is_exact(mbx, ctx, copies):
    from oracle.scheduler_ref import Ddim, Dpm2M
    rng = np.random.default_rng(copies)
    n, hw = 3, 40
    d = Ddim(6, 0.99, trailing=True)
    g = np.float32(2.5)
    x = rng.standard_normal((n, hw, 4)).astype(np.float32)
    xd, prev = ctx.upload(x), ctx.empty((n, hw, 4))
    solver = [Dpm2M() for _ in range(n)]
    want = x.copy()
    for i in range(len(d.timesteps)):
        eps = rng.standard_normal((n * copies, hw, 4)).astype(np.float32)
        coef = (ctypes.c_float * 5)()
        order = ctypes.c_int32()
        mbx.check(mbx.abi.lib().mbx_dpm_coefficients(6, 0.99, 1, i, 2, coef, ctypes.byref(order)))
        ed = ctx.upload(eps)
        mbx.check(mbx.abi.lib().mbx_cfg_dpm_step(ctx.handle, ed.vp, n, hw, copies, g, coef, order.value, xd.vp,
                                                 prev.vp))
        for j in range(n):
            e = (eps[2 * j] + g * (eps[2 * j + 1] - eps[2 * j])).astype(np.float32) if copies == 2 else eps[j]
            if i == 2:
                solver[j].restart()
            want[j] = solver[j].step(d, e, i, want[j])
        assert np.array_equal(xd.numpy(), want), i
