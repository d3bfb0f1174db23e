"""CPU tests of the any-size imaging path and the Fast preset's scheduler: the
oracle restatements against the reference's fixtures and known answers, and the
library's host-side functions (crop window, Lanczos3 coefficient tables, DPM
coefficients) against the oracle. No GPU call is made.

Pins:
  * Lanczos3: byte-exact with Pillow's Image.LANCZOS (fixtures lz* written by
    tests/golden/make_golden.py; upstream resizes the crop window with it, and the
    reference's fast_image_resize follows the same convolution formulation);
  * compensated paste: the reference's upstream fixture (comp.*), byte-exact;
  * crop window: the reference's own cases (src/imaging/crop.rs:66-133);
  * dilation: cv2 anchor semantics (src/imaging/mod.rs:96-129);
  * DPM-Solver++(2M): the reference's diffusers values (src/scheduler.rs:203-237).
"""
import ctypes
import os

import numpy as np
import pytest
from safetensors.numpy import load_file

from conftest import load_package

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def golden():
    return load_file(os.path.join(HERE, "golden", "imaging_ref.safetensors"))


def test_lanczos_oracle_is_byte_exact_with_pillow(golden):
    from oracle import imaging_ref
    for k in ("lz1", "lz2", "lz3", "lz4"):
        src, want = golden[f"{k}.src"], golden[f"{k}.dst"]
        got = imaging_ref.resize_u8(src, want.shape[0])
        bad = int((got != want).sum())
        assert bad == 0, f"{k}: {bad} bytes differ from Pillow"


def test_lanczos_same_size_is_a_copy():
    from oracle import imaging_ref
    a = np.random.default_rng(1).integers(0, 256, (40, 40, 3), dtype=np.uint8)
    assert np.array_equal(imaging_ref.resize_u8(a, 40), a)


def test_lanczos_flat_colour_stays_flat():
    # src/imaging/resize.rs:121-146: a flat colour survives the resize (within 2/255 there;
    # exactly here, the coefficients sum to 2^22).
    from oracle import imaging_ref
    a = np.empty((100, 100, 3), np.uint8)
    a[...] = (40, 120, 200)
    for d in (512, 37):
        out = imaging_ref.resize_u8(a, d)
        assert np.all(np.abs(out.astype(int) - np.array([40, 120, 200])) <= 2)


@pytest.mark.parametrize("src,dst", [(300, 128), (96, 128), (77, 64), (128, 45), (4096, 512), (512, 3000), (513, 512),
                                     (1, 512)])
def test_library_lanczos_table_matches_oracle(src, dst):
    from oracle import imaging_ref
    mbx = load_package()
    k = ctypes.c_int64()
    mbx.check(mbx.lib().mbx_lanczos_table(src, dst, None, None, ctypes.byref(k)))
    bounds = np.zeros((dst, 2), np.int32)
    coeffs = np.zeros((dst, k.value), np.int32)
    mbx.check(mbx.lib().mbx_lanczos_table(src, dst, bounds.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                          coeffs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(k)))
    wb, wk = imaging_ref.lanczos_table(src, dst)
    assert np.array_equal(bounds, wb)
    assert np.array_equal(coeffs, wk)


def _lib_crop(mbx, box, w, h, model=512):
    win = (ctypes.c_int64 * 3)()
    rect = mbx.abi.Rect()
    mbx.check(mbx.lib().mbx_crop_window(*box, w, h, model, win, ctypes.byref(rect)))
    return (win[0], win[1], win[2]), (rect.x, rect.y, rect.width, rect.height)


# (bbox, image w, image h) -> window (x, y, side), from src/imaging/crop.rs:66-121.
CROP_CASES = [
    ((100, 100, 40, 40), 2000, 2000, (0, 0, 512)),
    ((900, 900, 40, 40), 2000, 2000, (664, 664, 512)),
    ((0, 0, 512, 512), 512, 512, (0, 0, 512)),
    ((100, 100, 300, 300), 512, 512, (0, 0, 512)),
    ((5, 5, 2, 2), 512, 512, (0, 0, 512)),
    ((100, 100, 600, 600), 800, 800, (0, 0, 800)),
    ((200, 50, 500, 300), 1000, 400, (0, -300, 1000)),
    ((500, 500, 600, 400), 2000, 1500, (200, 100, 1200)),
    ((1900, 10, 80, 80), 2000, 2000, (1488, 0, 512)),
    ((100, 50, 100, 100), 300, 200, (0, -50, 300)),
]


@pytest.mark.parametrize("box,w,h,want", CROP_CASES)
def test_crop_window_reference_cases(box, w, h, want):
    from oracle import imaging_ref
    assert imaging_ref.crop_plan(box, w, h) == want
    mbx = load_package()
    win, rect = _lib_crop(mbx, box, w, h)
    assert win == want
    assert rect == imaging_ref.source_rect(want, w, h)


def test_crop_window_always_contains_the_mask():
    # The property of src/imaging/crop.rs:123-133, library and oracle on the same draws.
    from oracle import imaging_ref
    mbx = load_package()
    rng = np.random.default_rng(9)
    for _ in range(3000):
        iw, ih = (int(v) for v in 1 + rng.integers(0, 3000, 2))
        x, y = int(rng.integers(0, iw)), int(rng.integers(0, ih))
        box = (x, y, 1 + int(rng.integers(0, iw - x)), 1 + int(rng.integers(0, ih - y)))
        win, rect = _lib_crop(mbx, box, iw, ih)
        assert win == imaging_ref.crop_plan(box, iw, ih)
        px, py, side = win
        assert px <= box[0] and py <= box[1]
        assert px + side >= box[0] + box[2] and py + side >= box[1] + box[3]
        assert rect[0] + rect[2] <= iw and rect[1] + rect[3] <= ih


def test_crop_window_rejects_a_bbox_outside_the_image():
    mbx = load_package()
    with pytest.raises(mbx.MbxError) as e:
        _lib_crop(mbx, (90, 0, 20, 5), 100, 100)
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT


def test_window_to_model_replicates_edges_and_zero_pads_the_mask():
    # src/imaging/resize.rs:121-146: 100x60 image, window of side 100 padded by 20 rows.
    from oracle import imaging_ref
    img = np.empty((60, 100, 3), np.uint8)
    img[...] = (40, 120, 200)
    mask = np.full((60, 100), 255, np.uint8)
    rgb, binary = imaging_ref.window_to_model(img, mask, (0, -20, 100), 512)
    assert np.all(np.abs(rgb.astype(int) - np.array([40, 120, 200])) <= 2)
    assert binary[2, 256] == 0 and binary[256, 256] == 255 and binary[509, 256] == 0
    back = imaging_ref.model_to_window(np.full((512, 512, 3), 0.5, np.float32), 100)
    assert back.shape == (100, 100, 3) and np.all(back == 127)
    same = imaging_ref.model_to_window(np.full((512, 512, 3), 0.999, np.float32), 512)
    assert np.all(same == 254)


def _paste_at_origin(image, result, mask, mode):
    from oracle import imaging_ref
    h, w = mask.shape
    side = max(w, h)
    padded = np.zeros((side, side, 3), np.uint8)
    padded[:h, :w] = result
    return imaging_ref.paste(image, mask, padded, (0, 0, side), mode)[0]


def test_compensated_paste_is_byte_exact_with_upstream(golden):
    from oracle import imaging_ref
    for k in ("a", "b", "c"):
        g = lambda name: golden[f"comp.{k}.{name}"].astype(np.uint8)
        got = _paste_at_origin(g("image"), g("result"), g("mask"), imaging_ref.PASTE_FEATHER_COMPENSATE)
        assert int((got != g("out")).sum()) == 0, k
        plain = _paste_at_origin(g("image"), g("result"), g("mask"), imaging_ref.PASTE_FEATHER)
        assert not np.array_equal(plain, got)


def test_compensation_falls_back_to_feather_without_a_ring_or_a_mask():
    # src/imaging/blend.rs:302-326.
    from oracle import imaging_ref
    w, h = 24, 20
    image = (np.arange(w * h * 3) * 7 % 251).astype(np.uint8).reshape(h, w, 3)
    result = (np.arange(w * h * 3) * 13 % 241).astype(np.uint8).reshape(h, w, 3)
    full = np.full((h, w), 255, np.uint8)
    assert np.array_equal(_paste_at_origin(image, result, full, imaging_ref.PASTE_FEATHER_COMPENSATE),
                          _paste_at_origin(image, result, full, imaging_ref.PASTE_FEATHER))
    empty = np.zeros((16, 16), np.uint8)
    im2, re2 = np.full((16, 16, 3), 90, np.uint8), np.full((16, 16, 3), 200, np.uint8)
    assert np.array_equal(_paste_at_origin(im2, re2, empty, imaging_ref.PASTE_FEATHER_COMPENSATE),
                          _paste_at_origin(im2, re2, empty, imaging_ref.PASTE_FEATHER))


def test_feather_paste_keeps_the_outside_and_blends_the_edge():
    # src/imaging/blend.rs:257-279: a window larger than the image writes only the inside.
    from oracle import imaging_ref
    w, h = 40, 30
    img = np.full((h, w, 3), 10, np.uint8)
    m = np.zeros((h, w), np.uint8)
    m[5:25, 10:30] = 255
    out, rect = imaging_ref.paste(img, m, np.full((40, 40, 3), 250, np.uint8), (0, 0, 40),
                                  imaging_ref.PASTE_FEATHER)
    assert rect == (0, 0, 40, 30)
    assert out[0, 0, 0] == 10 and out[15, 20, 0] == 250 and 10 < out[15, 9, 0] < 250


def test_dilation_follows_the_cv2_anchor():
    from oracle import imaging_ref
    m = np.zeros((7, 9), np.uint8)
    m[3, 4] = 255
    m[0, 0] = 200
    d = imaging_ref.dilate(m, 3)
    assert int((d == 255).sum()) == 13 and d[2, 3] == 255 and d[4, 5] == 255 and d[2, 6] == 0
    d = imaging_ref.dilate(m, 2)
    assert d[3, 4] == 255 and d[2, 3] == 0 and d[4, 5] == 255
    assert int((imaging_ref.dilate(m, 1) == 255).sum()) == 2
    assert not imaging_ref.dilate(np.full((7, 9), 127, np.uint8), 3).any()


DPM_WANT = [
    [1.228850083e+00, -2.980257470e+00, 4.364194085e+00],
    [2.418310907e+00, -5.782050465e+00, 8.090883333e+00],
    [3.814012762e+00, -9.051524459e+00, 1.235500469e+01],
    [4.986929961e+00, -1.177817121e+01, 1.581279684e+01],
    [5.635935287e+00, -1.324560079e+01, 1.747831563e+01],
]


def test_dpm_oracle_matches_the_reference_values():
    from oracle.scheduler_ref import Ddim, Dpm2M
    d = Ddim(5, 1.0, trailing=True)
    assert d.timesteps == [999, 799, 599, 399, 199]
    x = np.array([0.5, -1.25, 2.0], np.float32)
    s = Dpm2M()
    for i, want in enumerate(DPM_WANT):
        k = np.float32(1.0) + np.float32(0.2) * np.float32(i)
        x = s.step(d, np.array([0.1, -0.3, 0.7], np.float32) * k, i, x)
        assert np.all(np.abs(x - want) <= 2e-5 * np.abs(want))


def test_dpm_restart_makes_the_next_step_first_order():
    from oracle.scheduler_ref import Ddim, Dpm2M
    d = Ddim(5, 1.0, trailing=True)
    eps = np.array([0.1, -0.3, 0.7], np.float32)
    fresh, restarted = Dpm2M(), Dpm2M()
    restarted.step(d, eps, 0, np.array([1.0, 2.0, 3.0], np.float32))
    restarted.restart()
    a = fresh.step(d, eps, 1, np.array([0.5, -1.25, 2.0], np.float32))
    b = restarted.step(d, eps, 1, np.array([0.5, -1.25, 2.0], np.float32))
    assert np.array_equal(a, b)


def _lib_dpm(mbx, steps, strength, trailing, i, restart):
    coef = (ctypes.c_float * 5)()
    order = ctypes.c_int32()
    mbx.check(mbx.lib().mbx_dpm_coefficients(steps, strength, int(trailing), i, restart, coef, ctypes.byref(order)))
    return np.array(coef[:], np.float32), order.value


def test_library_dpm_step_reproduces_the_reference_values():
    # The device kernel's arithmetic (f32, reference order) on the library's coefficients.
    mbx = load_package()
    f = np.float32
    x = np.array([0.5, -1.25, 2.0], np.float32)
    prev = None
    for i, want in enumerate(DPM_WANT):
        c, order = _lib_dpm(mbx, 5, 1.0, True, i, -1)
        assert order == (0 if i == 4 else (1 if i == 0 else 2))
        k = f(1.0) + f(0.2) * f(i)
        e = np.array([0.1, -0.3, 0.7], np.float32) * k
        x0 = ((x - c[0] * e) * c[1]).astype(np.float32)
        if order == 0:
            x = x0
        elif order == 1:
            x = (c[2] * x + c[3] * x0).astype(np.float32)
        else:
            x = (c[2] * x + c[3] * x0 - c[4] * prev).astype(np.float32)
        prev = x0
        assert np.all(np.abs(x - want) <= 2e-5 * np.abs(want))


def test_library_dpm_coefficients_follow_the_oracle_with_a_restart():
    # Fast preset: 10 trailing steps at strength 0.99, history restarted at step 3.
    from oracle.scheduler_ref import Ddim, dpm_coefficients
    mbx = load_package()
    d = Ddim(10, 0.99, trailing=True)
    for i in range(len(d.timesteps)):
        c, order = _lib_dpm(mbx, 10, 0.99, True, i, 3)
        alpha, sigma, lam = dpm_coefficients(d, d.timesteps[i])
        assert c[0] == np.float32(sigma) and c[1] == np.float32(1.0 / alpha)
        if i + 1 == len(d.timesteps):
            assert order == 0
            continue
        assert order == (1 if i in (0, 3) else 2)
