"""GPU parity of the engine (include/moebius_cuda_engine.h) against the CPU
oracle composed in the reference's order: the UNet (src/unet/*), the VAE
encoder (src/vae/encoder.rs) and whole inpaints (src/pipeline.rs): both
presets, every paste mode, mask dilation and images of any size, with
caller-supplied noise, on seeded random-init weights in the converter's
format. Scaled-down networks of the same structure (widths 64/128/256,
latent 16; VAE widths 32/64/128/128) keep the oracle fast; the full-size
network runs one UNet step, a 2-step inpaint and the benchmark's batch of
8 Exact inpaints (19 DDIM steps). Gates (BASELINE
north_star): max relative error ≤ 1e-3 (f32 weights, 3xTF32) / 5e-3 (f16
weights, 2xTF32) per network output, 8-bit PSNR ≥ 45 dB end to end."""
import ctypes
import os

import numpy as np
import pytest

from conftest import load_package, max_rel_err

pytestmark = pytest.mark.gpu

TINY_UNET = ((64, 128, 256), 16)
TINY_VAE = (32, 64, 128, 128)


def psnr8(a, b):
    mse = np.mean((a.astype(np.float64) - b.astype(np.float64)) ** 2)
    return float("inf") if mse == 0 else 10 * np.log10(255.0 ** 2 / mse)


def _weights(tmp_path_factory, name, unet=TINY_UNET, vae=TINY_VAE, f16=True, seed=0):
    syn = load_package().synthetic
    d = str(tmp_path_factory.mktemp(name))
    syn.write_weights_dir(d, seed=seed, f16=f16, unet_widths=unet[0], latent=unet[1], vae_widths=vae)
    wu, _ = syn.read_safetensors(os.path.join(d, "unet.safetensors"))
    wv, _ = syn.read_safetensors(os.path.join(d, "vae.safetensors"))
    return d, wu, wv


# fixture name -> (weights directory, engine)
_WEIGHT_DIRS = {}


@pytest.fixture(scope="module", params=["f16", "f32"])
def tiny(request, tmp_path_factory, mbx, ctx):
    d, wu, wv = _weights(tmp_path_factory, f"tiny_{request.param}", f16=request.param == "f16")
    eng = mbx.engine.Engine(d, 0)
    eng.set_stream(ctx.stream)
    _WEIGHT_DIRS[f"tiny_{request.param}"] = (d, eng)
    yield eng, wu, wv, request.param
    _WEIGHT_DIRS.pop(f"tiny_{request.param}", None)
    eng.close()


@pytest.fixture(scope="module")
def full(tmp_path_factory, mbx, ctx):
    syn = mbx.synthetic
    d, wu, wv = _weights(tmp_path_factory, "full", unet=(syn.UNET_WIDTHS, syn.UNET_LATENT), vae=syn.VAE_WIDTHS)
    eng = mbx.engine.Engine(d, 0)
    eng.set_stream(ctx.stream)
    yield eng, wu, wv
    eng.close()


def _gate(wdtype):
    return 1e-3 if wdtype == "f32" else 5e-3


def test_engine_reads_the_network_shape(tiny):
    eng = tiny[0]
    assert (eng.latent, eng.side, eng.widths) == (16, 128, (64, 128, 256))


@pytest.mark.parametrize("items,cfg,t", [(2, True, 900), (4, True, 450), (1, False, 0)])
def test_unet_forward_matches_oracle(ctx, tiny, items, cfg, t):
    from oracle import unet_ref
    eng, wu, _, wdtype = tiny
    rng = np.random.default_rng(items + t)
    x = rng.standard_normal((items, 16, 16, 9)).astype(np.float32)
    xd, eps = ctx.upload(x), ctx.empty((items, 16, 16, 4))
    eng.unet_forward(xd.ptr, items, t, cfg, eps.ptr)
    got = eps.numpy()
    branches = [i % 2 for i in range(items)] if cfg else [1] * items
    want = unet_ref.forward(wu, x, t, branches)
    assert max_rel_err(got, want) <= _gate(wdtype)


def test_vae_encode_decode_match_oracle(ctx, tiny):
    from oracle import vae_ref
    eng, _, wv, wdtype = tiny
    rng = np.random.default_rng(8)
    img = rng.uniform(-1, 1, (2, 64, 64, 3)).astype(np.float32)
    noise = rng.standard_normal((2, 8, 8, 4)).astype(np.float32)
    z = ctx.empty((2, 8, 8, 4))
    imgd, nd = ctx.upload(img), ctx.upload(noise)
    eng.vae_encode(imgd.ptr, nd.ptr, 2, 64, 64, z.ptr)
    assert max_rel_err(z.numpy(), vae_ref.encode(wv, img, noise)) <= _gate(wdtype)
    lat = (rng.standard_normal((2, 8, 8, 4)) * 0.13025).astype(np.float32)
    out = ctx.empty((2, 64, 64, 3))
    latd = ctx.upload(lat)
    eng.vae_decode(latd.ptr, 2, 8, 8, out.ptr)
    assert max_rel_err(out.numpy(), vae_ref.decode(wv, lat)) <= _gate(wdtype)


def _inputs(rng, n, side, ch=3):
    lat = side // 8
    img = rng.integers(0, 256, (n, side, side, ch), dtype=np.uint8)
    yy, xx = np.mgrid[:side, :side]
    masks = np.zeros((n, side, side), np.uint8)
    for i in range(n):
        cy, cx = rng.uniform(0.3, 0.7, 2) * side
        ry, rx = rng.uniform(0.15, 0.3, 2) * side
        masks[i] = ((((yy - cy) / ry) ** 2 + ((xx - cx) / rx) ** 2) <= 1) * rng.integers(128, 256)
    nv = rng.standard_normal((2 * n, lat, lat, 4)).astype(np.float32)
    ni = rng.standard_normal((n, lat, lat, 4)).astype(np.float32)
    no = rng.standard_normal((n, 4)).astype(np.float32)
    return img, masks, nv, ni, no


def test_inpaint_batch_matches_oracle(mbx, tiny):
    """Three inpaints in one batch (the last with an empty mask), Exact preset, 19 DDIM steps."""
    from oracle import pipeline_ref, unet_ref
    eng, wu, wv, _ = tiny
    rng = np.random.default_rng(21)
    img, masks, nv, ni, no = _inputs(rng, 3, 128)
    masks[2] = 0
    got = img.copy()
    eng.inpaint_batch(got, masks, noise=(nv, ni, no))
    ehs = unet_ref.conditioning(wu)
    for i in range(2):
        want = pipeline_ref.inpaint(wu, wv, img[i], masks[i], nv[2 * i:2 * i + 2], ni[i], no[i], ehs=ehs)
        assert psnr8(got[i], want) >= 45.0
        assert not np.array_equal(got[i], img[i])
    assert np.array_equal(got[2], img[2]), "an empty mask changes nothing"


def test_batch_items_are_independent(mbx, tiny):
    eng = tiny[0]
    rng = np.random.default_rng(22)
    img, masks, nv, ni, no = _inputs(rng, 2, 128, ch=4)
    both = img.copy()
    eng.inpaint_batch(both, masks, noise=(nv, ni, no), p=mbx.engine.params(steps=4))
    one = img[1:].copy()
    eng.inpaint_batch(one, masks[1:], noise=(nv[2:], ni[1:], no[1:]), p=mbx.engine.params(steps=4))
    assert np.array_equal(both[1:], one)
    assert np.array_equal(both[..., 3], img[..., 3]), "alpha is preserved"


def test_single_image_api(mbx, tiny):
    eng = tiny[0]
    rng = np.random.default_rng(23)
    img, masks, *_ = _inputs(rng, 1, 128, ch=4)
    # Strided image rows (reference moebius_inpaint takes a row stride).
    canvas = np.zeros((128, 128 + 7, 4), np.uint8)
    canvas[:, :128] = img[0]
    view = canvas[:, :128]
    rect = eng.inpaint(view, masks[0], mbx.engine.params(steps=3, seed=5))
    assert rect == (0, 0, 128, 128)
    past = np.argwhere(canvas[:, 128:] != 0)
    assert past.size == 0, f"bytes past the row width changed: {past[:8].tolist()} of {len(past)}"
    assert np.array_equal(view[..., 3], img[0, ..., 3])
    again = np.ascontiguousarray(img[0]).copy()
    eng.inpaint(again, masks[0], mbx.engine.params(steps=3, seed=5))
    assert np.array_equal(again, view), "seeded noise is deterministic"
    blank = img[0].copy()
    assert eng.inpaint(blank, np.zeros((128, 128), np.uint8)) == (0, 0, 0, 0)
    assert np.array_equal(blank, img[0])


def test_engine_rejects_bad_requests(mbx, tiny):
    eng = tiny[0]
    img = np.zeros((64, 64, 3), np.uint8)
    full = np.full((64, 64), 255, np.uint8)
    for p in (mbx.engine.params(preset=7), mbx.engine.params(paste=9), mbx.engine.params(steps=1001)):
        with pytest.raises(mbx.MbxError) as e:
            eng.inpaint(img, full, p)
        assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT
    with pytest.raises(mbx.MbxError) as e:
        mbx.check(mbx.abi.lib().mbx_inpaint(eng.handle, img.ctypes.data, 64, 64, 64 * 3 - 1, 3, full.ctypes.data, 64,
                                            None, mbx.abi.PROGRESS_FN(), None, None))
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT
    with pytest.raises(mbx.MbxError) as e:
        mbx.check(mbx.abi.lib().mbx_inpaint(eng.handle, img.ctypes.data, 64, 64, 64 * 2, 2, full.ctypes.data, 64,
                                            None, mbx.abi.PROGRESS_FN(), None, None))
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT
    with pytest.raises(mbx.MbxError) as e:  # batch call: model-size images only
        eng.inpaint_batch(np.zeros((1, 64, 64, 3), np.uint8), full[None])
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT


def _single_noise(rng, lat):
    return (rng.standard_normal((2, lat, lat, 4)).astype(np.float32),
            rng.standard_normal((lat, lat, 4)).astype(np.float32),
            rng.standard_normal(4).astype(np.float32))


# Image sizes other than the model side (128 here): a window as large as the image's long
# side, padded above and below (300 x 200, RGBA with a row stride), a window inside a larger
# image (700 x 500), an image smaller than the model (90 x 60: upscaled window), each through
# the crop window, Lanczos3 both ways and the paste.
@pytest.mark.parametrize("w,h,ch,paste,r", [(300, 200, 4, 0, 0.3), (700, 500, 3, 3, 0.1), (90, 60, 3, 1, 0.2)])
def test_any_size_inpaint_matches_oracle(mbx, tiny, w, h, ch, paste, r):
    from oracle import pipeline_ref, unet_ref
    eng, wu, wv, _ = tiny
    rng = np.random.default_rng(w + h)
    img = rng.integers(0, 256, (h, w, ch), dtype=np.uint8)
    yy, xx = np.mgrid[:h, :w]
    cy, cx = rng.uniform(0.3, 0.7) * h, rng.uniform(0.3, 0.7) * w
    mask = (((((yy - cy) / (r * h)) ** 2 + ((xx - cx) / (r * w)) ** 2) <= 1) * 200).astype(np.uint8)
    noise = _single_noise(rng, 16)
    canvas = np.zeros((h, w * ch + 9), np.uint8)
    view = canvas[:, :w * ch].reshape(h, w, ch)
    view[...] = img
    rect = eng.inpaint(view, mask, mbx.engine.params(steps=4, paste=paste), noise=noise)
    want, want_rect = pipeline_ref.run(wu, wv, img, mask, *noise, params=dict(steps=4, paste=paste or 2),
                                       ehs=unet_ref.conditioning(wu))
    assert rect == want_rect
    assert psnr8(view, want) >= 45.0
    x, y, rw, rh = rect
    outside = np.ones((h, w), bool)
    outside[y:y + rh, x:x + rw] = False
    assert np.array_equal(view[outside], img[outside]), "only the changed rectangle is written"
    assert not canvas[:, w * ch:].any(), "bytes past the row width are untouched"
    if ch == 4:
        assert np.array_equal(view[..., 3], img[..., 3])


def test_fast_preset_matches_oracle(mbx, tiny):
    """Fast: trailing DPM-Solver++(2M), CFG for the first 3 steps then conditional only, ROI
    encode; here 5 steps so the oracle stays quick (3 CFG + 2 conditional-only, one restart)."""
    from oracle import pipeline_ref, unet_ref
    eng, wu, wv, _ = tiny
    rng = np.random.default_rng(41)
    img, masks, nv, ni, no = _inputs(rng, 2, 128)
    masks[1] = 0
    masks[1, 20:40, 30:50] = 255  # a small mask: its ROI window is smaller than the latent
    got = img.copy()
    p = mbx.engine.params(preset=mbx.abi.PRESET_FAST, steps=5)
    eng.inpaint_batch(got, masks, p, noise=(nv, ni, no))
    ehs = unet_ref.conditioning(wu)
    for i in range(2):
        want = pipeline_ref.run(wu, wv, img[i], masks[i], nv[2 * i:2 * i + 2], ni[i], no[i],
                                params=dict(pipeline_ref.FAST, steps=5), ehs=ehs)[0]
        assert psnr8(got[i], want) >= 45.0, i
    single = img[1].copy()
    eng.inpaint(single, masks[1], p, noise=(nv[2:4], ni[1], no[1]))
    assert np.array_equal(single, got[1]), "single and batch calls agree"


def test_batch_paste_modes_and_dilation_match_oracle(mbx, tiny):
    from oracle import pipeline_ref, unet_ref
    eng, wu, wv, _ = tiny
    rng = np.random.default_rng(43)
    img, masks, nv, ni, no = _inputs(rng, 2, 128, ch=4)
    ehs = unet_ref.conditioning(wu)
    for paste, dilate in ((1, 0), (3, 5)):
        got = img.copy()
        eng.inpaint_batch(got, masks, mbx.engine.params(steps=3, paste=paste, mask_dilate=dilate), noise=(nv, ni, no))
        for i in range(2):
            want = pipeline_ref.run(wu, wv, img[i], masks[i], nv[2 * i:2 * i + 2], ni[i], no[i],
                                    params=dict(steps=3, paste=paste, mask_dilate=dilate), ehs=ehs)[0]
            assert psnr8(got[i], want) >= 45.0, (paste, dilate, i)


def test_progress_reports_and_cancel_leaves_image_untouched(mbx, tiny):
    eng = tiny[0]
    rng = np.random.default_rng(24)
    img, masks, *_ = _inputs(rng, 1, 128)
    seen = []

    def progress(stage, done, total):
        seen.append((stage, done, total))
        return stage == 1 and done == 2  # cancel after the second denoising step

    work = img[0].copy()
    with pytest.raises(mbx.MbxError) as e:
        eng.inpaint(work, masks[0], mbx.engine.params(steps=5), progress)
    assert e.value.code == mbx.abi.ERR_CANCELLED
    assert np.array_equal(work, img[0])
    assert seen == [(0, 0, 1), (0, 1, 1), (1, 1, 4), (1, 2, 4)]
    seen.clear()
    eng.inpaint(work, masks[0], mbx.engine.params(steps=5), lambda s, d, t: seen.append((s, d, t)) and False)
    assert seen[-3:] == [(1, 4, 4), (2, 0, 1), (2, 1, 1)]


def test_full_size_unet_step_matches_oracle(ctx, full):
    from oracle import unet_ref
    eng, wu, _ = full
    rng = np.random.default_rng(31)
    x = rng.standard_normal((2, 64, 64, 9)).astype(np.float32)
    eps = ctx.empty((2, 64, 64, 4))
    xd = ctx.upload(x)
    eng.unet_forward(xd.ptr, 2, 900, True, eps.ptr)
    want = unet_ref.forward(wu, x, 900, [0, 1])
    assert max_rel_err(eps.numpy(), want) <= 5e-3


def test_full_size_inpaint_matches_oracle(mbx, full):
    """One 512² inpaint, Exact preset with 3 steps (2 denoising steps), f16 weights."""
    from oracle import pipeline_ref
    eng, wu, wv = full
    rng = np.random.default_rng(32)
    img, masks, nv, ni, no = _inputs(rng, 1, 512)
    got = img.copy()
    eng.inpaint_batch(got, masks, mbx.engine.params(steps=3), noise=(nv, ni, no))
    want = pipeline_ref.inpaint(wu, wv, img[0], masks[0], nv, ni[0], no[0], steps=3)
    assert psnr8(got[0], want) >= 45.0


def test_full_size_exact_batch_of_8_matches_oracle(mbx, ctx, full):
    """The benchmark's configuration: 8 full-size 512² Exact inpaints in one batch (20 steps at
    strength 0.99 = 19 DDIM steps, CFG 2.5, the UNet replayed from the graph captured at batch
    16), f16 weights, random-ellipse masks covering 10-40 %. Items 0 and 5 against the oracle
    pipeline with the same noise (src/pipeline.rs:217-373, src/preset.rs:59-72); the
    device-buffer call the benchmark times gives the same bytes as the host-buffer call."""
    from oracle import pipeline_ref, unet_ref
    eng, wu, wv = full
    syn = mbx.synthetic
    rng = np.random.default_rng(1234)
    n = 8
    img = rng.integers(0, 256, (n, 512, 512, 3), dtype=np.uint8)
    masks = syn.ellipse_masks(rng, n, 512)
    nv = rng.standard_normal((2 * n, 64, 64, 4), dtype=np.float32)
    ni = rng.standard_normal((n, 64, 64, 4), dtype=np.float32)
    no = rng.standard_normal((n, 4), dtype=np.float32)
    got = img.copy()
    eng.inpaint_batch(got, masks, noise=(nv, ni, no))
    # The device-buffer path (what the benchmark's `value` times). It returns once the work is
    # enqueued on the engine's stream (the session context's), so that stream is synchronised
    # before the result is read through another context.
    c2 = mbx.Context(0)
    try:
        dpx, dm = c2.upload(img, np.uint8), c2.upload(masks, np.uint8)
        dnv, dni, dno = c2.upload(nv), c2.upload(ni), c2.upload(no)
        c2.synchronize()
        eng.inpaint_batch_device(dpx.ptr, dm.ptr, n, 512, 3, mbx.engine.params(), (dnv.ptr, dni.ptr, dno.ptr))
        ctx.synchronize()
        got_dev = dpx.numpy()
    finally:
        c2.close()
    assert np.array_equal(got_dev, got), "device-buffer and host-buffer calls agree"
    ehs = unet_ref.conditioning(wu)
    for i in (0, 5):
        want = pipeline_ref.inpaint(wu, wv, img[i], masks[i], nv[2 * i:2 * i + 2], ni[i], no[i], ehs=ehs)
        assert psnr8(got[i], want) >= 45.0, f"item {i}"
        assert not np.array_equal(got[i], img[i])


def test_moebius_cpu_dropin_runs_the_engine(mbx, tiny):
    """The reference-named C API (include/moebius_cpu.h) on a real weights directory: an inpaint
    through moebius_inpaint gives the same bytes and rectangle as mbx_inpaint with the same seed."""
    import ctypes
    eng = tiny[0]
    d = _WEIGHT_DIRS[f"tiny_{tiny[3]}"][0]
    lib = mbx.abi.lib()
    h = ctypes.c_void_p()
    mbx.check(lib.moebius_engine_create(d.encode(), 7, ctypes.byref(h)))
    try:
        rng = np.random.default_rng(24)
        img, masks, *_ = _inputs(rng, 1, 128, ch=4)
        p = mbx.engine.params(steps=3, seed=11)
        want = img[0].copy()
        rect_want = eng.inpaint(want, masks[0], p)
        got = img[0].copy()
        rect = mbx.abi.Rect()
        st = lib.moebius_inpaint(h, got.ctypes.data_as(ctypes.c_void_p), 128, 128, 128 * 4, 4,
                                 masks[0].ctypes.data_as(ctypes.c_void_p), 128, ctypes.byref(p),
                                 mbx.abi.PROGRESS_FN(), None, ctypes.byref(rect))
        assert st == 0, lib.moebius_last_error()
        assert np.array_equal(got, want)
        assert (rect.x, rect.y, rect.width, rect.height) == rect_want
        # Reference status codes: a bad channel count is MOEBIUS_ERR_INVALID_ARGUMENT.
        st = lib.moebius_inpaint(h, got.ctypes.data_as(ctypes.c_void_p), 128, 128, 128 * 4, 2,
                                 masks[0].ctypes.data_as(ctypes.c_void_p), 128, None, mbx.abi.PROGRESS_FN(), None,
                                 None)
        assert st == 1
    finally:
        lib.moebius_engine_destroy(h)
