"""TEST INFRASTRUCTURE ONLY: one inpaint composed from the oracle pieces in the
reference's order (src/pipeline.rs:163-373, src/preset.rs:55-83, src/imaging/*,
src/scheduler.rs), with caller-supplied noise as the reference's parity runs use
(Engine::inpaint_with_noise, pipeline.rs:150-161). Any image size: mask
dilation, bbox, square crop window, Lanczos3 resampling to and from the model
size, every paste mode; the Exact (DDIM, CFG every step) and Fast
(DPM-Solver++(2M), trailing spacing, CFG for the first steps, ROI encode)
presets.
"""
from __future__ import annotations

import numpy as np

from . import imaging_ref, unet_ref, vae_ref
from .scheduler_ref import Ddim, Dpm2M

f32 = np.float32

EXACT = dict(steps=20, strength=0.99, trailing=False, solver="ddim", guidance=2.5, noise_offset=0.0357,
             cfg_steps=None, roi_encode=False, paste=imaging_ref.PASTE_FEATHER, mask_dilate=0)
FAST = dict(EXACT, steps=10, trailing=True, solver="dpm", cfg_steps=3, roi_encode=True)
ROI_MARGIN = 8


def roi_window(mask_lat, margin):
    """Latent bbox of mask_lat > 0.5 grown by `margin` and clamped, (x, y, w, h) or None
    (src/vae/mod.rs:64-78)."""
    n = mask_lat.shape[0]
    ys, xs = np.nonzero(mask_lat > 0.5)
    if ys.size == 0:
        return None
    x0, y0 = max(int(xs.min()) - margin, 0), max(int(ys.min()) - margin, 0)
    x1, y1 = min(int(xs.max()) + margin, n - 1), min(int(ys.max()) + margin, n - 1)
    return x0, y0, x1 - x0 + 1, y1 - y0 + 1


def run(wu, wv, image, mask, noise_vae, noise_init, noise_offset, params=None, ehs=None, trace=None):
    """image [h, w, ch] u8 (RGB/RGBA), mask [h, w] u8, noise_vae [2, L, L, 4] (image, masked),
    noise_init [L, L, 4], noise_offset [4] -> (inpainted image u8, changed rect (x, y, w, h))."""
    p = dict(EXACT, **(params or {}))
    L = noise_init.shape[0]
    S = 8 * L
    h, w = mask.shape
    if p["mask_dilate"] > 0:                                   # pipeline.rs:191-197
        mask = imaging_ref.dilate(mask, p["mask_dilate"])
    box = imaging_ref.bbox(mask)
    if box is None:                                            # pipeline.rs:198-200
        return image.copy(), (0, 0, 0, 0)
    plan = imaging_ref.crop_plan(box, w, h, S)                 # pipeline.rs:201
    rgb_u8, binary = imaging_ref.window_to_model(image, mask, plan, S)
    rgb, _ = imaging_ref.to_model(rgb_u8, binary)              # pipeline.rs:236
    keep = np.where(binary >= 128, f32(0.0), f32(1.0))
    masked = (rgb * keep[..., None]).astype(f32)              # pipeline.rs:237-244
    mask_lat = (binary[::8, ::8] >= 128).astype(f32)          # pipeline.rs:247-252

    window = roi_window(mask_lat, ROI_MARGIN) if p["roi_encode"] else None
    if window is not None and (window[2] < L or window[3] < L):  # pipeline.rs:255-275
        rx, ry, rw, rh = window
        z_masked = vae_ref.encode(wv, masked[None], noise_vae[1:2])[0]
        crop = rgb[8 * ry:8 * (ry + rh), 8 * rx:8 * (rx + rw)]
        part = vae_ref.encode(wv, crop[None], noise_vae[0:1, ry:ry + rh, rx:rx + rw])[0]
        ix, iy, iw, ih = roi_window(mask_lat, ROI_MARGIN // 2)
        z_img = z_masked.copy()
        z_img[iy:iy + ih, ix:ix + iw] = part[iy - ry:iy - ry + ih, ix - rx:ix - rx + iw]
    else:
        z = vae_ref.encode(wv, np.stack([rgb, masked]), noise_vae)
        z_img, z_masked = z[0], z[1]

    init = (np.asarray(noise_init, f32) + f32(p["noise_offset"]) * np.asarray(noise_offset, f32)).astype(f32)
    ddim = Ddim(p["steps"], p["strength"], p["trailing"])
    ts = ddim.timesteps
    x = init.copy() if ddim.pure_noise_start else ddim.add_noise(z_img, init, ts[0])
    ehs = unet_ref.conditioning(wu) if ehs is None else ehs
    g = f32(p["guidance"])
    dpm = Dpm2M()
    for i, t in enumerate(ts):                                 # pipeline.rs:313-346
        inp = np.concatenate([x, mask_lat[..., None], z_masked], axis=-1)[None]
        if p["cfg_steps"] is None or i < p["cfg_steps"]:
            e = unet_ref.forward(wu, np.concatenate([inp, inp]), t, [0, 1], ehs)
            eps = (e[0] + g * (e[1] - e[0])).astype(f32)
        else:
            eps = unet_ref.forward(wu, inp, t, [1], ehs)[0]
        if p["solver"] == "ddim":
            x = ddim.step(eps, t, x)
        else:
            if p["cfg_steps"] == i:
                dpm.restart()
            x = dpm.step(ddim, eps, i, x)
    dec = vae_ref.decode(wv, x[None])[0]                      # pipeline.rs:355-366
    if trace is not None:
        trace["latents"] = x
        trace["decoded"] = dec
        trace["plan"] = plan
    result = imaging_ref.model_to_window(dec, plan[2])        # pipeline.rs:370
    return imaging_ref.paste(image, mask, result, plan, p["paste"])


def inpaint(wu, wv, image, mask, noise_vae, noise_init, noise_offset, steps=20, strength=0.99, guidance=2.5,
            noise_offset_scale=0.0357, ehs=None, trace=None):
    """Exact preset on a model-size image (used whole): the inpainted image."""
    params = dict(steps=steps, strength=strength, guidance=guidance, noise_offset=noise_offset_scale)
    return run(wu, wv, image, mask, noise_vae, noise_init, noise_offset, params, ehs, trace)[0]
