"""TEST INFRASTRUCTURE ONLY: one Exact-preset inpaint of a model-size image,
composed from the oracle pieces in the reference's order (src/pipeline.rs:215-373,
src/preset.rs:312-328, src/imaging/*), with caller-supplied noise as the
reference's parity runs use (Engine::inpaint_with_noise, pipeline.rs:150-161).
"""
from __future__ import annotations

import numpy as np

from . import imaging_ref, unet_ref, vae_ref
from .scheduler_ref import Ddim

f32 = np.float32


def inpaint(wu, wv, image, mask, noise_vae, noise_init, noise_offset, steps=20, strength=0.99, guidance=2.5,
            noise_offset_scale=0.0357, ehs=None, trace=None):
    """image [S, S, ch] u8, mask [S, S] u8, noise_vae [2, L, L, 4] (image, masked), noise_init
    [L, L, 4], noise_offset [4] -> the inpainted image (u8, same shape). `trace`, when a dict,
    receives the final latents and the decoded image."""
    if not (mask >= 128).any():
        return image.copy()                                    # pipeline.rs:202-204
    rgb, binary = imaging_ref.to_model(image, mask)           # pipeline.rs:236
    keep = np.where(binary >= 128, f32(0.0), f32(1.0))
    masked = (rgb * keep[..., None]).astype(np.float32)      # pipeline.rs:237-244
    mask_lat = (binary[::8, ::8] >= 128).astype(np.float32)  # pipeline.rs:247-252
    z = vae_ref.encode(wv, np.stack([rgb, masked]), noise_vae)
    z_img, z_masked = z[0], z[1]
    init = (np.asarray(noise_init, f32) + f32(noise_offset_scale) * np.asarray(noise_offset, f32)).astype(f32)
    ddim = Ddim(steps, strength)
    ts = ddim.timesteps
    x = init.copy() if ddim.pure_noise_start else ddim.add_noise(z_img, init, ts[0])
    ehs = unet_ref.conditioning(wu) if ehs is None else ehs
    g = f32(guidance)
    for t in ts:                                              # pipeline.rs:317-345
        inp = np.concatenate([x, mask_lat[..., None], z_masked], axis=-1)[None]
        e = unet_ref.forward(wu, np.concatenate([inp, inp]), t, [0, 1], ehs)
        eps = (e[0] + g * (e[1] - e[0])).astype(f32)
        x = ddim.step(eps, t, x)
    dec = vae_ref.decode(wv, x[None])[0]                      # pipeline.rs:355-366
    if trace is not None:
        trace["latents"] = x
        trace["decoded"] = dec
    return imaging_ref.feather_paste(image, mask, imaging_ref.to_u8(dec))
