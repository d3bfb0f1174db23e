"""Python front end of the engine API (include/moebius_cuda_engine.h): the
moebius-cpu inpainting engine (UNet + VAE + Exact pipeline) on one GPU.

    eng = Engine(weights_dir, device=0)
    eng.inpaint(pixels, mask)                          # one image, in place (mbx_inpaint)
    eng.inpaint_batch(pixels, masks, noise=...)        # n images, in place (mbx_inpaint_batch)

``weights_dir`` holds ``unet.safetensors`` and ``vae.safetensors`` in the
reference converter's format (``synthetic.write_weights_dir`` writes seeded
random ones).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import numpy as np

from . import abi
from .abi import InpaintParams, check, lib


def params(preset=abi.PRESET_EXACT, steps=0, guidance=0.0, seed=0, paste=abi.PASTE_DEFAULT,
           mask_dilate=0) -> InpaintParams:
    return InpaintParams(preset, steps, guidance, seed, paste, mask_dilate)


def _ptr(a) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data) if isinstance(a, np.ndarray) else ctypes.c_void_p(int(a))


class Engine:
    def __init__(self, weights_dir: str, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().mbx_engine_create(weights_dir.encode(), device, ctypes.byref(h)))
        self.handle = h
        lat, side = ctypes.c_int64(), ctypes.c_int64()
        widths = (ctypes.c_int64 * 3)()
        check(lib().mbx_engine_info(h, ctypes.byref(lat), ctypes.byref(side), widths))
        self.latent, self.side, self.widths = lat.value, side.value, tuple(widths)

    def close(self) -> None:
        if self.handle:
            lib().mbx_engine_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def launch_count(self) -> int:
        return int(lib().mbx_engine_launch_count(self.handle))

    def set_stream(self, stream_ptr: Optional[int]) -> None:
        check(lib().mbx_engine_set_stream(self.handle, ctypes.c_void_p(stream_ptr or 0)))

    def inpaint(self, pixels: np.ndarray, mask: np.ndarray, p: Optional[InpaintParams] = None,
                progress: Optional[Callable[[int, int, int], bool]] = None, noise=None):
        """In place on an [h, w, 3|4] uint8 image of any size (row stride may exceed w·channels);
        returns the changed rectangle (x, y, width, height). noise = (vae [2, L, L, 4], init
        [L, L, 4], offset [4]) float32 (mbx_inpaint_with_noise) or None (seeded, mbx_inpaint)."""
        assert pixels.dtype == np.uint8 and mask.dtype == np.uint8
        assert pixels.strides[1] == pixels.shape[2] and pixels.strides[2] == 1 and mask.strides[1] == 1
        h, w, ch = pixels.shape
        rect = abi.Rect()
        cb = abi.PROGRESS_FN(lambda _u, s, d, t: int(bool(progress(s, d, t)))) if progress else abi.PROGRESS_FN()
        pp = ctypes.byref(p) if p is not None else None
        if noise is None:
            check(lib().mbx_inpaint(self.handle, _ptr(pixels), w, h, pixels.strides[0], ch, _ptr(mask),
                                    mask.strides[0], pp, cb, None, ctypes.byref(rect)))
        else:
            nz = [np.ascontiguousarray(a, np.float32) for a in noise]
            check(lib().mbx_inpaint_with_noise(self.handle, _ptr(pixels), w, h, pixels.strides[0], ch, _ptr(mask),
                                               mask.strides[0], pp, *[_ptr(a) for a in nz], cb, None,
                                               ctypes.byref(rect)))
        return rect.x, rect.y, rect.width, rect.height

    def inpaint_batch(self, pixels: np.ndarray, masks: np.ndarray, p: Optional[InpaintParams] = None, noise=None,
                      progress: Optional[Callable[[int, int, int], bool]] = None) -> None:
        """In place on host arrays pixels [n, S, S, ch] uint8, masks [n, S, S] uint8; noise =
        (vae [2n, L, L, 4], init [n, L, L, 4], offset [n, 4]) float32 or None (seeded)."""
        assert pixels.dtype == np.uint8 and pixels.flags["C_CONTIGUOUS"]
        masks = np.ascontiguousarray(masks, np.uint8)
        n, s, _, ch = pixels.shape
        nz = [None, None, None] if noise is None else [np.ascontiguousarray(a, np.float32) for a in noise]
        cb = abi.PROGRESS_FN(lambda _u, st, d, t: int(bool(progress(st, d, t)))) if progress else abi.PROGRESS_FN()
        check(lib().mbx_inpaint_batch(self.handle, _ptr(pixels), _ptr(masks), n, s, ch,
                                      ctypes.byref(p) if p is not None else None,
                                      *[_ptr(a) if a is not None else None for a in nz], 0, cb, None))

    def inpaint_batch_device(self, pixels_ptr: int, masks_ptr: int, n: int, side: int, channels: int,
                             p: Optional[InpaintParams] = None, noise_ptrs=(None, None, None)) -> None:
        """Device-buffer variant (every pointer on the engine's device)."""
        check(lib().mbx_inpaint_batch(self.handle, ctypes.c_void_p(pixels_ptr), ctypes.c_void_p(masks_ptr), n, side,
                                      channels, ctypes.byref(p) if p is not None else None,
                                      *[ctypes.c_void_p(q) if q else None for q in noise_ptrs], 1,
                                      abi.PROGRESS_FN(), None))

    def unet_forward(self, x_ptr: int, items: int, timestep: int, cfg: bool, eps_ptr: int) -> None:
        check(lib().mbx_engine_unet_forward(self.handle, ctypes.c_void_p(x_ptr), items, timestep, int(cfg),
                                            ctypes.c_void_p(eps_ptr)))

    def vae_encode(self, images_ptr: int, noise_ptr: int, b: int, h: int, w: int, z_ptr: int) -> None:
        check(lib().mbx_engine_vae_encode(self.handle, ctypes.c_void_p(images_ptr), ctypes.c_void_p(noise_ptr), b, h,
                                          w, ctypes.c_void_p(z_ptr)))

    def vae_decode(self, latents_ptr: int, b: int, h: int, w: int, out_ptr: int) -> None:
        check(lib().mbx_engine_vae_decode(self.handle, ctypes.c_void_p(latents_ptr), b, h, w,
                                          ctypes.c_void_p(out_ptr)))
