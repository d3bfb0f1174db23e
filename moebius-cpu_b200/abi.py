"""ctypes binding of libmoebius_cuda.so (declared in include/moebius_cuda.h).

Loading fails loudly: there is no CPU fallback. ``symbols()`` lists every
entry point the header declares so a test can check the library exports them.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "lib", "libmoebius_cuda.so")
HEADER = os.path.join(REPO, "include", "moebius_cuda.h")
ENGINE_HEADER = os.path.join(REPO, "include", "moebius_cuda_engine.h")
COMPAT_HEADER = os.path.join(REPO, "include", "moebius_cpu.h")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_WEIGHTS = 2
ERR_UNSUPPORTED_DEVICE = 3
ERR_CANCELLED = 4
ERR_IO = 5
ERR_INTERNAL = 6
ERR_OUT_OF_MEMORY = 7
ERR_CUDA = 8
ERR_TIMEOUT = 9

DTYPE_F32 = 0
DTYPE_F16 = 1

EPILOGUE_NONE = 0
EPILOGUE_RELU = 1
EPILOGUE_GLU_SILU = 2

ACT_NONE = 0
ACT_SILU = 1

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t
_f32 = ctypes.c_float
_pvp = ctypes.POINTER(ctypes.c_void_p)
_pi64 = ctypes.POINTER(ctypes.c_int64)
_psz = ctypes.POINTER(ctypes.c_size_t)
_pi32 = ctypes.POINTER(ctypes.c_int32)
_pf32 = ctypes.POINTER(ctypes.c_float)
_u32 = ctypes.c_uint32
_f64 = ctypes.c_double

PRESET_EXACT = 0
PRESET_FAST = 1
PASTE_DEFAULT = 0
PASTE_NONE = 1
PASTE_FEATHER = 2
PASTE_FEATHER_COMPENSATE = 3


class InpaintParams(ctypes.Structure):
    """mbx_inpaint_params (the reference's MoebiusParams); zero = Exact defaults."""
    _fields_ = [("preset", ctypes.c_uint32), ("steps", ctypes.c_uint32), ("guidance", ctypes.c_float),
                ("seed", ctypes.c_uint64), ("paste", ctypes.c_uint32), ("mask_dilate", ctypes.c_uint32)]


class Rect(ctypes.Structure):
    _fields_ = [("x", ctypes.c_uint32), ("y", ctypes.c_uint32), ("width", ctypes.c_uint32),
                ("height", ctypes.c_uint32)]


PROGRESS_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32)

# name -> (restype, argtypes)
SIGNATURES = {
    "mbx_abi_version": (ctypes.c_uint32, []),
    "mbx_last_error": (ctypes.c_char_p, []),
    "mbx_ctx_create": (_i32, [_i32, _pvp]),
    "mbx_ctx_destroy": (None, [_vp]),
    "mbx_ctx_set_stream": (_i32, [_vp, _vp]),
    "mbx_ctx_stream": (_vp, [_vp]),
    "mbx_ctx_synchronize": (_i32, [_vp]),
    "mbx_ctx_launch_count": (_u64, [_vp]),
    "mbx_selftest_wait_timeout": (_i32, [_vp, _i64]),
    "mbx_alloc": (_i32, [_vp, _sz, _pvp]),
    "mbx_free": (_i32, [_vp, _vp]),
    "mbx_pool_release_below": (_i32, [_vp, _sz]),
    "mbx_pool_stats": (_i32, [_vp, _psz, _psz]),
    "mbx_host_alloc": (_i32, [_sz, _pvp]),
    "mbx_host_free": (_i32, [_vp]),
    "mbx_memcpy_h2d": (_i32, [_vp, _vp, _vp, _sz]),
    "mbx_memcpy_d2h": (_i32, [_vp, _vp, _vp, _sz]),
    "mbx_memcpy_d2d": (_i32, [_vp, _vp, _vp, _sz]),
    "mbx_param_create": (_i32, [_vp, _vp, _i32, _i64, _i64, _i64, _pvp]),
    "mbx_param_destroy": (None, [_vp, _vp]),
    "mbx_param_info": (_i32, [_vp, _pi64, _pi64, _pi64, _pi32]),
    "mbx_silu_inplace": (_i32, [_vp, _vp, _i64]),
    "mbx_add_inplace": (_i32, [_vp, _vp, _vp, _i64]),
    "mbx_bias_temb_add": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mbx_concat_channels": (_i32, [_vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "mbx_group_norm_affine": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp, _vp, _vp, _vp]),
    "mbx_group_norm_apply": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _i32, _vp, _vp]),
    "mbx_group_norm_forward": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp, _vp, _i32, _vp]),
    "mbx_group_norm_forward_noalloc": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _vp, _vp, _i32,
                                              _vp]),
    "mbx_layer_norm": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _f32, _vp]),
    "mbx_depthwise3x3": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _vp]),
    "mbx_depthwise3x3_fused": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _vp, _vp, _i32, _vp]),
    "mbx_conv1x1": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "mbx_conv3x3_output_hw": (_i32, [_i64, _i64, _i64, _pi64, _i32, _pi64, _pi64]),
    "mbx_conv3x3": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _pi64, _i32, _vp, _vp, _i32, _vp,
                           _vp]),
    "mbx_conv_group_norm_affine": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _pi64, _i32, _vp, _vp,
                                          _i32, _vp, _i32, _vp, _i64, _f32, _vp, _vp, _vp, _vp, _vp]),
    "mbx_matmul": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32]),
    "mbx_softmax_rows": (_i32, [_vp, _vp, _i64, _i64, _f32, _f32]),
    "mbx_gemm": (_i32, [_vp, _vp, _vp, _i64, _i64, _vp, _i64, _i32, _vp, _vp]),
    "mbx_scale_add": (_i32, [_vp, _vp, _i64, _f32, _f32, _vp]),
    "mbx_conv1x1_fused": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp]),
    "mbx_lambda_content": (_i32, [_vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mbx_self_lambda_position": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mbx_cross_lambda_position": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mbx_inpaint_prepare": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "mbx_vae_sample": (_i32, [_vp, _vp, _vp, _i64, _f32, _vp]),
    "mbx_latents_init": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _f32, _f32, _i32, _vp]),
    "mbx_unet_input": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "mbx_cfg_ddim_step": (_i32, [_vp, _vp, _i64, _i64, _i64, _f32, _pf32, _vp]),
    "mbx_gaussian_blur_u8": (_i32, [_vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp]),
    "mbx_feather_paste": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mbx_cfg_dpm_step": (_i32, [_vp, _vp, _i64, _i64, _i64, _f32, _pf32, _i32, _vp, _vp]),
    "mbx_dpm_coefficients": (_i32, [_u32, _f64, _i32, _i64, _i64, _pf32, _pi32]),
    "mbx_crop_window": (_i32, [_u32, _u32, _u32, _u32, _u32, _u32, _i64, _pi64, ctypes.POINTER(Rect)]),
    "mbx_lanczos_table": (_i32, [_i64, _i64, _pi32, _pi32, _pi64]),
    "mbx_mask_dilate": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "mbx_mask_bbox": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mbx_window_to_model": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                   _i64, _i64, _i64, _vp, _vp]),
    "mbx_model_to_window": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp]),
    "mbx_paste": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                         _i64, _vp, _u32, _vp]),
    # include/moebius_cuda_engine.h
    "mbx_engine_create": (_i32, [ctypes.c_char_p, _i32, _pvp]),
    "mbx_engine_destroy": (None, [_vp]),
    "mbx_engine_set_stream": (_i32, [_vp, _vp]),
    "mbx_engine_info": (_i32, [_vp, _pi64, _pi64, _pi64]),
    "mbx_engine_launch_count": (_u64, [_vp]),
    "mbx_inpaint": (_i32, [_vp, _vp, _u32, _u32, _u32, _u32, _vp, _u32, ctypes.POINTER(InpaintParams), PROGRESS_FN,
                           _vp, ctypes.POINTER(Rect)]),
    "mbx_inpaint_with_noise": (_i32, [_vp, _vp, _u32, _u32, _u32, _u32, _vp, _u32, ctypes.POINTER(InpaintParams),
                                      _vp, _vp, _vp, PROGRESS_FN, _vp, ctypes.POINTER(Rect)]),
    "mbx_inpaint_batch": (_i32, [_vp, _vp, _vp, _i64, _u32, _u32, ctypes.POINTER(InpaintParams), _vp, _vp, _vp,
                                 _i32, PROGRESS_FN, _vp]),
    "mbx_engine_unet_forward": (_i32, [_vp, _vp, _i64, _i64, _i32, _vp]),
    "mbx_engine_vae_encode": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "mbx_engine_vae_decode": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp]),
    "mbx_ddim_timesteps": (_i32, [_u32, _f64, _i32, _pi64, _pi64]),
    "mbx_ddim_alphas_cumprod": (_i32, [_pf32]),
}

# include/moebius_cpu.h: the reference's own C API names (a drop-in for moebius-cpu hosts).
COMPAT_SIGNATURES = {
    "moebius_abi_version": (ctypes.c_uint32, []),
    "moebius_last_error": (ctypes.c_char_p, []),
    "moebius_engine_create": (_i32, [ctypes.c_char_p, _u32, _pvp]),
    "moebius_engine_destroy": (None, [_vp]),
    "moebius_inpaint": (_i32, [_vp, _vp, _u32, _u32, _u32, _u32, _vp, _u32, ctypes.POINTER(InpaintParams),
                               PROGRESS_FN, _vp, ctypes.POINTER(Rect)]),
}

_lib = None


class MbxError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"moebius-cuda error {code}: {message}")
        self.code = code


def header_symbols() -> list[str]:
    """Function names declared in include/moebius_cuda.h and include/moebius_cuda_engine.h."""
    text = open(HEADER).read() + open(ENGINE_HEADER).read()
    return sorted(set(re.findall(r"\b(mbx_[a-z0-9_]+)\s*\(", text)) - {"mbx_progress_fn"})


def compat_header_symbols() -> list[str]:
    """Function names declared in include/moebius_cpu.h."""
    return sorted(set(re.findall(r"\b(moebius_[a-z0-9_]+)\s*\(", open(COMPAT_HEADER).read())))


def lib() -> ctypes.CDLL:
    """The loaded library with argtypes set. Raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C moebius-cpu_b200/csrc` "
                               "(or __graft_entry__.build()); there is no CPU fallback")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in {**SIGNATURES, **COMPAT_SIGNATURES}.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != OK:
        raise MbxError(status, lib().mbx_last_error().decode(errors="replace"))
