"""moebius-cuda: the moebius-cpu engine kernel layer on B200 (sm_100a).

Python front end over the C ABI (``include/moebius_cuda.h``) used by the tests
and the benchmark. Device tensors are NHWC float32 buffers owned by a
``Context`` (its stream-ordered caching pool); every op is asynchronous on the
context stream and mirrors one reference engine call:

=====================  ==========================================================
``group_norm``         GroupNorm::forward (src/engine/norm.rs:41-53)
``group_norm_affine``  GroupNorm::affine (src/engine/norm.rs:57-105)
``group_norm_apply``   apply_affine (src/engine/norm.rs:134-147)
``layer_norm``         layer_norm (src/engine/norm.rs:151-172)
``depthwise3x3``       depthwise3x3 (src/engine/depthwise.rs:31-59)
``conv1x1``            Conv1x1::forward (src/engine/conv.rs:38-55)
``conv3x3``            Conv3x3::forward / forward_prologue / forward_im2col
                       (src/engine/conv.rs:83-130)
``silu_inplace``       ops::silu_inplace (src/engine/ops.rs:11-13)
``add_inplace``        ops::add_inplace (src/engine/ops.rs:16-19)
``concat_channels``    Tensor::concat_channels_into (src/engine/tensor.rs:59-73)
``bias_temb_add``      conv bias prefill + resnet temb add (src/engine/conv.rs:170-190,
                       src/unet/blocks.rs:98)
``matmul``             gemm::matmul (src/engine/gemm.rs:63-132)
=====================  ==========================================================

Import with ``importlib.import_module("moebius-cpu_b200")`` (the directory
name is not a Python identifier).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from . import abi
from .abi import MbxError, check, lib

__all__ = ["Context", "DeviceTensor", "Param", "MbxError", "abi", "group_norm", "group_norm_affine",
           "group_norm_apply", "layer_norm", "depthwise3x3", "conv1x1", "conv3x3", "conv3x3_output_hw",
           "silu_inplace", "add_inplace", "concat_channels", "bias_temb_add", "matmul", "conv_group_norm_affine",
           "EPILOGUES"]

EPILOGUES = {"none": abi.EPILOGUE_NONE, "relu": abi.EPILOGUE_RELU, "glu_silu": abi.EPILOGUE_GLU_SILU}


class Context:
    """One device, one stream, one caching pool (mbx_ctx)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().mbx_ctx_create(device, ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self) -> None:
        if self.handle:
            lib().mbx_ctx_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def synchronize(self) -> None:
        check(lib().mbx_ctx_synchronize(self.handle))

    def set_stream(self, stream_ptr: Optional[int]) -> None:
        check(lib().mbx_ctx_set_stream(self.handle, ctypes.c_void_p(stream_ptr or 0)))

    @property
    def stream(self) -> int:
        return lib().mbx_ctx_stream(self.handle) or 0

    @property
    def launch_count(self) -> int:
        return int(lib().mbx_ctx_launch_count(self.handle))

    def pool_stats(self) -> tuple[int, int]:
        cached, used = ctypes.c_size_t(), ctypes.c_size_t()
        check(lib().mbx_pool_stats(self.handle, ctypes.byref(cached), ctypes.byref(used)))
        return cached.value, used.value

    def release_below(self, min_bytes: int) -> None:
        check(lib().mbx_pool_release_below(self.handle, min_bytes))

    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        check(lib().mbx_alloc(self.handle, nbytes, ctypes.byref(p)))
        return p.value

    def free(self, ptr: int) -> None:
        check(lib().mbx_free(self.handle, ctypes.c_void_p(ptr)))

    def copy_h2d(self, dst: int, src_host: int, nbytes: int) -> None:
        check(lib().mbx_memcpy_h2d(self.handle, ctypes.c_void_p(dst), ctypes.c_void_p(src_host), nbytes))

    def copy_d2h(self, dst_host: int, src: int, nbytes: int) -> None:
        check(lib().mbx_memcpy_d2h(self.handle, ctypes.c_void_p(dst_host), ctypes.c_void_p(src), nbytes))

    @staticmethod
    def host_alloc(nbytes: int) -> int:
        """Page-locked host memory (mbx_host_alloc); release with host_free."""
        p = ctypes.c_void_p()
        check(lib().mbx_host_alloc(nbytes, ctypes.byref(p)))
        return p.value

    @staticmethod
    def host_free(ptr: int) -> None:
        check(lib().mbx_host_free(ctypes.c_void_p(ptr)))

    def empty(self, shape: Sequence[int], dtype=np.float32) -> "DeviceTensor":
        return DeviceTensor(self, tuple(int(s) for s in shape), dtype=dtype)

    def upload(self, arr, dtype=np.float32) -> "DeviceTensor":
        """Copies a host array to a new device buffer (float32 unless `dtype` says otherwise)."""
        a = np.ascontiguousarray(arr, dtype=dtype)
        t = DeviceTensor(self, a.shape, dtype=a.dtype)
        if a.size:
            check(lib().mbx_memcpy_h2d(self.handle, ctypes.c_void_p(t.ptr), a.ctypes.data_as(ctypes.c_void_p),
                                       a.nbytes))
        return t


class DeviceTensor:
    """A device buffer from the context's pool, with a shape (float32 NHWC unless `dtype` says otherwise)."""

    def __init__(self, ctx: Context, shape: tuple, ptr: Optional[int] = None, dtype=np.float32):
        self.ctx = ctx
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)
        self.size = int(np.prod(self.shape)) if self.shape else 1
        self.nbytes = self.dtype.itemsize * self.size
        self.owned = ptr is None
        self.ptr = ctx.alloc(self.nbytes) if ptr is None else int(ptr)

    @classmethod
    def wrap(cls, ctx: Context, ptr: int, shape: Sequence[int], dtype=np.float32) -> "DeviceTensor":
        """A view of caller-owned device memory (e.g. a torch tensor's data_ptr()); never freed here."""
        return cls(ctx, tuple(int(s) for s in shape), ptr=ptr, dtype=dtype)

    def __del__(self):
        # Owned blocks go back to the context's pool (stream-ordered, so safe while queued
        # kernels still read them: only later work on the same stream can reuse the block).
        try:
            if self.ptr and self.owned and self.ctx.handle:
                self.ctx.free(self.ptr)
                self.ptr = 0
        except Exception:
            pass

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        if self.size:
            check(lib().mbx_memcpy_d2h(self.ctx.handle, out.ctypes.data_as(ctypes.c_void_p),
                                       ctypes.c_void_p(self.ptr), self.nbytes))
        self.ctx.synchronize()
        return out

    def free(self) -> None:
        if self.ptr and self.owned:
            self.ctx.free(self.ptr)
        self.ptr = 0

    @property
    def vp(self) -> ctypes.c_void_p:
        return ctypes.c_void_p(self.ptr)


class Param:
    """A dense conv weight (Param, src/engine/param.rs): [c_out, c_in] or [c_out, 3, 3, c_in]."""

    def __init__(self, ctx: Context, weight, dtype: str = "f32"):
        w = np.asarray(weight)
        if w.ndim == 2:
            c_out, taps, c_in = w.shape[0], 1, w.shape[1]
        elif w.ndim == 4 and w.shape[1:3] == (3, 3):
            c_out, taps, c_in = w.shape[0], 9, w.shape[3]
        else:
            raise ValueError("weight must be [c_out, c_in] or [c_out, 3, 3, c_in]")
        if dtype == "f16":
            data = np.ascontiguousarray(w, dtype=np.float16)
            code = abi.DTYPE_F16
        elif dtype == "f32":
            data = np.ascontiguousarray(w, dtype=np.float32)
            code = abi.DTYPE_F32
        else:
            raise ValueError("dtype must be 'f32' or 'f16'")
        h = ctypes.c_void_p()
        check(lib().mbx_param_create(ctx.handle, data.ctypes.data_as(ctypes.c_void_p), code, c_out, taps, c_in,
                                     ctypes.byref(h)))
        self.ctx, self.handle = ctx, h
        self.c_out, self.taps, self.c_in, self.dtype = c_out, taps, c_in, dtype

    def close(self) -> None:
        if self.handle:
            lib().mbx_param_destroy(self.ctx.handle, self.handle)
            self.handle = None


def _vp(t: Optional[DeviceTensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.ptr) if t is not None else ctypes.c_void_p(0)


def _nhwc(x: DeviceTensor):
    if len(x.shape) != 4:
        raise ValueError("expected an NHWC tensor")
    return x.shape


def silu_inplace(x: DeviceTensor) -> DeviceTensor:
    check(lib().mbx_silu_inplace(x.ctx.handle, x.vp, x.size))
    return x


def add_inplace(a: DeviceTensor, b: DeviceTensor) -> DeviceTensor:
    if a.size != b.size:
        raise ValueError("add length mismatch")
    check(lib().mbx_add_inplace(a.ctx.handle, a.vp, b.vp, a.size))
    return a


def bias_temb_add(x: DeviceTensor, bias: Optional[DeviceTensor] = None, temb: Optional[DeviceTensor] = None,
                  out: Optional[DeviceTensor] = None) -> DeviceTensor:
    n, c = x.shape[0], x.shape[-1]
    out = out or x.ctx.empty(x.shape)
    check(lib().mbx_bias_temb_add(x.ctx.handle, x.vp, n, x.size // (n * c), c, _vp(bias), _vp(temb), out.vp))
    return out


def concat_channels(a: DeviceTensor, b: DeviceTensor, out: Optional[DeviceTensor] = None) -> DeviceTensor:
    if a.shape[:-1] != b.shape[:-1]:
        raise ValueError("concat_channels: spatial shapes differ")
    ca, cb = a.shape[-1], b.shape[-1]
    out = out or a.ctx.empty(a.shape[:-1] + (ca + cb,))
    check(lib().mbx_concat_channels(a.ctx.handle, a.vp, ca, b.vp, cb, a.size // ca, out.vp))
    return out


def group_norm_affine(x: DeviceTensor, groups: int, eps: float, gamma: DeviceTensor, beta: DeviceTensor,
                      add: Optional[DeviceTensor] = None):
    n, h, w, c = _nhwc(x)
    scale, shift = x.ctx.empty((n, c)), x.ctx.empty((n, c))
    check(lib().mbx_group_norm_affine(x.ctx.handle, x.vp, n, h, w, c, groups, eps, gamma.vp, beta.vp, _vp(add),
                                      scale.vp, shift.vp))
    return scale, shift


def group_norm_apply(x: DeviceTensor, scale: DeviceTensor, shift: DeviceTensor, silu: bool = False,
                     residual: Optional[DeviceTensor] = None, out: Optional[DeviceTensor] = None) -> DeviceTensor:
    n, c = x.shape[0], x.shape[-1]
    out = out or x.ctx.empty(x.shape)
    check(lib().mbx_group_norm_apply(x.ctx.handle, x.vp, n, x.size // (n * c), c, scale.vp, shift.vp, int(silu),
                                     _vp(residual), out.vp))
    return out


def group_norm(x: DeviceTensor, groups: int, eps: float, gamma: DeviceTensor, beta: DeviceTensor,
               add: Optional[DeviceTensor] = None, silu: bool = False,
               out: Optional[DeviceTensor] = None) -> DeviceTensor:
    n, h, w, c = _nhwc(x)
    out = out or x.ctx.empty(x.shape)
    check(lib().mbx_group_norm_forward(x.ctx.handle, x.vp, n, h, w, c, groups, eps, gamma.vp, beta.vp, _vp(add),
                                       int(silu), out.vp))
    return out


def layer_norm(x: DeviceTensor, gamma: DeviceTensor, beta: DeviceTensor, eps: float,
               out: Optional[DeviceTensor] = None) -> DeviceTensor:
    c = x.shape[-1]
    out = out or x.ctx.empty(x.shape)
    check(lib().mbx_layer_norm(x.ctx.handle, x.vp, x.size // c, c, gamma.vp, beta.vp, eps, out.vp))
    return out


def depthwise3x3(x: DeviceTensor, weight: DeviceTensor, bias: DeviceTensor, epilogue: str = "none",
                 out: Optional[DeviceTensor] = None, prologue=None) -> DeviceTensor:
    """prologue = (scale [n, c], shift [n, c], silu): the input is read as [SiLU](x*scale + shift)."""
    n, h, w, c = _nhwc(x)
    ep = EPILOGUES[epilogue]
    out = out or x.ctx.empty((n, h, w, c // 2 if ep == abi.EPILOGUE_GLU_SILU else c))
    if prologue is None:
        check(lib().mbx_depthwise3x3(x.ctx.handle, x.vp, n, h, w, c, weight.vp, bias.vp, ep, out.vp))
    else:
        sc, sh, silu = prologue
        check(lib().mbx_depthwise3x3_fused(x.ctx.handle, x.vp, n, h, w, c, sc.vp, sh.vp, int(silu), weight.vp,
                                           bias.vp, ep, out.vp))
    return out


def conv1x1(x: DeviceTensor, weight: Param, bias: Optional[DeviceTensor] = None,
            residual: Optional[DeviceTensor] = None, out: Optional[DeviceTensor] = None) -> DeviceTensor:
    n, h, w, c = _nhwc(x)
    out = out or x.ctx.empty((n, h, w, weight.c_out))
    check(lib().mbx_conv1x1(x.ctx.handle, x.vp, n, h, w, c, weight.handle, _vp(bias), _vp(residual), out.vp))
    return out


def conv3x3_output_hw(h: int, w: int, stride: int = 1, pad=(1, 1, 1, 1), upsample2x: bool = False):
    ho, wo = ctypes.c_int64(), ctypes.c_int64()
    p = (ctypes.c_int64 * 4)(*pad)
    check(lib().mbx_conv3x3_output_hw(h, w, stride, p, int(upsample2x), ctypes.byref(ho), ctypes.byref(wo)))
    return ho.value, wo.value


def conv3x3(x: DeviceTensor, weight: Param, bias: Optional[DeviceTensor] = None, stride: int = 1,
            pad=(1, 1, 1, 1), upsample2x: bool = False, prologue=None, residual: Optional[DeviceTensor] = None,
            out: Optional[DeviceTensor] = None) -> DeviceTensor:
    """prologue = (scale [n, c_in], shift [n, c_in], silu) device tensors, or None."""
    n, h, w, c = _nhwc(x)
    ho, wo = conv3x3_output_hw(h, w, stride, pad, upsample2x)
    out = out or x.ctx.empty((n, ho, wo, weight.c_out))
    p = (ctypes.c_int64 * 4)(*pad)
    ps, pz, silu = (None, None, 0) if prologue is None else (prologue[0], prologue[1], int(prologue[2]))
    check(lib().mbx_conv3x3(x.ctx.handle, x.vp, n, h, w, c, weight.handle, _vp(bias), stride, p, int(upsample2x),
                            _vp(ps), _vp(pz), silu, _vp(residual), out.vp))
    return out


def conv_group_norm_affine(x: DeviceTensor, weight: Param, groups: int, eps: float, gamma: DeviceTensor,
                          beta: DeviceTensor, bias: Optional[DeviceTensor] = None, add: Optional[DeviceTensor] = None,
                          stride: int = 1, pad=(1, 1, 1, 1), upsample2x: bool = False, prologue=None,
                          residual: Optional[DeviceTensor] = None, act: int = abi.ACT_NONE,
                          out: Optional[DeviceTensor] = None):
    """A 1x1 or 3x3 conv (by the weight's taps) plus the GroupNorm affine of its output from statistics
    gathered in the conv's epilogue (mbx_conv_group_norm_affine): returns (out, scale [n, c_out],
    shift [n, c_out])."""
    n, h, w, c = _nhwc(x)
    ho, wo = conv3x3_output_hw(h, w, stride, pad, upsample2x) if weight.taps == 9 else (h, w)
    out = out or x.ctx.empty((n, ho, wo, weight.c_out))
    scale, shift = x.ctx.empty((n, weight.c_out)), x.ctx.empty((n, weight.c_out))
    p = (ctypes.c_int64 * 4)(*pad)
    ps, pz, silu = (None, None, 0) if prologue is None else (prologue[0], prologue[1], int(prologue[2]))
    check(lib().mbx_conv_group_norm_affine(x.ctx.handle, x.vp, n, h, w, c, weight.handle, _vp(bias), stride, p,
                                           int(upsample2x), _vp(ps), _vp(pz), silu, _vp(residual), int(act), out.vp,
                                           groups, eps, gamma.vp, beta.vp, _vp(add), scale.vp, shift.vp))
    return out, scale, shift


def matmul(a: DeviceTensor, b: DeviceTensor, c: Optional[DeviceTensor] = None,
           accumulate: bool = False) -> DeviceTensor:
    """c (+)= a @ b for dense row-major 2-D device tensors."""
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    c = c or a.ctx.empty((m, n))
    check(lib().mbx_matmul(a.ctx.handle, c.vp, a.vp, m, k, k, 1, b.vp, n, n, 1, int(accumulate)))
    return c


from . import engine, synthetic  # noqa: E402  (engine API; seeded converter-format weights)
