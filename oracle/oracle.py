"""TEST INFRASTRUCTURE ONLY: numpy front end of the CPU oracle (``liboracle.so``).

The oracle restates the moebius-cpu engine kernels (reference ``src/engine/*.rs``)
on the CPU; ``ref_engine.cpp`` cites the reference lines per function. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU baseline and
``--impl reference`` arm) import this module. The product package never does.

All arrays are float32, C-contiguous, NHWC. Functions allocate and return their
outputs, mirroring the reference's "kernel reshapes `out`" convention.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def build() -> str:
    """Compiles liboracle.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.ora_exp.restype = ctypes.c_float
        _lib.ora_exp.argtypes = [ctypes.c_float]
        _lib.ora_silu.restype = ctypes.c_float
        _lib.ora_silu.argtypes = [ctypes.c_float]
        _lib.ora_get_threads.restype = ctypes.c_int
        _lib.ora_layer_norm.argtypes = [_f, _i64, _i64, _f, _f, ctypes.c_float, _f]
        _lib.ora_group_norm_affine.argtypes = [_f, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _f, _f, _f, _f, _f]
        _lib.ora_group_norm_forward.argtypes = [_f, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _f, _f, _f,
                                                ctypes.c_int, _f]
        _ci = ctypes.c_int
        _pad = ctypes.POINTER(ctypes.c_int64)
        _lib.ora_set_threads.argtypes = [_ci]
        _lib.ora_silu_inplace.argtypes = [_f, _i64]
        _lib.ora_add_inplace.argtypes = [_f, _f, _i64]
        _lib.ora_bias_temb_add.argtypes = [_f, _i64, _i64, _i64, _f, _f, _f]
        _lib.ora_concat_channels.argtypes = [_f, _i64, _f, _i64, _i64, _f]
        _lib.ora_group_norm_apply.argtypes = [_f, _i64, _i64, _i64, _f, _f, _ci, _f]
        _lib.ora_depthwise3x3.argtypes = [_f, _i64, _i64, _i64, _i64, _f, _f, _ci, _f]
        _lib.ora_conv1x1.argtypes = [_f, _i64, _i64, _f, _i64, _f, _f, _f]
        conv_args = [_f, _i64, _i64, _i64, _i64, _f, _i64, _f, _i64, _pad, _ci, _f, _f, _ci, _f]
        _lib.ora_conv3x3.argtypes = conv_args
        _lib.ora_conv3x3_im2col.argtypes = conv_args
        _lib.ora_matmul.argtypes = [_f, _f, _i64, _i64, _i64, _i64, _f, _i64, _i64, _i64, _ci]
        _lib.ora_gemm_nt.argtypes = [_i64, _i64, _i64, _f, _f, _f, _ci]
        _lib.ora_softmax_rows.argtypes = [_f, _i64, _i64, ctypes.c_float]
        _lib.ora_softmax_lambda.argtypes = [_f, _f, _i64, _i64, _i64, _f]
        _lib.ora_tap_filter.argtypes = [_f, _f, _f, _i64, _i64, _i64]
        _lib.ora_position_term.argtypes = [_f, _f, _f, _f, _i64, _i64]
        _lib.ora_timestep_sinusoid.argtypes = [_i64, _i64, _f]
        _lib.ora_vae_sample.argtypes = [_f, _f, _i64, _f]
    return _lib


def set_threads(n: int = 0) -> int:
    """Sets the OpenMP thread count (0 = all cores); returns the count in use."""
    lib().ora_set_threads(int(n))
    return lib().ora_get_threads()


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "oracle wants contiguous float32"
    return a.ctypes.data_as(_f)


def _c(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def exp(x: float) -> float:
    return lib().ora_exp(x)


def silu_scalar(x: float) -> float:
    return lib().ora_silu(x)


def silu(x):
    y = _c(x).copy()
    lib().ora_silu_inplace(_p(y), _i64(y.size))
    return y


def add(a, b):
    y = _c(a).copy()
    b = _c(b)
    assert y.size == b.size
    lib().ora_add_inplace(_p(y), _p(b), _i64(y.size))
    return y


def bias_temb_add(x, bias=None, temb=None):
    x = _c(x)
    n, c = x.shape[0], x.shape[-1]
    out = np.empty_like(x)
    lib().ora_bias_temb_add(_p(x), _i64(n), _i64(x.size // (n * c)), _i64(c), _p(_c(bias)), _p(_c(temb)), _p(out))
    return out


def concat_channels(a, b):
    a, b = _c(a), _c(b)
    assert a.shape[:-1] == b.shape[:-1]
    out = np.empty(a.shape[:-1] + (a.shape[-1] + b.shape[-1],), np.float32)
    pixels = a.size // a.shape[-1]
    lib().ora_concat_channels(_p(a), _i64(a.shape[-1]), _p(b), _i64(b.shape[-1]), _i64(pixels), _p(out))
    return out


def group_norm_affine(x, groups, eps, gamma, beta, add=None):
    """GroupNorm::affine: returns (scale [n,c], shift [n,c])."""
    x = _c(x)
    n, h, w, c = x.shape
    scale = np.empty((n, c), np.float32)
    shift = np.empty((n, c), np.float32)
    lib().ora_group_norm_affine(_p(x), n, h, w, c, groups, eps, _p(_c(gamma)), _p(_c(beta)), _p(_c(add)),
                                _p(scale), _p(shift))
    return scale, shift


def group_norm_apply(x, scale, shift, silu=False):
    x = _c(x)
    n, c = x.shape[0], x.shape[-1]
    out = np.empty_like(x)
    lib().ora_group_norm_apply(_p(x), _i64(n), _i64(x.size // (n * c)), _i64(c), _p(_c(scale)), _p(_c(shift)),
                               ctypes.c_int(int(silu)), _p(out))
    return out


def group_norm(x, groups, eps, gamma, beta, add=None, silu=False):
    """GroupNorm::forward."""
    x = _c(x)
    n, h, w, c = x.shape
    out = np.empty_like(x)
    lib().ora_group_norm_forward(_p(x), n, h, w, c, groups, eps, _p(_c(gamma)), _p(_c(beta)), _p(_c(add)),
                                 int(silu), _p(out))
    return out


def layer_norm(x, gamma, beta, eps):
    x = _c(x)
    c = x.shape[-1]
    out = np.empty_like(x)
    lib().ora_layer_norm(_p(x), x.size // c, c, _p(_c(gamma)), _p(_c(beta)), eps, _p(out))
    return out


EPILOGUES = {"none": 0, "relu": 1, "glu_silu": 2}


def depthwise3x3(x, weight, bias, epilogue="none"):
    x = _c(x)
    n, h, w, c = x.shape
    ep = EPILOGUES[epilogue]
    out = np.empty((n, h, w, c // 2 if ep == 2 else c), np.float32)
    lib().ora_depthwise3x3(_p(x), _i64(n), _i64(h), _i64(w), _i64(c), _p(_c(weight)), _p(_c(bias)),
                           ctypes.c_int(ep), _p(out))
    return out


def conv1x1(x, weight, bias=None, residual=None):
    """Conv1x1::forward: weight [c_out, c_in]."""
    x = _c(x)
    c_in = x.shape[-1]
    c_out = weight.shape[0]
    out = np.empty(x.shape[:-1] + (c_out,), np.float32)
    lib().ora_conv1x1(_p(x), _i64(x.size // c_in), _i64(c_in), _p(_c(weight)), _i64(c_out), _p(_c(bias)),
                      _p(_c(residual)), _p(out))
    return out


def conv3x3_output_hw(h, w, stride=1, pad=(1, 1, 1, 1), upsample2x=False):
    up = 2 if upsample2x else 1
    return (h * up + pad[0] + pad[2] - 3) // stride + 1, (w * up + pad[1] + pad[3] - 3) // stride + 1


def conv3x3(x, weight, bias=None, stride=1, pad=(1, 1, 1, 1), upsample2x=False, prologue=None, im2col=False):
    """Conv3x3::forward / forward_prologue / forward_im2col.

    weight [c_out, 3, 3, c_in]; prologue = (scale [n,c_in], shift [n,c_in], silu) or None.
    """
    x = _c(x)
    n, h, w, c_in = x.shape
    c_out = weight.shape[0]
    ho, wo = conv3x3_output_hw(h, w, stride, pad, upsample2x)
    out = np.empty((n, ho, wo, c_out), np.float32)
    pad_arr = (ctypes.c_int64 * 4)(*pad)
    ps, pz, psilu = (None, None, 0) if prologue is None else (_c(prologue[0]), _c(prologue[1]), int(prologue[2]))
    fn = lib().ora_conv3x3_im2col if im2col else lib().ora_conv3x3
    fn(_p(x), _i64(n), _i64(h), _i64(w), _i64(c_in), _p(_c(weight)), _i64(c_out), _p(_c(bias)), _i64(stride),
       pad_arr, ctypes.c_int(int(upsample2x)), _p(ps), _p(pz), ctypes.c_int(psilu), _p(out))
    return out


def matmul(a, b, c=None):
    """c (+)= a @ b for dense 2-D float32 arrays (gemm::matmul)."""
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[1]
    acc = c is not None
    out = _c(c).copy() if acc else np.empty((m, n), np.float32)
    lib().ora_matmul(_p(out), _p(a), _i64(m), _i64(k), _i64(k), _i64(1), _p(b), _i64(n), _i64(n), _i64(1),
                     ctypes.c_int(int(acc)))
    return out


def gemm_nt(a, b):
    """a [m, k] @ b[n, k]^T (the engine GEMM with a transposed weight view)."""
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[0]
    out = np.empty((m, n), np.float32)
    lib().ora_gemm_nt(m, n, k, _p(a), _p(b), _p(out), 0)
    return out


def softmax_rows(x, scale):
    """softmax_rows (src/vae/mod.rs:279-293) on a copy of the 2-D array x."""
    y = _c(x).copy()
    lib().ora_softmax_rows(_p(y), y.shape[0], y.shape[1], scale)
    return y


def softmax_lambda(keys, v):
    """softmax_lambda (src/unet/lambda.rs:318-359): keys [rows, k], v [rows, vd] -> [k, vd]."""
    keys = _c(keys).copy()
    v = _c(v)
    rows, k = keys.shape
    vd = v.shape[1]
    lam = np.empty((k, vd), np.float32)
    lib().ora_softmax_lambda(_p(keys), _p(v), rows, k, vd, _p(lam))
    return lam


def tap_filter(a, v, o, hh, ww):
    """tap_filter (src/unet/lambda.rs:154-184) into o [hw, 8·vd] in place; a [hw·8, 226], v [hw, vd]."""
    a, v = _c(a), _c(v)
    assert o.dtype == np.float32 and o.flags["C_CONTIGUOUS"]
    lib().ora_tap_filter(_p(a), _p(v), _p(o), hh, ww, v.shape[-1])
    return o


def position_term(q, e, v, o):
    """position_term (src/unet/lambda.rs:276-295) into o [hw, 8k] in place."""
    q, e, v = _c(q), _c(e), _c(v)
    assert o.dtype == np.float32 and o.flags["C_CONTIGUOUS"]
    k = v.shape[-1]
    lib().ora_position_term(_p(q), _p(e), _p(v), _p(o), q.size // (8 * k), k)
    return o


def timestep_sinusoid(t, dim):
    out = np.empty(dim, np.float32)
    lib().ora_timestep_sinusoid(int(t), dim, _p(out))
    return out


def vae_sample(moments, noise):
    """sample (src/vae/encoder.rs:219-230): moments [..., 8], noise [..., 4] -> z [..., 4]."""
    moments, noise = _c(moments), _c(noise)
    z = np.empty_like(noise)
    lib().ora_vae_sample(_p(moments), _p(noise), noise.size // 4, _p(z))
    return z
