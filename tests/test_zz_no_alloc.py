"""mbx_group_norm_forward_noalloc: the GroupNorm entry point for callers that
cannot allocate device memory (hosts that plan every byte themselves, or code
on another framework's stream), whose scratch is a fixed array in the library.

Called through the C ABI and compared with mbx_group_norm_forward (which takes
its scratch from the context's pool) and with the CPU oracle's GroupNorm on two
calls in a row, with different shapes, so the second call cannot lean on the
first call's scratch contents. A warmed-up call leaves the device's free memory
(cudaMemGetInfo) unchanged: it allocates nothing. This file is collected last,
and passes on its own in a fresh process too.
"""
import ctypes

import numpy as np
import pytest

from conftest import scaled_err

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the scaled-error tolerance of the other GroupNorm tests


def _p(t):
    return ctypes.c_void_p(t.ptr) if t is not None else ctypes.c_void_p(0)


def _noalloc(mbx, ctx, x, groups, eps, gamma, beta, add, silu, out):
    n, h, w, c = x.shape
    return mbx.abi.lib().mbx_group_norm_forward_noalloc(ctypes.c_void_p(ctx.stream), _p(x), n, h, w, c, groups,
                                                        eps, _p(gamma), _p(beta), _p(add), int(silu), _p(out))


@pytest.mark.parametrize("silu", [True, False])
def test_noalloc_matches_pool_entry_point_twice(mbx, ctx, oracle, silu):
    rng = np.random.default_rng(2026)
    cases = [((2, 64, 64, 320), 32, 1e-5, True), ((8, 32, 32, 512), 32, 1e-6, False)]
    for shape, groups, eps, with_add in cases:
        n, c = shape[0], shape[-1]
        xh = (rng.standard_normal(shape) * 2 + 0.3).astype(np.float32)
        gh = rng.normal(1.0, 0.1, c).astype(np.float32)
        bh = rng.normal(0.0, 0.1, c).astype(np.float32)
        ah = rng.standard_normal((n, c)).astype(np.float32) if with_add else None
        x, gamma, beta = ctx.upload(xh), ctx.upload(gh), ctx.upload(bh)
        add = ctx.upload(ah) if with_add else None
        want = mbx.group_norm(x, groups, eps, gamma, beta, add=add, silu=silu).numpy()
        out = ctx.empty(shape)
        mbx.check(_noalloc(mbx, ctx, x, groups, eps, gamma, beta, add, silu, out))
        ctx.synchronize()
        got = out.numpy()
        assert scaled_err(got, want) <= TOL
        assert scaled_err(got, oracle.group_norm(xh, groups, eps, gh, bh, add=ah, silu=silu)) <= TOL


def test_noalloc_allocates_nothing(mbx, ctx):
    import torch
    rng = np.random.default_rng(7)
    shape = (4, 64, 64, 256)
    x = ctx.upload(rng.standard_normal(shape).astype(np.float32))
    g = ctx.upload(np.ones(256, np.float32))
    b = ctx.upload(np.zeros(256, np.float32))
    out = ctx.empty(shape)
    mbx.check(_noalloc(mbx, ctx, x, 32, 1e-6, g, b, None, True, out))  # warm-up: module and scratch resident
    ctx.synchronize()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(0)
    pool0 = ctx.pool_stats()
    for _ in range(3):
        mbx.check(_noalloc(mbx, ctx, x, 32, 1e-6, g, b, None, True, out))
    ctx.synchronize()
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0, "device memory changed across calls"
    assert ctx.pool_stats() == pool0


def test_noalloc_rejects_problems_beyond_its_scratch(mbx, ctx):
    x = ctx.upload(np.zeros((1, 4, 4, 64), np.float32))
    g = ctx.upload(np.ones(64, np.float32))
    # 64 items of 512x512 in 32 groups need 64 * 1024 * 32 * 16 B = 32 MiB of partials (> 8 MiB).
    st = mbx.abi.lib().mbx_group_norm_forward_noalloc(ctypes.c_void_p(ctx.stream), _p(x), 64, 512, 512, 64, 32,
                                                      1e-6, _p(g), _p(g), None, 1, _p(x))
    assert st == mbx.abi.ERR_INVALID_ARGUMENT
    assert b"maximum" in mbx.abi.lib().mbx_last_error()
    ctx.synchronize()
