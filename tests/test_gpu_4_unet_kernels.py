"""GPU parity of the UNet- and pipeline-specific kernels against the CPU oracle
the λ layers (src/unet/lambda.rs), the fused 1×1 conv
(GroupNorm prologue, SiLU epilogue), and the per-inpaint element kernels
(src/pipeline.rs, src/scheduler.rs, src/vae/encoder.rs, src/imaging/*).
Gates: ≤ 1e-5 relative for the f32 λ arithmetic, bit-exact for the integer /
byte work and for the element kernels written in the reference's operation
order."""
import ctypes

import numpy as np
import pytest

from conftest import load_golden, max_rel_err, scaled_err

pytestmark = pytest.mark.gpu


def _at(t, byte_offset):
    return ctypes.c_void_p(t.ptr + byte_offset)


@pytest.mark.parametrize("items,rows,k", [(2, 4096, 40), (3, 1024, 80), (2, 256, 160), (2, 10, 8), (1, 300, 24)])
def test_lambda_content(mbx, ctx, oracle, items, rows, k):
    rng = np.random.default_rng(rows + k)
    kv = (rng.standard_normal((items, rows, 2 * k)) * 2).astype(np.float32)
    d = ctx.upload(kv)
    lam = ctx.empty((items, k, k))
    mbx.check(mbx.abi.lib().mbx_lambda_content(ctx.handle, d.vp, 2 * k, _at(d, 4 * k), 2 * k, items, rows, k, k,
                                                 lam.vp))
    got = lam.numpy()
    for b in range(items):
        want = oracle.softmax_lambda(kv[b, :, :k], kv[b, :, k:])
        assert max_rel_err(got[b], want) <= 1e-5


def _self_case(rng, n, h, w, k):
    c = 8 * k
    q = rng.standard_normal((n, h, w, c)).astype(np.float32)
    kv = rng.standard_normal((n, h, w, 2 * k)).astype(np.float32)
    lam = (rng.standard_normal((n, k, k)) * 0.2).astype(np.float32)
    waug = (rng.standard_normal((k, 226)) / 15).astype(np.float32)
    return q, kv, lam, waug


@pytest.mark.parametrize("n,h,w,k", [(2, 64, 64, 40), (2, 32, 32, 80), (2, 16, 16, 160), (1, 13, 10, 8),
                                     (2, 5, 4, 16), (1, 9, 9, 32)])
def test_self_lambda_position(mbx, ctx, oracle, n, h, w, k):
    rng = np.random.default_rng(n * h * w + k)
    q, kv, lam, waug = _self_case(rng, n, h, w, k)
    c, hw = 8 * k, h * w
    out0 = rng.standard_normal((n, h, w, c)).astype(np.float32)
    a = np.zeros((n * hw * 8, 228), np.float32)
    a[:, :226] = oracle.gemm_nt(q.reshape(-1, k), np.ascontiguousarray(waug.T))
    qd, kvd, lamd, ad, out = (ctx.upload(t) for t in (q, kv, lam, a, out0))
    mbx.check(mbx.abi.lib().mbx_self_lambda_position(ctx.handle, qd.vp, lamd.vp, ad.vp, 228, _at(kvd, 4 * k), 2 * k,
                                                       n, h, w, k, out.vp))
    got = out.numpy()
    for b in range(n):
        o = oracle.gemm_nt(q[b].reshape(hw * 8, k), np.ascontiguousarray(lam[b].T))
        ab = np.ascontiguousarray(a[b * hw * 8:(b + 1) * hw * 8, :226])
        oracle.tap_filter(ab, np.ascontiguousarray(kv[b].reshape(hw, 2 * k)[:, k:]), o, h, w)
        assert max_rel_err(got[b] - out0[b], o.reshape(h, w, c)) <= 1e-5


@pytest.mark.parametrize("n,hw,k,period", [(4, 4096, 40, 2), (2, 1024, 80, 2), (2, 256, 160, 1), (3, 64, 8, 2),
                                           (2, 100, 24, 2)])
def test_cross_lambda_position(mbx, ctx, oracle, n, hw, k, period):
    rng = np.random.default_rng(hw + k + period)
    c = 8 * k
    q = rng.standard_normal((n, hw, c)).astype(np.float32)
    e = (rng.standard_normal((hw, 10, k)) / np.sqrt(k)).astype(np.float32)
    lam = (rng.standard_normal((2, k, k)) * 0.2).astype(np.float32)
    vt = rng.standard_normal((2, 10, k)).astype(np.float32)
    out0 = rng.standard_normal((n, hw, c)).astype(np.float32)
    qd, ed, lamd, vd, out = (ctx.upload(t) for t in (q, e, lam, vt, out0))
    first = 1 if period == 1 else 0  # cond-only batches read the cond tables
    mbx.check(mbx.abi.lib().mbx_cross_lambda_position(ctx.handle, qd.vp, ed.vp, _at(lamd, first * 4 * k * k),
                                                        _at(vd, first * 4 * 10 * k), period, n, hw, k, out.vp))
    got = out.numpy()
    for b in range(n):
        br = 1 if period == 1 else b % 2
        o = oracle.gemm_nt(q[b].reshape(hw * 8, k), np.ascontiguousarray(lam[br].T))
        oracle.position_term(q[b], e, vt[br], o)
        assert max_rel_err(got[b] - out0[b], o.reshape(hw, c)) <= 1e-5


@pytest.mark.parametrize("n,h,w,ci,co,wdtype,res", [(2, 16, 16, 64, 96, "f32", True), (3, 7, 9, 40, 33, "f32", False),
                                                    (2, 20, 20, 128, 160, "f16", True)])
def test_conv1x1_fused_prologue_and_silu(mbx, ctx, oracle, n, h, w, ci, co, wdtype, res):
    rng = np.random.default_rng(ci + co)
    x = rng.standard_normal((n, h, w, ci)).astype(np.float32)
    scale = (rng.standard_normal((n, ci)) * 0.5 + 1).astype(np.float32)
    shift = (rng.standard_normal((n, ci)) * 0.3).astype(np.float32)
    wt = (rng.standard_normal((co, ci)) / np.sqrt(ci)).astype(np.float32)
    if wdtype == "f16":
        wt = wt.astype(np.float16).astype(np.float32)
    bias = (rng.standard_normal(co) * 0.1).astype(np.float32)
    r = rng.standard_normal((n, h, w, co)).astype(np.float32) if res else None
    p = mbx.Param(ctx, wt, wdtype)
    xd, sd, td, bd = ctx.upload(x), ctx.upload(scale), ctx.upload(shift), ctx.upload(bias)
    rd = ctx.upload(r) if res else None
    out = ctx.empty((n, h, w, co))
    mbx.check(mbx.abi.lib().mbx_conv1x1_fused(ctx.handle, xd.vp, n, h, w, ci, p.handle, bd.vp, sd.vp, td.vp, 1,
                                                rd.vp if res else None, mbx.abi.ACT_SILU, out.vp))
    got = out.numpy()
    p.close()
    y = oracle.group_norm_apply(x, scale, shift, silu=True)
    want = oracle.silu(oracle.conv1x1(y, wt, bias, r))
    assert max_rel_err(got, want) <= 1e-5
    assert scaled_err(got, want) <= 1e-4


def _ellipse(side, cy, cx, ry, rx):
    yy, xx = np.mgrid[:side, :side]
    return ((((yy - cy) / ry) ** 2 + ((xx - cx) / rx) ** 2) <= 1).astype(np.uint8) * 255


@pytest.mark.parametrize("ch", [3, 4])
def test_inpaint_prepare_matches_to_model(mbx, ctx, ch):
    from oracle.imaging_ref import to_model
    rng = np.random.default_rng(ch)
    n, s = 3, 64
    img = rng.integers(0, 256, (n, s, s, ch), dtype=np.uint8)
    masks = np.stack([_ellipse(s, 30, 20, 10, 15), np.zeros((s, s), np.uint8),
                      rng.integers(0, 256, (s, s), dtype=np.uint8)])
    imd, md = ctx.upload(img, np.uint8), ctx.upload(masks, np.uint8)
    images, binary = ctx.empty((2 * n, s, s, 3)), ctx.empty((n, s, s), np.uint8)
    lat, flags = ctx.empty((n, s // 8, s // 8)), ctx.empty((n,), np.int32)
    mbx.check(mbx.abi.lib().mbx_inpaint_prepare(ctx.handle, imd.vp, md.vp, n, s, s, ch, images.vp, binary.vp, lat.vp,
                                                  flags.vp))
    gi, gb, gl = images.numpy(), binary.numpy(), lat.numpy()
    for i in range(n):
        rgb, b = to_model(img[i], masks[i])
        keep = np.where(b >= 128, np.float32(0), np.float32(1))
        assert np.array_equal(gi[2 * i], rgb) and np.array_equal(gi[2 * i + 1], rgb * keep[..., None])
        assert np.array_equal(gb[i], b)
        assert np.array_equal(gl[i], (b[::8, ::8] >= 128).astype(np.float32))
    assert list(flags.numpy()) == [1, 0, 1]


@pytest.mark.parametrize("case", ["a", "b", "c", "e1", "e2"])
def test_gaussian_blur_byte_exact(mbx, ctx, case):
    f = load_golden("imaging_ref.safetensors")
    m = f[f"{case}.mask"].astype(np.uint8)
    h, w = m.shape
    md, out, scratch = ctx.upload(m, np.uint8), ctx.empty((h, w), np.uint8), ctx.empty((h, w), np.uint8)
    mbx.check(mbx.abi.lib().mbx_gaussian_blur_u8(ctx.handle, md.vp, 1, h, w, ctypes.c_float(3.0), scratch.vp,
                                                   out.vp))
    assert np.array_equal(out.numpy(), f[f"{case}.blurred"].astype(np.uint8))


def test_feather_paste_byte_exact(mbx, ctx):
    from oracle.imaging_ref import feather_paste, pil_gaussian_blur
    rng = np.random.default_rng(9)
    n, s = 3, 96
    img = rng.integers(0, 256, (n, s, s, 4), dtype=np.uint8)
    masks = np.stack([_ellipse(s, 40, 50, 20, 30), _ellipse(s, 10, 90, 30, 12), np.zeros((s, s), np.uint8)])
    dec = (rng.random((n, s, s, 3)) * 1.2 - 0.1).astype(np.float32)
    blurred = np.stack([pil_gaussian_blur(np.where(m >= 128, 255, 0).astype(np.uint8)) for m in masks])
    flags = np.array([1, 1, 0], np.int32)
    imd, decd = ctx.upload(img, np.uint8), ctx.upload(dec)
    bd, fd = ctx.upload(blurred, np.uint8), ctx.upload(flags, np.int32)
    mbx.check(mbx.abi.lib().mbx_feather_paste(ctx.handle, decd.vp, bd.vp, imd.vp, n, s, s, 4, fd.vp))
    got = imd.numpy()
    from oracle.imaging_ref import to_u8
    for i in range(2):
        assert np.array_equal(got[i], feather_paste(img[i], masks[i], to_u8(dec[i])))
    assert np.array_equal(got[2], img[2]), "an empty mask leaves the image untouched"
    assert np.array_equal(got[..., 3], img[..., 3]), "alpha is preserved"


def test_vae_sample(mbx, ctx, oracle):
    rng = np.random.default_rng(4)
    mom = (rng.standard_normal((2, 16, 16, 8)) * 3).astype(np.float32)
    mom[0, 0, 0, 4:] = [-100, 100, -30, 20]  # logvar clamp edges
    noise = rng.standard_normal((2, 16, 16, 4)).astype(np.float32)
    z = ctx.empty((2, 16, 16, 4))
    md, nd = ctx.upload(mom), ctx.upload(noise)  # held: a dropped buffer returns to the pool at once
    mbx.check(mbx.abi.lib().mbx_vae_sample(ctx.handle, md.vp, nd.vp, 2 * 256, ctypes.c_float(0.13025), z.vp))
    assert max_rel_err(z.numpy(), oracle.vae_sample(mom, noise)) <= 1e-6


def test_latents_init_unet_input_and_ddim_step_are_exact(mbx, ctx):
    from oracle.scheduler_ref import Ddim
    rng = np.random.default_rng(6)
    n, lat = 3, 8
    hw = lat * lat
    z = rng.standard_normal((2 * n, lat, lat, 4)).astype(np.float32)
    ni = rng.standard_normal((n, lat, lat, 4)).astype(np.float32)
    no = rng.standard_normal((n, 4)).astype(np.float32)
    ml = (rng.random((n, lat, lat)) > 0.5).astype(np.float32)
    d = Ddim(20, 0.99)
    t0 = d.timesteps[0]
    a0 = d.ac[t0]
    zd, nid, nod, mld = ctx.upload(z), ctx.upload(ni), ctx.upload(no), ctx.upload(ml)
    x = ctx.empty((n, lat, lat, 4))
    L = mbx.abi.lib()
    mbx.check(L.mbx_latents_init(ctx.handle, zd.vp, nid.vp, nod.vp, n, hw, ctypes.c_float(0.0357),
                                 ctypes.c_float(np.sqrt(a0)), ctypes.c_float(np.sqrt(np.float32(1) - a0)), 0, x.vp))
    init = (ni + np.float32(0.0357) * no[:, None, None, :]).astype(np.float32)
    want_x = np.stack([d.add_noise(z[2 * i], init[i], t0) for i in range(n)])
    assert np.array_equal(x.numpy(), want_x)
    inp = ctx.empty((2 * n, lat, lat, 9))
    mbx.check(L.mbx_unet_input(ctx.handle, x.vp, mld.vp, zd.vp, n, hw, 2, inp.vp))
    got_in = inp.numpy()
    for i in range(n):
        want = np.concatenate([want_x[i], ml[i][..., None], z[2 * i + 1]], axis=-1)
        assert np.array_equal(got_in[2 * i], want) and np.array_equal(got_in[2 * i + 1], want)
    eps = rng.standard_normal((2 * n, lat, lat, 4)).astype(np.float32)
    t = d.timesteps[3]
    a_t, a_prev = d.ac[t], d.ac[t - d.step_ratio]
    coef = (ctypes.c_float * 4)(np.sqrt(np.float32(1) - a_t), np.sqrt(a_t), np.sqrt(a_prev),
                                np.sqrt(np.float32(1) - a_prev))
    epsd = ctx.upload(eps)
    mbx.check(L.mbx_cfg_ddim_step(ctx.handle, epsd.vp, n, hw, 2, ctypes.c_float(2.5), coef, x.vp))
    g = np.float32(2.5)
    want = np.stack([d.step((eps[2 * i] + g * (eps[2 * i + 1] - eps[2 * i])).astype(np.float32), t, want_x[i])
                     for i in range(n)])
    assert np.array_equal(x.numpy(), want)
