"""CPU checks of the oracle's UNet / pipeline pieces and of the library's
host-side schedule, pinned on the reference's own test values:

* DDIM: src/scheduler.rs:181-255 (timesteps, ᾱ, step, add_noise), for the
  numpy restatement and for the library's mbx_ddim_* entry points;
* Pillow blur: the reference's fixture (tests/fixtures/blur.safetensors, copied
  to tests/golden/imaging_ref.safetensors) plus two 512² masks from Pillow;
* λ layers: the oracle's reassociated forms (as the reference computes them,
  src/unet/lambda.rs:15-24) against float64 restatements of the definitions
  in lambda.rs:7-14 and 27-38 (λp materialised);
* the synthetic weights against the converted weight manifest.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_golden, load_package, max_rel_err


def close(got, want, rel):
    # src/scheduler.rs:175-179
    for g, w in zip(np.ravel(got), np.ravel(want)):
        assert abs(float(g) - w) <= rel * max(abs(w), 1e-3), (g, w)


def test_ddim_timesteps_match_reference():
    from oracle.scheduler_ref import Ddim
    d = Ddim(20, 0.99)
    assert d.timesteps == [i * 50 for i in range(18, -1, -1)]
    assert not d.pure_noise_start
    assert Ddim(7, 0.99).timesteps == [710, 568, 426, 284, 142, 0]
    full = Ddim(20, 1.0)
    assert len(full.timesteps) == 20 and full.timesteps[0] == 950 and full.pure_noise_start
    assert Ddim(4, 1.0, trailing=True).timesteps == [999, 749, 499, 249]


def test_ddim_values_match_reference():
    from oracle.scheduler_ref import Ddim, alphas_cumprod
    ac = alphas_cumprod()
    close([ac[t] for t in (0, 1, 500, 900, 999)],
          [9.991499782e-01, 9.982960224e-01, 2.763324678e-01, 1.415113267e-02, 4.660095088e-03], 1e-5)
    d = Ddim(20, 0.99)
    x = np.array([0.5, -1.25, 2.0], np.float32)
    eps = np.array([0.1, -0.3, 0.7], np.float32)
    for t, want in [(900, [6.129949689e-01, -1.518200040e+00, 2.366255760e+00]),
                    (50, [4.927129745e-01, -1.221965790e+00, 1.911952496e+00]),
                    (0, [4.972958863e-01, -1.241781354e+00, 1.980433226e+00])]:
        close(d.step(eps, t, x), want, 1e-5)
    close(d.add_noise(x, eps, 900), [1.587691903e-01, -4.465679526e-01, 9.329465032e-01], 1e-5)


def test_library_ddim_schedule_matches_reference():
    import ctypes
    from oracle.scheduler_ref import alphas_cumprod
    mbx = load_package()
    lib = mbx.abi.lib()
    out = (ctypes.c_int64 * 1000)()
    n = ctypes.c_int64()
    for steps, strength, trailing, want in [(20, 0.99, 0, [i * 50 for i in range(18, -1, -1)]),
                                            (7, 0.99, 0, [710, 568, 426, 284, 142, 0]),
                                            (4, 1.0, 1, [999, 749, 499, 249])]:
        mbx.check(lib.mbx_ddim_timesteps(steps, strength, trailing, out, ctypes.byref(n)))
        assert list(out[:n.value]) == want
    ac = np.zeros(1000, np.float32)
    mbx.check(lib.mbx_ddim_alphas_cumprod(ac.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
    assert np.array_equal(ac, alphas_cumprod()), "library and oracle schedules differ bit for bit"
    assert lib.mbx_ddim_timesteps(0, 0.99, 0, out, ctypes.byref(n)) == mbx.abi.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("case", ["a", "b", "c", "e1", "e2"])
def test_pil_blur_is_byte_exact(case):
    from oracle.imaging_ref import pil_gaussian_blur
    f = load_golden("imaging_ref.safetensors")
    got = pil_gaussian_blur(f[f"{case}.mask"].astype(np.uint8), 3.0)
    assert np.array_equal(got, f[f"{case}.blurred"].astype(np.uint8))


def test_feather_paste_keeps_outside_and_blends_edge():
    # src/imaging/blend.rs:253-275 (whole-image window)
    from oracle.imaging_ref import feather_paste
    w, h = 40, 30
    img = np.full((h, w, 3), 10, np.uint8)
    m = np.zeros((h, w), np.uint8)
    m[5:25, 10:30] = 255
    out = feather_paste(img, m, np.full((h, w, 3), 250, np.uint8))
    assert out[0, 0, 0] == 10 and out[15, 20, 0] == 250
    assert 10 < out[15, 9, 0] < 250


def test_to_u8_truncates_and_clamps():
    # src/imaging/blend.rs:222-231
    from oracle.imaging_ref import to_u8
    assert list(to_u8(np.array([0.99999, 1.2, -0.1, 0.5, 1.0, 0.0, np.nan], np.float32))) == [254, 255, 0, 127,
                                                                                               255, 0, 0]


def _naive_self_lambda(q, kt, vt, wpos, bpos, hh, ww):
    """lambda.rs:7-14 in float64 with λp materialised: Y = Yc + Yp."""
    hw, k = kt.shape
    q = q.reshape(hw, 8, k).astype(np.float64)
    e = np.exp(kt - kt.max(axis=0))
    ks = e / e.sum(axis=0)
    lam_c = ks.T @ vt                                            # [k, v]
    yc = q @ lam_c                                               # [hw, 8, v]
    vmap = vt.reshape(hh, ww, k).astype(np.float64)
    vpad = np.pad(vmap, ((7, 7), (7, 7), (0, 0)))
    lam_p = np.zeros((hh, ww, k, k))
    for ky in range(15):
        for kx in range(15):
            lam_p += wpos[None, None, :, ky * 15 + kx, None] * vpad[ky:ky + hh, kx:kx + ww, None, :]
    lam_p += bpos[None, None, :, None]
    yp = np.einsum("phk,pkv->phv", q, lam_p.reshape(hw, k, k))
    return (yc + yp).reshape(hh, ww, 8 * k)


def test_self_lambda_oracle_matches_definition(oracle):
    from oracle import unet_ref
    rng = np.random.default_rng(1)
    hh, ww, c = 9, 11, 64
    k = c // 8
    x = rng.standard_normal((1, hh, ww, c)).astype(np.float32)
    w = {"a.to_q.weight": rng.standard_normal((c, c)).astype(np.float32) / 8,
         "a.to_q.bias": rng.standard_normal(c).astype(np.float32) * 0.1,
         "a.to_k.weight": rng.standard_normal((k, c)).astype(np.float32) / 8,
         "a.to_v.weight": rng.standard_normal((k, c)).astype(np.float32) / 8,
         "a.to_v.bias": rng.standard_normal(k).astype(np.float32) * 0.1,
         "a.pos_conv.weight": rng.standard_normal((k, 225)).astype(np.float32) / 15,
         "a.pos_conv.bias": rng.standard_normal(k).astype(np.float32) * 0.1}
    got = unet_ref.self_lambda(w, "a", x)[0]
    x64 = x[0].reshape(-1, c).astype(np.float64)
    q = x64 @ w["a.to_q.weight"].T + w["a.to_q.bias"]
    kt = x64 @ w["a.to_k.weight"].T
    vt = x64 @ w["a.to_v.weight"].T + w["a.to_v.bias"]
    want = _naive_self_lambda(q, kt, vt, w["a.pos_conv.weight"].astype(np.float64), w["a.pos_conv.bias"], hh, ww)
    assert max_rel_err(got, want) < 2e-5


def test_cross_lambda_oracle_matches_definition(oracle):
    from oracle import unet_ref
    rng = np.random.default_rng(2)
    hh, ww, c = 4, 6, 64
    k = c // 8
    x = rng.standard_normal((2, hh, ww, c)).astype(np.float32)
    ehs = rng.standard_normal((2, 10, 768)).astype(np.float32)
    w = {"a.to_q.weight": rng.standard_normal((c, c)).astype(np.float32) / 8,
         "a.to_q.bias": rng.standard_normal(c).astype(np.float32) * 0.1,
         "a.to_k.weight": rng.standard_normal((k, 768)).astype(np.float32) / 28,
         "a.to_v.weight": rng.standard_normal((k, 768)).astype(np.float32) / 28,
         "a.to_v.bias": rng.standard_normal(k).astype(np.float32) * 0.1,
         "a.rel_pos_emb": rng.standard_normal((hh * ww, 10, k)).astype(np.float32) / 3}
    consts = unet_ref.cross_constants(w, "a", ehs)
    got = unet_ref.cross_lambda(w, "a", x, [1, 0], consts)
    for b, br in enumerate([1, 0]):
        x64 = x[b].reshape(-1, c).astype(np.float64)
        q = (x64 @ w["a.to_q.weight"].T + w["a.to_q.bias"]).reshape(-1, 8, k)
        keys = ehs[br].astype(np.float64) @ w["a.to_k.weight"].T
        v = ehs[br].astype(np.float64) @ w["a.to_v.weight"].T + w["a.to_v.bias"]
        e = np.exp(keys - keys.max(axis=0))
        lam_c = (e / e.sum(axis=0)).T @ v
        lam_p = np.einsum("pmk,mv->pkv", w["a.rel_pos_emb"].astype(np.float64), v)   # E·V, lambda.rs:39-40
        want = np.einsum("phk,kv->phv", q, lam_c) + np.einsum("phk,pkv->phv", q, lam_p)
        assert max_rel_err(got[b].reshape(-1, 8, k), want) < 2e-5


def test_timestep_sinusoid_matches_definition(oracle):
    s = oracle.timestep_sinusoid(900, 320)
    i = np.arange(160)
    arg = 900.0 * np.exp(-np.log(10000.0) * i / 160)
    assert np.allclose(s[:160], np.cos(arg), atol=2e-4) and np.allclose(s[160:], np.sin(arg), atol=2e-4)


def test_synthetic_weights_match_the_converted_manifest():
    syn = load_package().synthetic
    manifest = json.load(open(os.path.join(GOLDEN, "weights_manifest.json")))
    for section, shapes in (("unet", syn.unet_shapes()), ("vae", syn.vae_shapes())):
        got = {n: list(s) for n, (s, _) in shapes.items()}
        assert got == manifest[section]


def test_safetensors_round_trip(tmp_path):
    syn = load_package().synthetic
    t = {"a": np.arange(6, dtype=np.float32).reshape(2, 3), "b.c": np.ones((4,), np.float16)}
    p = str(tmp_path / "x.safetensors")
    syn.write_safetensors(p, t, {"scaling_factor": "0.13025"})
    back, meta = syn.read_safetensors(p)
    assert meta == {"scaling_factor": "0.13025"}
    assert all(np.array_equal(back[k], t[k]) and back[k].dtype == t[k].dtype for k in t)
    from safetensors.numpy import load_file
    other = load_file(p)
    assert all(np.array_equal(other[k], t[k]) for k in t)


def test_tiny_oracle_inpaint_keeps_empty_masks_and_is_deterministic():
    syn = load_package().synthetic
    from oracle import pipeline_ref
    wu = syn.random_weights(syn.unet_shapes((64, 128, 256), 16), 0)
    wv = syn.random_weights(syn.vae_shapes((32, 64, 128, 128)), 1)
    rng = np.random.default_rng(3)
    img = rng.integers(0, 256, (128, 128, 3), dtype=np.uint8)
    nv = rng.standard_normal((2, 16, 16, 4)).astype(np.float32)
    ni = rng.standard_normal((16, 16, 4)).astype(np.float32)
    no = rng.standard_normal(4).astype(np.float32)
    empty = np.zeros((128, 128), np.uint8)
    assert np.array_equal(pipeline_ref.inpaint(wu, wv, img, empty, nv, ni, no, steps=3), img)
    mask = empty.copy()
    mask[30:80, 40:100] = 200
    a = pipeline_ref.inpaint(wu, wv, img, mask, nv, ni, no, steps=3)
    b = pipeline_ref.inpaint(wu, wv, img, mask, nv, ni, no, steps=3)
    assert np.array_equal(a, b)
    assert (a[40:70, 50:90] != img[40:70, 50:90]).any()
    assert np.array_equal(a[120:, :10], img[120:, :10]), "far from the mask the source is untouched"
