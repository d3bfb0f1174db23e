"""The CPU oracle pinned against the reference's own golden vectors and tests.

Every case of the reference's tests/kernels.rs runs here against the oracle
with the reference's tolerances: fixture cases against the reference's
PyTorch fixture (copied to tests/golden/kernels_ref.safetensors), the
f64-definition cases against float64 restatements of the same loops. The
math.rs KATs (src/engine/math.rs:42-65) pin the oracle's exp/SiLU.
"""
import math

import numpy as np
import pytest

from conftest import rel_l2, scaled_err


def test_exp_matches_float64(oracle):
    # src/engine/math.rs:50-61
    worst = 0.0
    x = -87.0
    while x < 88.0:
        got, want = oracle.exp(np.float32(x)), math.exp(float(np.float32(x)))
        worst = max(worst, abs((got - want) / want))
        x += 0.0137 * 37  # a coarser walk of the same range
    assert worst < 3e-7
    assert oracle.exp(-1000.0) == oracle.exp(-87.33655)
    assert math.isfinite(oracle.exp(1000.0))


def test_silu_matches_definition(oracle):
    # src/engine/math.rs:63-72
    for i in range(-2000, 2000, 7):
        x = float(np.float32(i * 0.01))
        want = x / (1.0 + math.exp(-x))
        assert abs(oracle.silu_scalar(x) - want) <= 1e-6 * (1.0 + abs(want))
    assert abs(oracle.silu_scalar(-200.0)) < 1e-30
    assert oracle.silu_scalar(200.0) == 200.0


def test_conv1x1_bias_and_residual(oracle, ref_fixture):
    f = ref_fixture
    assert scaled_err(oracle.conv1x1(f["c1.x"], f["c1.w"], f["c1.b"]), f["c1.y"]) <= 1e-5
    assert scaled_err(oracle.conv1x1(f["c1.x"], f["c1.w"], f["c1.b"], f["c1.r"]), f["c1.yr"]) <= 1e-5


def test_conv1x1_f16_weights_match_rounded_f32(oracle, ref_fixture):
    # tests/kernels.rs:54-63: f16 storage is exactly the f32 weights rounded to f16.
    f = ref_fixture
    rounded = f["c1.w"].astype(np.float16).astype(np.float32)
    a = oracle.conv1x1(f["c1.x"], rounded)
    b = oracle.conv1x1(f["c1.x"], rounded.copy())
    assert scaled_err(a, b) <= 1e-6


@pytest.mark.parametrize("name,stride,pad,up", [
    ("c3.same", 1, (1, 1, 1, 1), False),
    ("c3.s2p1", 2, (1, 1, 1, 1), False),
    ("c3.s2vae", 2, (0, 0, 1, 1), False),
    ("c3.up", 1, (1, 1, 1, 1), True),
])
def test_conv3x3_variants(oracle, ref_fixture, name, stride, pad, up):
    f = ref_fixture
    got = oracle.conv3x3(f["c3.x"], f["c3.w"], f["c3.b"], stride, pad, up)
    assert scaled_err(got, f[name]) <= 1e-5
    got = oracle.conv3x3(f["c3.x"], f["c3.w"], f["c3.b"], stride, pad, up, im2col=True)
    assert scaled_err(got, f[name]) <= 1e-5


def naive_conv3x3_same(x, wt):
    """f64 direct 3×3 same conv: x [n,h,w,c], wt [o,3,3,c]."""
    n, h, w, c = x.shape
    xp = np.zeros((n, h + 2, w + 2, c))
    xp[:, 1:-1, 1:-1] = x
    out = np.zeros((n, h, w, wt.shape[0]))
    for ky in range(3):
        for kx in range(3):
            out += np.einsum("nhwc,oc->nhwo", xp[:, ky:ky + h, kx:kx + w], wt[:, ky, kx].astype(np.float64))
    return out


def test_conv3x3_band_boundaries(oracle):
    # tests/kernels.rs:87-116: c_in = 1024 forces several im2col bands.
    n, h, w, c = 1, 40, 30, 1024
    i = np.arange(n * h * w * c, dtype=np.int64)
    x = (((i * 7919) % 211) / 211.0 - 0.5).astype(np.float32).reshape(n, h, w, c)
    j = np.arange(2 * 9 * c, dtype=np.int64)
    wt = (((j * 104_729) % 97) / 970.0 - 0.05).astype(np.float32).reshape(2, 3, 3, c)
    want = naive_conv3x3_same(x.astype(np.float64), wt)
    assert scaled_err(oracle.conv3x3(x, wt), want) <= 2e-5
    assert scaled_err(oracle.conv3x3(x, wt, im2col=True), want) <= 2e-5


def test_depthwise_epilogues(oracle, ref_fixture):
    f = ref_fixture
    assert scaled_err(oracle.depthwise3x3(f["dw.x"], f["dw.w"], f["dw.b"], "relu"), f["dw.relu"]) <= 1e-5
    assert scaled_err(oracle.depthwise3x3(f["dw.x"], f["dw.w"], f["dw.b"], "glu_silu"), f["dw.glu"]) <= 1e-5


def depthwise_f64(x, wt, b, ep):
    n, h, w, c = x.shape
    xp = np.zeros((n, h + 2, w + 2, c))
    xp[:, 1:-1, 1:-1] = x
    y = np.broadcast_to(b.astype(np.float64), (n, h, w, c)).copy()
    for ky in range(3):
        for kx in range(3):
            y += xp[:, ky:ky + h, kx:kx + w] * wt[ky, kx].astype(np.float64)
    if ep == "relu":
        return np.maximum(y, 0.0)
    if ep == "glu_silu":
        v, g = y[..., :c // 2], y[..., c // 2:]
        return v * g / (1.0 + np.exp(-g))
    return y


@pytest.mark.parametrize("h,w,c,ep", [(5, 7, 64, "relu"), (4, 9, 70, "none"), (3, 5, 140, "glu_silu"),
                                      (2, 4, 64, "glu_silu")])
def test_depthwise_register_blocks_and_tails(oracle, h, w, c, ep):
    # tests/kernels.rs:173-213
    i = np.arange(h * w * c, dtype=np.int64)
    x = (((i * 7919) % 211) / 211.0 - 0.5).astype(np.float32).reshape(1, h, w, c)
    j = np.arange(9 * c, dtype=np.int64)
    wt = (((j * 31) % 17) / 17.0 - 0.5).astype(np.float32).reshape(3, 3, c)
    b = (np.arange(c) * 0.01 - 0.2).astype(np.float32)
    assert scaled_err(oracle.depthwise3x3(x, wt, b, ep), depthwise_f64(x, wt, b, ep)) <= 1e-5


def test_group_norm_plain_and_fused(oracle, ref_fixture):
    f = ref_fixture
    got = oracle.group_norm(f["gn.x"], 32, 1e-6, f["gn.gamma"], f["gn.beta"])
    assert scaled_err(got, f["gn.y"]) <= 1e-5
    got = oracle.group_norm(f["gn.x"], 32, 1e-5, f["gn.gamma"], f["gn.beta"], f["gn.add"], silu=True)
    assert scaled_err(got, f["gn.y_add_silu"]) <= 1e-5


def test_layer_norm_tokens(oracle, ref_fixture):
    f = ref_fixture
    x = f["ln.x"].reshape(3, 17, 1, 44)
    got = oracle.layer_norm(x, f["ln.gamma"], f["ln.beta"], 1e-5)
    assert scaled_err(got.reshape(3, 17, 44), f["ln.y"]) <= 1e-5


@pytest.mark.parametrize("n,h,w,ci,co,up", [(2, 37, 23, 24, 40, False), (1, 9, 13, 16, 8, True),
                                            (1, 6, 5, 768, 720, False)])
def test_winograd_matches_direct_on_multiband_odd_sizes(oracle, n, h, w, ci, co, up):
    # tests/kernels.rs:154-170 (f16-rounded weights, as Param::f16_from)
    i = np.arange(n * h * w * ci, dtype=np.int64)
    x = (((i * 7919) % 401) / 401.0 - 0.5).astype(np.float32).reshape(n, h, w, ci)
    j = np.arange(co * 9 * ci, dtype=np.int64)
    wt = (((j * 104_729) % 113) / 1130.0 - 0.05).astype(np.float16).astype(np.float32).reshape(co, 3, 3, ci)
    b = (np.arange(co) * 0.01).astype(np.float32)
    fast = oracle.conv3x3(x, wt, b, upsample2x=up)
    direct = oracle.conv3x3(x, wt, b, upsample2x=up, im2col=True)
    assert scaled_err(fast, direct) <= 2e-5


def lcg(seed):
    s = seed

    def nxt():
        nonlocal s
        s = (s * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        return ((s >> 40) / float(1 << 24)) * 2.0 - 1.0
    return nxt


@pytest.mark.parametrize("n,h,w,ci,groups,co", [(2, 7, 9, 40, 8, 24), (2, 37, 23, 64, 32, 16)])
@pytest.mark.parametrize("up", [False, True])
def test_prologue_matches_group_norm_then_conv(oracle, n, h, w, ci, groups, co, up):
    # tests/kernels.rs:233-264 (the 768-channel case is replaced by 64 channels to keep the CPU suite fast)
    rng = np.random.default_rng(7 + ci)
    x = (rng.uniform(-1, 1, (n, h, w, ci)) * 3.0 + 0.7).astype(np.float32)
    gamma = (1.0 + 0.5 * rng.uniform(-1, 1, ci)).astype(np.float32)
    beta = rng.uniform(-1, 1, ci).astype(np.float32)
    wt = (rng.uniform(-1, 1, (co, 3, 3, ci)) * 0.05).astype(np.float16).astype(np.float32)
    bias = (np.arange(co) * 0.01).astype(np.float32)
    a = oracle.group_norm(x, groups, 1e-6, gamma, beta, silu=True)
    want = oracle.conv3x3(a, wt, bias, upsample2x=up)
    scale, shift = oracle.group_norm_affine(x, groups, 1e-6, gamma, beta)
    got = oracle.conv3x3(x, wt, bias, upsample2x=up, prologue=(scale, shift, True))
    assert rel_l2(got, want) <= 1e-6


def test_extra_fixture_cases(oracle, extra_fixture):
    f = extra_fixture
    got = oracle.group_norm(f["gn64.x"], 32, 1e-6, f["gn64.gamma"], f["gn64.beta"], f["gn64.add"], silu=True)
    assert scaled_err(got, f["gn64.y"]) <= 1e-5
    got = oracle.conv1x1(f["c1o.x"], f["c1o.w"], f["c1o.b"], f["c1o.r"])
    assert scaled_err(got, f["c1o.y"]) <= 1e-5
    scale, shift = oracle.group_norm_affine(f["pro.x"], 8, 1e-6, f["pro.gamma"], f["pro.beta"])
    for key, up in (("pro.y", False), ("pro.yup", True)):
        got = oracle.conv3x3(f["pro.x"], f["pro.w"], f["pro.b"], upsample2x=up, prologue=(scale, shift, True))
        assert scaled_err(got, f[key]) <= 1e-5
    assert scaled_err(oracle.conv3x3(f["c3n.x"], f["c3n.w"], f["c3n.b"]), f["c3n.y"]) <= 1e-5
    assert scaled_err(oracle.depthwise3x3(f["dw70.x"], f["dw70.w"], f["dw70.b"]), f["dw70.y"]) <= 1e-5
    assert scaled_err(oracle.depthwise3x3(f["dw140.x"], f["dw140.w"], f["dw140.b"], "glu_silu"),
                      f["dw140.y"]) <= 1e-5
    x = f["ln320.x"].reshape(2, 37, 1, 320)
    got = oracle.layer_norm(x, f["ln320.gamma"], f["ln320.beta"], 1e-5).reshape(2, 37, 320)
    assert scaled_err(got, f["ln320.y"]) <= 1e-5
    assert scaled_err(oracle.bias_temb_add(f["bt.x"], f["bt.bias"], f["bt.temb"]), f["bt.y"]) <= 1e-6
    assert scaled_err(oracle.add(f["bt.x"], f["bt.r"]), f["bt.sum"]) <= 1e-6
    assert scaled_err(oracle.silu(f["bt.x"]), f["bt.silu"]) <= 1e-6


def test_concat_channels_interleaves_per_pixel(oracle):
    # src/engine/tensor.rs:86-95
    a = np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 2, 2)
    b = np.array([10, 20, 30, 40, 50, 60], np.float32).reshape(1, 1, 2, 3)
    c = oracle.concat_channels(a, b)
    assert c.shape == (1, 1, 2, 5)
    assert c.ravel().tolist() == [1, 2, 10, 20, 30, 3, 4, 40, 50, 60]


def test_matmul_matches_naive(oracle):
    # src/engine/gemm.rs:138-160
    m, k, n = 7, 5, 3
    a = np.sin(np.arange(m * k) * 0.37).astype(np.float32).reshape(m, k)
    w = np.cos(np.arange(n * k) * 0.11).astype(np.float32).reshape(n, k)
    want = a.astype(np.float64) @ w.T.astype(np.float64)
    got = oracle.matmul(a, np.ascontiguousarray(w.T))
    assert np.max(np.abs(got - want)) < 1e-5
    got2 = oracle.matmul(a, np.ascontiguousarray(w.T), got)
    assert np.max(np.abs(got2 - 2 * want)) < 1e-5
