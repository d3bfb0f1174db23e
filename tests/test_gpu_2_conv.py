"""GPU parity of the tensor-core convolutions (tcgen05 implicit GEMM) through
the C ABI: every conv case of the reference's tests/kernels.rs at its
tolerances, the fused GroupNorm prologue, and BASELINE-shaped single-block /
conv-sweep inputs against the CPU oracle with the per-kernel gates
(max relative error ≤ 1e-3 for f32 weights (3×TF32), ≤ 5e-3 for f16 weights).
"""
import numpy as np
import pytest

from conftest import max_rel_err, rel_l2, scaled_err

pytestmark = pytest.mark.gpu

REF_TOL = 1e-5
GATE_F32 = 1e-3
GATE_F16 = 5e-3


def up(ctx, a):
    return ctx.upload(a)


def test_conv1x1_bias_and_residual(mbx, ctx, ref_fixture):
    f = ref_fixture
    w = mbx.Param(ctx, f["c1.w"])
    x, b = up(ctx, f["c1.x"]), up(ctx, f["c1.b"])
    assert scaled_err(mbx.conv1x1(x, w, b).numpy(), f["c1.y"]) <= REF_TOL
    assert scaled_err(mbx.conv1x1(x, w, b, residual=up(ctx, f["c1.r"])).numpy(), f["c1.yr"]) <= REF_TOL
    w.close()


def test_conv1x1_f16_weights_match_rounded_f32(mbx, ctx, ref_fixture):
    # tests/kernels.rs:54-63
    f = ref_fixture
    x = up(ctx, f["c1.x"])
    w16 = mbx.Param(ctx, f["c1.w"], "f16")
    w32 = mbx.Param(ctx, f["c1.w"].astype(np.float16).astype(np.float32))
    assert scaled_err(mbx.conv1x1(x, w16).numpy(), mbx.conv1x1(x, w32).numpy()) <= 1e-6


@pytest.mark.parametrize("name,stride,pad,upx", [
    ("c3.same", 1, (1, 1, 1, 1), False),
    ("c3.s2p1", 2, (1, 1, 1, 1), False),
    ("c3.s2vae", 2, (0, 0, 1, 1), False),
    ("c3.up", 1, (1, 1, 1, 1), True),
])
def test_conv3x3_variants(mbx, ctx, ref_fixture, name, stride, pad, upx):
    f = ref_fixture
    w = mbx.Param(ctx, f["c3.w"])
    got = mbx.conv3x3(up(ctx, f["c3.x"]), w, up(ctx, f["c3.b"]), stride, pad, upx).numpy()
    assert scaled_err(got, f[name]) <= REF_TOL


def test_extra_fixture_convs(mbx, ctx, extra_fixture):
    f = extra_fixture
    w = mbx.Param(ctx, f["c1o.w"])
    got = mbx.conv1x1(up(ctx, f["c1o.x"]), w, up(ctx, f["c1o.b"]), residual=up(ctx, f["c1o.r"])).numpy()
    assert scaled_err(got, f["c1o.y"]) <= REF_TOL
    w = mbx.Param(ctx, f["c3n.w"])
    assert scaled_err(mbx.conv3x3(up(ctx, f["c3n.x"]), w, up(ctx, f["c3n.b"])).numpy(), f["c3n.y"]) <= REF_TOL
    # GN(+SiLU) prologue fused into the conv, plain and upsampled; padding stays zero.
    x = up(ctx, f["pro.x"])
    sc, sh = mbx.group_norm_affine(x, 8, 1e-6, up(ctx, f["pro.gamma"]), up(ctx, f["pro.beta"]))
    w = mbx.Param(ctx, f["pro.w"])
    b = up(ctx, f["pro.b"])
    for key, upx in (("pro.y", False), ("pro.yup", True)):
        got = mbx.conv3x3(x, w, b, upsample2x=upx, prologue=(sc, sh, True)).numpy()
        assert scaled_err(got, f[key]) <= REF_TOL


def naive_conv3x3_same(x, wt):
    n, h, w, c = x.shape
    xp = np.zeros((n, h + 2, w + 2, c))
    xp[:, 1:-1, 1:-1] = x
    out = np.zeros((n, h, w, wt.shape[0]))
    for ky in range(3):
        for kx in range(3):
            out += np.einsum("nhwc,oc->nhwo", xp[:, ky:ky + h, kx:kx + w], wt[:, ky, kx].astype(np.float64))
    return out


def test_conv3x3_band_boundaries(mbx, ctx):
    # tests/kernels.rs:87-116 (c_in = 1024: many K chunks; 1200 output pixels = 10 M tiles)
    n, h, w, c = 1, 40, 30, 1024
    i = np.arange(n * h * w * c, dtype=np.int64)
    x = (((i * 7919) % 211) / 211.0 - 0.5).astype(np.float32).reshape(n, h, w, c)
    j = np.arange(2 * 9 * c, dtype=np.int64)
    wt = (((j * 104_729) % 97) / 970.0 - 0.05).astype(np.float32).reshape(2, 3, 3, c)
    got = mbx.conv3x3(up(ctx, x), mbx.Param(ctx, wt)).numpy()
    assert scaled_err(got, naive_conv3x3_same(x.astype(np.float64), wt)) <= 2e-5


@pytest.mark.parametrize("n,h,w,ci,co,upx", [(2, 37, 23, 24, 40, False), (1, 9, 13, 16, 8, True),
                                             (1, 6, 5, 768, 720, False)])
def test_f16_weights_match_direct_on_odd_sizes(mbx, ctx, oracle, n, h, w, ci, co, upx):
    # tests/kernels.rs:154-170: the GPU direct conv with f16 weights vs the oracle's im2col path.
    i = np.arange(n * h * w * ci, dtype=np.int64)
    x = (((i * 7919) % 401) / 401.0 - 0.5).astype(np.float32).reshape(n, h, w, ci)
    j = np.arange(co * 9 * ci, dtype=np.int64)
    wt = (((j * 104_729) % 113) / 1130.0 - 0.05).astype(np.float32).reshape(co, 3, 3, ci)
    b = (np.arange(co) * 0.01).astype(np.float32)
    got = mbx.conv3x3(up(ctx, x), mbx.Param(ctx, wt, "f16"), up(ctx, b), upsample2x=upx).numpy()
    want = oracle.conv3x3(x, wt.astype(np.float16).astype(np.float32), b, upsample2x=upx, im2col=True)
    assert scaled_err(got, want) <= 2e-5


def lcg(seed):
    s = seed

    def nxt(k):
        nonlocal s
        out = np.empty(k, np.float32)
        for i in range(k):
            s = (s * 6364136223846793005 + 1442695040888963407) % (1 << 64)
            out[i] = ((s >> 40) / float(1 << 24)) * 2.0 - 1.0
        return out
    return nxt


@pytest.mark.parametrize("n,h,w,ci,groups,co", [(2, 7, 9, 40, 8, 24), (2, 37, 23, 768, 32, 16),
                                                 (2, 32, 32, 64, 32, 48)])  # the last: TMA-fed A tiles
@pytest.mark.parametrize("upx", [False, True])
def test_prologue_matches_group_norm_then_conv(mbx, ctx, n, h, w, ci, groups, co, upx):
    # tests/kernels.rs:233-264, both sides on the GPU.
    rng = np.random.default_rng(7 + ci)
    x = (rng.uniform(-1, 1, (n, h, w, ci)) * 3.0 + 0.7).astype(np.float32)
    gamma = (1.0 + 0.5 * rng.uniform(-1, 1, ci)).astype(np.float32)
    beta = rng.uniform(-1, 1, ci).astype(np.float32)
    wt = (rng.uniform(-1, 1, (co, 3, 3, ci)) * 0.05).astype(np.float32)
    bias = (np.arange(co) * 0.01).astype(np.float32)
    xd, g, b = up(ctx, x), up(ctx, gamma), up(ctx, beta)
    wp, bd = mbx.Param(ctx, wt, "f16"), up(ctx, bias)
    a = mbx.group_norm(xd, groups, 1e-6, g, b, silu=True)
    want = mbx.conv3x3(a, wp, bd, upsample2x=upx).numpy()
    sc, sh = mbx.group_norm_affine(xd, groups, 1e-6, g, b)
    got = mbx.conv3x3(xd, wp, bd, upsample2x=upx, prologue=(sc, sh, True)).numpy()
    assert rel_l2(got, want) <= 1e-6


def test_single_block_config(mbx, ctx, oracle):
    """x [1,64,64,256] ~N(0,1); GN(32, eps 1e-6, γ~N(1,0.02), β~N(0,0.02)) + SiLU;
    3×3 conv 256→256 (w ~N(0, 1/√2304), bias ~N(0, 0.01)); + x. Fused on the GPU as GN stats →
    conv with the GN prologue and the residual in the epilogue."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 64, 64, 256)).astype(np.float32)
    gamma = rng.normal(1.0, 0.02, 256).astype(np.float32)
    beta = rng.normal(0.0, 0.02, 256).astype(np.float32)
    wt = rng.normal(0.0, 1.0 / np.sqrt(2304.0), (256, 3, 3, 256)).astype(np.float32)
    bias = rng.normal(0.0, 0.01, 256).astype(np.float32)
    want = oracle.conv3x3(oracle.group_norm(x, 32, 1e-6, gamma, beta, silu=True), wt, bias)
    want = oracle.add(want, x)
    for dtype, gate in (("f32", GATE_F32), ("f16", GATE_F16)):
        wref = wt if dtype == "f32" else wt.astype(np.float16).astype(np.float32)
        want_d = want if dtype == "f32" else oracle.add(
            oracle.conv3x3(oracle.group_norm(x, 32, 1e-6, gamma, beta, silu=True), wref, bias), x)
        xd = up(ctx, x)
        sc, sh = mbx.group_norm_affine(xd, 32, 1e-6, up(ctx, gamma), up(ctx, beta))
        got = mbx.conv3x3(xd, mbx.Param(ctx, wt, dtype), up(ctx, bias), prologue=(sc, sh, True),
                          residual=xd).numpy()
        assert max_rel_err(got, want_d) <= gate
        assert scaled_err(got, want_d) <= 1e-4


@pytest.mark.parametrize("k", [1, 3])
@pytest.mark.parametrize("hw,ci,co", [(64, 128, 128), (64, 256, 512), (64, 512, 256), (128, 128, 256)])
@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_conv_sweep_matches_oracle(mbx, ctx, oracle, k, hw, ci, co, dtype):
    """BASELINE config 3 shapes at B = 1 (B = 8 at 256×256 below): w ~N(0, 1/√fan_in), fused
    bias + residual epilogue."""
    rng = np.random.default_rng(hw + ci + co + k)
    x = rng.standard_normal((1, hw, hw, ci)).astype(np.float32)
    shape = (co, ci) if k == 1 else (co, 3, 3, ci)
    wt = rng.normal(0.0, 1.0 / np.sqrt(ci * k * k), shape).astype(np.float32)
    bias = rng.normal(0.0, 0.01, co).astype(np.float32)
    res = rng.standard_normal((1, hw, hw, co)).astype(np.float32)
    wref = wt if dtype == "f32" else wt.astype(np.float16).astype(np.float32)
    if k == 1:
        want = oracle.conv1x1(x, wref, bias, res)
        got = mbx.conv1x1(up(ctx, x), mbx.Param(ctx, wt, dtype), up(ctx, bias), up(ctx, res)).numpy()
    else:
        want = oracle.add(oracle.conv3x3(x, wref, bias), res)
        got = mbx.conv3x3(up(ctx, x), mbx.Param(ctx, wt, dtype), up(ctx, bias), residual=up(ctx, res)).numpy()
    assert max_rel_err(got, want) <= (GATE_F32 if dtype == "f32" else GATE_F16)
    assert scaled_err(got, want) <= 2e-5


@pytest.mark.parametrize("k,ci,co,dtype", [
    (3, 512, 512, "f16"),  # the benchmark's roofline shape
    (3, 512, 512, "f32"),
    (3, 256, 256, "f16"),
    (3, 128, 512, "f32"),
    (1, 512, 512, "f16"),
    (1, 256, 128, "f32"),
])
def test_conv_sweep_b8_256_matches_oracle(mbx, ctx, oracle, k, ci, co, dtype):
    """BASELINE config 3 at its largest size, [8, 256, 256, c_in]: the 3×3 convs take the TMA
    path that loads A as 128-pixel pieces of 256-pixel rows (a 4-D box, zero fill as the
    padding), the 1×1 convs the 2-D A box; whole outputs against the oracle (its Winograd path
    for the 3×3), fused bias + residual epilogue."""
    rng = np.random.default_rng(8 * ci + co + k)
    shape = (8, 256, 256, ci)
    x = rng.standard_normal(shape, dtype=np.float32)
    wshape = (co, ci) if k == 1 else (co, 3, 3, ci)
    wt = rng.normal(0.0, 1.0 / np.sqrt(ci * k * k), wshape).astype(np.float32)
    bias = rng.normal(0.0, 0.01, co).astype(np.float32)
    res = rng.standard_normal((8, 256, 256, co), dtype=np.float32)
    wref = wt if dtype == "f32" else wt.astype(np.float16).astype(np.float32)
    p = mbx.Param(ctx, wt, dtype)
    if k == 1:
        got = mbx.conv1x1(up(ctx, x), p, up(ctx, bias), up(ctx, res)).numpy()
        want = oracle.conv1x1(x, wref, bias, res)
    else:
        got = mbx.conv3x3(up(ctx, x), p, up(ctx, bias), residual=up(ctx, res)).numpy()
        want = oracle.add(oracle.conv3x3(x, wref, bias), res)
    p.close()
    assert max_rel_err(got, want) <= (GATE_F32 if dtype == "f32" else GATE_F16)
    assert scaled_err(got, want) <= 2e-5


@pytest.mark.parametrize("shape,stride,pad,upx,co", [
    ((2, 64, 64, 320), 2, (1, 1, 1, 1), False, 320),     # UNet Downsample2D, level 0
    ((1, 128, 128, 128), 2, (0, 0, 1, 1), False, 128),   # VAE encoder Downsample2D
    ((2, 16, 16, 1280), 1, (1, 1, 1, 1), True, 1280),    # UNet Upsample2D, level 2
    ((1, 64, 64, 4), 1, (1, 1, 1, 1), False, 512),       # VAE decoder conv_in (4 channels)
    ((1, 64, 64, 128), 1, (1, 1, 1, 1), False, 3),       # VAE conv_out (3 channels)
    # Upsampled inputs at each tile geometry: 128 / wo output rows per tile (wo 32, 64, 128) and
    # 128-pixel pieces of a row (wo 256, 512). Upsampled convs gather A with cp.async (no TMA box).
    ((2, 16, 16, 64), 1, (1, 1, 1, 1), True, 96),
    ((1, 32, 32, 64), 1, (1, 1, 1, 1), True, 160),
    ((2, 64, 64, 96), 1, (1, 1, 1, 1), True, 64),
    ((1, 128, 128, 32), 1, (1, 1, 1, 1), True, 64),
    ((1, 256, 256, 32), 1, (1, 1, 1, 1), True, 32),
])
def test_unet_vae_conv_shapes(mbx, ctx, oracle, shape, stride, pad, upx, co):
    rng = np.random.default_rng(shape[-1] + co)
    ci = shape[-1]
    x = rng.standard_normal(shape).astype(np.float32)
    wt = rng.normal(0.0, 1.0 / np.sqrt(9 * ci), (co, 3, 3, ci)).astype(np.float32)
    bias = rng.normal(0.0, 0.01, co).astype(np.float32)
    want = oracle.conv3x3(x, wt, bias, stride, pad, upx)
    got = mbx.conv3x3(up(ctx, x), mbx.Param(ctx, wt), up(ctx, bias), stride, pad, upx).numpy()
    assert max_rel_err(got, want) <= GATE_F32
    assert scaled_err(got, want) <= 2e-5


def test_conv_errors(mbx, ctx):
    w = mbx.Param(ctx, np.zeros((8, 3, 3, 16), np.float32))
    with pytest.raises(mbx.MbxError) as e:
        mbx.conv3x3(up(ctx, np.zeros((1, 4, 4, 12), np.float32)), w)  # wrong c_in
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT
    with pytest.raises(mbx.MbxError):
        mbx.conv1x1(up(ctx, np.zeros((1, 4, 4, 16), np.float32)), w)  # 3×3 weight given to a 1×1 conv
    ctx.synchronize()


def test_device_error_word_is_clear(mbx, ctx):
    """No bounded wait gave up during the tests above (mbx_ctx_synchronize reports MBX_ERR_TIMEOUT otherwise)."""
    ctx.synchronize()


def test_bounded_wait_gives_up_and_the_context_recovers(mbx, ctx, ref_fixture):
    """A device wait that runs out, in the form that faults nothing: one thread waits on a
    barrier that nothing arrives at (no copy issued) with a limit of 2e7 cycles (about 10 ms).
    mbx_ctx_synchronize reports MBX_ERR_TIMEOUT with the kernel and site, clears the record,
    and the same context then runs a conv that matches the reference fixture."""
    lib = mbx.abi.lib()
    ctx.synchronize()
    mbx.check(lib.mbx_selftest_wait_timeout(ctx.handle, 20_000_000))
    assert lib.mbx_ctx_synchronize(ctx.handle) == mbx.abi.ERR_TIMEOUT
    msg = lib.mbx_last_error()
    assert b"timed out" in msg and b"kernel 4" in msg and b"site 12" in msg, msg
    ctx.synchronize()  # the record was cleared
    assert lib.mbx_selftest_wait_timeout(ctx.handle, 0) == mbx.abi.ERR_INVALID_ARGUMENT
    f = ref_fixture
    w = mbx.Param(ctx, f["c1.w"])
    got = mbx.conv1x1(up(ctx, f["c1.x"]), w, up(ctx, f["c1.b"])).numpy()
    w.close()
    assert scaled_err(got, f["c1.y"]) <= REF_TOL
    ctx.synchronize()


@pytest.mark.parametrize("shape,k,co,dtype,with_add,with_res,act,upx", [
    ((16, 64, 64, 320), 1, 320, "f16", True, True, 0, False),   # UNet DwConv2d pointwise → norm2 (+ temb)
    ((2, 32, 32, 640), 1, 640, "f16", True, False, 0, False),
    ((2, 64, 64, 128), 3, 256, "f32", False, False, 0, False),  # VAE resnet conv1 → norm2
    ((1, 64, 64, 64), 3, 128, "f16", False, True, 0, True),     # upsampled 3×3: output 128 × 128
    ((1, 32, 32, 96), 1, 160, "f16", False, False, 1, False),   # SiLU epilogue, 160-wide N tiles
    ((2, 10, 12, 64), 1, 96, "f16", True, False, 0, False),     # 120-pixel maps: the separate statistics pass
])
def test_conv_group_norm_affine(mbx, ctx, oracle, shape, k, co, dtype, with_add, with_res, act, upx):
    """mbx_conv_group_norm_affine: the conv's output is the plain conv's bit for bit, and the
    GroupNorm affine built from the epilogue's statistics equals the separate statistics pass on
    that output at the GroupNorm tolerance, and the oracle's conv + GroupNorm::affine at the gates
    (src/engine/conv.rs:38-102, src/engine/norm.rs:57-129)."""
    rng = np.random.default_rng(sum(shape) + co + k)
    n, h, w, ci = shape
    groups = 32
    x = rng.standard_normal(shape).astype(np.float32)
    wshape = (co, ci) if k == 1 else (co, 3, 3, ci)
    wt = rng.normal(0.0, 1.0 / np.sqrt(ci * k * k), wshape).astype(np.float32)
    bias = rng.normal(0.0, 0.01, co).astype(np.float32)
    ho, wo = (2 * h, 2 * w) if upx else (h, w)
    res = rng.standard_normal((n, ho, wo, co)).astype(np.float32) if with_res else None
    add = rng.normal(0.0, 0.5, (n, co)).astype(np.float32) if with_add else None
    gamma = rng.normal(1.0, 0.1, co).astype(np.float32)
    beta = rng.normal(0.0, 0.1, co).astype(np.float32)
    p = mbx.Param(ctx, wt, dtype)
    xd, bd = up(ctx, x), up(ctx, bias)
    rd = up(ctx, res) if with_res else None
    ad = up(ctx, add) if with_add else None
    gd, betad = up(ctx, gamma), up(ctx, beta)
    out, sc, sh = mbx.conv_group_norm_affine(xd, p, groups, 1e-5, gd, betad, bias=bd, add=ad, upsample2x=upx,
                                             residual=rd, act=act)
    if k == 1:
        plain = ctx.empty((n, ho, wo, co))
        mbx.check(mbx.abi.lib().mbx_conv1x1_fused(ctx.handle, xd.vp, n, h, w, ci, p.handle, bd.vp, None, None, 0,
                                                 rd.vp if rd else None, act, plain.vp))
    else:
        plain = mbx.conv3x3(xd, p, bd, upsample2x=upx, residual=rd)
    got = out.numpy()
    assert np.array_equal(got, plain.numpy())
    sc2, sh2 = mbx.group_norm_affine(plain, groups, 1e-5, gd, betad, add=ad)
    assert scaled_err(sc.numpy(), sc2.numpy()) <= REF_TOL
    assert scaled_err(sh.numpy(), sh2.numpy()) <= REF_TOL
    wref = wt if dtype == "f32" else wt.astype(np.float16).astype(np.float32)
    want = oracle.conv1x1(x, wref, bias, res) if k == 1 else oracle.conv3x3(x, wref, bias, upsample2x=upx)
    if k == 3 and with_res:
        want = oracle.add(want, res)
    if act:
        want = oracle.silu(want)
    wsc, wsh = oracle.group_norm_affine(want, groups, 1e-5, gamma, beta, add=add)
    gate = GATE_F32 if dtype == "f32" else GATE_F16
    assert max_rel_err(got, want) <= gate
    assert max_rel_err(sc.numpy(), wsc) <= gate
    assert max_rel_err(sh.numpy(), wsh) <= gate
    p.close()
