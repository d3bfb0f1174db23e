"""GPU parity of the memory-bound kernels (GroupNorm, LayerNorm, depthwise,
elementwise) through the C ABI, against (1) the reference's PyTorch fixture
and the extra fixtures at the reference's tolerance (scaled error ≤ 1e-5,
tests/kernels.rs:29-38), and (2) the CPU oracle on BASELINE-shaped inputs
(memory-bound sweep shapes) with the per-kernel gate max relative error ≤ 1e-3.
"""
import numpy as np
import pytest

from conftest import max_rel_err, scaled_err

pytestmark = pytest.mark.gpu

REF_TOL = 1e-5
GATE = 1e-3


def up(ctx, a):
    return ctx.upload(a)


def test_group_norm_plain_and_fused(mbx, ctx, ref_fixture):
    f = ref_fixture
    x = up(ctx, f["gn.x"])
    g, b = up(ctx, f["gn.gamma"]), up(ctx, f["gn.beta"])
    assert scaled_err(mbx.group_norm(x, 32, 1e-6, g, b).numpy(), f["gn.y"]) <= REF_TOL
    add = up(ctx, f["gn.add"])
    got = mbx.group_norm(x, 32, 1e-5, g, b, add=add, silu=True).numpy()
    assert scaled_err(got, f["gn.y_add_silu"]) <= REF_TOL


def test_group_norm_two_channels_per_group(mbx, ctx, extra_fixture):
    f = extra_fixture
    got = mbx.group_norm(up(ctx, f["gn64.x"]), 32, 1e-6, up(ctx, f["gn64.gamma"]), up(ctx, f["gn64.beta"]),
                         add=up(ctx, f["gn64.add"]), silu=True).numpy()
    assert scaled_err(got, f["gn64.y"]) <= REF_TOL


def test_group_norm_affine_matches_oracle(mbx, ctx, oracle):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((2, 9, 13, 96)) * 2 + 0.5).astype(np.float32)
    gamma = rng.normal(1, 0.02, 96).astype(np.float32)
    beta = rng.normal(0, 0.02, 96).astype(np.float32)
    add = rng.standard_normal((2, 96)).astype(np.float32)
    sc, sh = mbx.group_norm_affine(up(ctx, x), 32, 1e-5, up(ctx, gamma), up(ctx, beta), up(ctx, add))
    wsc, wsh = oracle.group_norm_affine(x, 32, 1e-5, gamma, beta, add)
    assert max_rel_err(sc.numpy(), wsc) <= 1e-5
    assert scaled_err(sh.numpy(), wsh) <= 1e-5


def test_group_norm_apply_with_residual(mbx, ctx, oracle):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((2, 5, 7, 64)).astype(np.float32)
    r = rng.standard_normal((2, 5, 7, 64)).astype(np.float32)
    sc = rng.normal(1, 0.1, (2, 64)).astype(np.float32)
    sh = rng.normal(0, 0.1, (2, 64)).astype(np.float32)
    got = mbx.group_norm_apply(up(ctx, x), up(ctx, sc), up(ctx, sh), silu=True, residual=up(ctx, r)).numpy()
    want = oracle.add(oracle.group_norm_apply(x, sc, sh, silu=True), r)
    assert scaled_err(got, want) <= 1e-6


@pytest.mark.parametrize("shape", [(1, 32, 32, 64), (2, 64, 64, 128), (1, 128, 128, 256), (8, 32, 32, 512),
                                   (1, 64, 64, 320), (2, 16, 16, 2560)])
@pytest.mark.parametrize("silu", [False, True])
def test_group_norm_sweep_matches_oracle(mbx, ctx, oracle, shape, silu):
    rng = np.random.default_rng(sum(shape))
    n, h, w, c = shape
    x = rng.standard_normal(shape).astype(np.float32)
    gamma = rng.normal(1, 0.02, c).astype(np.float32)
    beta = rng.normal(0, 0.02, c).astype(np.float32)
    got = mbx.group_norm(up(ctx, x), 32, 1e-6, up(ctx, gamma), up(ctx, beta), silu=silu).numpy()
    want = oracle.group_norm(x, 32, 1e-6, gamma, beta, silu=silu)
    assert max_rel_err(got, want) <= GATE
    assert scaled_err(got, want) <= 1e-5


def test_group_norm_ragged_channels_scalar_path(mbx, ctx, oracle):
    # 36 channels in 12 groups: 4-wide vectors but 3 channels per group; 30 channels in 10 groups: scalar path.
    rng = np.random.default_rng(5)
    for c, g in ((36, 12), (30, 10)):
        x = rng.standard_normal((3, 7, 5, c)).astype(np.float32)
        gamma, beta = rng.normal(1, 0.3, c).astype(np.float32), rng.normal(0, 0.3, c).astype(np.float32)
        got = mbx.group_norm(up(ctx, x), g, 1e-5, up(ctx, gamma), up(ctx, beta), silu=True).numpy()
        assert scaled_err(got, oracle.group_norm(x, g, 1e-5, gamma, beta, silu=True)) <= REF_TOL


def test_layer_norm(mbx, ctx, ref_fixture, extra_fixture, oracle):
    f = ref_fixture
    got = mbx.layer_norm(up(ctx, f["ln.x"].reshape(3, 17, 1, 44)), up(ctx, f["ln.gamma"]), up(ctx, f["ln.beta"]),
                         1e-5).numpy()
    assert scaled_err(got.reshape(3, 17, 44), f["ln.y"]) <= REF_TOL
    e = extra_fixture
    got = mbx.layer_norm(up(ctx, e["ln320.x"].reshape(2, 37, 1, 320)), up(ctx, e["ln320.gamma"]),
                         up(ctx, e["ln320.beta"]), 1e-5).numpy()
    assert scaled_err(got.reshape(2, 37, 320), e["ln320.y"]) <= REF_TOL
    rng = np.random.default_rng(3)
    for c in (640, 1280, 13):
        x = rng.standard_normal((2, 16, 16, c)).astype(np.float32)
        g, b = rng.standard_normal(c).astype(np.float32), rng.standard_normal(c).astype(np.float32)
        got = mbx.layer_norm(up(ctx, x), up(ctx, g), up(ctx, b), 1e-5).numpy()
        assert scaled_err(got, oracle.layer_norm(x, g, b, 1e-5)) <= REF_TOL


def test_depthwise_epilogues(mbx, ctx, ref_fixture):
    f = ref_fixture
    x, w, b = up(ctx, f["dw.x"]), up(ctx, f["dw.w"]), up(ctx, f["dw.b"])
    assert scaled_err(mbx.depthwise3x3(x, w, b, "relu").numpy(), f["dw.relu"]) <= REF_TOL
    assert scaled_err(mbx.depthwise3x3(x, w, b, "glu_silu").numpy(), f["dw.glu"]) <= REF_TOL


def test_depthwise_tails(mbx, ctx, extra_fixture):
    f = extra_fixture
    got = mbx.depthwise3x3(up(ctx, f["dw70.x"]), up(ctx, f["dw70.w"]), up(ctx, f["dw70.b"])).numpy()
    assert scaled_err(got, f["dw70.y"]) <= REF_TOL
    got = mbx.depthwise3x3(up(ctx, f["dw140.x"]), up(ctx, f["dw140.w"]), up(ctx, f["dw140.b"]), "glu_silu").numpy()
    assert scaled_err(got, f["dw140.y"]) <= REF_TOL


@pytest.mark.parametrize("shape,ep", [((1, 32, 32, 64), "none"), ((8, 64, 64, 128), "relu"),
                                      ((2, 64, 64, 1600), "glu_silu"), ((2, 16, 16, 6400), "glu_silu"),
                                      ((1, 5, 7, 9), "relu"), ((2, 33, 17, 13), "none"), ((1, 1, 1, 8), "relu"),
                                      ((1, 40, 3, 26), "glu_silu"),
                                      # TMA-tiled kernel: ragged 16 × 16 tiles and a partial channel box
                                      ((1, 37, 45, 72), "glu_silu"), ((2, 20, 50, 96), "relu"),
                                      ((1, 18, 18, 36), "none"),
                                      # several tiles per persistent CTA: the two-stage ring wraps and
                                      # the channel block (and so the taps) changes between tiles
                                      ((4, 128, 128, 96), "none"), ((3, 48, 80, 200), "relu")])
def test_depthwise_matches_oracle(mbx, ctx, oracle, shape, ep):
    rng = np.random.default_rng(shape[-1] + len(ep))
    c = shape[-1]
    x = rng.standard_normal(shape).astype(np.float32)
    w = (rng.standard_normal((3, 3, c)) / np.sqrt(3.0)).astype(np.float32)
    b = rng.normal(0, 0.01, c).astype(np.float32)
    got = mbx.depthwise3x3(up(ctx, x), up(ctx, w), up(ctx, b), ep).numpy()
    want = oracle.depthwise3x3(x, w, b, ep)
    assert scaled_err(got, want) <= REF_TOL
    assert max_rel_err(got, want) <= GATE


@pytest.mark.parametrize("shape,ep,silu", [((2, 20, 50, 96), "relu", True), ((1, 37, 45, 72), "none", True),
                                           ((1, 40, 40, 64), "glu_silu", False), ((2, 64, 64, 320), "relu", True),
                                           # shapes the tiled kernel does not take: GroupNorm to scratch first
                                           ((2, 9, 9, 40), "relu", True), ((1, 20, 20, 12), "none", True)])
def test_depthwise_group_norm_prologue(mbx, ctx, oracle, shape, ep, silu):
    """mbx_depthwise3x3_fused equals GroupNorm apply + depthwise bit for bit, and the oracle's
    GroupNorm (with a per-item add, as the resnets' time embedding) + depthwise at the gate."""
    import math
    rng = np.random.default_rng(sum(shape) + len(ep))
    n, h, w, c = shape
    groups = math.gcd(c, 32)
    x = (rng.standard_normal(shape) * 2 + 0.5).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, c).astype(np.float32)
    beta = rng.normal(0, 0.2, c).astype(np.float32)
    add = rng.normal(0, 0.5, (n, c)).astype(np.float32)
    wt = (rng.standard_normal((3, 3, c)) / np.sqrt(3.0)).astype(np.float32)
    b = rng.normal(0, 0.01, c).astype(np.float32)
    xd, wd, bd = up(ctx, x), up(ctx, wt), up(ctx, b)
    sc, sh = mbx.group_norm_affine(xd, groups, 1e-5, up(ctx, gamma), up(ctx, beta), add=up(ctx, add))
    two_pass = mbx.depthwise3x3(mbx.group_norm_apply(xd, sc, sh, silu), wd, bd, ep).numpy()
    got = mbx.depthwise3x3(xd, wd, bd, ep, prologue=(sc, sh, silu)).numpy()
    assert np.array_equal(got, two_pass)
    want = oracle.depthwise3x3(oracle.group_norm(x, groups, 1e-5, gamma, beta, add=add, silu=silu), wt, b, ep)
    assert max_rel_err(got, want) <= GATE


def test_elementwise_fixture(mbx, ctx, extra_fixture):
    f = extra_fixture
    x = up(ctx, f["bt.x"])
    assert scaled_err(mbx.bias_temb_add(x, up(ctx, f["bt.bias"]), up(ctx, f["bt.temb"])).numpy(), f["bt.y"]) <= 1e-6
    a = up(ctx, f["bt.x"])
    mbx.add_inplace(a, up(ctx, f["bt.r"]))
    assert scaled_err(a.numpy(), f["bt.sum"]) <= 1e-6
    s = up(ctx, f["bt.x"])
    mbx.silu_inplace(s)
    assert scaled_err(s.numpy(), f["bt.silu"]) <= 1e-6


@pytest.mark.parametrize("shape", [(8, 64, 64, 512), (1, 32, 32, 64), (3, 5, 7, 13), (2, 1, 1, 1)])
def test_elementwise_matches_oracle(mbx, ctx, oracle, shape):
    rng = np.random.default_rng(sum(shape))
    n, c = shape[0], shape[-1]
    x = rng.standard_normal(shape).astype(np.float32)
    r = rng.standard_normal(shape).astype(np.float32)
    bias = rng.normal(0, 0.01, c).astype(np.float32)
    temb = rng.standard_normal((n, c)).astype(np.float32)
    got = mbx.bias_temb_add(up(ctx, x), up(ctx, bias), up(ctx, temb)).numpy()
    assert np.array_equal(got, oracle.bias_temb_add(x, bias, temb))
    got = mbx.bias_temb_add(up(ctx, x), None, up(ctx, temb)).numpy()
    assert np.array_equal(got, oracle.bias_temb_add(x, None, temb))
    a = up(ctx, x)
    mbx.add_inplace(a, up(ctx, r))
    assert np.array_equal(a.numpy(), oracle.add(x, r))
    s = up(ctx, x)
    mbx.silu_inplace(s)
    assert scaled_err(s.numpy(), oracle.silu(x)) <= 1e-6


def test_concat_channels(mbx, ctx, oracle):
    rng = np.random.default_rng(9)
    for ca, cb in ((1280, 1280), (13, 7), (640, 320)):
        a = rng.standard_normal((2, 5, 6, ca)).astype(np.float32)
        b = rng.standard_normal((2, 5, 6, cb)).astype(np.float32)
        got = mbx.concat_channels(up(ctx, a), up(ctx, b)).numpy()
        assert np.array_equal(got, oracle.concat_channels(a, b))


def test_matmul_strided(mbx, ctx, oracle):
    rng = np.random.default_rng(4)
    for m, k, n in ((7, 5, 3), (67, 129, 45), (300, 64, 257)):
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        c = rng.standard_normal((m, n)).astype(np.float32)
        got = mbx.matmul(up(ctx, a), up(ctx, b)).numpy()
        want = a.astype(np.float64) @ b.astype(np.float64)
        assert np.max(np.abs(got - want)) < 1e-4 * max(1, np.sqrt(k))
        cd = up(ctx, c)
        mbx.matmul(up(ctx, a), up(ctx, b), cd, accumulate=True)
        assert np.max(np.abs(cd.numpy() - (want + c))) < 1e-4 * max(1, np.sqrt(k))


def test_empty_inputs_are_no_ops(mbx, ctx):
    x = ctx.empty((0, 4, 4, 8))
    g, b = up(ctx, np.ones(8, np.float32)), up(ctx, np.zeros(8, np.float32))
    mbx.group_norm(x, 4, 1e-6, g, b)
    mbx.depthwise3x3(x, up(ctx, np.ones((3, 3, 8), np.float32)), b)
    mbx.silu_inplace(ctx.empty((0,)))
    ctx.synchronize()


def test_shape_errors_are_reported_not_aborted(mbx, ctx):
    x = up(ctx, np.zeros((1, 4, 4, 30), np.float32))
    g = up(ctx, np.ones(30, np.float32))
    with pytest.raises(mbx.MbxError) as e:
        mbx.group_norm(x, 32, 1e-6, g, g)  # 30 channels, 32 groups
    assert e.value.code == mbx.abi.ERR_INVALID_ARGUMENT
    with pytest.raises(mbx.MbxError):
        mbx.depthwise3x3(up(ctx, np.zeros((1, 2, 2, 3), np.float32)), up(ctx, np.zeros((3, 3, 3), np.float32)),
                         up(ctx, np.zeros(3, np.float32)), "glu_silu")  # odd channels for GLU
    ctx.synchronize()


def test_pool_reuses_blocks(mbx, ctx):
    a = ctx.empty((1024, 1024))
    p = a.ptr
    a.free()
    b = ctx.empty((1024, 1024))
    assert b.ptr == p, "a freed block of the same size is handed back (Scratch::tensor_for)"
    b.free()
    cached, _ = ctx.pool_stats()
    assert cached >= 4 << 20
    ctx.release_below(1 << 40)
    cached, _ = ctx.pool_stats()
    assert cached == 0


@pytest.mark.parametrize("shape,add,silu", [((8, 128, 128, 256), False, True), ((2, 256, 256, 512), True, True),
                                            ((4, 512, 512, 64), False, False)])
def test_group_norm_large_tensors(mbx, ctx, oracle, shape, add, silu):
    """Tensors larger than L2 (the statistics pass and the apply pass both stream from DRAM)."""
    rng = np.random.default_rng(shape[-1] * 7 + shape[0])
    n, h, w, c = shape
    x = (rng.standard_normal(shape, dtype=np.float32) * 1.5 + 0.2).astype(np.float32)
    gamma = rng.normal(1, 0.02, c).astype(np.float32)
    beta = rng.normal(0, 0.02, c).astype(np.float32)
    a = rng.standard_normal((n, c)).astype(np.float32) if add else None
    got = mbx.group_norm(up(ctx, x), 32, 1e-6, up(ctx, gamma), up(ctx, beta), add=up(ctx, a) if add else None,
                         silu=silu).numpy()
    want = oracle.group_norm(x, 32, 1e-6, gamma, beta, a, silu=silu)
    assert max_rel_err(got, want) <= GATE
    assert scaled_err(got, want) <= REF_TOL
