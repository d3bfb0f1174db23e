"""CPU-only checks of the C-ABI library: it loads, exports every symbol the
header declares, and its host-side argument handling behaves like the
reference's C ABI (status codes + thread-local message, src/ffi.rs:1-103)
without touching a GPU."""
import ctypes

import pytest

from conftest import load_package


def test_library_exports_every_header_symbol():
    mbx = load_package()
    declared = mbx.abi.header_symbols()
    assert len(declared) >= 30
    lib = mbx.abi.lib()
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"
    assert sorted(mbx.abi.SIGNATURES) == declared, "ctypes signature table out of sync with the header"


def test_abi_version_and_error_string():
    mbx = load_package()
    lib = mbx.abi.lib()
    assert lib.mbx_abi_version() == 1
    assert lib.mbx_last_error() is not None


def test_conv3x3_output_hw_matches_reference_formula():
    # Conv3x3::output_hw, src/engine/conv.rs:77-81
    mbx = load_package()
    cases = [((9, 11, 1, (1, 1, 1, 1), False), (9, 11)), ((9, 11, 2, (1, 1, 1, 1), False), (5, 6)),
             ((9, 11, 2, (0, 0, 1, 1), False), (4, 5)), ((9, 11, 1, (1, 1, 1, 1), True), (18, 22)),
             ((64, 64, 2, (1, 1, 1, 1), False), (32, 32)), ((512, 512, 2, (0, 0, 1, 1), False), (256, 256))]
    for (h, w, s, pad, up), want in cases:
        assert mbx.conv3x3_output_hw(h, w, s, pad, up) == want


def test_invalid_arguments_return_status_and_message():
    mbx = load_package()
    lib = mbx.abi.lib()
    ho, wo = ctypes.c_int64(), ctypes.c_int64()
    pad = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    st = lib.mbx_conv3x3_output_hw(1, 1, 3, pad, 0, ctypes.byref(ho), ctypes.byref(wo))
    assert st == mbx.abi.ERR_INVALID_ARGUMENT
    assert b"stride" in lib.mbx_last_error()
    # Null context: reported, never dereferenced.
    assert lib.mbx_silu_inplace(None, None, 4) == mbx.abi.ERR_INVALID_ARGUMENT
    assert b"context" in lib.mbx_last_error()
    assert lib.mbx_ctx_create(0, None) == mbx.abi.ERR_INVALID_ARGUMENT
    assert lib.mbx_depthwise3x3_fused(None, None, 1, 4, 4, 8, None, None, 1, None, None, 1, None) == \
        mbx.abi.ERR_INVALID_ARGUMENT
    assert b"context" in lib.mbx_last_error()


def test_context_needs_a_b200():
    """Without a GPU (this CPU container) creation fails with UNSUPPORTED_DEVICE, like the
    reference's MOEBIUS_ERR_UNSUPPORTED_CPU on a CPU without AVX2/FMA."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    mbx = load_package()
    with pytest.raises(mbx.MbxError) as e:
        mbx.Context(0)
    assert e.value.code == mbx.abi.ERR_UNSUPPORTED_DEVICE
