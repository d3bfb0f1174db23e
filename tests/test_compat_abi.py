"""CPU-only checks of the moebius-cpu drop-in (include/moebius_cpu.h): the
reference's outer C API names (moebius_abi_version, moebius_last_error,
moebius_engine_create / destroy, moebius_inpaint; reference
include/moebius_cpu.h:48-67, src/ffi.rs:105-233) exported by
libmoebius_cuda.so.

A small C host that calls every entry point the way a moebius-cpu host would
is compiled with gcc against this repository's header and linked to the
library. Where the reference checkout is available (MOEBIUS_REFERENCE_ROOT,
default: a `reference` directory beside this repository), the same host is also compiled against the
reference's own header, unmodified, and linked to this library, and the
struct layouts seen through both headers are compared. Without a GPU,
engine creation must fail with the reference's MOEBIUS_ERR_UNSUPPORTED_CPU
(3) and a message; argument errors come back as the reference reports them.
"""
import ctypes
import os
import shutil
import subprocess

import pytest

from conftest import REPO, load_package

LIBDIR = os.path.join(REPO, "moebius-cpu_b200", "lib")
OUR_INCLUDE = os.path.join(REPO, "include")
REF_ROOT = os.environ.get("MOEBIUS_REFERENCE_ROOT", os.path.join(os.path.dirname(REPO), "reference"))
REF_INCLUDE = os.path.join(REF_ROOT, "include")

HOST_C = r"""
#include <stddef.h>
#include <stdio.h>
#include <string.h>
#include "moebius_cpu.h"

static int32_t on_progress(void *user, uint32_t stage, uint32_t done, uint32_t total) {
    (void)user; (void)stage; (void)done; (void)total;
    return 0;
}

int main(void) {
    /* Layout of the shared structs, as this header declares them. */
    printf("layout %zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(MoebiusParams), offsetof(MoebiusParams, steps),
           offsetof(MoebiusParams, guidance), offsetof(MoebiusParams, seed), offsetof(MoebiusParams, paste),
           offsetof(MoebiusParams, mask_dilate), sizeof(MoebiusRect), offsetof(MoebiusRect, height));
    printf("abi %u %u\n", moebius_abi_version(), (unsigned)MOEBIUS_ABI_VERSION);
    printf("last_error_not_null %d\n", moebius_last_error() != NULL);
    MoebiusEngine *engine = (MoebiusEngine *)0x1;
    int32_t st = moebius_engine_create(NULL, 0, &engine);
    printf("create_null_dir %d %d\n", st, engine == (MoebiusEngine *)0x1);
    engine = (MoebiusEngine *)0x1;
    st = moebius_engine_create("/nonexistent-weights", 4, &engine);
    printf("create %d %d %s\n", st, engine == (MoebiusEngine *)0x1, moebius_last_error());
    uint8_t px[4 * 4 * 3] = {0}, mask[4 * 4] = {0};
    MoebiusParams p;
    memset(&p, 0, sizeof p);
    p.preset = MOEBIUS_PRESET_EXACT;
    p.paste = MOEBIUS_PASTE_FEATHER;
    MoebiusRect changed = {1, 2, 3, 4};
    st = moebius_inpaint(NULL, px, 4, 4, 12, 3, mask, 4, &p, on_progress, NULL, &changed);
    printf("inpaint_null_engine %d\n", st);
    moebius_engine_destroy(NULL);
    printf("codes %d %d %d %d %d %d %d\n", MOEBIUS_OK, MOEBIUS_ERR_INVALID_ARGUMENT, MOEBIUS_ERR_WEIGHTS,
           MOEBIUS_ERR_UNSUPPORTED_CPU, MOEBIUS_ERR_CANCELLED, MOEBIUS_ERR_IO, MOEBIUS_ERR_INTERNAL);
    return 0;
}
"""


def _gpu_present():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def _build_and_run(tmp_path, include_dir, tag):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not installed")
    src = tmp_path / f"host_{tag}.c"
    src.write_text(HOST_C)
    exe = tmp_path / f"host_{tag}"
    subprocess.run([gcc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", include_dir, str(src), "-o", str(exe),
                    "-L", LIBDIR, "-lmoebius_cuda", f"-Wl,-rpath,{LIBDIR}"], check=True, capture_output=True)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")  # no device: creation must fail cleanly
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, env=env).stdout
    return {ln.split()[0]: ln.split()[1:] for ln in out.splitlines() if ln.strip()}


def test_library_exports_the_reference_names():
    mbx = load_package()
    declared = mbx.abi.compat_header_symbols()
    assert declared == ["moebius_abi_version", "moebius_engine_create", "moebius_engine_destroy",
                        "moebius_inpaint", "moebius_last_error"]
    lib = mbx.abi.lib()
    assert all(hasattr(lib, s) for s in declared)
    assert sorted(mbx.abi.COMPAT_SIGNATURES) == declared
    assert lib.moebius_abi_version() == 1
    assert lib.moebius_last_error() is not None


def test_c_host_against_our_header(tmp_path):
    load_package().abi.lib()  # the library is built
    r = _build_and_run(tmp_path, OUR_INCLUDE, "ours")
    assert r["abi"] == ["1", "1"]
    assert r["last_error_not_null"] == ["1"]
    # MOEBIUS_ERR_INVALID_ARGUMENT; *out is written only on success (src/ffi.rs:120-139)
    assert r["create_null_dir"] == ["1", "1"]
    assert r["inpaint_null_engine"] == ["1"]
    assert r["codes"] == ["0", "1", "2", "3", "4", "5", "6"]
    if not _gpu_present():
        assert r["create"][:2] == ["3", "1"], r["create"]  # MOEBIUS_ERR_UNSUPPORTED_CPU, *out untouched
        assert len(r["create"]) > 2, "a message in moebius_last_error()"


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_INCLUDE, "moebius_cpu.h")),
                    reason="reference checkout not available")
def test_c_host_against_the_reference_header_links_and_matches(tmp_path):
    """The reference's unmodified header, this library: the host compiles, links, runs, and
    sees the same constants and struct layouts as through this repository's header."""
    load_package().abi.lib()
    ours = _build_and_run(tmp_path, OUR_INCLUDE, "ours")
    ref = _build_and_run(tmp_path, REF_INCLUDE, "ref")
    assert ref["layout"] == ours["layout"]
    assert ref["codes"] == ours["codes"]
    assert ref["abi"] == ours["abi"]
    assert ref["create_null_dir"] == ours["create_null_dir"]
    assert ref["inpaint_null_engine"] == ours["inpaint_null_engine"]
    assert ref["create"][:2] == ours["create"][:2]


def test_params_struct_matches_the_engine_params():
    """moebius_inpaint forwards MoebiusParams as mbx_inpaint_params: same layout."""
    mbx = load_package()
    assert ctypes.sizeof(mbx.abi.InpaintParams) == 32
    assert mbx.abi.InpaintParams.seed.offset == 16
