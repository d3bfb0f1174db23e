"""Two GPUs driven from one process, the way include/moebius_cuda_engine.h
tells hosts to use several devices: one engine per device, each driven from
its own host thread. Kernel attributes that belong to a device (the dynamic
shared-memory limit of the conv, depthwise and λ kernels) must be set on each
device, from any thread. Each device's batch must be bit-identical to the
same batch run alone on device 0 first. The reference allows concurrent
inpaints by construction (src/pipeline.rs:119-136). Skipped with fewer than
two GPUs."""
import os
import threading

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu


def _batch(rng, n, side=128):
    lat = side // 8
    syn = load_package().synthetic
    img = rng.integers(0, 256, (n, side, side, 3), dtype=np.uint8)
    masks = syn.ellipse_masks(rng, n, side)
    nv = rng.standard_normal((2 * n, lat, lat, 4), dtype=np.float32)
    ni = rng.standard_normal((n, lat, lat, 4), dtype=np.float32)
    no = rng.standard_normal((n, 4), dtype=np.float32)
    return img, masks, (nv, ni, no)


def test_two_engines_on_two_devices_from_two_threads(mbx, ctx, tmp_path_factory):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    syn = mbx.synthetic
    d = str(tmp_path_factory.mktemp("two_devices"))
    syn.write_weights_dir(d, seed=0, f16=True, unet_widths=(64, 128, 256), latent=16, vae_widths=(32, 64, 128, 128))
    rng = np.random.default_rng(77)
    batches = [_batch(rng, 2), _batch(rng, 3)]
    p = mbx.engine.params(steps=4)

    # Alone, on device 0 (this also configures device 0's kernels first).
    want = []
    with mbx.engine.Engine(d, 0) as e0:
        for img, masks, noise in batches:
            out = img.copy()
            e0.inpaint_batch(out, masks, p, noise=noise)
            want.append(out)

    # Together: device 1 runs batch 0 and device 0 runs batch 1, each engine created and
    # driven by its own thread.
    got, errors = [None, None], []

    def work(device, which):
        try:
            img, masks, noise = batches[which]
            with mbx.engine.Engine(d, device) as e:
                for _ in range(2):
                    out = img.copy()
                    e.inpaint_batch(out, masks, p, noise=noise)
                got[which] = out
        except Exception as exc:  # reported below
            errors.append((device, repr(exc)))

    threads = [threading.Thread(target=work, args=(1, 0)), threading.Thread(target=work, args=(0, 1))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not errors, errors
    for which in (0, 1):
        assert got[which] is not None
        assert np.array_equal(got[which], want[which]), f"batch {which} differs from its single-device run"
    assert not np.array_equal(want[0], batches[0][0])
