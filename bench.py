#!/usr/bin/env python
"""Benchmark of the moebius-cuda engine kernel layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload (the memory-bound sweep, at its largest shape):
one step runs the sweep's four ops over an NHWC f32 batch [8, 512, 512, 512]
(4 GiB, larger than L2, so no flush is needed between steps):

    y1 = SiLU(GroupNorm32(x))           8 B/elt  (read x, write y1)
    y2 = y1 + bias[c] + temb[item, c]   8 B/elt
    y2 += x        (residual add)      12 B/elt
    y4 = depthwise3x3(y2) + bias        8 B/elt

The metric is algorithmic bytes per second (36 B/elt per step), whole job.
Each rank owns its own batch (independent inputs, no collective on the data
path: weak scaling); torch.distributed only carries the barrier and the
max-over-ranks of the device time.

Printed on rank 0 as one JSON line, also with the roofline of the dominant
op, the CPU baseline (the oracle port on the host cores), the end-to-end
number through the C ABI with pinned host buffers (H2D of x, D2H of y4 in
the timed region), the tensor-core conv sweep's largest shape, the SM clocks
sampled during the timed region and the count of this library's kernel
launches.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

SHAPE = (8, 512, 512, 512)
CPU_SAMPLE = (1, 128, 256, 512)
BYTES_PER_ELT = {"group_norm_silu": 8, "bias_temb_add": 8, "residual_add": 12, "depthwise3x3": 8}
METRIC = ("memory-bound sweep throughput (GroupNorm32+SiLU, bias+temb add, residual add, depthwise 3x3) "
          "in algorithmic GB/s")
UNIT = "GB/s"
CONV_SHAPE = (8, 256, 256, 512, 512)  # n, h, w, c_in, c_out: the conv sweep's largest 3x3 case


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def config(args):
    return {"workload": "BASELINE configs[1] memory-bound sweep, largest shape; 4 ops per step",
            "shape_nhwc": list(SHAPE), "groups": 32, "eps": 1e-6, "dtype": "f32",
            "per_rank_batch": SHAPE[0], "global_batch": SHAPE[0] * args.gpus, "parallelism": f"dp{args.gpus}",
            "l2": "inputs (4 GiB per tensor) larger than L2; no flush"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_uuid: str | None):
        self.uuid = gpu_uuid
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- helpers
def traffic_from_profiles(kernel_key: str):
    """Per-launch DRAM traffic (bytes) of a kernel at the bench shape, from a committed ncu summary."""
    pdir = os.path.join(REPO, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if kernel_key in name:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(os.path.join(pdir, name)).read())
            if m:
                return float(m.group(1))
    return None


def cpu_baseline(steps=3):
    """The oracle (CPU restatement of the reference kernels) on a bounded sample, all host threads."""
    from oracle import oracle
    threads = oracle.set_threads(0)
    rng = np.random.default_rng(1234)
    n, h, w, c = CPU_SAMPLE
    x = rng.standard_normal(CPU_SAMPLE, dtype=np.float32)
    gamma = (1.0 + 0.02 * rng.standard_normal(c)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(c)).astype(np.float32)
    bias = (0.01 * rng.standard_normal(c)).astype(np.float32)
    temb = rng.standard_normal((n, c), dtype=np.float32)
    dw_w = (rng.standard_normal((3, 3, c)) / np.sqrt(3.0)).astype(np.float32)
    dw_b = (0.01 * rng.standard_normal(c)).astype(np.float32)
    best = None
    for _ in range(steps):
        t0 = time.perf_counter()
        y1 = oracle.group_norm(x, 32, 1e-6, gamma, beta, silu=True)
        y2 = oracle.bias_temb_add(y1, bias, temb)
        y2 = oracle.add(y2, x)
        oracle.depthwise3x3(y2, dw_w, dw_b, "none")
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    elems = int(np.prod(CPU_SAMPLE))
    gbs = sum(BYTES_PER_ELT.values()) * elems / best / 1e9
    return {"value": round(gbs, 2), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"the same 4-op step on {list(CPU_SAMPLE)} (oracle/ref_engine.cpp, OpenMP), best of {steps}",
            "seconds_per_sample_step": round(best, 4)}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    return world, rank, local, dist


def tf32_peak(torch):
    """Dense TF32 throughput of cuBLAS (8192^3 matmul, TF32 on), burst best of 10: the conv roofline."""
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device="cuda")
    b = torch.randn(8192, 8192, device="cuda")
    for _ in range(3):
        torch.matmul(a, b)
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e) / 1e3)
    torch.backends.cuda.matmul.allow_tf32 = False
    del a, b
    return 2 * 8192 ** 3 / best / 1e12


def decoder_flops(lat_h, lat_w):
    """Direct-conv FLOPs of one decoder pass (1×1 and 3×3 convs, attention GEMMs)."""
    vae = importlib.import_module("moebius-cpu_b200.vae")
    total, h, w = 0.0, lat_h, lat_w
    shapes = vae.decoder_weight_shapes()
    # conv layers run at the resolution of their level
    res = {"post_quant_conv": (h, w), "decoder.conv_in": (h, w), "decoder.mid_block": (h, w),
           "decoder.conv_out": (8 * h, 8 * w), "decoder.conv_norm_out": (8 * h, 8 * w)}
    for name, shp in shapes.items():
        if not name.endswith(".weight") or len(shp) < 2:
            continue
        if name.startswith("decoder.up_blocks."):
            lvl = int(name.split(".")[2])
            hh, ww = h << lvl, w << lvl
            if ".upsamplers." in name:
                hh, ww = hh * 2, ww * 2
        else:
            key = next(k for k in res if name.startswith(k))
            hh, ww = res[key]
        taps = 9 if len(shp) == 4 else 1
        total += 2.0 * hh * ww * shp[0] * shp[-1] * taps
    hw = h * w
    total += 2 * 2.0 * hw * hw * vae.VAE_BLOCK_OUT[-1]  # q·kᵀ and p·v
    return total


def bench_vae_decoder(mbx, ctx, torch, small=False):
    vae = importlib.import_module("moebius-cpu_b200.vae")
    lat_hw = 16 if small else 64
    w = vae.random_decoder_weights(0, f16=True)
    dec = vae.Decoder(ctx, w, "f16")
    out = {"workload": f"BASELINE configs[3]: VAE decoder, latent [B,{lat_hw},{lat_hw},4] -> "
                       f"[B,{8 * lat_hw},{8 * lat_hw},3], seeded random-init f16 weights (2xTF32)",
           "gflop_per_image": round(decoder_flops(lat_hw, lat_hw) / 1e9, 1)}
    gen = torch.Generator(device="cuda").manual_seed(7)
    for bsz in (1, 8):
        lat = torch.randn(bsz, lat_hw, lat_hw, 4, device="cuda", generator=gen) * vae.SCALING_FACTOR
        L = mbx.DeviceTensor.wrap(ctx, lat.data_ptr(), tuple(lat.shape))
        for _ in range(2):
            dec.decode(L)
        torch.cuda.synchronize()
        reps = 3
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(reps):
            img = dec.decode(L)
        e_ev.record()
        e_ev.synchronize()
        ms = s_ev.elapsed_time(e_ev) / reps
        out[f"b{bsz}"] = {"ms": round(ms, 2), "images_per_s": round(bsz / (ms / 1e3), 2),
                          "useful_tflops": round(bsz * decoder_flops(lat_hw, lat_hw) / (ms / 1e3) / 1e12, 1)}
        del img
    dec.close()
    return out


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch

    world, rank, local, dist = init_dist()
    torch.cuda.set_device(local)
    mbx = importlib.import_module("moebius-cpu_b200")
    ctx = mbx.Context(local)
    # One explicit stream for torch's events and this library's kernels (the legacy
    # default stream has handle 0, which mbx_ctx_set_stream reads as "own stream").
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    assert ctx.stream == stream.cuda_stream
    dev = torch.device("cuda", local)
    n, h, w, c = SHAPE
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    x = torch.randn(SHAPE, device=dev, generator=gen)
    gamma = 1.0 + 0.02 * torch.randn(c, device=dev, generator=gen)
    beta = 0.02 * torch.randn(c, device=dev, generator=gen)
    bias = 0.01 * torch.randn(c, device=dev, generator=gen)
    temb = torch.randn(n, c, device=dev, generator=gen)
    dw_w = torch.randn(3, 3, c, device=dev, generator=gen) / 3 ** 0.5
    dw_b = 0.01 * torch.randn(c, device=dev, generator=gen)
    y1, y2, y4 = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    W = lambda t: mbx.DeviceTensor.wrap(ctx, t.data_ptr(), tuple(t.shape))  # noqa: E731
    X, G, B, BI, TE, DW, DB = map(W, (x, gamma, beta, bias, temb, dw_w, dw_b))
    Y1, Y2, Y4 = W(y1), W(y2), W(y4)

    ops = [
        ("group_norm_silu", lambda: mbx.group_norm(X, 32, 1e-6, G, B, silu=True, out=Y1)),
        ("bias_temb_add", lambda: mbx.bias_temb_add(Y1, BI, TE, out=Y2)),
        ("residual_add", lambda: mbx.add_inplace(Y2, X)),
        ("depthwise3x3", lambda: mbx.depthwise3x3(Y2, DW, DB, "none", out=Y4)),
    ]

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        for _, f in ops:
            f()
    barrier()
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid) if hasattr(
        torch.cuda.get_device_properties(dev), "uuid") else None)
    if sampler.uuid and not sampler.uuid.startswith("GPU-"):
        sampler.uuid = "GPU-" + sampler.uuid
    sampler.start()
    time.sleep(0.3)
    ev = {name: [] for name, _ in ops}
    launches0 = ctx.launch_count
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        for name, f in ops:
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            f()
            e_ev.record()
            ev[name].append((s_ev, e_ev))
    end.record()
    barrier()
    launches = ctx.launch_count - launches0
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / args.steps
    op_ms = {k: float(np.mean([a.elapsed_time(b) for a, b in v])) for k, v in ev.items()}
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    elems = int(np.prod(SHAPE))
    step_bytes = sum(BYTES_PER_ELT.values()) * elems
    value = world * step_bytes / (ms_max / 1e3) / 1e9

    # Parity spot-check of this very run (size-independent properties on the device result).
    ok = bool(torch.isfinite(y4).all().item())

    # End to end through the C ABI with pinned host buffers: H2D x, the 4 ops, D2H y4.
    e2e = None
    if not args.skip_e2e:
        nbytes = x.numel() * 4
        hx = mbx.Context.host_alloc(nbytes)
        hy = mbx.Context.host_alloc(nbytes)
        try:
            ctx.copy_d2h(hx, x.data_ptr(), nbytes)
            ctx.synchronize()
            e2e_steps = max(1, min(3, args.steps))
            barrier()
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(e2e_steps):
                ctx.copy_h2d(x.data_ptr(), hx, nbytes)
                for _, f in ops:
                    f()
                ctx.copy_d2h(hy, y4.data_ptr(), nbytes)
            e_ev.record()
            barrier()
            e_ms = s_ev.elapsed_time(e_ev) / e2e_steps
            te = torch.tensor([e_ms], device=dev, dtype=torch.float64)
            if dist:
                dist.all_reduce(te, op=dist.ReduceOp.MAX)
            e2e = {"value": round(world * step_bytes / (float(te.item()) / 1e3) / 1e9, 2), "unit": UNIT,
                   "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes, "ms_per_step": round(float(te.item()), 3),
                   "path": "mbx C ABI: mbx_memcpy_h2d from pinned host, 4 ops, mbx_memcpy_d2h to pinned host"}
        finally:
            mbx.Context.host_free(hx)
            mbx.Context.host_free(hy)

    # Tensor-core conv sweep, largest 3x3 shape (f16 and f32 weights).
    conv = None
    if not args.skip_conv and rank == 0:
        cn, chh, cww, cci, cco = CONV_SHAPE
        del y1, y2
        torch.cuda.empty_cache()
        cx = torch.randn(cn, chh, cww, cci, device=dev, generator=gen)
        cy = torch.empty(cn, chh, cww, cco, device=dev)
        wt = (torch.randn(cco, 3, 3, cci, generator=torch.Generator().manual_seed(7)) / (9 * cci) ** 0.5).numpy()
        cb = 0.01 * torch.randn(cco, device=dev, generator=gen)
        CX, CY, CB = W(cx), W(cy), W(cb)
        flops = 2.0 * cn * chh * cww * 9 * cci * cco
        tf32 = tf32_peak(torch)
        conv = {"shape": f"[{cn},{chh},{cww},{cci}] -> {cco}, 3x3 pad 1, bias", "tf32_dense_peak_tflops": round(tf32, 1),
                "tf32_peak_source": "measured here: cuBLAS 8192^3 TF32 matmul, best of 10"}
        for dtype in ("f16", "f32"):
            p = mbx.Param(ctx, wt, dtype)
            for _ in range(2):
                mbx.conv3x3(CX, p, CB, out=CY)
            torch.cuda.synchronize()
            reps = 5
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(reps):
                mbx.conv3x3(CX, p, CB, out=CY)
            e_ev.record()
            e_ev.synchronize()
            cms = s_ev.elapsed_time(e_ev) / reps
            mmas = 2 if dtype == "f16" else 3
            useful = flops / (cms / 1e3) / 1e12
            conv[dtype] = {"ms": round(cms, 3), "useful_tflops": round(useful, 1),
                           "issued_tflops": round(useful * mmas, 1), "mma_per_product": mmas,
                           "issued_frac_of_tf32_peak": round(useful * mmas / tf32, 3)}
            p.close()

    # the full VAE decoder (64×64 latent → 512×512 RGB), B = 1 and B = 8.
    vae_line = None
    if not args.skip_vae and rank == 0:
        vae_line = bench_vae_decoder(mbx, ctx, torch, small=args.small)

    hbm, peak_kind = peaks()
    dom = max(op_ms, key=op_ms.get)
    achieved = BYTES_PER_ELT[dom] * elems / (op_ms[dom] / 1e3) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) NHWC f32, generated on device)",
            "config": config(args),
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": BYTES_PER_ELT[dom] * elems,
                         "traffic": traffic_from_profiles(dom)},
            "ops_ms": {k: round(v, 4) for k, v in op_ms.items()},
            "ops_frac_of_hbm": {k: round(BYTES_PER_ELT[k] * elems / (v / 1e3) / 1e9 / hbm, 4)
                                for k, v in op_ms.items()},
            "e2e": e2e, "gpu_launches": launches, "clocks": clocks, "result_finite": ok,
            "conv": conv,
            "vae_decoder": vae_line,
        }
        if not args.skip_cpu:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle
    threads = oracle.set_threads(0)
    rng = np.random.default_rng(1234)
    n, h, w, c = CPU_SAMPLE
    x = rng.standard_normal(CPU_SAMPLE, dtype=np.float32)
    gamma = (1.0 + 0.02 * rng.standard_normal(c)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(c)).astype(np.float32)
    bias = (0.01 * rng.standard_normal(c)).astype(np.float32)
    temb = rng.standard_normal((n, c), dtype=np.float32)
    dw_w = (rng.standard_normal((3, 3, c)) / np.sqrt(3.0)).astype(np.float32)
    dw_b = (0.01 * rng.standard_normal(c)).astype(np.float32)

    def step():
        y1 = oracle.group_norm(x, 32, 1e-6, gamma, beta, silu=True)
        y2 = oracle.bias_temb_add(y1, bias, temb)
        y2 = oracle.add(y2, x)
        oracle.depthwise3x3(y2, dw_w, dw_b, "none")

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    elems = int(np.prod(CPU_SAMPLE))
    value = sum(BYTES_PER_ELT.values()) * elems / dt / 1e9
    sample = (f"each step: the same 4-op step on {list(CPU_SAMPLE)} (a bounded sample of the "
              f"{list(SHAPE)} workload); oracle/ref_engine.cpp, the C++ restatement of the reference's "
              "Rust kernels (the Rust crate cannot be built here: no cargo)")
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) NHWC f32)", "config": config(args),
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-conv", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-vae", action="store_true")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: [1,256,256,512] sweep (128 MiB, above L2) and a [1,128,128,512] conv")
    args = ap.parse_args()
    if args.small:
        global SHAPE, CONV_SHAPE
        SHAPE = (1, 256, 256, 512)
        CONV_SHAPE = (1, 128, 128, 512, 512)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
