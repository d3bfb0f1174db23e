#!/usr/bin/env python
"""Benchmark of moebius-cuda on B200: Exact-preset 512² inpaints per second.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload: end-to-end Exact inpaints of 512×512 RGB u8
images ~U[0,255] with binary masks of random filled ellipses covering 10-40 %,
seeded latent noise, the 0.22B Moebius UNet + SDXL VAE with seeded
random-init f16 weights in the reference converter's format (no checkpoint
offline), preset.rs Exact: 20 steps at strength 0.99 (19 DDIM steps from
t = 900), CFG 2.5 (UNet batch 2 per inpaint), noise offset 0.0357, VAE encode
of [image, masked] and decode, Pillow-blur feathered paste.

One step = one batch of B inpaints per GPU (default 8): prepare → VAE encode
(2B images) → 19 × (UNet at batch 2B replayed from a CUDA graph, CFG + DDIM)
→ VAE decode (B) → blur + paste. `value` = inpaints/s of the whole job with
the inputs already in HBM (device-timed, max over ranks; L2 flushed between
steps); `e2e` = the same through mbx_inpaint_batch with pinned host buffers
(pixels, masks and noise copied in and the pixels out inside the timed region).
Each rank owns its own inpaints (weak scaling, no collective on the data path;
torch.distributed carries only the barrier and the max of the device times).

Also in the line: the roofline of the dominant kernel (the tcgen05 implicit-
GEMM conv, timed live on the conv sweep's largest 3×3 shape against the
measured cuBLAS TF32 peak), the memory-bound sweep (its
largest shape, against the measured HBM copy bandwidth), the VAE decoder
(configs[3], B = 1 and 8), the CPU baseline (the oracle on the host cores), SM
clocks sampled during the timed region and this library's kernel launches.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import re
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "512x512 Exact-preset inpaints/s (UNet + VAE + DDIM, CFG 2.5, 19 steps), whole job"
UNIT = "inpaints/s"
SIDE = 512
LATENT = 64
STEPS_EXACT = 20
# The reference's own per-inpaint FLOP count (upstream count: UNet 632 GFLOP/step × 19
# + VAE encode 2233 + decode 2515 GFLOP), used to express inpaints/s as TFLOP/s.
INPAINT_TFLOP = 16.76
SWEEP_SHAPE = (8, 512, 512, 512)
BYTES_PER_ELT = {"group_norm_silu": 8, "bias_temb_add": 8, "residual_add": 12, "depthwise3x3": 8}
CONV_SHAPE = (8, 256, 256, 512, 512, 9)  # n, h, w, c_in, c_out, taps: the conv sweep's largest 3×3 case
SWEEP_OVERRIDE = None  # --sweep-shape: another memory-sweep shape (profiling cases)
L2_FLUSH_BYTES = 256 << 20


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def config(args):
    return {"workload": "BASELINE configs[4]: end-to-end Exact inpaint, 512x512 RGB, random-ellipse masks "
                        "10-40 %, 0.22B UNet + SDXL VAE (seeded random-init f16 weights)",
            "model": "moebius student UNet (320/640/1280, lambda layers) + SDXL VAE", "image": [SIDE, SIDE, 3],
            "per_rank_batch": args.batch, "global_batch": args.batch * args.gpus, "parallelism": f"dp{args.gpus}",
            "preset": {"steps": STEPS_EXACT, "strength": 0.99, "denoise_steps": 19, "guidance": 2.5,
                       "noise_offset": 0.0357, "scheduler": "DDIM leading", "paste": "feather"},
            "weights": "f16 GEMM weights (2xTF32 products), f32 accumulation",
            "l2": f"flushed between steps ({L2_FLUSH_BYTES >> 20} MiB write)"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
               "-i", str(self.index)]
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


def traffic_from_profiles(kernel_key: str):
    """Per-launch DRAM traffic (bytes) at the bench shape, from a committed ncu summary."""
    pdir = os.path.join(REPO, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if kernel_key in name:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(os.path.join(pdir, name)).read())
            if m:
                return float(m.group(1))
    return None


def traffic_ratios_from_profiles():
    """DRAM bytes ÷ algorithmic bytes per memory-bound op, from the committed ncu summaries."""
    pdir = os.path.join(REPO, "profiles")
    out = {}
    if os.path.isdir(pdir):
        for name in sorted(os.listdir(pdir)):
            for m in re.finditer(r"traffic_ratio_([a-z0-9_]+):\s*([0-9.]+)", open(os.path.join(pdir, name)).read()):
                out[m.group(1)] = float(m.group(2))
    return out


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local, dist


def weights_dir(rank, dist, small):
    """Seeded converter-format weights, written once per box (rank 0) and shared by the ranks."""
    syn = importlib.import_module("moebius-cpu_b200.synthetic")
    tag = "small" if small else "full"
    d = os.path.join(tempfile.gettempdir(), f"moebius_b200_bench_weights_{tag}_seed0")
    done = os.path.join(d, "complete")
    if rank == 0 and not os.path.exists(done):
        if small:
            syn.write_weights_dir(d, seed=0, f16=True, unet_widths=(64, 128, 256), latent=16,
                                  vae_widths=(32, 64, 128, 128))
        else:
            syn.write_weights_dir(d, seed=0, f16=True)
        open(done, "w").close()
    if dist:
        dist.barrier()
    return d


def synthetic_inputs(rank, n, side):
    """Seeded images ~U[0,255], ellipse masks (10-40 %), and the pipeline's noise tensors."""
    syn = importlib.import_module("moebius-cpu_b200.synthetic")
    rng = np.random.default_rng(1234 + rank)
    lat = side // 8
    img = rng.integers(0, 256, (n, side, side, 3), dtype=np.uint8)
    masks = syn.ellipse_masks(rng, n, side)
    nv = rng.standard_normal((2 * n, lat, lat, 4), dtype=np.float32)
    ni = rng.standard_normal((n, lat, lat, 4), dtype=np.float32)
    no = rng.standard_normal((n, 4), dtype=np.float32)
    return img, masks, nv, ni, no


# --------------------------------------------------------------------------- CPU baseline (the oracle)
def cpu_inpaint_baseline(small=False):
    """The oracle on a bounded sample of one inpaint: one UNet CFG step (batch 2), the VAE encode
    of [image, masked] and the decode, each timed once on all host threads; an inpaint costs
    19 UNet steps + encode + decode (the element work between them is negligible)."""
    from oracle import oracle, unet_ref, vae_ref
    syn = importlib.import_module("moebius-cpu_b200.synthetic")
    threads = oracle.set_threads(0)
    if small:
        wu = syn.random_weights(syn.unet_shapes((64, 128, 256), 16), 0)
        wv = syn.random_weights(syn.vae_shapes((32, 64, 128, 128)), 1)
        side = 128
    else:
        wu = syn.random_weights(syn.unet_shapes(), 0)
        wv = syn.random_weights(syn.vae_shapes(), 1)
        side = SIDE
    lat = side // 8
    rng = np.random.default_rng(99)
    ehs = unet_ref.conditioning(wu)
    x = rng.standard_normal((2, lat, lat, 9)).astype(np.float32)
    t0 = time.perf_counter()
    unet_ref.forward(wu, x, 900, [0, 1], ehs)
    t_unet = time.perf_counter() - t0
    img = rng.uniform(-1, 1, (2, side, side, 3)).astype(np.float32)
    noise = rng.standard_normal((2, lat, lat, 4)).astype(np.float32)
    t0 = time.perf_counter()
    z = vae_ref.encode(wv, img, noise)
    t_enc = time.perf_counter() - t0
    t0 = time.perf_counter()
    vae_ref.decode(wv, z[:1])
    t_dec = time.perf_counter() - t0
    per = 19 * t_unet + t_enc + t_dec
    return {"value": round(1.0 / per, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"one {side}x{side} inpaint timed by parts on the oracle (oracle/, C++ + OpenMP restatement "
                       "of the reference's Rust engine, which cannot be built here): 1 UNet CFG step at batch 2 "
                       f"({t_unet:.2f} s) x 19 + VAE encode of 2 images ({t_enc:.2f} s) + decode ({t_dec:.2f} s)"),
            "seconds_per_inpaint": round(per, 2)}


# --------------------------------------------------------------------------- secondary measurements
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


def bench_conv(mbx, ctx, torch, dev, small):
    """The tcgen05 implicit-GEMM conv on the conv sweep's largest 3×3 shape (f16 and f32 weights);
    --conv-shape selects another shape, a 1×1 conv with taps = 1."""
    cn, chh, cww, cci, cco, taps = CONV_SHAPE
    gen = torch.Generator(device=dev).manual_seed(7)
    cx = torch.randn(cn, chh, cww, cci, device=dev, generator=gen)
    cy = torch.empty(cn, chh, cww, cco, device=dev)
    wshape = (cco, 3, 3, cci) if taps == 9 else (cco, cci)
    wt = (torch.randn(*wshape, generator=torch.Generator().manual_seed(7)) / (taps * cci) ** 0.5).numpy()
    conv = mbx.conv3x3 if taps == 9 else mbx.conv1x1
    cb = 0.01 * torch.randn(cco, device=dev, generator=gen)
    W = lambda t: mbx.DeviceTensor.wrap(ctx, t.data_ptr(), tuple(t.shape))  # noqa: E731
    CX, CY, CB = W(cx), W(cy), W(cb)
    flops = 2.0 * cn * chh * cww * taps * cci * cco
    tf32 = tf32_peak(torch)
    kind = "3x3 pad 1" if taps == 9 else "1x1"
    out = {"shape": f"[{cn},{chh},{cww},{cci}] -> {cco}, {kind}, bias", "tf32_dense_peak_tflops": round(tf32, 1),
           "tf32_peak_source": "measured here: cuBLAS 8192^3 TF32 matmul, best of 10", "flops_per_launch": flops}
    for dtype in ("f16", "f32"):
        p = mbx.Param(ctx, wt, dtype)
        for _ in range(2):
            conv(CX, p, CB, out=CY)
        torch.cuda.synchronize()
        reps = 5
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(reps):
            conv(CX, p, CB, out=CY)
        e_ev.record()
        e_ev.synchronize()
        cms = s_ev.elapsed_time(e_ev) / reps
        mmas = 2 if dtype == "f16" else 3
        useful = flops / (cms / 1e3) / 1e12
        out[dtype] = {"ms": round(cms, 3), "useful_tflops": round(useful, 1), "issued_tflops": round(useful * mmas, 1),
                      "mma_per_product": mmas, "useful_frac_of_tf32_peak": round(useful / tf32, 3),
                      "issued_frac_of_tf32_peak": round(useful * mmas / tf32, 3)}
        p.close()
    return out


def bench_memory_sweep(mbx, ctx, torch, dev, small, hbm, shape=None):
    """BASELINE configs[1] at its largest shape (or `shape`): the four memory-bound ops, algorithmic
    GB/s at the reference's byte rule (input + output bytes, examples/kernel_bench.rs:93,106)."""
    shape = shape or ((1, 256, 256, 512) if small else SWEEP_SHAPE)
    n, h, w, c = shape
    gen = torch.Generator(device=dev).manual_seed(1234)
    x = torch.randn(shape, device=dev, generator=gen)
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
    ops = [("group_norm_silu", lambda: mbx.group_norm(X, 32, 1e-6, G, B, silu=True, out=Y1)),
           ("bias_temb_add", lambda: mbx.bias_temb_add(Y1, BI, TE, out=Y2)),
           ("residual_add", lambda: mbx.add_inplace(Y2, X)),
           ("depthwise3x3", lambda: mbx.depthwise3x3(Y2, DW, DB, "none", out=Y4))]
    for _ in range(3):
        for _, f in ops:
            f()
    torch.cuda.synchronize()
    ev = {name: [] for name, _ in ops}
    for _ in range(5):
        for name, f in ops:
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            f()
            e_ev.record()
            ev[name].append((s_ev, e_ev))
    torch.cuda.synchronize()
    elems = int(np.prod(shape))
    op_ms = {k: float(np.mean([a.elapsed_time(b) for a, b in v])) for k, v in ev.items()}
    total_ms = sum(op_ms.values())
    return {"workload": f"BASELINE configs[1], shape {list(shape)} (inputs larger than L2)",
            "gbs": round(sum(BYTES_PER_ELT.values()) * elems / (total_ms / 1e3) / 1e9, 1),
            "ops_ms": {k: round(v, 4) for k, v in op_ms.items()},
            "ops_frac_of_hbm": {k: round(BYTES_PER_ELT[k] * elems / (v / 1e3) / 1e9 / hbm, 4)
                                for k, v in op_ms.items()},
            "traffic_ratio_ncu": {k: v for k, v in traffic_ratios_from_profiles().items()},
            "traffic_ratio_note": "DRAM bytes (ncu, profiles/*.md, [8,128,128,512]) / algorithmic bytes"}


def bench_gn_fused(mbx, ctx, torch, dev, hbm, shape):
    """GroupNorm(32) + SiLU when its statistics come from the producing conv's epilogue
    (mbx_conv_group_norm_affine), on the memory sweep's shape: the producer is a 1×1 conv c → c (f16
    weights). The GroupNorm's own cost is then the statistics' extra cost inside the conv (conv with
    statistics, fold and finalize, minus the plain conv) plus the apply pass (8 B/elt)."""
    n, h, w, c = shape
    gen = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(shape, device=dev, generator=gen)
    y, z = torch.empty_like(x), torch.empty_like(x)
    gamma = 1.0 + 0.02 * torch.randn(c, device=dev, generator=gen)
    beta = 0.02 * torch.randn(c, device=dev, generator=gen)
    W = lambda t: mbx.DeviceTensor.wrap(ctx, t.data_ptr(), tuple(t.shape))  # noqa: E731
    X, Y, Z, G, B = W(x), W(y), W(z), W(gamma), W(beta)
    wt = (torch.randn(c, c, generator=torch.Generator().manual_seed(5)) / c ** 0.5).numpy()
    p = mbx.Param(ctx, wt, "f16")
    state = {}

    def stats():
        _, state["sc"], state["sh"] = mbx.conv_group_norm_affine(X, p, 32, 1e-6, G, B, out=Y)

    ops = [("conv_plain", lambda: mbx.conv1x1(X, p, out=Y)), ("conv_with_statistics", stats),
           ("apply_silu", lambda: mbx.group_norm_apply(Y, state["sc"], state["sh"], silu=True, out=Z))]
    for _ in range(3):
        for _, f in ops:
            f()
    torch.cuda.synchronize()
    ev = {name: [] for name, _ in ops}
    for _ in range(5):
        for name, f in ops:
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            f()
            e_ev.record()
            ev[name].append((s_ev, e_ev))
    torch.cuda.synchronize()
    p.close()
    ms = {k: float(np.mean([a.elapsed_time(b) for a, b in v])) for k, v in ev.items()}
    elems = x.numel()
    gn_ms = max(ms["conv_with_statistics"] - ms["conv_plain"], 0.0) + ms["apply_silu"]
    return {"workload": f"{list(shape)}: 1x1 conv {c}->{c} (f16 weights) producing the GroupNorm input",
            "ms": {k: round(v, 4) for k, v in ms.items()},
            "statistics_extra_ms": round(ms["conv_with_statistics"] - ms["conv_plain"], 4),
            "group_norm_silu_ms": round(gn_ms, 4),
            "group_norm_silu_frac_of_hbm": round(8 * elems / (gn_ms / 1e3) / 1e9 / hbm, 4),
            "apply_frac_of_hbm": round(8 * elems / (ms["apply_silu"] / 1e3) / 1e9 / hbm, 4)}


def bench_unet_memory_kernels(mbx, ctx, torch, dev, hbm, batch=16):
    """The UNet's own memory-bound shapes at the headline batch (8 inpaints × the CFG pair), bytes
    counted as the reference counts them (input + output): the level-0 MixFFN depthwise with the
    GLU·SiLU epilogue [16,64,64,1600] → 800 channels (4 B per input + 4 B per output element), the
    level-0 LayerNorm over 16·4096 tokens of 320 channels (8 B/elt), and the DWConv2d depthwise with
    its GroupNorm + SiLU prologue and ReLU [16,64,64,320] (8 B/elt)."""
    gen = torch.Generator(device=dev).manual_seed(99)
    W = lambda t: mbx.DeviceTensor.wrap(ctx, t.data_ptr(), tuple(t.shape))  # noqa: E731
    x = torch.randn(batch, 64, 64, 1600, device=dev, generator=gen)
    glu_w = torch.randn(3, 3, 1600, device=dev, generator=gen) / 3
    glu_b = 0.01 * torch.randn(1600, device=dev, generator=gen)
    glu_y = torch.empty(batch, 64, 64, 800, device=dev)
    t = torch.randn(batch * 4096, 320, device=dev, generator=gen)
    ln_g = 1 + 0.02 * torch.randn(320, device=dev, generator=gen)
    ln_b = 0.02 * torch.randn(320, device=dev, generator=gen)
    ln_y = torch.empty_like(t)
    r = torch.randn(batch, 64, 64, 320, device=dev, generator=gen)
    r_w = torch.randn(3, 3, 320, device=dev, generator=gen) / 3
    r_b = 0.01 * torch.randn(320, device=dev, generator=gen)
    sc = 1 + 0.1 * torch.randn(batch, 320, device=dev, generator=gen)
    sh = 0.1 * torch.randn(batch, 320, device=dev, generator=gen)
    r_y = torch.empty_like(r)
    X, GW, GB, GY = W(x), W(glu_w), W(glu_b), W(glu_y)
    T, LG, LB, LY = W(t), W(ln_g), W(ln_b), W(ln_y)
    R, RW, RB, SC, SH, RY = W(r), W(r_w), W(r_b), W(sc), W(sh), W(r_y)
    ops = [("depthwise3x3_glu_silu", lambda: mbx.depthwise3x3(X, GW, GB, "glu_silu", out=GY),
            (x.numel() + glu_y.numel()) * 4),
           ("layer_norm", lambda: mbx.layer_norm(T, LG, LB, 1e-5, out=LY), 8 * t.numel()),
           ("depthwise3x3_gn_prologue_relu",
            lambda: mbx.depthwise3x3(R, RW, RB, "relu", out=RY, prologue=(SC, SH, True)), 8 * r.numel())]
    for _ in range(3):
        for _, f, _ in ops:
            f()
    torch.cuda.synchronize()
    out = {"workload": f"UNet level-0 shapes at batch {batch} (inputs larger than L2)"}
    for name, f, nbytes in ops:
        evs = []
        for _ in range(5):
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            f()
            e_ev.record()
            evs.append((s_ev, e_ev))
        torch.cuda.synchronize()
        ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
        out[name] = {"ms": round(ms, 4), "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                     "frac_of_hbm": round(nbytes / (ms / 1e3) / 1e9 / hbm, 4)}
    return out


def bench_vae_decoder(eng, torch, dev, latent):
    """the VAE decoder at B = 1 and 8 through the engine."""
    out = {"workload": f"BASELINE configs[3]: VAE decoder, latent [B,{latent},{latent},4] -> "
                       f"[B,{8 * latent},{8 * latent},3], seeded random-init f16 weights (2xTF32)"}
    gen = torch.Generator(device=dev).manual_seed(7)
    for bsz in (1, 8):
        lat = torch.randn(bsz, latent, latent, 4, device=dev, generator=gen) * 0.13025
        img = torch.empty(bsz, 8 * latent, 8 * latent, 3, device=dev)
        for _ in range(2):
            eng.vae_decode(lat.data_ptr(), bsz, latent, latent, img.data_ptr())
        torch.cuda.synchronize()
        reps = 3
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(reps):
            eng.vae_decode(lat.data_ptr(), bsz, latent, latent, img.data_ptr())
        e_ev.record()
        e_ev.synchronize()
        ms = s_ev.elapsed_time(e_ev) / reps
        out[f"b{bsz}"] = {"ms": round(ms, 2), "images_per_s": round(bsz / (ms / 1e3), 2)}
    return out


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch

    world, rank, local, dist = init_dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    mbx = importlib.import_module("moebius-cpu_b200")
    side = 128 if args.small else SIDE
    # One explicit stream for torch's events and the engine's kernels.
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    eng = None
    if not (args.skip_inpaint and args.skip_vae):
        eng = mbx.engine.Engine(weights_dir(rank, dist, args.small), local)
        eng.set_stream(stream.cuda_stream)
    if args.component:
        return run_component(args, mbx, torch, dev, eng, world, rank, dist)
    if args.skip_inpaint:
        return run_secondary_only(args, mbx, torch, dev, eng, stream, world, rank, dist)
    n = args.batch
    img, masks, nv, ni, no = synthetic_inputs(rank, n, side)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    d_src, d_masks, d_nv, d_ni, d_no = t(img), t(masks), t(nv), t(ni), t(no)
    d_work = torch.empty_like(d_src)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    p = mbx.engine.params()

    def step():
        d_work.copy_(d_src)
        eng.inpaint_batch_device(d_work.data_ptr(), d_masks.data_ptr(), n, side, 3, p,
                                 (d_nv.data_ptr(), d_ni.data_ptr(), d_no.data_ptr()))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):  # the first one also captures the UNet graph for this batch size
        step()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    launches0 = eng.launch_count
    evs = []
    for _ in range(args.steps):
        flush.zero_()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        step()
        e_ev.record()
        evs.append((s_ev, e_ev))
    barrier()
    launches = eng.launch_count - launches0
    clocks = sampler.stop()
    ms = float(sum(a.elapsed_time(b) for a, b in evs)) / args.steps
    tt = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_max = float(tt.item())
    value = world * n / (ms_max / 1e3)
    changed = float((d_work != d_src).any(dim=-1).float().mean().item())

    # End to end through mbx_inpaint_batch with pinned host buffers (copies inside the timed region).
    e2e = None
    if not args.skip_e2e:
        hosts = {}
        try:
            for name, a in (("img", img), ("masks", masks), ("nv", nv), ("ni", ni), ("no", no)):
                ptr = mbx.Context.host_alloc(a.nbytes)
                buf = np.ctypeslib.as_array((ctypes.c_uint8 * a.nbytes).from_address(ptr)).view(a.dtype)
                hosts[name] = (ptr, buf.reshape(a.shape))
                hosts[name][1][...] = a
            work_ptr = mbx.Context.host_alloc(img.nbytes)
            work = np.ctypeslib.as_array((ctypes.c_uint8 * img.nbytes).from_address(work_ptr)).reshape(img.shape)
            lib = mbx.abi.lib()
            e2e_steps = max(1, min(3, args.steps))

            def host_step():
                mbx.abi.check(lib.mbx_inpaint_batch(eng.handle, ctypes.c_void_p(work_ptr),
                                                    ctypes.c_void_p(hosts["masks"][0]), n, side, 3, ctypes.byref(p),
                                                    ctypes.c_void_p(hosts["nv"][0]), ctypes.c_void_p(hosts["ni"][0]),
                                                    ctypes.c_void_p(hosts["no"][0]), 0, mbx.abi.PROGRESS_FN(), None))

            work[...] = hosts["img"][1]
            host_step()
            barrier()
            tot = 0.0
            for _ in range(e2e_steps):
                work[...] = hosts["img"][1]  # fresh pixels (the call inpaints in place); outside the timing
                flush.zero_()
                s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_ev.record()
                host_step()
                e_ev.record()
                e_ev.synchronize()
                tot += s_ev.elapsed_time(e_ev)
            barrier()
            te = torch.tensor([tot / e2e_steps], device=dev, dtype=torch.float64)
            if dist:
                dist.all_reduce(te, op=dist.ReduceOp.MAX)
            h2d = img.nbytes + masks.nbytes + nv.nbytes + ni.nbytes + no.nbytes
            e2e = {"value": round(world * n / (float(te.item()) / 1e3), 3), "unit": UNIT,
                   "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(img.nbytes),
                   "ms_per_step": round(float(te.item()), 2),
                   "path": "mbx_inpaint_batch(device_buffers=0) from pinned host memory: H2D pixels, masks, noise; "
                           "whole pipeline; D2H pixels"}
            mbx.Context.host_free(work_ptr)
        finally:
            for ptr, _ in hosts.values():
                mbx.Context.host_free(ptr)

    components = None
    if rank == 0 and not args.skip_components:
        components = {k: round(component_ms(eng, torch, dev, k, n, side // 8, 2, 3), 2)
                      for k in ("unet", "vae_encode", "vae_decode")}
        components["note"] = (f"ms per call at the step's batch: one UNet step at batch {2 * n} (eager, no graph), "
                              f"VAE encode of {2 * n} images, decode of {n}")
    hbm, peak_kind = peaks()
    conv = sweep = vae_line = unet_mem = gn_fused = None
    if rank == 0:
        ctxm = mbx.Context(local)
        ctxm.set_stream(stream.cuda_stream)
        if not args.skip_conv:
            conv = bench_conv(mbx, ctxm, torch, dev, args.small)
        if not args.skip_sweep:
            sweep = bench_memory_sweep(mbx, ctxm, torch, dev, args.small, hbm, SWEEP_OVERRIDE)
            unet_mem = bench_unet_memory_kernels(mbx, ctxm, torch, dev, hbm)
            gn_fused = bench_gn_fused(mbx, ctxm, torch, dev, hbm, (1, 256, 256, 512) if args.small else SWEEP_SHAPE)
        if not args.skip_vae:
            vae_line = bench_vae_decoder(eng, torch, dev, side // 8)
        ctxm.close()
    if rank == 0:
        roof = None
        if conv:
            ach = conv["f16"]["useful_tflops"]
            roof = {"bound": "tensor", "kernel": "conv_tc_kernel (tcgen05 implicit-GEMM 3x3, f16 weights, 2xTF32)",
                    "achieved": ach, "peak": conv["tf32_dense_peak_tflops"], "unit": "TFLOP/s",
                    "frac": round(ach / conv["tf32_dense_peak_tflops"], 4),
                    "peak_kind": "measured here (cuBLAS TF32 dense, burst); MEASURED_PEAKS.json holds no TF32 figure",
                    "issued_frac": conv["f16"]["issued_frac_of_tf32_peak"],
                    "algorithmic_flops_per_launch": conv["flops_per_launch"], "shape": conv["shape"],
                    "traffic": traffic_from_profiles("conv_tc_3x3")}
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded U[0,255] images, random-ellipse masks, N(0,1) noise; random-init weights)",
            "config": config(args),
            "implied_tflops": round(value * INPAINT_TFLOP, 1),
            "roofline": roof, "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
            "result_changed_pixel_frac": round(changed, 4), "components_ms": components,
            "conv": conv, "memory_sweep": sweep, "group_norm_fused": gn_fused, "unet_memory_kernels": unet_mem,
            "vae_decoder": vae_line,
            "hbm_peak_gbs": hbm, "hbm_peak_kind": peak_kind,
        }
        # The CPU baseline is timed at N = 1 only: under torchrun the other ranks would be
        # polling a collective meanwhile, taking host cores from the timed CPU run.
        if not args.skip_cpu and world == 1:
            line["cpu_baseline"] = cpu_inpaint_baseline(args.small)
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def component_ms(eng, torch, dev, name, n, latent, warmup, steps, nvtx=False):
    """Device time of one pipeline component at the headline batch: the UNet step at batch 2n
    (eager, no graph), the VAE encode of 2n images or the VAE decode of n latents."""
    gen = torch.Generator(device=dev).manual_seed(5)
    side = latent * 8
    if name == "unet":
        x = torch.randn(2 * n, latent, latent, 9, device=dev, generator=gen)
        y = torch.empty(2 * n, latent, latent, 4, device=dev)
        call = lambda: eng.unet_forward(x.data_ptr(), 2 * n, 900, True, y.data_ptr())  # noqa: E731
    elif name == "vae_encode":
        x = torch.rand(2 * n, side, side, 3, device=dev, generator=gen) * 2 - 1
        z = torch.randn(2 * n, latent, latent, 4, device=dev, generator=gen)
        y = torch.empty(2 * n, latent, latent, 4, device=dev)
        call = lambda: eng.vae_encode(x.data_ptr(), z.data_ptr(), 2 * n, side, side, y.data_ptr())  # noqa: E731
    else:
        x = torch.randn(n, latent, latent, 4, device=dev, generator=gen) * 0.13025
        y = torch.empty(n, side, side, 3, device=dev)
        call = lambda: eng.vae_decode(x.data_ptr(), n, latent, latent, y.data_ptr())  # noqa: E731
    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    tot = 0.0
    for i in range(steps):
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if nvtx and i == steps - 1:
            torch.cuda.nvtx.range_push(name)
        s_ev.record()
        call()
        e_ev.record()
        if nvtx and i == steps - 1:
            torch.cuda.nvtx.range_pop()
        e_ev.synchronize()
        tot += s_ev.elapsed_time(e_ev)
    return tot / steps


def run_component(args, mbx, torch, dev, eng, world, rank, dist):
    """--component NAME: one pipeline component alone (profiling case; the last timed call is
    wrapped in an NVTX range named NAME for ncu --nvtx-include)."""
    latent = (128 if args.small else SIDE) // 8
    ms = component_ms(eng, torch, dev, args.component, args.batch, latent, args.warmup, args.steps, nvtx=True)
    if rank == 0:
        print(json.dumps({"component": args.component, "batch_inpaints": args.batch, "ms": round(ms, 3),
                          "n_gpus": world}), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_secondary_only(args, mbx, torch, dev, eng, stream, world, rank, dist):
    """--skip-inpaint: only the kernel-level measurements (profiling cases); no headline value."""
    hbm, peak_kind = peaks()
    out = {"metric": METRIC, "value": None, "unit": UNIT, "n_gpus": world, "note": "--skip-inpaint: kernel cases only"}
    if rank == 0:
        ctxm = mbx.Context(dev.index)
        ctxm.set_stream(stream.cuda_stream)
        if not args.skip_conv:
            out["conv"] = bench_conv(mbx, ctxm, torch, dev, args.small)
        if not args.skip_sweep:
            out["memory_sweep"] = bench_memory_sweep(mbx, ctxm, torch, dev, args.small, hbm, SWEEP_OVERRIDE)
            out["unet_memory_kernels"] = bench_unet_memory_kernels(mbx, ctxm, torch, dev, hbm)
            out["group_norm_fused"] = bench_gn_fused(mbx, ctxm, torch, dev, hbm, SWEEP_OVERRIDE or SWEEP_SHAPE)
        if not args.skip_vae:
            out["vae_decoder"] = bench_vae_decoder(eng, torch, dev, (128 if args.small else SIDE) // 8)
        ctxm.close()
        print(json.dumps(out), flush=True)
    if eng:
        eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU path, restated by the oracle (the Rust crate cannot be built here),
    on all host threads. Each step is one UNet CFG step (batch 2), the bulk of an inpaint; the
    VAE encode + decode of one inpaint is timed once and amortised over its 19 steps."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle, unet_ref, vae_ref
    syn = importlib.import_module("moebius-cpu_b200.synthetic")
    threads = oracle.set_threads(0)
    side = 128 if args.small else SIDE
    if args.small:
        wu = syn.random_weights(syn.unet_shapes((64, 128, 256), 16), 0)
        wv = syn.random_weights(syn.vae_shapes((32, 64, 128, 128)), 1)
    else:
        wu = syn.random_weights(syn.unet_shapes(), 0)
        wv = syn.random_weights(syn.vae_shapes(), 1)
    lat = side // 8
    rng = np.random.default_rng(99)
    ehs = unet_ref.conditioning(wu)
    img = rng.uniform(-1, 1, (2, side, side, 3)).astype(np.float32)
    noise = rng.standard_normal((2, lat, lat, 4)).astype(np.float32)
    t0 = time.perf_counter()
    z = vae_ref.encode(wv, img, noise)
    vae_ref.decode(wv, z[:1])
    t_vae = time.perf_counter() - t0
    x = rng.standard_normal((2, lat, lat, 9)).astype(np.float32)
    for _ in range(args.warmup):
        unet_ref.forward(wu, x, 900, [0, 1], ehs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        unet_ref.forward(wu, x, 900, [0, 1], ehs)
    t_step = (time.perf_counter() - t0) / args.steps
    per = 19 * t_step + t_vae
    value = 1.0 / per
    sample = (f"each step: one UNet CFG step at batch 2 ({t_step:.2f} s) of a {side}x{side} inpaint; VAE encode of 2 "
              f"images + decode of 1 timed once ({t_vae:.2f} s); inpaints/s = 1 / (19 x step + VAE); oracle/ "
              "(C++ + OpenMP restatement of the reference's Rust engine: cargo is absent, the crate cannot be built)")
    line = {"metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_step * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded inputs, random-init weights)", "config": config(args), "impl": "reference",
            "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=8, help="inpaints per GPU per step")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-conv", action="store_true")
    ap.add_argument("--skip-sweep", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-vae", action="store_true")
    ap.add_argument("--skip-inpaint", action="store_true", help="kernel-level measurements only")
    ap.add_argument("--skip-components", action="store_true")
    ap.add_argument("--component", choices=["unet", "vae_encode", "vae_decode"], default=None,
                    help="time one pipeline component alone (profiling case)")
    ap.add_argument("--conv-shape", default=None,
                    help="n,h,w,c_in,c_out[,taps] of the conv measurement (taps 9: 3x3, 1: 1x1)")
    ap.add_argument("--sweep-shape", default=None, help="n,h,w,c of the memory-sweep measurement")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: a scaled-down network (64/128/256, 128x128 images) and small sweeps")
    args = ap.parse_args()
    global CONV_SHAPE, SWEEP_OVERRIDE
    if args.sweep_shape:
        SWEEP_OVERRIDE = tuple(int(v) for v in args.sweep_shape.split(","))
        if len(SWEEP_OVERRIDE) != 4:
            ap.error("--sweep-shape takes n,h,w,c")
    if args.conv_shape:
        vals = tuple(int(v) for v in args.conv_shape.split(","))
        if len(vals) not in (5, 6) or (len(vals) == 6 and vals[5] not in (1, 9)):
            ap.error("--conv-shape takes n,h,w,c_in,c_out[,taps] with taps 1 or 9")
        CONV_SHAPE = vals if len(vals) == 6 else vals + (9,)
    elif args.small:
        CONV_SHAPE = (1, 128, 128, 512, 512, 9)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
