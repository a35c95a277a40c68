"""DA3-BASE ViT encoder images/s on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl vestra|reference]
                    [--math bf16|q8|f32] [--images 64] [--grid 24x36]

A step is one 12-layer encoder forward over a global batch of `--images`
synthetic images (64 at 504x336; random-init weights
W~N(0,0.02), b~N(0,0.01), LayerScale 1e-5; tokens ~N(0,1)), through the C ABI
(vk_encoder_forward).  Images are independent, so under torchrun every rank
runs its contiguous shard of the batch (strong scaling, no collective on the
data path); time is the max over ranks of CUDA-event time around K steps.
The line also carries the weak-scaling figure (64 images per GPU), the
timed NCCL gather of the outputs to rank 0, and the rest of config 5's
sweep (16 images at 1008x672, Q8_0 weights) at the same GPU count.

`e2e` is the same metric through vk_encoder_forward_host_async: pinned host tokens
in, host result out, copies pipelined with the compute inside the timed
region.  `--impl reference` times the reference's CPU fast path (the
AVX-512 restatement in oracle/, all host cores) on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "vestra-kernels_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

E, H, F, LAYERS = 768, 12, 3072, 12
METRIC = "DA3-BASE ViT encoder images/sec @504x336, 1/2/4/8 B200; % of roofline"


def gflop_per_image(tokens: int) -> float:
    """Algorithmic work per image (12 layers): 2*T*E*(3E+E+F+F) for the
    projections plus 4*H*T^2*64 for attention."""
    proj = 2.0 * tokens * E * (3 * E + E + F + F)
    attn = 4.0 * H * tokens * tokens * 64
    return LAYERS * (proj + attn) / 1e9


def make_layers(seed: int = 0):
    r = np.random.default_rng(seed)
    f = lambda *s, sc: (r.standard_normal(s, dtype=np.float32) * np.float32(sc))
    out = []
    for _ in range(LAYERS):
        out.append({
            "ln1_g": np.ones(E, np.float32), "ln1_b": np.zeros(E, np.float32),
            "qkv_w": f(E, 3 * E, sc=0.02), "qkv_b": f(3 * E, sc=0.01),
            "proj_w": f(E, E, sc=0.02), "proj_b": f(E, sc=0.01), "ls1": np.full(E, 1e-5, np.float32),
            "ln2_g": np.ones(E, np.float32), "ln2_b": np.zeros(E, np.float32),
            "fc1_w": f(E, F, sc=0.02), "fc1_b": f(F, sc=0.01),
            "fc2_w": f(F, E, sc=0.02), "fc2_b": f(E, sc=0.01), "ls2": np.full(E, 1e-5, np.float32),
        })
    return out


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return {"hbm_gbs": p["hbm_gbs"], "bf16": p["bf16_tflops"], "bf16_sustained": p["bf16_tflops_sustained"],
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []
        self.active = False  # only samples taken inside a timed region count

    def mark(self, active: bool):
        self.active = active

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            if self.active:
                self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU legs
def cpu_reference_seconds_per_image(grid_h, grid_w, layers, reps: int = 1):
    """Times the reference's AVX-512 fast path (oracle/vk_cpu_ref.c, all host
    threads) on one image, 12 layers, `reps` times; returns seconds/image."""
    from oracle import oracle

    oracle.set_cpu_ref_threads(os.cpu_count())  # all host threads, whatever OMP_NUM_THREADS says
    T = grid_h * grid_w + 1
    x = np.random.default_rng(1).standard_normal((T, E), dtype=np.float32)
    times = []
    for _ in range(reps):
        y = x
        t0 = time.perf_counter()
        for layer in layers:
            y = oracle.cpu_ref_encoder_layer(y, layer, grid_h, grid_w)
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


INT8_DENSE_SPEC_TOPS = 4500.0  # B200 dense int8, NVIDIA's spec sheet (the 9 POPS figure is with 2:4 sparsity)


def int8_peak_tops():
    """Dense int8 tensor throughput measured here: torch._int_mm (a cuBLASLt
    int8 GEMM, 8192^3, 2 ops per multiply-add), best of 5 after warm-up.
    A denominator only; None where the call is unavailable."""
    import torch

    try:
        n = 8192
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        return 2.0 * n ** 3 / (best / 1e3) / 1e12
    except Exception:
        return None


def traffic_from_profiles():
    """DRAM bytes per launch of the projection GEMM from the committed ncu
    summary (profiles/gemm_bf16_encoder64.md, line `traffic_bytes_per_launch:`)."""
    path = os.path.join(ROOT, "profiles", "gemm_bf16_encoder64.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":")[1].split()[0])
    except OSError:
        pass
    return None


def run_reference(args, rank, world):
    if rank != 0:
        return
    gh, gw = args.grid
    layers = make_layers(0)
    cores = os.cpu_count()
    cpu_reference_seconds_per_image(gh, gw, layers[:1], 1)  # page in
    for _ in range(args.warmup):
        cpu_reference_seconds_per_image(gh, gw, layers[:2], 1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_seconds_per_image(gh, gw, layers, 1)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"DA3-BASE 12-layer encoder, 1 image per step @ {gh}x{gw} patches "
                               f"({gh * gw + 1} tokens), random-init weights", "images_per_step": 1,
                   "tokens": gh * gw + 1, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": cores, "kind": "port",
                         "sample": "1 image x 12 layers per step (reference AVX-512 path restated in C, OpenMP)"},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU leg
def l2_note(B, T):
    """Whether the per-layer activations outgrow the 126 MB L2 (no flush is
    done between steps, so only then do steps stream from HBM)."""
    mb = B * T * (E * 4 + 5 * E * 2 + F * 2) / 1e6
    if mb > 126:
        return "working set larger than L2: %.0f MB of activations per layer (126 MB L2), no flush" % mb
    return "working set %.0f MB fits in the 126 MB L2 (no flush): a latency figure, not a bandwidth one" % mb


def patch_embed_ms(vk, ctx, B, gh, gw, steps, math):
    """CUDA-event ms per call of the batched patch embedding (random-init
    weights, images ~U(0, 1)), or None for Q8_0 math (f32 / bf16 only)."""
    import torch

    if math == vk.MATH_Q8_0:
        return None
    r = np.random.default_rng(3)
    h, w, n = 14 * gh, 14 * gw, gh * gw
    pe = vk.PatchEmbed(ctx, (r.standard_normal((588, E)) * 0.02).astype(np.float32),
                       (r.standard_normal(E) * 0.01).astype(np.float32),
                       (r.standard_normal(E) * 0.02).astype(np.float32), channels=3, patch=14, math=math)
    imgs = torch.rand(B, 3, h, w, device="cuda")
    pos = torch.randn(n + 1, E, device="cuda") * 0.02
    toks = torch.empty(B, n + 1, E, device="cuda")
    for _ in range(3):
        pe(imgs, pos, toks, B, h, w)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        pe(imgs, pos, toks, B, h, w)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


# representative DPT-head consumer shapes at 336 x 504 (grid 24 x 36): the
# encoder output to CHW, a 3x3 fusion convolution on the 4x-upsampled map,
# the align-corners 2x resize, and the final resize + UV add + 3x3 head
# convolution fused (src/conv.rs:304)
DPT_FUSION = (128, 128, 96, 144)
DPT_RESIZE = (128, 96, 144, 192, 288)
DPT_FINAL = (64, 32, 192, 288, 336, 504)
FP32_SIMT_NOMINAL = 148 * 128 * 2 * 1.965e9 / 1e12  # TFLOP/s at the maximum SM clock (nominal, not measured)


def dpt_consumers(vk, ctx, B, gh, gw, reps=5):
    """CUDA-event ms per call over B images of the DPT head's consumers of the
    encoder output (random-init filters, N(0,1) maps), each with its roofline."""
    import torch

    def timed(fn):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    r = np.random.default_rng(5)
    peaks = load_peaks()
    res = {}
    n = gh * gw
    tm = torch.randn(B * n * E, device="cuda")
    chw = torch.empty_like(tm)
    ms = timed(lambda: vk.token_to_chw_batched(tm, B, n, E, chw, ctx=ctx))
    gbs = 2 * tm.numel() * 4 / ms / 1e6
    res["token_to_chw"] = {"ms": round(ms, 4), "gbs": gbs, "frac_of_hbm": gbs / peaks["hbm_gbs"]}
    del tm, chw
    ci, co, h, w = DPT_FUSION
    wt = (r.standard_normal(co * ci * 9) * 0.05).astype(np.float32)
    x = torch.randn(B * ci * h * w, device="cuda")
    y = torch.empty(B * co * h * w, device="cuda")
    bias = torch.zeros(co, device="cuda")
    for mname, m in (("bf16", vk.MATH_BF16), ("f32", vk.MATH_F32)):
        f = vk.WinogradF2Filter(ctx, wt, ci, co, math=m)
        ms = timed(lambda: vk.conv3x3_batched(x, B, h, w, f, bias, y, ctx=ctx))
        direct = 2.0 * 9 * ci * co * h * w * B / (ms / 1e3) / 1e12
        wino = 2.0 * 16 * ci * co * ((h + 1) // 2) * ((w + 1) // 2) * B / (ms / 1e3) / 1e12
        if m == vk.MATH_BF16:  # implicit GEMM on the tensor cores: the direct convolution's FLOPs
            res["conv3x3_%dx%d_%dx%d_bf16" % (ci, co, h, w)] = {
                "ms": round(ms, 4), "tflops": direct, "frac": direct / peaks["bf16_sustained"],
                "of": "measured bf16 sustained (tensor)", "includes": "the channels-last bf16 copy of the input"}
        else:  # Winograd F(2x2, 3x3) on the SIMT cores: its transform-domain products
            res["conv3x3_%dx%d_%dx%d_f32" % (ci, co, h, w)] = {
                "ms": round(ms, 4), "winograd_tflops": wino, "frac": wino / FP32_SIMT_NOMINAL,
                "of": "nominal fp32 SIMT", "direct_equiv_tflops": direct}
    del x, y
    c, ih, iw, oh, ow = DPT_RESIZE
    x = torch.randn(B * c * ih * iw, device="cuda")
    y = torch.empty(B * c * oh * ow, device="cuda")
    ms = timed(lambda: vk.bilinear_resize_align_corners(x, B * c, ih, iw, oh, ow, y, ctx=ctx))
    gbs = (x.numel() + y.numel()) * 4 / ms / 1e6
    res["resize_ac_%dx%d_to_%dx%d" % (ih, iw, oh, ow)] = {"ms": round(ms, 4), "gbs": gbs,
                                                         "frac_of_hbm": gbs / peaks["hbm_gbs"]}
    del x, y
    ci, co, ih, iw, oh, ow = DPT_FINAL
    wt = (r.standard_normal(co * ci * 9) * 0.05).astype(np.float32)
    x = torch.randn(B * ci * ih * iw, device="cuda")
    add = torch.randn(ci * oh * ow, device="cuda")
    y = torch.empty(B * co * oh * ow, device="cuda")
    bias = torch.zeros(co, device="cuda")
    for mname, m in (("bf16", vk.MATH_BF16), ("f32", vk.MATH_F32)):
        f = vk.WinogradF2Filter(ctx, wt, ci, co, math=m)
        ms = timed(lambda: vk.conv3x3_batched(x, B, ih, iw, f, bias, y, resize_to=(oh, ow), add=add, ctx=ctx))
        res["resize_ac_conv3x3_%dx%d_to_%dx%d_%s" % (ci, co, oh, ow, mname)] = {
            "ms": round(ms, 4), "direct_equiv_tflops": 2.0 * 9 * ci * co * oh * ow * B / (ms / 1e3) / 1e12}
    res["note"] = ("outside `value`. Convolutions: bf16 math = implicit GEMM on the tensor cores (direct FLOPs), "
                   "f32 math = the reference's Winograd arithmetic on the SIMT cores (nominal peak %.1f TFLOP/s: "
                   "148 SMs x 128 lanes x 2 x 1965 MHz); resize / transpose against measured HBM" % FP32_SIMT_NOMINAL)
    return res


def time_encoder(vk, ctx, math, total, gh, gw, steps, warmup, rank, world, clk=None):
    """One configuration: `total` images sharded image-wise over the ranks
    (image_shard), K timed steps of the device path and K of the host path.
    Returns the rank-max device and e2e milliseconds plus what the line
    reports about the step."""
    import torch

    from vestra_kernels.sharding import image_shard, max_over_ranks

    T = gh * gw + 1
    first, B = image_shard(total, rank, world)
    enc = vk.Encoder(ctx, make_layers(0), math=math)
    g = torch.Generator(device="cuda").manual_seed(1234)
    x_all = torch.randn(total, T, E, device="cuda", generator=g)
    x = x_all[first:first + B].contiguous()
    del x_all
    out = torch.empty_like(x)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(warmup):
        enc.forward(x, out, B, gh, gw)
    ctx.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    if clk is not None:
        clk.mark(True)
    start.record()
    for _ in range(steps):
        enc.forward(x, out, B, gh, gw)
    stop.record()
    barrier()
    if clk is not None:
        clk.mark(False)
    ms = start.elapsed_time(stop)
    launches = enc.last_launches() * steps

    # end to end: pinned host buffers through the C ABI.  Warm-up: every
    # slot of the three-slot ring runs eager, then captured, then replayed,
    # so no graph capture falls inside the timed region
    hin = x.cpu().pin_memory()
    hout = torch.empty_like(hin).pin_memory()
    enc.forward_host(hin, hout, B, gh, gw)
    for _ in range(3 * warmup):
        enc.forward_host_async(hin, hout, B, gh, gw)
    ctx.synchronize()
    barrier()
    if clk is not None:
        clk.mark(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        enc.forward_host_async(hin, hout, B, gh, gw)  # every step copies its tokens in and its result out
    e1.record()
    barrier()
    if clk is not None:
        clk.mark(False)
    e2e_ms = e0.elapsed_time(e1)
    res = {"ms": max_over_ranks(ms), "e2e_ms": max_over_ranks(e2e_ms), "launches": launches, "enc": enc, "x": x,
           "out": out, "B": B, "h2d": int(hin.numel() * 4), "d2h": int(hout.numel() * 4)}
    res["value"] = total / (res["ms"] / 1e3 / steps)
    res["e2e"] = total / (res["e2e_ms"] / 1e3 / steps)
    return res


def run_vestra(args, rank, world, local_rank):
    import torch

    import vestra_kernels as vk
    from vestra_kernels.sharding import gather_images, max_over_ranks

    torch.cuda.set_device(local_rank)
    math = {"bf16": vk.MATH_BF16, "q8": vk.MATH_Q8_0, "f32": vk.MATH_F32}[args.math]
    gh, gw = args.grid
    T = gh * gw + 1
    total = args.images
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)  # a real stream: the encoder is graph-captured on it
    ctx = vk.Context(local_rank, stream=stream)
    if args.dpt_only:
        if rank == 0:
            print(json.dumps({"dpt_consumers": dpt_consumers(vk, ctx, total, gh, gw, reps=args.steps),
                              "images": total}), flush=True)
        return

    with ClockSampler(local_rank) as clk:
        r = time_encoder(vk, ctx, math, total, gh, gw, args.steps, args.warmup, rank, world, clk)
    B, x, out, enc = r["B"], r["x"], r["out"], r["enc"]
    ms, value, e2e_value = r["ms"], r["value"], r["e2e"]

    # the optional final gather of the outputs to rank 0 (NCCL), timed alone
    gather = None
    if world > 1:
        for _ in range(2):
            gather_images(out, total)
        torch.distributed.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(3):
            gather_images(out, total)
        torch.cuda.synchronize()
        gms = max_over_ranks((time.perf_counter() - t0) / 3 * 1e3)
        gather = {"ms": gms, "bytes": total * T * E * 4,
                  "note": "all ranks' f32 outputs to rank 0 with NCCL all_gather, wall clock, outside `value`"}

    # weak scaling beside the strong figure: 64 images on every GPU
    weak = None
    if world > 1 and not args.no_sweep:
        w = time_encoder(vk, ctx, math, total * world, gh, gw, args.steps, args.warmup, rank, world)
        weak = {"value": w["value"], "e2e": w["e2e"], "images_per_gpu": total, "global_batch": total * world}
        del w

    # the rest of BASELINE config 5's sweep, at the same GPU count
    sweep = None
    if not args.no_sweep and args.math == "bf16" and (gh, gw) == (24, 36) and total == 64:
        sweep = {}
        for name, m, n_img, sh, sw in (("16img_3457tok_bf16", vk.MATH_BF16, 16, 48, 72),
                                       ("64img_865tok_q8_0", vk.MATH_Q8_0, 64, 24, 36),
                                       ("16img_3457tok_q8_0", vk.MATH_Q8_0, 16, 48, 72)):
            k = max(3, args.steps // 4)
            w = time_encoder(vk, ctx, m, n_img, sh, sw, k, args.warmup, rank, world)
            sweep[name] = {"images_per_s": w["value"], "e2e_images_per_s": w["e2e"], "steps": k,
                           "ms_per_step": w["ms"] / k, "tokens": sh * sw + 1, "global_batch": n_img,
                           "whole_step_tflops": gflop_per_image(sh * sw + 1) * w["value"] / world / 1e3}
            if m == vk.MATH_Q8_0:
                if "int8_peak_tops" not in sweep:
                    p8 = int8_peak_tops()
                    sweep["int8_peak_tops"] = {"value": p8 if p8 is not None else INT8_DENSE_SPEC_TOPS,
                                               "kind": "measured here (torch._int_mm 8192^3)" if p8 is not None
                                               else "spec sheet, not measured"}
                sweep[name]["whole_step_frac_of_int8"] = (sweep[name]["whole_step_tflops"]
                                                          / sweep["int8_peak_tops"]["value"])
            del w

    # per-kernel device time (eager forward with events between kernels)
    slots = enc.profile(x, out, B, gh, gw)
    pe_ms = patch_embed_ms(vk, ctx, B, gh, gw, args.steps, math)
    dpt = dpt_consumers(vk, ctx, B, gh, gw) if not args.no_dpt else None
    if rank != 0:
        return

    peaks = load_peaks()
    gf = gflop_per_image(T)
    # dominant kernel: the projection GEMM (slots 1, 3, 5, 6 of each block)
    proj_flop = 2.0 * B * T * E * (3 * E + E + F + F) * LAYERS
    gemm_ms = sum(slots[i] for i in (1, 3, 5, 6)) if math != vk.MATH_F32 else sum(slots[i] for i in (1, 6, 8, 9))
    attn_ms = slots[2] if math != vk.MATH_F32 else slots[4]
    gemm_tflops = proj_flop / (gemm_ms / 1e3) / 1e12
    attn_tflops = (4.0 * H * T * T * 64 * B * LAYERS) / (attn_ms / 1e3) / 1e12
    peak = peaks["bf16_sustained"]
    peak_kind = f"bf16 dense sustained, {peaks['source']}"
    if math == vk.MATH_Q8_0:  # the Q8_0 GEMMs run on the int8 tensor cores
        measured = int8_peak_tops()
        if measured is not None:
            peak, peak_kind = measured, "int8 dense, measured here (torch._int_mm 8192^3, best of 5)"
        else:
            peak, peak_kind = INT8_DENSE_SPEC_TOPS, "int8 dense, spec sheet (not measured)"
    total_ms_eager = sum(slots)
    line = {
        "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": {"bf16": "bf16", "q8": "int8", "f32": "f32"}[args.math], "data": "synthetic",
        "config": {"workload": f"DA3-BASE 12-layer ViT encoder, {total} images @ {gh * 14}x{gw * 14} "
                               f"({T} tokens) sharded image-wise over {world} GPU(s), random-init weights, "
                               f"tokens ~N(0,1)",
                   "global_batch": total, "images_per_gpu": B, "tokens": T, "layers": LAYERS,
                   "math": args.math, "parallelism": f"image-sharded x{world}, no collective on the data path",
                   "l2": l2_note(B, T)},
        "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": r["d2h"]},
        "gpu_launches": r["launches"],
        "roofline": {"bound": "tensor", "kernel": "k_gemm_bf16 (projection GEMMs)" if math == vk.MATH_BF16 else
                     ("k_gemm_q8" if math == vk.MATH_Q8_0 else "k_gemm_f32"),
                     "achieved": gemm_tflops, "peak": peak,
                     "unit": "TOPS" if math == vk.MATH_Q8_0 else "TFLOP/s", "frac": gemm_tflops / peak,
                     "peak_kind": peak_kind,
                     "traffic": traffic_from_profiles() if math == vk.MATH_BF16 else None,
                     "whole_step_tflops": gf * value / world / 1e3,
                     "whole_step_frac": gf * value / world / 1e3 / peak,
                     "whole_step_frac_of_burst": gf * value / world / 1e3 / peaks["bf16"],
                     "attention_tflops": attn_tflops,
                     "slot_ms": dict(zip(["ln1", "qkv", "attention", "proj", "ln2", "fc1", "fc2"]
                                         if math != vk.MATH_F32 else
                                         ["ln1", "qkv", "rope_q", "rope_k", "attention", "to_tokens", "proj",
                                          "ln2", "fc1", "fc2"], [round(v, 4) for v in slots])),
                     "kernel_ms": {"layernorm": slots[0] + slots[4] if math != vk.MATH_F32 else slots[0] + slots[7],
                                   "gemm": gemm_ms, "attention": attn_ms, "eager_total": total_ms_eager}},
        "clocks": clk.summary(),
        "gather": gather,
        "weak_scaling": weak,
        "sweep": sweep,
        "patch_embed": None if pe_ms is None else {
            "ms_per_step": round(pe_ms, 4), "images_per_s": B / (pe_ms / 1e3),
            "tflops": 2.0 * B * gh * gw * 588 * E / (pe_ms / 1e3) / 1e12,
            "note": "patchify + 588->768 projection + cls/position assembly of this GPU's shard, outside `value`"},
        "dpt_consumers": dpt,
    }
    if world == 1 and not args.no_cpu:
        s = cpu_reference_seconds_per_image(gh, gw, make_layers(0), reps=1)
        line["cpu_baseline"] = {"value": 1.0 / s, "unit": "images/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": "1 image x 12 layers (reference AVX-512 path restated in C, OpenMP)"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vestra", choices=["vestra", "reference"])
    ap.add_argument("--math", default="bf16", choices=["bf16", "q8", "f32"])
    ap.add_argument("--images", type=int, default=64)
    ap.add_argument("--grid", default="24x36")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-dpt", action="store_true", help="skip the DPT-consumer timings")
    ap.add_argument("--no-sweep", action="store_true", help="skip the sweep and weak-scaling configurations")
    ap.add_argument("--dpt-only", action="store_true",
                    help="run only the DPT-consumer kernels on --images images (for profiling)")
    args = ap.parse_args()
    args.grid = tuple(int(v) for v in args.grid.split("x"))
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_vestra(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch

            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
