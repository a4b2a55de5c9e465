#!/usr/bin/env python
"""Benchmark of the DSINE refine-ops unit on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg4]
                    [--impl ours|reference]

A step is one pass of the unit over one batch: the initial RayReLU, I AngMF
iterations and the convex 8x upsample (+ L2, crop), i.e. one bvml_refine
call. The default workload is BASELINE.json config 4 -- B = 256 frames of
720x1280 per GPU (grid 90x160), fp16 storage, 5x5 window at dilation 1, 5
iterations -- the configuration its Mpixel/s metric is swept on over 1/2/4/8
GPUs. Under torchrun every rank processes its own 256 frames (image-parallel,
no collective on the data path: weak scaling); time is the max over ranks.

Inputs are seeded synthetic tensors with the benchmark generators'
distributions (no dataset exists for this path). They total ~9.4 GB per GPU,
far above the 126 MB L2, so no L2 flush is needed between steps.

The JSON line carries, beyond the driver contract:
  roofline      the dominant kernel's algorithmic bytes per launch over its
                average launch time (CUDA events recorded between the fused
                unit's launches, on its stream, in a second pass of the same
                steps right after the timed ones, so that the timed steps
                carry no extra stream operations) against
                MEASURED_PEAKS.json's HBM copy bandwidth;
  unit_roofline the same for the whole step (the fused refinement);
  e2e           the same metric through the host-buffer API
                (brovisionml_b200.pipeline), pinned host inputs copied in and
                the result copied out every step;
  cpu_baseline  the reference's own CPU ops (oracle/_ref) on this host's
                cores, on a bounded sample of the same workload (rank 0, N=1).

``--impl reference`` times the reference CPU implementation alone (rank 0;
other ranks exit) and prints the same metric with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: full-res H, W, frames per GPU, window, dilation, iterations, storage, full-res RayReLU
    "cfg4": dict(H=720, W=1280, B=256, ps=5, dil=1, iters=5, f16=True, rr=False),
    "cfg2": dict(H=1024, W=1024, B=16, ps=5, dil=2, iters=5, f16=False, rr=False),
    "cfg2h": dict(H=1024, W=1024, B=16, ps=5, dil=2, iters=5, f16=True, rr=False),
    "cfg1": dict(H=480, W=640, B=1, ps=5, dil=1, iters=5, f16=False, rr=True),
    "cfg3": dict(H=4096, W=4096, B=1, ps=7, dil=1, iters=5, f16=False, rr=False),
}
FALLBACK_HBM_GBS = 6650.0


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock and clock-event reasons of one GPU, polled through NVML every
    ~5 ms in a background thread during the timed region (nvidia-smi's
    fastest loop is too coarse for a region of tens of milliseconds)."""

    # NVML clocks-event-reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, device_index: int, uuid: str | None = None):
        self.index = device_index
        self.uuid = uuid
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self.error = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = None
            if self.uuid:
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(self.uuid)
                except Exception:
                    h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # sampling is reported, never required
            self.error = str(e)
            return self
        self._stop = threading.Event()

        def poll():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    self.samples.append((mhz, rs, pw))
                except Exception as e:
                    self.error = str(e)
                    return
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz,
                    "reasons": ["unsampled" + (f": {self.error}" if self.error else "")]}
        mhz = [m for m, _, _ in self.samples]
        reasons = sorted({k for _, r, _ in self.samples for k, bit in self.REASONS.items()
                          if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(mhz), "power_w_max": round(max(p for _, _, p in self.samples), 1),
                "samples": len(self.samples), "reasons": reasons, "source": "nvml"}


# ----------------------------------------------------------------- inputs

def make_device_inputs(cfg, seed, device, torch, logits=False):
    """Seeded synthetic inputs on the GPU, generator distributions of the
    benchmark configurations (oracle.gen_unit draws the same laws on CPU).
    logits: prob / angle as raw head outputs instead (N(0, 2.5) and
    N(-2.5, 1.5) logits, for the path that activates them on load)."""
    H, W, B, ps, iters = cfg["H"], cfg["W"], cfg["B"], cfg["ps"], cfg["iters"]
    h, w = H // 8, W // 8
    P = ps * ps
    dt = torch.float16 if cfg["f16"] else torch.float32
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    fx = fy = 0.8 * W
    cx, cy = W / 2.0, H / 2.0
    fu, cu = fx * w / W, (cx + 0.5) * w / W
    fv, cv = fy * h / H, (cy + 0.5) * h / H
    ys, xs = torch.meshgrid(torch.arange(h, device=device, dtype=torch.float64),
                            torch.arange(w, device=device, dtype=torch.float64), indexing="ij")
    rx = ((xs + 0.5) - cu) / fu
    ry = ((ys + 0.5) - cv) / fv
    ray = torch.stack([rx, ry, torch.ones_like(rx)])
    ray = (ray / ray.norm(dim=0, keepdim=True)).float().contiguous()
    n = torch.randn((B, 3, h, w), generator=g, device=device)
    n = n / n.norm(dim=1, keepdim=True).clamp_min(1e-12)
    s = torch.sign((n * ray[None]).sum(1, keepdim=True))
    s[s == 0] = 1
    normal0 = (n * s).to(dt).contiguous()
    del n, s
    prob, xy, angle = [], [], []
    for _ in range(iters):
        xy.append(torch.randn((B, 2 * P, h, w), generator=g, device=device).to(dt))
        if logits:
            angle.append((torch.randn((B, P, h, w), generator=g, device=device) * 1.5
                          - 2.5).to(dt))
            prob.append((torch.randn((B, P, h, w), generator=g, device=device) * 2.5).to(dt))
            continue
        angle.append((torch.rand((B, P, h, w), generator=g, device=device) * 0.3).to(dt))
        lg = torch.randn((B, P, h, w), generator=g, device=device)
        prob.append(torch.softmax(lg, dim=1).to(dt))
        del lg
    mask = torch.empty((B, 576, h, w), device=device, dtype=dt)
    for b0 in range(0, B, 16):
        mask[b0:b0 + 16] = torch.randn((min(16, B - b0), 576, h, w), generator=g,
                                       device=device).to(dt)
    return dict(normal0=normal0, prob=prob, xy=xy, angle=angle, mask=mask, ray8=ray, fu=fu,
                cu=cu, fv=fv, cv=cv, h=h, w=w, dt=dt)


# ----------------------------------------------------------------- CPU reference

def cpu_reference_sample(cfg, threads=0, seconds_min=10.0):
    """Time the reference CPU ops (oracle/_ref, threaded over frames) on a
    bounded sample: one distinct generated frame repeated over `frames`
    output frames. Returns (Mpx/s, threads, frames, seconds, kind)."""
    from oracle import oracle as O

    if cfg["ps"] != 5 or cfg["dil"] != 1 or not O.ref_available():
        kind = "port"
    else:
        kind = "reference"
    u = O.gen_unit(cfg["H"], cfg["W"], 1, ps=cfg["ps"], dil=cfg["dil"], iters=cfg["iters"],
                   seed=123)
    if cfg["f16"]:
        u = O.to_f16_storage(u)
    nthreads = threads or os.cpu_count() or 1
    per_frame_px = cfg["H"] * cfg["W"]

    def run(frames):
        t0 = time.perf_counter()
        if kind == "reference":
            O.ref_unit_mt(u, threads=nthreads, full_res_ray_relu=cfg["rr"], frames=frames)
        else:  # the restatement (non-reference windows), one frame per call
            for _ in range(frames):
                O.refine_unit(u, full_res_ray_relu=cfg["rr"])
        return time.perf_counter() - t0

    frames = nthreads if kind == "reference" else 1
    dt = run(frames)  # also the warm-up
    # grow to a sample of at least `seconds_min` of CPU work (wall x threads),
    # whole rounds of one frame per thread, then time it warm
    cores = nthreads if kind == "reference" else 1
    cpu_s = dt * cores
    if cpu_s < seconds_min:
        frames = math.ceil(frames * seconds_min / max(cpu_s, 1e-3))
        if kind == "reference":
            frames = math.ceil(frames / nthreads) * nthreads
    dt = run(frames)
    return frames * per_frame_px / dt / 1e6, cores, frames, dt, kind


def reference_arm(args, cfg):
    """--impl reference: the reference's own CPU path, all host threads."""
    from oracle import oracle as O

    nthreads = os.cpu_count() or 1
    kind = "reference" if (O.ref_available() and cfg["ps"] == 5 and cfg["dil"] == 1) else "port"
    u = O.gen_unit(cfg["H"], cfg["W"], 1, ps=cfg["ps"], dil=cfg["dil"], iters=cfg["iters"],
                   seed=123)
    if cfg["f16"]:
        u = O.to_f16_storage(u)
    frames = nthreads if kind == "reference" else 1
    out = np.empty((frames, 3, cfg["H"], cfg["W"]), np.float32)

    def step():
        if kind == "reference":
            O.ref_unit_mt(u, threads=nthreads, full_res_ray_relu=cfg["rr"], frames=frames, out=out)
        else:
            O.refine_unit(u, full_res_ray_relu=cfg["rr"])

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = frames * cfg["H"] * cfg["W"] / dt / 1e6
    line = {
        "impl": "reference", "metric": metric_name(), "value": round(value, 3),
        "unit": "Mpixel/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded generators)",
        "config": workload_config(args, cfg, extra={"sample_frames": frames}),
        "cpu_baseline": {"value": round(value, 3), "unit": "Mpixel/s", "cores": nthreads,
                         "kind": kind,
                         "sample": f"{frames} frames of {cfg['W']}x{cfg['H']} per step "
                                   f"(one generated frame repeated), reference dsine_ops.cpp "
                                   f"CPU twin (fp32 storage, fp64 math) + restated upsample"},
        "e2e": {"value": round(value, 3), "unit": "Mpixel/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def stage_flops_per_px(iters: int) -> float:
    """Model FLOPs per grid pixel of the ConvGRU + heads as the reference
    computes them (unpadded channels): convz, convr, convq 5x5 over 130 -> 64
    per iteration; per head 3x3 66 -> 128, 1x1 128 -> 128, 1x1 128 -> out
    (25, 50, 25, 576)."""
    gru = 2 * (3 * 64) * 130 * 25
    heads = 4 * (2 * 128 * 66 * 9 + 2 * 128 * 128) + 2 * 128 * (25 + 50 + 25 + 576)
    return float(iters * (gru + heads))


def stage_executed_flops(iters: int, B: int, h: int, w: int) -> float:
    """FLOPs the tensor cores run for the same result (unpadded channels): the
    fixed inputs' terms once (feat 64 -> 192 over 5x5 per frame; uv 2 -> 192
    over 5x5 and 2 -> 512 over 3x3 once for all frames), the up-mask head
    only in the last iteration (the only upsample that reaches the output),
    and per iteration only the hidden state
    (64 -> 192 over 5x5, 64 -> 512 over 3x3) and the 1x1 layers."""
    px = B * h * w
    once = 2 * 192 * 64 * 25 * px + (2 * 192 * 2 * 25 + 2 * 512 * 2 * 9) * h * w
    # (+ the extra K that adds the hoisted GRU terms as bf16 hi + lo)
    it = (2 * 192 * 64 * 25 + 2 * 128 * 256 + 2 * 64 * 128 + 2 * 384 * 64 * 9
          + 3 * 2 * 128 * 128 + 2 * 128 * 100)
    # the up-mask head (its 3x3 slice and two 1x1 layers), last iteration only
    mask = 2 * 128 * 64 * 9 + 2 * 128 * 128 + 2 * 128 * 576
    return float(once + (iters * it + mask) * px)


def stage_bench(args, cfg, device, rank, world, barrier, max_over_ranks):
    """--stage: a step is the whole refinement of B frames -- `iters`
    iterations of ConvGRU + heads (brovisionml_b200.refine_stage) and the
    fused ops on their raw outputs (refine(..., logits=True))."""
    import torch

    import brovisionml_b200 as bv
    from brovisionml_b200.refine_stage import RefineStage, StageOutputs, random_params

    B, H, W, I = cfg["B"], cfg["H"], cfg["W"], cfg["iters"]
    h, w = H // 8, W // 8
    dt = torch.float16 if cfg["f16"] else torch.float32
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    h0 = torch.tanh(torch.randn((B, 64, h, w), device=device, generator=g))
    feat = torch.relu(torch.randn((B, 64, h, w), device=device, generator=g))
    fx = 0.8 * W
    fu, cu, fv, cv = fx * w / W, (W / 2 + 0.5) * w / W, fx * h / H, (H / 2 + 0.5) * h / H
    ys, xs = torch.meshgrid(torch.arange(h, device=device), torch.arange(w, device=device),
                            indexing="ij")
    uv = torch.stack([((xs + 0.5) - cu) / fu, ((ys + 0.5) - cv) / fv]).float()
    n0 = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device=device, generator=g),
                                       dim=1).to(dt)
    st = RefineStage(random_params(device, seed=7), B, h, w, device=device, out_dtype=dt)
    mk = lambda c: torch.empty((B, c, h, w), device=device, dtype=dt)  # noqa: E731
    outs = [StageOutputs(mk(25), mk(50), mk(25), mk(576) if i == I - 1 else None)
            for i in range(I)]
    res = torch.empty((B, 3, H, W), device=device, dtype=dt)
    ws = torch.empty(bv.refine_workspace_bytes(B, h, w), device=device, dtype=torch.uint8)
    stream = torch.cuda.Stream(device)

    def stage():
        st.start(h0, feat, uv)
        for i in range(I):  # only the last iteration's up-mask reaches the output
            st.step(outs[i], up_mask=i == I - 1)

    def ops():
        bv.refine(n0, [o.prob for o in outs], [o.xy for o in outs], [o.angle for o in outs],
                  outs[-1].up_mask, fu, cu, fv, cv, out=res, workspace=ws, logits=True)

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            stage()
            ops()
        stream.synchronize()
        st.check_pipeline()
        barrier()
        torch.cuda.synchronize()
        uuid = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            pass
        marks = [[ev(), ev(), ev()] for _ in range(args.steps)]
        with ClockSampler(device.index, uuid) as clk:
            for k in range(args.steps):
                marks[k][0].record(stream)
                stage()
                marks[k][1].record(stream)
                ops()
                marks[k][2].record(stream)
            stream.synchronize()
        barrier()
        st.check_pipeline()
    step_ms = max_over_ranks(sum(m[0].elapsed_time(m[2]) for m in marks) / args.steps)
    stage_ms = max_over_ranks(sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps)
    ops_ms = max_over_ranks(sum(m[1].elapsed_time(m[2]) for m in marks) / args.steps)
    flops = stage_flops_per_px(I) * B * h * w
    tflops = flops / (stage_ms * 1e-3) / 1e12
    flops_x = stage_executed_flops(I, B, h, w)
    tflops_x = flops_x / (stage_ms * 1e-3) / 1e12
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops_sustained"])
        peak_src = "measured sustained (MEASURED_PEAKS.json bf16_tflops_sustained)"
    except Exception:
        peak, peak_src = 1400.0, "fallback sustained 1.4 PFLOP/s"
    line = {
        "metric": "Mpixel/s of the DSINE refinement (ConvGRU + heads + refine ops)",
        "value": round(world * B * H * W / (step_ms * 1e-3) / 1e6, 1), "unit": "Mpixel/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(step_ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (tensor cores, fp32 accumulate) + f32 ops",
        "storage": "f16" if cfg["f16"] else "f32",
        "data": "synthetic (random weights of the reference's shapes, seeded inputs)",
        "config": workload_config(args, cfg, {"stage": "ConvGRU 5x5 130->64 x3, 4 heads "
                                              "(3x3 66->128, 1x1 128->128, 1x1 128->out)"}),
        # per step: stage inputs 1, hoisted terms 3, 6 per iteration (zr, q,
        # heads 3x3, three head tails), the up-mask head 2 (last iteration),
        # AngMF I, upsample 1
        "gpu_launches": args.steps * (1 + 3 + 6 * I + 2 + I + 1),
        "stage": {"ms": round(stage_ms, 3), "tflops_model": round(tflops, 1),
                  "flops_model_per_step": flops, "tflops_executed": round(tflops_x, 1),
                  "flops_executed_per_step": flops_x},
        "ops": {"ms": round(ops_ms, 3)},
        "roofline": {"bound": "tensor", "kernel": "conv_tc (refine stage)",
                     "achieved": round(tflops_x, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops_x / peak, 4), "peak_source": peak_src,
                     "flops": "executed (hoisted feature/uv terms counted once)",
                     "traffic": None},
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def metric_name():
    return "Mpixel/s of DSINE refine ops (5 iters + upsample)"


def workload_config(args, cfg, extra=None):
    c = {"workload": args.config, "frames_per_gpu": cfg["B"],
         "image": f"{cfg['W']}x{cfg['H']}", "grid": f"{cfg['W'] // 8}x{cfg['H'] // 8}",
         "window": f"{cfg['ps']}x{cfg['ps']}", "dilation": cfg["dil"], "iters": cfg["iters"],
         "storage": "f16" if cfg["f16"] else "f32", "full_res_ray_relu": cfg["rr"],
         "parallelism": f"image-parallel x{args.gpus}",
         "l2": "inputs ~9 GB/GPU >> 126 MB L2 (no flush needed)" if args.config == "cfg4"
               else "inputs larger than L2" }
    if getattr(args, "logits", False):
        c["head_outputs"] = "raw logits, sigmoid / pi*sigmoid applied on load"
    if extra:
        c.update(extra)
    return c


# ----------------------------------------------------------------- our arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg4", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--frames", type=int, default=0, help="override frames per GPU")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--stage", action="store_true",
                    help="time the whole learned refinement: ConvGRU + heads on the tensor "
                         "cores (random weights of the reference's shapes), then the ops on "
                         "their raw outputs (device timing only)")
    ap.add_argument("--logits", action="store_true",
                    help="raw head outputs for prob / angle, activated on load (device "
                         "timing only)")
    args = ap.parse_args()
    if args.logits or args.stage:
        args.no_e2e = args.no_cpu = True
    args.steps = max(1, args.steps)
    cfg = dict(CONFIGS[args.config])
    if args.frames:
        cfg["B"] = args.frames

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            reference_arm(args, cfg)
        return

    import torch
    import torch.distributed as dist

    import brovisionml_b200 as bv
    from brovisionml_b200.pipeline import HostBatch, HostRefiner

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.stage:
        return stage_bench(args, cfg, device, rank, world, barrier, max_over_ranks)
    inp = make_device_inputs(cfg, 1000 + rank, device, torch, logits=args.logits)
    h, w, B, P, I = inp["h"], inp["w"], cfg["B"], cfg["ps"] ** 2, cfg["iters"]
    s = 2 if cfg["f16"] else 4
    out = torch.empty((B, 3, 8 * h, 8 * w), device=device, dtype=inp["dt"])
    ws = torch.empty(bv.refine_workspace_bytes(B, h, w), device=device, dtype=torch.uint8)
    stream = torch.cuda.Stream(device)

    def step():
        bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"], inp["fu"],
                  inp["cu"], inp["fv"], inp["cv"], ray8=inp["ray8"], ps=cfg["ps"],
                  dil=cfg["dil"], full_res_ray_relu=cfg["rr"], out=out, workspace=ws,
                  logits=args.logits)

    n_launch = I + 1
    import ctypes

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
        stream.synchronize()
        # per-launch probe events for every timed step
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_launch + 1)]
               for _ in range(args.steps)]
        for e in evs:  # torch creates the CUDA event at its first record
            for ev in e:
                ev.record(stream)
        stream.synchronize()
        arrs = [(ctypes.c_void_p * len(e))(*[ev.cuda_event for ev in e]) for e in evs]
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        uuid = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            pass
        # the timed steps run without probes (no extra stream operations)
        with ClockSampler(local, uuid) as clk:
            start.record(stream)
            for k in range(args.steps):
                step()
            stop.record(stream)
            stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        # the same steps again with probes, for the per-kernel breakdown
        for k in range(args.steps):
            bv.check(bv.lib.bvml_probe_events(arrs[k], len(evs[k])))
            step()
        bv.lib.bvml_probe_events(None, 0)
        stream.synchronize()
        barrier()
    clocks = clk.summary()
    ms_local = start.elapsed_time(stop) / args.steps
    ms = max_over_ranks(ms_local)
    out_px = world * B * cfg["H"] * cfg["W"]
    value = out_px / (ms / 1e3) / 1e6

    # per-kernel launch times from the probes
    per = np.array([[evs[k][j].elapsed_time(evs[k][j + 1]) for j in range(n_launch)]
                    for k in range(args.steps)])  # ms
    angmf_ms = per[:, :I].mean() if I else 0.0
    up_ms = per[:, I].mean()
    hw = h * w
    angmf_bytes = [B * hw * (4 * P * s + (3 * s if i == 0 else 12) + 12) + 12 * hw
                   for i in range(I)]
    up_bytes = B * hw * (576 * s + 12) + B * 3 * 64 * hw * s
    peak, peak_kind = hbm_peak()
    kernels = {
        "angmf": {"launches_per_step": I, "avg_ms": round(float(angmf_ms), 5),
                  "bytes_per_launch": int(np.mean(angmf_bytes)) if I else 0,
                  "share": round(float(per[:, :I].sum() / per.sum()), 4)},
        "upsample": {"launches_per_step": 1, "avg_ms": round(float(up_ms), 5),
                     "bytes_per_launch": int(up_bytes),
                     "share": round(float(per[:, I].sum() / per.sum()), 4)},
    }
    for k in kernels.values():
        k["gbs"] = round(k["bytes_per_launch"] / (k["avg_ms"] * 1e-3) / 1e9, 1) if k["avg_ms"] else 0
    dom = max(kernels, key=lambda k: kernels[k]["share"])
    traffic = None
    tp = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(tp):
        try:
            with open(tp) as f:
                t = json.load(f)
            key = f"{dom}:{args.config}"
            if key in t:
                traffic = int(t[key]["dram_bytes_per_grid_px"] * B * hw)
        except Exception:
            traffic = None
    achieved = kernels[dom]["gbs"]
    unit_bytes = s * (6 + I * 4 * P + 576 + 192) * B * hw
    unit_gbs = world * unit_bytes / (ms * 1e-3) / 1e9

    line = {
        "metric": metric_name(), "value": round(value, 1), "unit": "Mpixel/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "storage": "f16" if cfg["f16"] else "f32",
        "data": "synthetic (seeded generators, BASELINE config distributions)",
        "config": workload_config(args, cfg),
        "gpu_launches": args.steps * n_launch,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "traffic": traffic},
        "unit_roofline": {"bytes_per_step_per_gpu": int(unit_bytes),
                          "achieved": round(unit_gbs / world, 1), "frac": round(unit_gbs / world / peak, 4)},
        "kernels": kernels,
        "clocks": clocks,
    }

    # ------------------------------------------------------------- e2e
    if not args.no_e2e:
        hb = HostBatch(normal0=inp["normal0"].cpu().pin_memory(),
                       prob=[t.cpu().pin_memory() for t in inp["prob"]],
                       xy=[t.cpu().pin_memory() for t in inp["xy"]],
                       angle=[t.cpu().pin_memory() for t in inp["angle"]],
                       mask=inp["mask"].cpu().pin_memory(), ray8=inp["ray8"].cpu().pin_memory())
        out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        del inp
        torch.cuda.empty_cache()
        hr = HostRefiner(device, B, h, w, I, out.dtype, ps=cfg["ps"], chunk=32)
        e2e_steps = max(1, min(args.steps, 5))
        fu, cu, fv, cv = make_intrinsics(cfg)
        for _ in range(2):
            hr.run(hb, out_host, fu, cu, fv, cv, dil=cfg["dil"], full_res_ray_relu=cfg["rr"])
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            hr.run(hb, out_host, fu, cu, fv, cv, dil=cfg["dil"], full_res_ray_relu=cfg["rr"])
        torch.cuda.synchronize()
        e2e_local = (time.perf_counter() - t0) / e2e_steps
        barrier()
        e2e_s = max_over_ranks(e2e_local)
        line["e2e"] = {"value": round(out_px / e2e_s / 1e6, 1), "unit": "Mpixel/s",
                       "h2d_bytes_per_step": int(hr.h2d_bytes(hb)),
                       "d2h_bytes_per_step": int(out_host.numel() * out_host.element_size()),
                       "ms_per_step": round(e2e_s * 1e3, 2), "steps": e2e_steps,
                       "api": "brovisionml_b200.pipeline.HostRefiner (pinned host buffers)"}

    # ------------------------------------------------------------- CPU baseline
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            v, cores, frames, secs, kind = cpu_reference_sample(cfg)
            line["cpu_baseline"] = {
                "value": round(v, 3), "unit": "Mpixel/s", "cores": cores, "kind": kind,
                "sample": f"{frames} frames of {cfg['W']}x{cfg['H']} (one generated frame "
                          f"repeated), {secs:.1f} s wall x {cores} threads; reference "
                          f"dsine_ops.cpp CPU twin (fp32 storage, fp64 math) + restated "
                          f"upsample"}
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "unit": "Mpixel/s", "cores": 0,
                                    "kind": "reference", "sample": f"failed: {e}"}

    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def make_intrinsics(cfg):
    H, W = cfg["H"], cfg["W"]
    h, w = H // 8, W // 8
    fx = fy = 0.8 * W
    cx, cy = W / 2.0, H / 2.0
    return fx * w / W, (cx + 0.5) * w / W, fy * h / H, (cy + 0.5) * h / H


if __name__ == "__main__":
    main()
