#!/usr/bin/env python
"""Benchmark of the DSINE refine-ops unit on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg4]
                    [--impl ours|reference] [--frames F] [--no-weak]
                    [--no-bands] [--no-e2e] [--no-cpu]

A step is one pass of the unit over one batch: the initial RayReLU, I AngMF
iterations and the convex 8x upsample (+ L2, crop), i.e. one bvml_refine
call. The default workload is BASELINE.json config 4 -- 256 frames of
720x1280 IN TOTAL (grid 90x160), fp16 storage, 5x5 window at dilation 1, 5
iterations -- split image-parallel over the N ranks with
sharding.plan_frames (32 frames per GPU at N = 8): strong scaling, no
collective on the data path, time = max over ranks.

Inputs are seeded synthetic tensors with the benchmark generators'
distributions (no dataset exists for this path). At 256 frames they total
~9.4 GB on one GPU and 1.2 GB per GPU at N = 8, far above the 126 MB L2 in
both cases, so no L2 flush is needed between steps.

The JSON line carries, beyond the driver contract:
  roofline      the dominant kernel's algorithmic bytes per launch over its
                average launch time (CUDA events recorded between the fused
                unit's launches, on its stream, inside the timed steps
                themselves, so the per-launch times add up to ms_per_step)
                against MEASURED_PEAKS.json's HBM copy bandwidth;
  unit_roofline the same for the whole step (the fused refinement);
  weak          (N > 1) the same unit with 256 frames on EVERY rank;
  bands         config 3: one 4096^2 frame (grid 512^2, 7x7, fp32) as exact
                halo row bands over the N ranks, timed three ways: the band
                compute alone; compute + NCCL gather of the owned rows to
                rank 0 + device-to-host copy of the frame there; compute +
                each rank copying its owned rows into one shared pinned host
                frame (the gather to host over every GPU's own PCIe link);
  e2e           the same metric through the host-buffer API
                (brovisionml_b200.pipeline), pinned host inputs copied in and
                the result copied out every step;
  stage         (one GPU, 5x5 configs) the whole learned refinement of 64
                frames: ConvGRU + heads on the tensor cores with random weights
                of the reference's shapes, then the fused ops on their raw
                outputs; executed TFLOP/s against the measured tensor peak;
  cpu_baseline  the reference's own CPU ops (oracle/_ref) on this host's
                cores -- all cores and one thread -- on a bounded sample of
                the same workload (rank 0, N=1), with the angular error of
                the GPU result on that sample.

``--impl reference`` times the reference CPU implementation alone (rank 0;
other ranks exit) with the same sampling routine and prints the same metric
with "impl": "reference"; on a GPU box its line also carries
``reference_cuda``: the reference's own CUDA kernels (src/dsine_ops.cu,
compiled unchanged) timed on the GPU for the same frame size.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: full-res H, W, frames in total (split over the ranks), window,
    # dilation, iterations, storage, full-res RayReLU
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

def grid_intrinsics(H: int, W: int):
    """Grid (1/8) intrinsics of a frame with fx = fy = 0.8 W, cx = W/2,
    cy = H/2 (the reference's pre-"+0.5" intrinsics scaled to the grid as
    src/dsine_refine.cpp:232-237 does)."""
    h, w = H // 8, W // 8
    fx = fy = 0.8 * W
    cx, cy = W / 2.0, H / 2.0
    return fx * w / W, (cx + 0.5) * w / W, fy * h / H, (cy + 0.5) * h / H


def make_device_inputs(cfg, B, seed, device, torch, logits=False):
    """Seeded synthetic inputs of B frames on the GPU, generator
    distributions of the benchmark configurations (oracle.gen_unit draws the
    same laws on CPU). logits: prob / angle as raw head outputs instead
    (N(0, 2.5) and N(-2.5, 1.5) logits, for the path that activates them on
    load)."""
    H, W, ps, iters = cfg["H"], cfg["W"], cfg["ps"], cfg["iters"]
    h, w = H // 8, W // 8
    P = ps * ps
    dt = torch.float16 if cfg["f16"] else torch.float32
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    fu, cu, fv, cv = grid_intrinsics(H, W)
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


def frames_slice(inp, b0, b1):
    """The inputs of frames [b0, b1) (views: frames are the leading dim)."""
    out = dict(inp)
    for k in ("normal0", "mask"):
        out[k] = inp[k][b0:b1]
    for k in ("prob", "xy", "angle"):
        out[k] = [t[b0:b1] for t in inp[k]]
    return out


# ----------------------------------------------------------------- CPU reference

class RefSampler:
    """The reference's CPU ops on a bounded sample of the workload, over a
    persistent pool of host threads: one step is one frame per thread, each
    frame the reference twin's unit (oracle/_ref: ray_relu + I x
    angmf_propagate of src/dsine_ops.cpp, then the restated upsample / L2 /
    crop) on one generated frame of the configuration. Windows the reference
    does not have (dilation 2, 7x7) run the C restatement instead ("port").
    Both the bench's cpu_baseline leg and ``--impl reference`` time steps of
    this one routine."""

    def __init__(self, cfg, threads: int):
        from concurrent.futures import ThreadPoolExecutor

        from oracle import oracle as O

        self.O = O
        self.cfg = cfg
        self.threads = max(1, threads)
        self.kind = ("reference" if (O.ref_available() and cfg["ps"] == 5 and cfg["dil"] == 1)
                     else "port")
        u = O.gen_unit(cfg["H"], cfg["W"], 1, ps=cfg["ps"], dil=cfg["dil"], iters=cfg["iters"],
                       seed=123)
        self.u = O.to_f16_storage(u) if cfg["f16"] else u
        self.outs = [np.empty((1, 3, cfg["H"], cfg["W"]), np.float32)
                     for _ in range(self.threads)]
        self.pool = ThreadPoolExecutor(self.threads)

    def _frame(self, k: int):
        # the oracle libraries are ctypes calls, which release the GIL
        if self.kind == "reference":
            self.O.ref_unit_mt(self.u, threads=1, full_res_ray_relu=self.cfg["rr"], frames=1,
                               out=self.outs[k])
        else:
            self.outs[k][:] = self.O.refine_unit(self.u, full_res_ray_relu=self.cfg["rr"])

    def step(self) -> float:
        """One frame per thread; returns the wall seconds."""
        t0 = time.perf_counter()
        list(self.pool.map(self._frame, range(self.threads)))
        return time.perf_counter() - t0

    def frames_per_step(self) -> int:
        return self.threads

    def rate(self, steps: int, warmup: int = 1):
        """Mpixel/s over `steps` timed steps after `warmup` untimed ones."""
        for _ in range(warmup):
            self.step()
        secs = sum(self.step() for _ in range(steps))
        px = steps * self.threads * self.cfg["H"] * self.cfg["W"]
        return px / secs / 1e6, secs

    def close(self):
        self.pool.shutdown()

    def sample_text(self, steps: int, secs: float) -> str:
        c = self.cfg
        what = ("reference dsine_ops.cpp CPU twin (fp32 storage, fp64 math) + restated upsample"
                if self.kind == "reference" else
                "fp64 C restatement of dsine_ops.cpp (window not in the reference) + restated "
                "upsample")
        return (f"{steps} steps x {self.threads} frames of {c['W']}x{c['H']} (one generated "
                f"frame, {'fp16-rounded ' if c['f16'] else ''}inputs), {secs:.1f} s wall on "
                f"{self.threads} persistent host thread(s); {what}")


def reference_arm(args, cfg):
    """--impl reference: the reference's own CPU path, all host threads, the
    same per-step sample as the bench's cpu_baseline leg."""
    nthreads = os.cpu_count() or 1
    rs = RefSampler(cfg, nthreads)
    for _ in range(args.warmup):
        rs.step()
    secs = sum(rs.step() for _ in range(args.steps))
    rs.close()
    dt = secs / args.steps
    frames = rs.frames_per_step()
    value = frames * cfg["H"] * cfg["W"] / dt / 1e6
    line = {
        "impl": "reference", "metric": metric_name(), "value": round(value, 3),
        "unit": "Mpixel/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded generators)",
        "config": workload_config(args, cfg, int(os.environ.get("WORLD_SIZE", "1")),
                                  extra={"sample_frames_per_step": frames,
                                         "reference_ranks": "rank 0 alone on all host cores "
                                                            "(the reference's CPU path)"}),
        "cpu_baseline": {"value": round(value, 3), "unit": "Mpixel/s", "cores": nthreads,
                         "kind": rs.kind, "sample": rs.sample_text(args.steps, secs)},
        "e2e": {"value": round(value, 3), "unit": "Mpixel/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    line["reference_cuda"] = reference_cuda_leg(cfg)
    print(json.dumps(line), flush=True)


REFGPU_LIB = os.path.join(ROOT, "oracle", "_ref", "libbvml_refgpu.so")


def reference_cuda_leg(cfg, frames: int = 16, reps: int = 3):
    """The reference's own CUDA kernels (src/dsine_ops.cu compiled unchanged
    for sm_100a by oracle/Makefile) on this GPU, driven as Refiner::forward
    drives them (src/dsine_refine.cpp:241-272): per frame ray_relu_cuda, then
    `iters` x angmf_propagate_cuda, fp32 storage (the reference's only one),
    legacy default stream, CUDA events. `frames` frames of the workload's
    size; Mpixel/s in full-resolution output pixels like `value`, although
    this GPU path has no upsample (brotensor's, absent). None of this
    repository's kernels run here."""
    if cfg["ps"] != 5 or cfg["dil"] != 1:
        return {"unavailable": "the reference's CUDA kernel is 5x5, dilation 1 only"}
    try:
        import ctypes

        import torch
    except ImportError as e:  # pragma: no cover
        return {"unavailable": f"torch: {e}"}
    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    if not os.path.exists(REFGPU_LIB):
        return {"unavailable": "oracle/_ref/libbvml_refgpu.so not built (needs the reference "
                               "tree at build time)"}
    lib = ctypes.CDLL(REFGPU_LIB)
    lib.bvml_refgpu_unit.restype = ctypes.c_int
    lib.bvml_refgpu_unit.argtypes = ([ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 +
                                     [ctypes.c_double] * 4 + [ctypes.c_void_p])
    dev = torch.device("cuda", 0)
    c = dict(cfg, f16=False)
    inp = make_device_inputs(c, frames, 4242, dev, torch)
    h, w, iters = inp["h"], inp["w"], cfg["iters"]
    arr = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])  # noqa: E731
    prob, xy, ang = arr(inp["prob"]), arr(inp["xy"]), arr(inp["angle"])
    out = torch.empty((frames, 3, h, w), device=dev)

    def run():
        rc = lib.bvml_refgpu_unit(inp["normal0"].data_ptr(), inp["ray8"].data_ptr(), prob, xy,
                                  ang, iters, frames, h, w, inp["fu"], inp["cu"], inp["fv"],
                                  inp["cv"], out.data_ptr())
        if rc != 0:
            raise RuntimeError("reference CUDA kernels failed")

    stream = torch.cuda.default_stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(2):
            run()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    return {"value": round(frames * cfg["H"] * cfg["W"] / (ms * 1e-3) / 1e6, 1),
            "unit": "Mpixel/s", "ms_per_step": round(ms, 4), "frames": frames,
            "storage": "f32", "device": torch.cuda.get_device_name(dev),
            "what": "the reference's ray_relu_cuda + iters x angmf_propagate_cuda per frame "
                    "(src/dsine_ops.cu, fp64 math, one thread per pixel); no upsample on "
                    "this GPU path"}


# ----------------------------------------------------------------- stage bench

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
    # (+ the extra K that adds the hoisted GRU terms as fp16 hi + lo)
    it = (2 * 192 * 64 * 25 + 2 * 128 * 256 + 2 * 64 * 128 + 2 * 384 * 64 * 9
          + 3 * 2 * 128 * 128 + 2 * 128 * 100)
    # the up-mask head (its 3x3 slice and two 1x1 layers), last iteration only
    mask = 2 * 128 * 64 * 9 + 2 * 128 * 128 + 2 * 128 * 576
    return float(once + (iters * it + mask) * px)


def stage_measure(cfg, B, steps, warmup, device, seed, barrier, max_over_ranks):
    """Time the whole learned refinement of B frames: RefineStage.start +
    `iters` iterations of ConvGRU + heads (brovisionml_b200.refine_stage, random
    weights of the reference's shapes) and the fused ops on their raw outputs
    (refine(..., logits=True)); CUDA events per step. Returns the times (ms,
    max over ranks) and the clock summary."""
    import torch

    import brovisionml_b200 as bv
    from brovisionml_b200.refine_stage import RefineStage, StageOutputs, random_params

    H, W, I = cfg["H"], cfg["W"], cfg["iters"]
    h, w = H // 8, W // 8
    dt = torch.float16 if cfg["f16"] else torch.float32
    g = torch.Generator(device=device).manual_seed(seed)
    h0 = torch.tanh(torch.randn((B, 64, h, w), device=device, generator=g))
    feat = torch.relu(torch.randn((B, 64, h, w), device=device, generator=g))
    fu, cu, fv, cv = grid_intrinsics(H, W)
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
        for _ in range(max(3, warmup)):
            stage()
            ops()
        stream.synchronize()
        st.check_pipeline()
        barrier()
        torch.cuda.synchronize()
        marks = [[ev(), ev(), ev()] for _ in range(steps)]
        with ClockSampler(device.index, gpu_uuid(torch, device)) as clk:
            for k in range(steps):
                marks[k][0].record(stream)
                stage()
                marks[k][1].record(stream)
                ops()
                marks[k][2].record(stream)
            stream.synchronize()
        barrier()
        st.check_pipeline()
    return {
        "step_ms": max_over_ranks(sum(m[0].elapsed_time(m[2]) for m in marks) / steps),
        "stage_ms": max_over_ranks(sum(m[0].elapsed_time(m[1]) for m in marks) / steps),
        "ops_ms": max_over_ranks(sum(m[1].elapsed_time(m[2]) for m in marks) / steps),
        "clocks": clk.summary(),
    }


def tensor_peak():
    """The measured sustained dense bf16 peak (fp16 runs at the same rate)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return (float(json.load(f)["bf16_tflops_sustained"]),
                    "measured sustained (MEASURED_PEAKS.json bf16_tflops_sustained; dense fp16 "
                    "runs at the bf16 rate)")
    except Exception:
        return 1400.0, "fallback sustained 1.4 PFLOP/s"


def stage_key(cfg, B, steps, warmup, device):
    """The whole learned refinement measured inside the default run (one GPU):
    the tensor-core stage's executed TFLOP/s against the measured peak, the
    ops on its raw outputs, Mpixel/s of the whole refinement."""
    I = cfg["iters"]
    h, w = cfg["H"] // 8, cfg["W"] // 8
    t = stage_measure(cfg, B, steps, warmup, device, 1000, lambda: None, lambda v: v)
    peak, _ = tensor_peak()
    tf = stage_executed_flops(I, B, h, w) / (t["stage_ms"] * 1e-3) / 1e12
    return {"what": "whole learned refinement: ConvGRU + 4 heads on the tensor cores (random "
                    "weights of the reference's shapes) + the fused ops on their raw outputs",
            "frames": B, "value": round(B * cfg["H"] * cfg["W"] / (t["step_ms"] * 1e-3) / 1e6, 1),
            "unit": "Mpixel/s", "ms_per_step": round(t["step_ms"], 3),
            "stage_ms": round(t["stage_ms"], 3), "ops_ms": round(t["ops_ms"], 3),
            "tflops_executed": round(tf, 1), "tensor_frac": round(tf / peak, 4),
            "tflops_model": round(stage_flops_per_px(I) * B * h * w /
                                  (t["stage_ms"] * 1e-3) / 1e12, 1),
            "steps": steps, "clocks": t["clocks"]}


def stage_bench(args, cfg, device, rank, world, barrier, max_over_ranks):
    """--stage: a step is the whole refinement of B frames per GPU -- `iters`
    iterations of ConvGRU + heads (brovisionml_b200.refine_stage) and the
    fused ops on their raw outputs (refine(..., logits=True))."""
    B, H, W, I = cfg["B"], cfg["H"], cfg["W"], cfg["iters"]
    h, w = H // 8, W // 8
    t = stage_measure(cfg, B, args.steps, args.warmup, device, 1000 + rank, barrier,
                      max_over_ranks)
    step_ms, stage_ms, ops_ms = t["step_ms"], t["stage_ms"], t["ops_ms"]
    flops = stage_flops_per_px(I) * B * h * w
    tflops = flops / (stage_ms * 1e-3) / 1e12
    flops_x = stage_executed_flops(I, B, h, w)
    tflops_x = flops_x / (stage_ms * 1e-3) / 1e12
    peak, peak_src = tensor_peak()
    line = {
        "metric": "Mpixel/s of the DSINE refinement (ConvGRU + heads + refine ops)",
        "value": round(world * B * H * W / (step_ms * 1e-3) / 1e6, 1), "unit": "Mpixel/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(step_ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (tensor cores, fp32 accumulate) + f32 ops",
        "storage": "f16" if cfg["f16"] else "f32",
        "data": "synthetic (random weights of the reference's shapes, seeded inputs)",
        "config": workload_config(args, cfg, world, {"frames_per_gpu": B, "stage":
                                  "ConvGRU 5x5 130->64 x3, 4 heads (3x3 66->128, 1x1 128->128, "
                                  "1x1 128->out)"}),
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
        "clocks": t["clocks"],
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def stage_layers(args, cfg, device):
    """--stage-layers: run `steps` iterations of the refine stage on random
    weights over B frames of the configuration's grid and print each
    launch's time in the last iteration and of start (CUDA events, one GPU).
    Also the target for profiling one layer: start runs twice (3 conv_tc
    kernels each, the second one timed), then each iteration launches 5
    conv_tc kernels (zr, q, heads 3x3, the up-mask head's two 1x1) --
    numbers 6 + 5 k .. 10 + 5 k -- and 3 head_tail kernels (the prob, xy and
    angle heads' last two layers)."""
    import torch

    from brovisionml_b200.refine_stage import (FEATURE, HEADS, HIDDEN, RefineStage,
                                               random_params)

    B, h, w = cfg["B"], cfg["H"] // 8, cfg["W"] // 8
    st = RefineStage(random_params(device, seed=7), B, h, w, device=device)
    g = torch.Generator(device=device).manual_seed(1)
    h0 = torch.tanh(torch.randn((B, HIDDEN, h, w), device=device, generator=g))
    feat = torch.relu(torch.randn((B, FEATURE, h, w), device=device, generator=g))
    ys, xs = torch.meshgrid(torch.arange(h, device=device), torch.arange(w, device=device),
                            indexing="ij")
    uv = torch.stack([((xs + 0.5) - w / 2) / (0.8 * w), ((ys + 0.5) - h / 2) / (0.8 * w)])
    st.start(h0, feat, uv.float())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    st.start(h0, feat, uv.float())
    e1.record()
    marks = []

    def timed(fn):
        def run(*a, **k):
            m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            m0.record()
            fn(*a, **k)
            m1.record()
            marks.append((m0, m1))
        return run

    st._conv, st._tail = timed(st._conv), timed(st._tail)
    for _ in range(max(1, args.steps)):
        marks.clear()
        st.step()
    torch.cuda.synchronize()
    st.check_pipeline()
    names = (["zr", "q", "heads3x3"] + [f"{n}.2+4" for n, c in HEADS if c <= 64] +
             [f"{n}.{i}" for n, c in HEADS if c > 64 for i in (2, 4)])
    print(f"frames {B} grid {w}x{h}: start {e0.elapsed_time(e1):.3f} ms; " +
          " ".join(f"{n} {a.elapsed_time(b):.3f}" for n, (a, b) in zip(names, marks)))


def metric_name():
    return "Mpixel/s of DSINE refine ops (5 iters + upsample)"


def workload_config(args, cfg, world, extra=None):
    from brovisionml_b200.sharding import plan_frames

    split = [n for _, n in plan_frames(cfg["B"], world)]
    c = {"workload": args.config, "frames_total": cfg["B"], "frames_per_gpu": split,
         "image": f"{cfg['W']}x{cfg['H']}", "grid": f"{cfg['W'] // 8}x{cfg['H'] // 8}",
         "window": f"{cfg['ps']}x{cfg['ps']}", "dilation": cfg["dil"], "iters": cfg["iters"],
         "storage": "f16" if cfg["f16"] else "f32", "full_res_ray_relu": cfg["rr"],
         "parallelism": f"image-parallel x{world} (sharding.plan_frames; no collective on the "
                        f"data path)",
         "l2": "inputs >= 1.2 GB per GPU >> 126 MB L2 (no flush needed)" if args.config == "cfg4"
               else "inputs larger than L2"}
    if getattr(args, "logits", False):
        c["head_outputs"] = "raw logits, sigmoid / pi*sigmoid applied on load"
    if extra:
        c.update(extra)
    return c


def gpu_uuid(torch, device):
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        return None


# ----------------------------------------------------------------- config 3 bands

def bands_bench(args, device, rank, world, barrier, max_over_ranks, stream):
    """Config 3 as the path shards it over N GPUs: one 4096^2 frame (grid
    512^2, 7x7, dilation 1, 5 iterations, fp32), rank r refining the exact
    halo row band sharding.plan_bands(512, N, halo_rows(5, 7, 1))[r] and
    cropping its owned rows. Every rank generates the same frame (same seed)
    and keeps its band's rows, resident before timing."""
    import torch
    import torch.distributed as dist

    import brovisionml_b200 as bv
    from brovisionml_b200.sharding import band_intrinsics, gather_bands, halo_rows, plan_bands

    cfg = CONFIGS["cfg3"]
    H, W, I, ps = cfg["H"], cfg["W"], cfg["iters"], cfg["ps"]
    h, w = H // 8, W // 8
    bands = plan_bands(h, world, halo_rows(I, ps, cfg["dil"]))
    bd = bands[rank]
    full = make_device_inputs(cfg, 1, 777, device, torch)
    rows = lambda t: t[..., bd.comp0:bd.comp1, :].contiguous()  # noqa: E731
    inp = {k: ([rows(t) for t in v] if isinstance(v, list) else
               rows(v) if k in ("normal0", "mask", "ray8") else v) for k, v in full.items()}
    del full
    torch.cuda.empty_cache()
    own_h = 8 * (bd.own1 - bd.own0)
    out = torch.empty((1, 3, own_h, W), device=device, dtype=torch.float32)
    ws = torch.empty(bv.refine_workspace_bytes(1, bd.rows, w), device=device, dtype=torch.uint8)
    cvb = band_intrinsics(inp["cv"], bd)

    def compute():
        bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"], inp["fu"],
                  inp["cu"], inp["fv"], cvb, ray8=inp["ray8"], ps=ps, dil=cfg["dil"],
                  crop=(8 * bd.crop_top, 0, own_h, W), out=out, workspace=ws)

    host = torch.empty((3, H, W), dtype=torch.float32).pin_memory() if rank == 0 else None

    def gather_d2h():
        compute()
        frame = gather_bands(out[0], bands)  # NCCL gather of owned rows to rank 0
        if rank == 0:
            host.copy_(frame, non_blocking=True)

    # the shared pinned host frame: one /dev/shm file mapped by every rank
    shm = None
    shm_path = f"/dev/shm/bvml_bench_cfg3_{os.environ.get('MASTER_PORT', 'solo')}"
    shm_err = None
    try:
        if rank == 0:
            with open(shm_path, "wb") as f:
                f.truncate(3 * H * W * 4)
        barrier()
        shm = torch.from_file(shm_path, shared=True, size=3 * H * W,
                              dtype=torch.float32).view(3, H, W)
        rc = torch.cuda.cudart().cudaHostRegister(shm.data_ptr(), 3 * H * W * 4, 0)
        if int(rc) != 0:
            raise RuntimeError(f"cudaHostRegister: {rc}")
    except Exception as e:  # reported, never required
        shm_err = str(e)
        shm = None
    flag = torch.tensor([1 if shm is None else 0], device=device)
    if world > 1:
        dist.all_reduce(flag)
    use_shm = int(flag.item()) == 0

    def host_gather():
        compute()
        for c in range(3):  # one contiguous device-to-host copy per channel
            shm[c, 8 * bd.own0:8 * bd.own1].copy_(out[0, c], non_blocking=True)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                fn()
            stream.synchronize()
            barrier()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(args.steps):
                fn()
            t1.record(stream)
            t1.synchronize()
            torch.cuda.synchronize()
            barrier()
        return max_over_ranks(t0.elapsed_time(t1) / args.steps)

    px = H * W
    res = {"workload": "cfg3", "image": f"{W}x{H}", "window": "7x7", "iters": I,
           "storage": "f32", "halo_rows": halo_rows(I, ps, cfg["dil"]),
           "bands": [[b.own0, b.own1, b.comp0, b.comp1] for b in bands],
           "scaling": "strong (one frame over N GPUs)"}
    ms = timed(compute)
    res["compute"] = {"value": round(px / (ms * 1e-3) / 1e6, 1), "unit": "Mpixel/s",
                      "ms_per_step": round(ms, 4)}
    ms = timed(gather_d2h)
    res["gather_nccl_d2h"] = {
        "value": round(px / (ms * 1e-3) / 1e6, 1), "unit": "Mpixel/s", "ms_per_step": round(ms, 4),
        "what": "compute + NCCL gather of the owned rows to rank 0 + device-to-host copy of "
                "the frame on rank 0", "d2h_bytes_per_step": 3 * H * W * 4}
    if use_shm:
        ms = timed(host_gather)
        res["host_gather"] = {
            "value": round(px / (ms * 1e-3) / 1e6, 1), "unit": "Mpixel/s",
            "ms_per_step": round(ms, 4),
            "what": "compute + every rank copying its owned rows into one shared pinned host "
                    "frame (/dev/shm mapped by all ranks)",
            "d2h_bytes_per_step": 3 * H * W * 4}
        if rank == 0:
            ref = torch.empty((3, H, W), dtype=torch.float32)
            gather_d2h()
            torch.cuda.synchronize()
            ref.copy_(host)
            host_gather()
            torch.cuda.synchronize()
            barrier()
            res["host_gather"]["equal_to_nccl_gather"] = bool(torch.equal(ref, shm))
        else:
            gather_d2h()
            torch.cuda.synchronize()
            host_gather()
            torch.cuda.synchronize()
            barrier()
    else:
        res["host_gather"] = {"unavailable": shm_err or "shared host frame unavailable"}
    if shm is not None:
        torch.cuda.cudart().cudaHostUnregister(shm.data_ptr())
    barrier()
    if rank == 0 and os.path.exists(shm_path):
        os.unlink(shm_path)
    return res


# ----------------------------------------------------------------- our arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg4", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--frames", type=int, default=0,
                    help="override the frames in total (split over the ranks)")
    ap.add_argument("--no-weak", action="store_true",
                    help="skip the weak-scaling key (all frames on every rank)")
    ap.add_argument("--no-bands", action="store_true", help="skip the config-3 band key")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-stage-key", action="store_true",
                    help="skip the whole-learned-refinement key of the one-GPU run")
    ap.add_argument("--stage", action="store_true",
                    help="time the whole learned refinement: ConvGRU + heads on the tensor "
                         "cores (random weights of the reference's shapes), then the ops on "
                         "their raw outputs (device timing only; frames per GPU)")
    ap.add_argument("--stage-layers", action="store_true",
                    help="time each launch of one refine-stage iteration and of start "
                         "(CUDA events; --frames frames of 720p, default 16)")
    ap.add_argument("--logits", action="store_true",
                    help="raw head outputs for prob / angle, activated on load (device "
                         "timing only)")
    args = ap.parse_args()
    if args.logits or args.stage or args.stage_layers:
        args.no_e2e = args.no_cpu = args.no_bands = args.no_weak = True
        args.no_stage_key = True
    args.steps = max(1, args.steps)
    cfg = dict(CONFIGS[args.config])
    if args.frames:
        cfg["B"] = args.frames
    if args.stage and not args.frames:
        cfg["B"] = 64
    if args.stage_layers and not args.frames:
        cfg["B"] = 16

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
    from brovisionml_b200.sharding import plan_frames

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    try:
        if args.stage_layers:
            return stage_layers(args, cfg, device)
        if args.stage:
            return stage_bench(args, cfg, device, rank, world, barrier, max_over_ranks)
        return unit_bench(args, cfg, device, rank, world, barrier, max_over_ranks, torch, bv,
                          HostBatch, HostRefiner, plan_frames)
    finally:
        if world > 1:
            dist.destroy_process_group()


def unit_bench(args, cfg, device, rank, world, barrier, max_over_ranks, torch, bv, HostBatch,
               HostRefiner, plan_frames):
    split = plan_frames(cfg["B"], world)
    b_off, B = split[rank]
    weak = world > 1 and not args.no_weak
    B_alloc = max(B, cfg["B"] if weak else 0, 1)
    inp_all = make_device_inputs(cfg, B_alloc, 1000 + rank, device, torch, logits=args.logits)
    h, w, P, I = inp_all["h"], inp_all["w"], cfg["ps"] ** 2, cfg["iters"]
    s = 2 if cfg["f16"] else 4
    stream = torch.cuda.Stream(device)

    def unit(nf):
        """A step over nf frames: the fused unit, its output and workspace."""
        inp = frames_slice(inp_all, 0, nf)
        out = torch.empty((nf, 3, 8 * h, 8 * w), device=device, dtype=inp["dt"])
        ws = torch.empty(bv.refine_workspace_bytes(max(nf, 1), h, w), device=device,
                         dtype=torch.uint8)

        def step():
            if nf == 0:
                return
            bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"],
                      inp["fu"], inp["cu"], inp["fv"], inp["cv"], ray8=inp["ray8"],
                      ps=cfg["ps"], dil=cfg["dil"], full_res_ray_relu=cfg["rr"], out=out,
                      workspace=ws, logits=args.logits)
        step.ws = ws
        return step, out

    def time_steps(step, clocks=False, probes=None):
        """Device ms per step on this rank (W warm-up steps, then K timed
        steps bracketed by a barrier and a synchronize on both sides). probes:
        one array of CUDA events per timed step, armed for that step's unit
        (bvml_probe_events), so that every launch is timed inside the timed
        region itself, on the launching stream."""
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                step()
            stream.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.synchronize()
            clk = ClockSampler(local_index(device), gpu_uuid(torch, device)) if clocks else None
            if clk:
                clk.__enter__()
            start.record(stream)
            for k in range(args.steps):
                if probes is not None:
                    bv.check(bv.lib.bvml_probe_events(probes[k], len(probes[k])))
                step()
            if probes is not None:
                bv.lib.bvml_probe_events(None, 0)
            stop.record(stream)
            stream.synchronize()
            if clk:
                clk.__exit__(None, None, None)
            torch.cuda.synchronize()
            barrier()
        return start.elapsed_time(stop) / args.steps, clk

    # per-kernel launch times: probe events recorded between the unit's
    # launches during the timed steps themselves. The unit is two launches
    # (all AngMF iterations in one persistent launch, then the upsample) or,
    # for shapes the persistent kernel does not take, I + 1.
    import ctypes

    step, out = unit(B)
    ws_of_step = step.ws
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(I + 2)]
           for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for e in evs:  # torch creates the CUDA event at its first record
            for ev in e:
                ev.record(stream)
        stream.synchronize()
    arrs = [(ctypes.c_void_p * len(e))(*[ev.cuda_event for ev in e]) for e in evs]
    ms_local, clk = time_steps(step, clocks=True, probes=arrs if B else None)
    ms = max_over_ranks(ms_local)
    clocks = clk.summary()
    out_px = cfg["B"] * cfg["H"] * cfg["W"]
    value = out_px / (ms / 1e3) / 1e6
    n_rec = int(bv.lib.bvml_probe_recorded()) if B else 0
    if B:
        with torch.cuda.stream(stream):
            bv.check(bv.lib.bvml_refine_status(ctypes.c_void_p(ws_of_step.data_ptr()),
                                               ctypes.c_void_p(stream.cuda_stream)))
    barrier()
    n_launch = max(n_rec - 1, 1)
    fused = n_launch == 2 and I > 1
    peak, peak_kind = hbm_peak()
    hw = h * w
    kernels = {}
    dom = "angmf"
    angmf_bytes = [B * hw * (4 * P * s + (3 * s if i == 0 else 12) + 12) + 12 * hw
                   for i in range(I)]
    if B:
        per = np.array([[evs[k][j].elapsed_time(evs[k][j + 1]) for j in range(n_launch)]
                        for k in range(args.steps)])  # ms
        na = n_launch - 1  # AngMF launches per step
        up_bytes = B * hw * (576 * s + 12) + B * 3 * 64 * hw * s
        kernels = {
            "angmf": {"launches_per_step": na, "iterations_per_launch": I // max(na, 1),
                      "avg_ms": round(float(per[:, :na].mean()), 5) if na else 0.0,
                      "bytes_per_launch": int(sum(angmf_bytes) / max(na, 1)),
                      "share": round(float(per[:, :na].sum() / per.sum()), 4),
                      "kernel": "angmf_iters_kernel (persistent, all iterations)" if fused
                      else "angmf_staged_kernel (one launch per iteration)"},
            "upsample": {"launches_per_step": 1, "avg_ms": round(float(per[:, na].mean()), 5),
                         "bytes_per_launch": int(up_bytes),
                         "share": round(float(per[:, na].sum() / per.sum()), 4)},
        }
        for k in kernels.values():
            k["gbs"] = (round(k["bytes_per_launch"] / (k["avg_ms"] * 1e-3) / 1e9, 1)
                        if k["avg_ms"] else 0)
        dom = max(kernels, key=lambda k: kernels[k]["share"])
    traffic = None
    tp = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(tp) and B:
        try:
            with open(tp) as f:
                t = json.load(f)
            key = f"{dom}:{args.config}"
            if key in t:
                # per grid pixel of one pass (one AngMF iteration / the upsample)
                passes = I // max(kernels["angmf"]["launches_per_step"], 1) \
                    if dom == "angmf" else 1
                traffic = int(t[key]["dram_bytes_per_grid_px"] * B * hw * passes)
        except Exception:
            traffic = None
    achieved = kernels[dom]["gbs"] if kernels else 0.0
    unit_bytes = s * (6 + I * 4 * P + 576 + 192) * B * hw
    unit_gbs_rank = unit_bytes / (ms * 1e-3) / 1e9

    line = {
        "metric": metric_name(), "value": round(value, 1), "unit": "Mpixel/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "storage": "f16" if cfg["f16"] else "f32",
        "data": "synthetic (seeded generators, BASELINE config distributions)",
        "config": workload_config(args, cfg, world),
        "gpu_launches": args.steps * n_launch,
        "gpu_launches_note": "our kernels per step: " + (
            "1 persistent AngMF (all iterations) + 1 upsample" if fused else
            f"{n_launch - 1} AngMF + 1 upsample") + "; plus one cudaMemsetAsync of the sync words",
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "traffic": traffic, "rank": rank, "frames": B},
        "unit_roofline": {"bytes_per_step_per_gpu": int(unit_bytes), "rank": rank,
                          "achieved": round(unit_gbs_rank, 1),
                          "frac": round(unit_gbs_rank / peak, 4)},
        "kernels": kernels,
        "clocks": clocks,
    }

    # ------------------------------------------------------------- weak scaling
    if weak:
        wstep, _ = unit(cfg["B"])
        wms = max_over_ranks(time_steps(wstep)[0])
        line["weak"] = {"frames_per_gpu": cfg["B"], "frames_total": world * cfg["B"],
                        "value": round(world * out_px / (wms * 1e-3) / 1e6, 1),
                        "unit": "Mpixel/s", "ms_per_step": round(wms, 4)}
        del wstep
    del step, out
    torch.cuda.empty_cache()

    # ------------------------------------------------------------- config 3 bands
    if not args.no_bands and args.config == "cfg4":
        line["bands"] = bands_bench(args, device, rank, world, barrier, max_over_ranks, stream)
        torch.cuda.empty_cache()

    # ------------------------------------------------------------- e2e
    if not args.no_e2e:
        src = frames_slice(inp_all, 0, B)
        pin = lambda t: t.cpu().pin_memory()  # noqa: E731
        hb = HostBatch(normal0=pin(src["normal0"]), prob=[pin(t) for t in src["prob"]],
                       xy=[pin(t) for t in src["xy"]], angle=[pin(t) for t in src["angle"]],
                       mask=pin(src["mask"]), ray8=pin(src["ray8"]))
        out_host = torch.empty((B, 3, 8 * h, 8 * w), dtype=src["dt"]).pin_memory()
        del src, inp_all
        torch.cuda.empty_cache()
        hr = HostRefiner(device, max(B, 1), h, w, I, out_host.dtype, ps=cfg["ps"], chunk=32)
        e2e_steps = max(1, min(args.steps, 5))
        fu, cu, fv, cv = grid_intrinsics(cfg["H"], cfg["W"])

        def run():
            if B:
                hr.run(hb, out_host, fu, cu, fv, cv, dil=cfg["dil"],
                       full_res_ray_relu=cfg["rr"])
        for _ in range(2):
            run()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            run()
        torch.cuda.synchronize()
        e2e_local = (time.perf_counter() - t0) / e2e_steps
        barrier()
        e2e_s = max_over_ranks(e2e_local)
        line["e2e"] = {"value": round(out_px / e2e_s / 1e6, 1), "unit": "Mpixel/s",
                       "h2d_bytes_per_step": int(hr.h2d_bytes(hb)),
                       "d2h_bytes_per_step": int(out_host.numel() * out_host.element_size()),
                       "ms_per_step": round(e2e_s * 1e3, 2), "steps": e2e_steps,
                       "bytes": f"per rank (rank {rank}, {B} frames)",
                       "api": "brovisionml_b200.pipeline.HostRefiner (pinned host buffers)"}

    # ------------------------------------- the whole learned refinement (f3)
    if rank == 0 and world == 1 and not args.no_stage_key and cfg["ps"] == 5 and \
            cfg["dil"] == 1:
        try:
            line["stage"] = stage_key(cfg, min(64, cfg["B"]), min(args.steps, 10), args.warmup,
                                      device)
        except Exception as e:  # reported, never required for the ops' number
            line["stage"] = {"failed": str(e)[:300]}

    # ------------------------------------------------------------- CPU baseline
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            line["cpu_baseline"], line["accuracy"] = cpu_baseline_leg(cfg, device, torch, bv)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "unit": "Mpixel/s", "cores": 0,
                                    "kind": "reference", "sample": f"failed: {e}"}

    if rank == 0:
        print(json.dumps(line), flush=True)


def local_index(device):
    return device.index if device.index is not None else 0


def cpu_baseline_leg(cfg, device, torch, bv):
    """The reference CPU ops on all host cores and on one thread (the same
    sampling routine as --impl reference), and the angular error of the GPU
    path against the reference twin on the sampled frame."""
    from oracle import oracle as O

    nthreads = os.cpu_count() or 1
    rs = RefSampler(cfg, nthreads)
    v_all, secs_all = rs.rate(steps=3, warmup=1)
    rs.close()
    rs1 = RefSampler(cfg, 1)
    v_one, secs_one = rs1.rate(steps=2, warmup=1)
    want = rs1.outs[0]
    u = rs1.u
    rs1.close()
    base = {"value": round(v_all, 3), "unit": "Mpixel/s", "cores": nthreads, "kind": rs.kind,
            "sample": rs.sample_text(3, secs_all),
            "single_thread": {"value": round(v_one, 3), "unit": "Mpixel/s", "cores": 1,
                              "sample": rs1.sample_text(2, secs_one)}}
    dt = torch.float16 if cfg["f16"] else torch.float32
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device, dt)  # noqa: E731
    got = bv.refine(t(u.normal0), [t(a) for a in u.prob], [t(a) for a in u.xy],
                    [t(a) for a in u.angle], t(u.mask), u.fu, u.cu, u.fv, u.cv,
                    ray8=torch.from_numpy(u.ray8).to(device), ps=cfg["ps"], dil=cfg["dil"],
                    full_res_ray_relu=cfg["rr"])
    torch.cuda.synchronize()
    m = O.compare(got.float().cpu().numpy(), want)
    acc = {"against": f"{rs1.kind} CPU path on the sampled frame (same inputs)",
           "max_abs": m["max_abs"], "mean_abs": m["mean_abs"],
           "ang_mean_deg": m["ang_mean_deg"], "ang_p99_deg": m["ang_p99_deg"],
           "ang_max_deg": m["ang_max_deg"],
           "tolerance_max_abs": O.TOL_F16 if cfg["f16"] else O.TOL_F32}
    return base, acc


if __name__ == "__main__":
    main()
