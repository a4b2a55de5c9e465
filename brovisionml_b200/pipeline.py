"""Host-buffer entry point: refine B frames whose inputs live in (pinned) host
memory, overlapping the PCIe copies with the kernels.

The reference uploads its inputs (src/dsine.cpp:87-89, the ray at
src/dsine_refine.cpp:225-228), runs the ops, and downloads the result
(src/dsine.cpp:99-101) one frame at a time on the default stream. Here the
batch is cut into chunks of frames and three streams run a software
pipeline: host->device copies of chunk i+1, the fused refine of chunk i and
the device->host copy of chunk i-1 proceed together, double-buffered in
device memory. Copies are plain cudaMemcpyAsync (torch ``copy_`` with
``non_blocking``), one per tensor per chunk.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from .ops import refine, refine_workspace_bytes


@dataclass
class HostBatch:
    """Pinned host inputs of B frames (B,C,h,w) and the (3,h,w) fp32 ray."""
    normal0: torch.Tensor
    prob: Sequence[torch.Tensor]
    xy: Sequence[torch.Tensor]
    angle: Sequence[torch.Tensor]
    mask: torch.Tensor
    ray8: torch.Tensor | None = None


class HostRefiner:
    """Reusable device buffers + streams for ``refine_from_host`` on one GPU."""

    def __init__(self, device: torch.device | int, B: int, h: int, w: int, iters: int,
                 dtype: torch.dtype, *, ps: int = 5, chunk: int = 32):
        self.dev = torch.device("cuda", device) if isinstance(device, int) else device
        self.B, self.h, self.w, self.iters, self.dtype, self.ps = B, h, w, iters, dtype, ps
        self.chunk = max(1, min(chunk, B))
        P = ps * ps
        c = self.chunk
        mk = lambda *s: torch.empty(s, device=self.dev, dtype=dtype)  # noqa: E731
        self.sets = []
        for _ in range(2):
            self.sets.append({
                "normal0": mk(c, 3, h, w),
                "prob": [mk(c, P, h, w) for _ in range(iters)],
                "xy": [mk(c, 2 * P, h, w) for _ in range(iters)],
                "angle": [mk(c, P, h, w) for _ in range(iters)],
                "mask": mk(c, 576, h, w),
                "out": mk(c, 3, 8 * h, 8 * w),
            })
        self.ray = torch.empty((3, h, w), device=self.dev, dtype=torch.float32)
        self.ws = torch.empty(refine_workspace_bytes(c, h, w), device=self.dev, dtype=torch.uint8)
        self.s_in = torch.cuda.Stream(self.dev)
        self.s_run = torch.cuda.Stream(self.dev)
        self.s_out = torch.cuda.Stream(self.dev)

    def h2d_bytes(self, hb: HostBatch) -> int:
        ts = [hb.normal0, hb.mask, *hb.prob, *hb.xy, *hb.angle]
        n = sum(t.numel() * t.element_size() for t in ts)
        return n + (hb.ray8.numel() * 4 if hb.ray8 is not None else 0)

    def run(self, hb: HostBatch, out_host: torch.Tensor, fu: float, cu: float, fv: float,
            cv: float, *, dil: int = 1, full_res_ray_relu: bool = False) -> None:
        """Refine all B frames of ``hb`` into pinned ``out_host`` (B,3,8h,8w).
        Returns when ``out_host`` is complete."""
        B, c = hb.normal0.shape[0], self.chunk
        with torch.cuda.device(self.dev):
            if hb.ray8 is not None:
                with torch.cuda.stream(self.s_in):
                    self.ray.copy_(hb.ray8, non_blocking=True)
            ray_ready = torch.cuda.Event()
            ray_ready.record(self.s_in)
            in_done, run_done, out_done = {}, {}, {}
            chunks = [(b0, min(B, b0 + c)) for b0 in range(0, B, c)]
            for i, (b0, b1) in enumerate(chunks):
                st = self.sets[i % 2]
                n = b1 - b0
                with torch.cuda.stream(self.s_in):
                    if i >= 2:  # the set is free once chunk i-2 is computed
                        self.s_in.wait_event(run_done[i - 2])
                    st["normal0"][:n].copy_(hb.normal0[b0:b1], non_blocking=True)
                    for k in range(self.iters):
                        st["prob"][k][:n].copy_(hb.prob[k][b0:b1], non_blocking=True)
                        st["xy"][k][:n].copy_(hb.xy[k][b0:b1], non_blocking=True)
                        st["angle"][k][:n].copy_(hb.angle[k][b0:b1], non_blocking=True)
                    st["mask"][:n].copy_(hb.mask[b0:b1], non_blocking=True)
                    in_done[i] = torch.cuda.Event()
                    in_done[i].record(self.s_in)
                with torch.cuda.stream(self.s_run):
                    self.s_run.wait_event(in_done[i])
                    self.s_run.wait_event(ray_ready)
                    if i >= 2:  # out buffer of this set is free once copied out
                        self.s_run.wait_event(out_done[i - 2])
                    sl = lambda t: t[:n]  # noqa: E731
                    refine(sl(st["normal0"]), [sl(t) for t in st["prob"]],
                           [sl(t) for t in st["xy"]], [sl(t) for t in st["angle"]],
                           sl(st["mask"]), fu, cu, fv, cv,
                           ray8=self.ray if hb.ray8 is not None else None, ps=self.ps, dil=dil,
                           full_res_ray_relu=full_res_ray_relu, out=sl(st["out"]),
                           workspace=self.ws)
                    run_done[i] = torch.cuda.Event()
                    run_done[i].record(self.s_run)
                with torch.cuda.stream(self.s_out):
                    self.s_out.wait_event(run_done[i])
                    out_host[b0:b1].copy_(st["out"][:n], non_blocking=True)
                    out_done[i] = torch.cuda.Event()
                    out_done[i].record(self.s_out)
            self.s_out.synchronize()


def pin(t: torch.Tensor) -> torch.Tensor:
    return t.pin_memory() if not t.is_pinned() else t


# ------------------------------------------------------------ one large frame

@dataclass(frozen=True)
class BandJob:
    """One exact-halo row band of a large frame: compute grid rows
    [comp0, comp1), keep the owned ones, i.e. output rows
    [8 * own0, 8 * own1) of the frame, which are rows
    [crop_t, crop_t + out_h) of the band's 8x output."""
    own0: int
    own1: int
    comp0: int
    comp1: int
    crop_t: int
    out_h: int


def plan_band_jobs(h: int, n_bands: int, iters: int, ps: int, dil: int) -> list[BandJob]:
    """The band jobs of an h-row grid (brovisionml_b200.sharding.plan_bands
    with the exact halo of the unit)."""
    from .sharding import halo_rows, plan_bands

    bands = plan_bands(h, max(1, min(n_bands, h)), halo_rows(iters, ps, dil))
    return [BandJob(b.own0, b.own1, b.comp0, b.comp1, 8 * b.crop_top, 8 * (b.own1 - b.own0))
            for b in bands if b.own1 > b.own0]


@dataclass
class HostFrame:
    """Host inputs of ONE frame: normal0 (3,h,w), prob[i] (P,h,w),
    xy[i] (2P,h,w), angle[i] (P,h,w), mask (576,h,w), ray8 (3,h,w) fp32 or
    None (computed on the device for each band)."""
    normal0: torch.Tensor
    prob: Sequence[torch.Tensor]
    xy: Sequence[torch.Tensor]
    angle: Sequence[torch.Tensor]
    mask: torch.Tensor
    ray8: torch.Tensor | None = None


class BandFailure(RuntimeError):
    """One or more bands of refine_frame_banded failed; ``failures`` lists
    (band index, device, BandJob, exception) for each."""

    def __init__(self, failures):
        self.failures = failures
        parts = [f"band {k} (grid rows {j.own0}..{j.own1 - 1}) on cuda:{d}: "
                 f"{type(e).__name__}: {e}" for k, d, j, e in failures]
        super().__init__("dsine ops: refine_frame_banded: " + "; ".join(parts))


def _refine_band(frame: "HostFrame", out_host: torch.Tensor, d: int, j: BandJob, fu: float,
                 cu: float, fv: float, cv: float, w: int, ps: int, dil: int,
                 full_res_ray_relu: bool, logits: bool) -> None:
    """Upload one band's inputs to device d, refine it (cropped to its owned
    rows by the unit itself) and copy the owned rows into out_host."""
    from .sharding import Band, band_intrinsics

    dev = torch.device("cuda", d)
    with torch.cuda.device(dev):
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            rows = lambda t: t[:, j.comp0:j.comp1]  # noqa: E731
            up = lambda t: rows(t).contiguous().pin_memory().to(dev, non_blocking=True)  # noqa
            res = refine(up(frame.normal0)[None], [up(t)[None] for t in frame.prob],
                         [up(t)[None] for t in frame.xy], [up(t)[None] for t in frame.angle],
                         up(frame.mask)[None], fu, cu, fv,
                         band_intrinsics(cv, Band(j.own0, j.own1, j.comp0, j.comp1)),
                         ray8=up(frame.ray8) if frame.ray8 is not None else None, ps=ps,
                         dil=dil, full_res_ray_relu=full_res_ray_relu,
                         crop=(j.crop_t, 0, j.out_h, 8 * w), logits=logits)
            out_host[:, 8 * j.own0:8 * j.own1].copy_(res[0])
        stream.synchronize()


def refine_frame_banded(frame: HostFrame, out_host: torch.Tensor, fu: float, cu: float,
                        fv: float, cv: float, *, n_bands: int, devices: Sequence[int] = (0,),
                        ps: int = 5, dil: int = 1, full_res_ray_relu: bool = False,
                        logits: bool = False, timeout: float | None = None) -> None:
    """Refine one frame too large for one call (or for one GPU's memory) as
    exact-halo row bands: band k runs on devices[k % len(devices)] (one host
    thread per device, bands of a device in order), and each band's owned
    output rows are cropped by the fused unit itself and copied straight
    into ``out_host`` (3, 8h, 8w) -- the 3-channel crop-stitch. The halo
    (sharding.halo_rows) makes the result equal the whole-frame refine up to
    the fp32 rounding of the band-shifted principal point; the reference
    instead caps the resolution of a large frame (src/dsine.cpp:117-141).

    Failures: a band that raises stops its device's remaining bands and,
    through a shared flag, every other device's bands that have not started;
    all threads are joined and one BandFailure names every failed band with
    its grid rows, device and exception. ``timeout`` (seconds) bounds the
    whole call: threads still running then are reported in a TimeoutError
    naming their devices and the bands not finished (the threads are daemon
    threads, so a stuck device cannot keep the process alive)."""
    import threading
    import time

    iters = len(frame.prob)
    _, h, w = frame.normal0.shape
    jobs = plan_band_jobs(h, n_bands, iters, ps, dil)
    per_dev = {d: [(k, j) for k, j in enumerate(jobs) if devices[k % len(devices)] == d]
               for d in dict.fromkeys(devices)}
    failures = []
    finished = set()
    lock = threading.Lock()
    cancel = threading.Event()

    def work(d: int, my_jobs) -> None:
        for k, j in my_jobs:
            if cancel.is_set():
                return
            try:
                _refine_band(frame, out_host, d, j, fu, cu, fv, cv, w, ps, dil,
                             full_res_ray_relu, logits)
            except BaseException as e:  # surfaced on the calling thread
                with lock:
                    failures.append((k, d, j, e))
                cancel.set()
                return
            with lock:
                finished.add(k)

    threads = {d: threading.Thread(target=work, args=(d, js), daemon=True)
               for d, js in per_dev.items() if js}
    for t in threads.values():
        t.start()
    deadline = None if timeout is None else time.monotonic() + timeout
    for t in threads.values():
        t.join(None if deadline is None else max(0.0, deadline - time.monotonic()))
    stuck = [d for d, t in threads.items() if t.is_alive()]
    if stuck:
        cancel.set()
        with lock:
            pending = [k for k, _ in enumerate(jobs) if k not in finished and
                       not any(f[0] == k for f in failures)]
        raise TimeoutError(f"dsine ops: refine_frame_banded: devices {stuck} still busy after "
                           f"{timeout} s; bands not finished: {pending}")
    if failures:
        raise BandFailure(sorted(failures, key=lambda f: f[0]))


# ------------------------------------------------ the whole refinement, banded

def plan_refine_bands(h: int, n_bands: int, iters: int, ps: int = 5, dil: int = 1):
    """Exact-halo row bands of an h-row grid for the whole learned refinement
    (sharding.refine_halo_rows)."""
    from .sharding import plan_bands, refine_halo_rows

    bands = plan_bands(h, max(1, min(n_bands, h)), refine_halo_rows(iters, ps, dil))
    return [b for b in bands if b.own1 > b.own0]


def band_inputs(intrins, origH: int, band):
    """The band's raw intrinsics and padded image height: the band is an
    image of 8 * rows padded rows whose principal point is 8 * comp0 pixels
    higher (the grid intrinsics then follow src/dsine_refine.cpp:230-237 as
    for a whole frame)."""
    fx, fy, cx, cy = (float(v) for v in intrins)
    return (fx, fy, cx, cy - 8.0 * band.comp0), 8 * band.rows


def refine_frame_banded_full(normal: torch.Tensor, feature: torch.Tensor, hidden: torch.Tensor,
                             intrins, origH: int, origW: int, out: torch.Tensor, *,
                             n_bands: int, run_band, iters: int = 5, ps: int = 5,
                             dil: int = 1) -> None:
    """The whole learned refinement of ONE frame as exact-halo row bands.

    normal (3,h,w), feature and hidden (64,h,w): the decoder's outputs for
    the frame (host or device); out (3, 8h, 8w): the refined normals. Band k
    computes grid rows [comp0, comp1) -- its owned rows plus
    sharding.refine_halo_rows on each side, clipped to the frame -- and keeps
    its owned output rows, so the stitched frame equals the whole-frame
    refinement (the convolutions' zero padding and AngMF's replicate padding
    apply only at the true frame edges; inside, the halo rows carry real data
    and the rows the band edge contaminates are exactly the halo). This
    replaces the reference's resolution cap for large frames
    (src/dsine.cpp:117-141: downscale, run, upsample, renormalise).

    run_band(normal, feature, hidden, intrins, origH, origW, crop) refines one
    band, given as (1,C,rows,w) slices with the band's intrinsics, and
    returns its (1, 3, out_h, 8w) output for crop = (top, 0, out_h, 8w);
    banded_refiner() gives the runner for brovisionml_b200.refiner.Refiner on
    one or more GPUs."""
    _, h, w = normal.shape
    for b in plan_refine_bands(h, n_bands, iters, ps, dil):
        rows = lambda t: t[None, :, b.comp0:b.comp1]  # noqa: E731
        intr_b, origH_b = band_inputs(intrins, origH, b)
        res = run_band(rows(normal), rows(feature), rows(hidden), intr_b, origH_b, origW,
                       (8 * b.crop_top, 0, 8 * (b.own1 - b.own0), 8 * w))
        out[:, 8 * b.own0:8 * b.own1].copy_(res[0])


def banded_refiner(refiners, out_dtype: torch.dtype = torch.float32):
    """A run_band for refine_frame_banded_full over Refiner instances (one
    per device, each loaded and moved with .to(device)); bands go to the
    devices in turn."""
    state = {"k": 0}

    def run_band(normal, feature, hidden, intr, origH, origW, crop):
        r = refiners[state["k"] % len(refiners)]
        state["k"] += 1
        dev = r.device
        t = lambda x: x.to(dev, torch.float32).contiguous()  # noqa: E731
        return r.forward(t(normal), t(feature), t(hidden), intr, origH, origW, crop=crop,
                         out_dtype=out_dtype)
    return run_band
