"""The whole DSINE refinement on one GPU: the B200 counterpart of
``brovisionml::dsine::Refiner`` (include/brovisionml/dsine_refine.h,
src/dsine_refine.cpp:181-294) -- load / to / forward over B frames of one
camera.

forward = the stage inputs and the hoisted feature / uv terms (RefineStage.
start), 5 iterations of ConvGRU + heads on the tensor cores (the up-mask head
in the last one only: only the last upsample reaches the result), then the
refine ops on the heads' raw outputs (AngMF with the activations fused,
convex 8x upsample, L2-normalise, crop: ``refine(..., logits=True)``). The
uv map and the ray are computed on the device from the intrinsics, with the
reference's +0.5 principal-point convention (src/dsine_decoder.cpp:242-290).
"""
from __future__ import annotations

import os
import struct
import sys
import time
from typing import Sequence

import torch

from .ops import refine
from .refine_stage import RefineStage, load_params

ITERS = 5  # kIter, src/dsine_refine.cpp:251


def _f32(v: float) -> float:
    return struct.unpack("f", struct.pack("f", float(v)))[0]


def grid_intrinsics(intrins: Sequence[float], h8: int, w8: int, origH: int,
                    origW: int) -> tuple[float, float, float, float]:
    """(fu, cu, fv, cv) on the /8 grid from the raw preprocess intrinsics
    (fx, fy, cx, cy) and the padded image size (src/dsine_refine.cpp:230-237);
    the intrinsics are the reference's float fields (Intrinsics,
    include/brovisionml/dsine_preprocess.h), widened to double."""
    fx, fy, cx, cy = (_f32(v) for v in intrins)
    sw, sh = w8 / origW, h8 / origH
    return fx * sw, (cx + 0.5) * sw, fy * sh, (cy + 0.5) * sh


def build_uv(intrins: Sequence[float], h8: int, w8: int, origH: int, origW: int,
             device) -> torch.Tensor:
    """The (2, h8, w8) uv conditioning map, computed as the reference does
    (double arithmetic, rounded to float; src/dsine_decoder.cpp:242-275)."""
    fu, cu, fv, cv = grid_intrinsics(intrins, h8, w8, origH, origW)
    xs = torch.arange(w8, device=device, dtype=torch.float64) + 0.5
    ys = torch.arange(h8, device=device, dtype=torch.float64) + 0.5
    u = ((xs - cu) / fu).float()
    v = ((ys - cv) / fv).float()
    return torch.stack([u[None, :].expand(h8, w8), v[:, None].expand(h8, w8)]).contiguous()


def profile_enabled() -> bool:
    """The reference's BROVISIONML_PROFILE switch (src/profile.cpp:9-15): set
    and not starting with '0'."""
    v = os.environ.get("BROVISIONML_PROFILE", "")
    return bool(v) and v[0] != "0"


class _Marks:
    """BROVISIONML_PROFILE marks as src/profile.cpp:17-29 has them: each mark
    synchronises the device and prints the time since the previous one to
    stderr (the C refiner prints the same lines)."""

    def __init__(self, device) -> None:
        self.on = profile_enabled()
        self.device = device
        if self.on:
            torch.cuda.synchronize(device)
            self.last = time.perf_counter()

    def mark(self, name: str) -> None:
        if not self.on:
            return
        torch.cuda.synchronize(self.device)
        now = time.perf_counter()
        print(f"[brovisionml-prof] {name:<28} {(now - self.last) * 1e3:9.2f} ms", file=sys.stderr)
        self.last = now


class Refiner:
    """load(dir) / load_file(path) / to(device) / forward(...), as the
    reference's Refiner, for B frames at once."""

    def __init__(self) -> None:
        self.params: dict[str, torch.Tensor] | None = None
        self.device = torch.device("cpu")
        self._stages: dict[tuple, RefineStage] = {}
        self._graphs: dict[tuple, tuple] = {}

    def load(self, directory: str) -> None:
        self.load_file(os.path.join(directory, "model.safetensors"))

    def load_file(self, path: str) -> None:
        self.params = load_params(path)
        self._reset()

    def load_params(self, params: dict[str, torch.Tensor]) -> None:
        """Weights already in memory (the reference's names and shapes)."""
        self.params = {k: v.detach().float().cpu() for k, v in params.items()}
        self._reset()

    def _reset(self) -> None:
        self._graphs.clear()  # graphs hold the stages' buffers: release them first
        self._stages.clear()

    def to(self, device) -> "Refiner":
        device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("dsine refine: the B200 refiner runs on CUDA devices only")
        if device != self.device:
            self.device = device
            self._reset()
        return self

    def _stage(self, B: int, h: int, w: int, out_dtype: torch.dtype) -> RefineStage:
        if self.params is None:
            raise RuntimeError("dsine refine: forward() called before load()")
        if self.device.type != "cuda":
            raise RuntimeError("dsine refine: forward() called before to(cuda device)")
        key = (B, h, w, out_dtype)
        if key not in self._stages:
            self._stages[key] = RefineStage(self.params, B, h, w, device=self.device,
                                            out_dtype=out_dtype)
        return self._stages[key]

    def forward(self, normal: torch.Tensor, feature: torch.Tensor, hidden: torch.Tensor,
                intrins: Sequence[float], origH: int, origW: int,
                crop: tuple[int, int, int, int] | None = None,
                out_dtype: torch.dtype = torch.float16, check: bool = True,
                graph: bool = False) -> torch.Tensor:
        """normal (B,3,h8,w8), feature and hidden (B,64,h8,w8): the decoder's
        outputs on this device. intrins = raw (fx, fy, cx, cy); origH, origW
        the padded image size; crop = (pad_t, pad_l, orig_h, orig_w) of the
        DsineTransform (default: none). Returns (B,3,orig_h,orig_w) unit
        normals in out_dtype (the storage of the heads' outputs and of the
        result; fp16 or fp32). check=True synchronises once to raise if a
        tensor-core pipeline gave up; with check=False the call stays
        asynchronous on the current stream, like the reference's brotensor
        ops. graph=True replays a CUDA graph of the whole refinement (about
        60 launches), captured on the first call for this shape, intrinsics
        and crop: the inputs are copied into the graph's buffers and the
        result is returned as a new tensor; for small batches the host's
        launch work otherwise dominates."""
        if graph:
            return self._forward_graph(normal, feature, hidden, intrins, origH, origW, crop,
                                       out_dtype, check)
        B, _, h, w = normal.shape
        if tuple(feature.shape) != (B, 64, h, w) or tuple(hidden.shape) != (B, 64, h, w):
            raise RuntimeError("dsine refine: feature and hidden must be (B,64,h8,w8) like "
                               "the normal's grid")
        st = self._stage(B, h, w, out_dtype)
        marks = _Marks(self.device)
        fu, cu, fv, cv = grid_intrinsics(intrins, h, w, origH, origW)
        st.start(hidden, feature, build_uv(intrins, h, w, origH, origW, self.device))
        outs = [st.step(up_mask=i == ITERS - 1) for i in range(ITERS)]
        marks.mark("refine.stage")
        res = refine(normal.to(out_dtype).contiguous(), [o.prob for o in outs],
                     [o.xy for o in outs], [o.angle for o in outs], outs[-1].up_mask,
                     fu, cu, fv, cv, crop=crop, logits=True)
        marks.mark("refine.ops")
        if check:
            st.check_pipeline()
        return res

    def _forward_graph(self, normal, feature, hidden, intrins, origH, origW, crop, out_dtype,
                       check):
        B, _, h, w = normal.shape
        key = (B, h, w, out_dtype, tuple(float(v) for v in intrins), origH, origW,
               tuple(crop) if crop is not None else None)
        if key not in self._graphs:
            ins = [t.detach().clone() for t in (normal, feature, hidden)]
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):  # warm-up: kernel attributes, workspace
                self.forward(*ins, intrins, origH, origW, crop, out_dtype, check=False)
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self.forward(*ins, intrins, origH, origW, crop, out_dtype, check=False)
            self._graphs[key] = (g, ins, out)
        g, ins, out = self._graphs[key]
        for dst, src in zip(ins, (normal, feature, hidden)):
            dst.copy_(src)
        g.replay()
        res = out.clone()
        if check:
            self._stage(B, h, w, out_dtype).check_pipeline()
        return res
