"""The learned half of DSINE's refinement on the tensor cores: the ConvGRU and
the four prediction heads of ``Refiner::forward`` (src/dsine_refine.cpp:
95-158, 253-276), whose raw outputs feed the refine ops (``refine(...,
logits=True)``).

The convolutions are linear in their input channels, and two of the three
channel groups never change during a refinement: the decoder feature (64
channels) and uv (2) are the same in every iteration, and uv is the same for
every frame. So ``start`` convolves them once --

  gxu = conv5x5(uv, W_zr||q[:, 128:130])          (1,192/4,h,w,4) fp32 (C4), shared
  gx  = conv5x5(feat, W_zr||q[:, 64:128]) + gxu    per frame, stored as fp16
        halves hi = fp16(gx), lo = fp16(gx - hi), each 64-channel block (z, r,
        q) as hi then lo: (B,h,w,384), about 22 mantissa bits
  gu  = conv3x3(uv, W_heads3x3[:, 64:66])          (1,512/4,h,w,4) fp32, shared

-- and each iteration convolves only the hidden state and adds the hoisted
terms (the same products, summed in another order): gx by the tensor cores,
as an extra K block (its hi and lo times identity blocks) after the 5x5 taps,
so the epilogue reads
no per-pixel table; gu in the epilogue (one frame, L2-resident):

  z, r = sigmoid(conv5x5(h, W_zr[:, :64]) + gx[:128])   one GEMM (N = 128);
         the epilogue writes z and r*h
  q   = tanh(conv5x5(r*h, W_q[:, :64]) + gx[128:])      epilogue
         h = (1-z) h + z q (fp32 state) and its fp16 copy
  each head: conv3x3 -> ReLU -> conv1x1 -> ReLU -> conv1x1; the four 3x3
         layers as one GEMM (N = 512) over h with gu added; the two 1x1
         layers of prob (25), xy (50) and angle (25) as one kernel each with
         the intermediate on chip (bvml_head_tail_1x1), the up_mask (576)
         head's as two; the last layer writes planar NCHW (fp16 or fp32)
         logits.

(The GRU and heads never read the normals, so all iterations run first and
the ops unit consumes their outputs afterwards.) 3 tensor-core launches per
refinement plus 8 per iteration (6 without the up-mask head), no separate
elementwise or layout pass;
the 5x5 GEMMs contract 25 x 64 instead of 25 x 130 (padded: 192) channels,
the heads' 3x3 9 x 64 instead of 9 x 66 (padded: 128). Weights are the
reference's (OIHW fp32, safetensors names ``gru.convz`` ...
``up_prob_head.4``), rounded to fp16 once; activations are fp16 between
layers, the GRU state and the hoisted terms fp32.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass

import torch

from ._capi import EPI_C4_F32, EPI_GRU_Q, EPI_GRU_ZR, EPI_NHWC, EPI_PLANAR_F16, EPI_SPLIT_F16, \
    EPI_PLANAR_F32, ConvEpilogue, check, lib
from .ops import _cuda, _p, _stream, pack_conv_weight, pad64

HEADS = (("prob_head", 25), ("xy_head", 50), ("angle_head", 25), ("up_prob_head", 576))
HIDDEN = 64      # ConvGRU hidden channels
FEATURE = 64     # decoder feature channels (input_dim 66 = feature + uv)
HEAD_HIDDEN = 128


def random_params(device, seed: int = 0) -> dict[str, torch.Tensor]:
    """Random weights with the reference's shapes and names (no checkpoint is
    available here): convs with std 1/sqrt(fan_in), small biases."""
    g = torch.Generator(device=device).manual_seed(seed)
    p = {}
    for name, shape in param_shapes().items():
        if name.endswith(".weight"):
            fan_in = shape[1] * shape[2] * shape[3]
            p[name] = torch.randn(shape, device=device, generator=g) * fan_in ** -0.5
        else:
            p[name] = torch.randn(shape, device=device, generator=g) * 0.05
    return p


def param_shapes() -> dict[str, tuple[int, ...]]:
    """The refine stage's tensors as the reference names and shapes them
    (src/dsine_refine.cpp:51-92, 185-194): gru.conv{z,r,q} 5x5 over 130
    channels, per head .0 3x3 66 -> 128, .2 1x1 128 -> 128, .4 1x1 128 -> out."""
    cin = HIDDEN + FEATURE + 2
    shapes = {}
    for g in "zrq":
        shapes[f"gru.conv{g}.weight"] = (HIDDEN, cin, 5, 5)
        shapes[f"gru.conv{g}.bias"] = (HIDDEN,)
    for head, out in HEADS:
        for i, (co, ci, k) in zip((0, 2, 4), ((HEAD_HIDDEN, HIDDEN + 2, 3),
                                             (HEAD_HIDDEN, HEAD_HIDDEN, 1),
                                             (out, HEAD_HIDDEN, 1))):
            shapes[f"{head}.{i}.weight"] = (co, ci, k, k)
            shapes[f"{head}.{i}.bias"] = (co,)
    return shapes


_ST_DTYPES = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16}


def load_params(path: str) -> dict[str, torch.Tensor]:
    """The refine stage's weights from a safetensors file (the reference's
    Refiner::load_file, src/dsine_refine.cpp:185-194, and load_f32,
    src/weights_util.h): F32, F16 or BF16 tensors widened to fp32 on the
    host; other tensors in the file (encoder, decoder) are not read. Errors
    name the file and the tensor, as the reference's do."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        if n <= 0 or n > (1 << 30):
            raise RuntimeError(f"dsine refine: {path}: not a safetensors file")
        header = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, shape in param_shapes().items():
            meta = header.get(name)
            if meta is None:
                raise RuntimeError(f"dsine refine: {path}: missing tensor '{name}'")
            dt = _ST_DTYPES.get(meta["dtype"])
            if dt is None:
                raise RuntimeError(f"dsine refine: {path}: tensor '{name}' has dtype "
                                   f"{meta['dtype']} (F32, F16 or BF16 expected)")
            if tuple(meta["shape"]) != shape:
                raise RuntimeError(f"dsine refine: {path}: tensor '{name}' has shape "
                                   f"{tuple(meta['shape'])}, expected {shape}")
            b0, b1 = meta["data_offsets"]
            f.seek(base + b0)
            raw = bytearray(f.read(b1 - b0))
            if len(raw) != b1 - b0:
                raise RuntimeError(f"dsine refine: {path}: tensor '{name}' is truncated")
            out[name] = torch.frombuffer(raw, dtype=dt).reshape(shape).float()
    return out


@dataclass
class StageOutputs:
    """Raw head outputs of one iteration, planar (B,C,h,w). up_mask is None
    for an iteration run with ``up_mask=False``."""
    prob: torch.Tensor
    xy: torch.Tensor
    angle: torch.Tensor
    up_mask: torch.Tensor | None


class RefineStage:
    """ConvGRU + prediction heads for B frames of an (h, w) grid on one GPU."""

    def __init__(self, params: dict[str, torch.Tensor], B: int, h: int, w: int,
                 device: torch.device | int = 0, out_dtype: torch.dtype = torch.float16):
        self.dev = torch.device("cuda", device) if isinstance(device, int) else device
        self.B, self.h, self.w = B, h, w
        if out_dtype not in (torch.float16, torch.float32):
            raise RuntimeError("dsine ops: refine stage: outputs are fp16 or fp32")
        self.out_dtype = out_dtype
        d = self.dev
        f32 = lambda t: t.to(d, torch.float32).contiguous()  # noqa: E731
        H = HIDDEN
        # hidden-state parts of the weights (input channels [0, 64))
        wz, wr, wq = (params[f"gru.conv{g}.weight"].to(d) for g in "zrq")
        self.w_zr = pack_conv_weight(torch.cat([wz, wr])[:, :H], H, 128)
        self.b_zr = f32(torch.cat([params["gru.convz.bias"], params["gru.convr.bias"]]))
        self.w_q = pack_conv_weight(wq[:, :H], H, 64)
        self.b_q = f32(params["gru.convq.bias"])
        c0 = torch.cat([params[f"{n}.0.weight"] for n, _ in HEADS]).to(d)
        self.w_c0 = pack_conv_weight(c0[:, :H], H, 4 * HEAD_HIDDEN)
        self.b_c0 = f32(torch.cat([params[f"{n}.0.bias"] for n, _ in HEADS]))
        # the same layer without the up-mask head's slice (the last 128
        # channels), for iterations that skip that head
        assert HEADS[-1][0] == "up_prob_head"
        self.w_c0_3 = pack_conv_weight(c0[:3 * HEAD_HIDDEN, :H], H, 3 * HEAD_HIDDEN)
        self.b_c0_3 = self.b_c0[:3 * HEAD_HIDDEN].contiguous()
        # the fixed inputs' parts: feat + uv -> z, r, q; uv -> the heads' 3x3
        wg = torch.cat([wz, wr, wq])
        self.w_gx = pack_conv_weight(wg[:, H:H + FEATURE], 64, 192)
        # identity blocks: the extra K that adds hi + lo of the hoisted GRU
        # terms (z, r: blocks 0 and 1 of gx; q: block 2)
        iz = torch.zeros((1, 128, 256), device=d, dtype=torch.float16)
        for n in range(128):
            iz[0, n, (n // 64) * 128 + n % 64] = 1
            iz[0, n, (n // 64) * 128 + 64 + n % 64] = 1
        e64 = torch.eye(64, device=d, dtype=torch.float16)
        self.iz = iz
        self.iq = torch.cat([e64, e64], 1)[None].contiguous()   # (1, 64, 128)
        self.w_gxu = pack_conv_weight(wg[:, H + FEATURE:], 64, 192)
        self.w_gu = pack_conv_weight(c0[:, H:], 64, 4 * HEAD_HIDDEN)
        self.zeros = torch.zeros(4 * HEAD_HIDDEN, device=d)
        self.w_c2 = [pack_conv_weight(params[f"{n}.2.weight"].to(d), 128, 128) for n, _ in HEADS]
        self.b_c2 = [f32(params[f"{n}.2.bias"]) for n, _ in HEADS]
        self.w_c4 = [pack_conv_weight(params[f"{n}.4.weight"].to(d), 128, pad64(c))
                     for n, c in HEADS]
        self.b_c4 = [f32(params[f"{n}.4.bias"]) for n, _ in HEADS]
        bf = torch.float16
        mk = lambda c, dt=bf, n=B: torch.zeros((n, h, w, c), device=d, dtype=dt)  # noqa: E731
        self.hx, self.rhx = mk(H), mk(H)                     # h (fp16), r * h
        # per-pixel epilogue tensors in channel groups (C8 fp16, C4 fp32)
        self.z = torch.zeros((B, H // 8, h, w, 8), device=d, dtype=bf)
        self.h32 = torch.zeros((B, H // 4, h, w, 4), device=d)
        self.fx, self.ux = mk(FEATURE), mk(64, n=1)          # feat, [uv | 0]
        # hoisted terms, C4 fp32: the epilogues read them coalesced
        self.gx = mk(384)                                     # gx as hi | lo blocks
        self.gxu = torch.zeros((1, 192 // 4, h, w, 4), device=d)
        self.gu = torch.zeros((1, HEAD_HIDDEN, h, w, 4), device=d)
        self.t1, self.t2 = mk(4 * HEAD_HIDDEN), mk(4 * HEAD_HIDDEN)
        self.err = torch.zeros(1, device=d, dtype=torch.int32)

    @classmethod
    def from_safetensors(cls, path: str, B: int, h: int, w: int,
                         device: torch.device | int = 0,
                         out_dtype: torch.dtype = torch.float16) -> "RefineStage":
        """A stage with the weights of a DSINE checkpoint (model.safetensors)."""
        return cls(load_params(path), B, h, w, device=device, out_dtype=out_dtype)

    def _tail(self, k: int, c: int, code: int, dst: torch.Tensor) -> None:
        """Head k's two 1x1 layers in one launch (bvml_head_tail_1x1)."""
        check(lib.bvml_head_tail_1x1(
            _p(self.t1), 4 * HEAD_HIDDEN, k * HEAD_HIDDEN, _p(self.w_c2[k]), _p(self.b_c2[k]),
            _p(self.w_c4[k]), _p(self.b_c4[k]), self.B, self.h, self.w, c, code, _p(dst),
            _p(self.err), _stream(self.dev)))

    # one launch through the C ABI
    def _conv(self, x, cin_off, cin_pad, w, bias, cout, ks, **epi):
        e = ConvEpilogue(**{k: (_p(v) if isinstance(v, torch.Tensor) else v)
                            for k, v in epi.items()})
        check(lib.bvml_conv2d_nhwc_f16_ex(_p(x), x.shape[-1], cin_off, cin_pad, _p(w),
                                           _p(bias), x.shape[0], self.h, self.w, cout,
                                           w.shape[1], ks, ctypes.byref(e), _p(self.err),
                                           _stream(self.dev)))

    def start(self, h0: torch.Tensor, feat: torch.Tensor, uv: torch.Tensor) -> None:
        """Load the decoder's hidden state h0 (B,64,h,w), feature (B,64,h,w)
        and uv (2,h,w) (src/dsine_refine.cpp:245-248), and convolve the fixed
        inputs once (three convolutions)."""
        _cuda("refine stage", h0, feat, uv)
        self.err.zero_()  # each refinement reports its own pipeline status
        uvn = uv.permute(1, 2, 0)[None].to(torch.float16)
        h0 = h0.float().contiguous()
        feat = feat.float().contiguous()
        self.ux[..., :2] = uvn
        with torch.cuda.device(self.dev):
            check(lib.bvml_stage_inputs(_p(h0), _p(feat), self.B, self.h, self.w, _p(self.h32),
                                        _p(self.hx), _p(self.fx), _stream(self.dev)))
            self._conv(self.ux, 0, 64, self.w_gxu, self.zeros, 192, 5, mode=EPI_C4_F32,
                       out=self.gxu, out_c=192, out_off=0)
            self._conv(self.fx, 0, 64, self.w_gx, self.zeros, 192, 5, mode=EPI_SPLIT_F16,
                       out=self.gx, out_c=384, out_off=0, add=self.gxu, add_c=192,
                       add_shared=1)
            self._conv(self.ux, 0, 64, self.w_gu, self.zeros, 4 * HEAD_HIDDEN, 3,
                       mode=EPI_C4_F32, out=self.gu, out_c=4 * HEAD_HIDDEN, out_off=0)

    def step(self, out: StageOutputs | None = None, up_mask: bool = True) -> StageOutputs:
        """One iteration: GRU update, then the heads' raw outputs. The
        up-mask head feeds only the convex upsample, and only the last
        iteration's upsample reaches the refined normal
        (src/dsine_refine.cpp:270-282): iterations before the last can pass
        up_mask=False and skip its two 1x1 launches (the 576-channel layer is
        the stage's largest output) and its quarter of the heads' shared 3x3
        layer."""
        B, h, w = self.B, self.h, self.w
        if out is None:
            mk = lambda c: torch.empty((B, c, h, w), device=self.dev,  # noqa: E731
                                       dtype=self.out_dtype)
            out = StageOutputs(*(mk(c) if up_mask or name != "up_prob_head" else None
                                 for name, c in HEADS))
        with torch.cuda.device(self.dev):
            self._conv(self.hx, 0, HIDDEN, self.w_zr, self.b_zr, 128, 5, mode=EPI_GRU_ZR,
                       h32=self.h32, z=self.z, rh=self.rhx, rh_c=HIDDEN, xin=self.gx,
                       xin_c=256, xin_stride=384, wx=self.iz)
            self._conv(self.rhx, 0, HIDDEN, self.w_q, self.b_q, 64, 5, mode=EPI_GRU_Q,
                       h32=self.h32, z=self.z, hx=self.hx, hx_c=HIDDEN,
                       xin=self.gx[..., 256:], xin_c=128, xin_stride=384, wx=self.iq)
            w_c0, b_c0 = (self.w_c0, self.b_c0) if up_mask else (self.w_c0_3, self.b_c0_3)
            self._conv(self.hx, 0, HIDDEN, w_c0, b_c0, b_c0.numel(), 3, mode=EPI_NHWC, act=1,
                       out=self.t1, out_c=4 * HEAD_HIDDEN, out_off=0, add=self.gu,
                       add_c=4 * HEAD_HIDDEN, add_shared=1)
            planar = EPI_PLANAR_F16 if self.out_dtype == torch.float16 else EPI_PLANAR_F32
            dsts = (out.prob, out.xy, out.angle, out.up_mask)
            code = 1 if self.out_dtype == torch.float16 else 0
            for k, (name, c) in enumerate(HEADS):
                if name == "up_prob_head" and not up_mask:
                    continue
                if c <= 64:  # 1x1 -> ReLU -> 1x1 in one kernel, intermediate on chip
                    self._tail(k, c, code, dsts[k])
                    continue
                self._conv(self.t1, k * HEAD_HIDDEN, HEAD_HIDDEN, self.w_c2[k], self.b_c2[k],
                           HEAD_HIDDEN, 1, mode=EPI_NHWC, act=1, out=self.t2,
                           out_c=4 * HEAD_HIDDEN, out_off=k * HEAD_HIDDEN)
                self._conv(self.t2, k * HEAD_HIDDEN, HEAD_HIDDEN, self.w_c4[k], self.b_c4[k], c,
                           1, mode=planar, out=dsts[k])
        return out

    def check_pipeline(self) -> None:
        """Raise if any launch since the last start() or check gave up (one
        device sync). The error word is cleared after it is read, so each
        check reports only the launches since the previous one."""
        code = int(self.err.item())
        if code != 0:
            self.err.zero_()
            raise RuntimeError(f"dsine cuda: refine stage: pipeline gave up (code {code})")


def reference_stage(params, h0, feat, uv, iters: int, *, emulate_f16: bool = True,
                    dtype: torch.dtype = torch.float32):
    """Plain PyTorch restatement of the same computation (the reference's
    formulas, src/dsine_refine.cpp:118-158), for tests, in fp32 (or `dtype`,
    e.g. float64 where a test needs results independent of summation order).
    With emulate_f16 the weights and the activations between layers are
    rounded to fp16 exactly where RefineStage rounds them, so the two differ
    only in summation order."""
    F = torch.nn.functional
    q16 = (lambda t: t.to(torch.float16).to(dtype)) if emulate_f16 else (lambda t: t)
    W = {k: (q16(v.to(dtype)) if k.endswith("weight") else v.to(dtype))
         for k, v in params.items()}
    B = h0.shape[0]
    uvb = uv[None].expand(B, -1, -1, -1).to(dtype)
    h = h0.to(dtype)
    feat = feat.to(dtype)
    outs = []
    for _ in range(iters):
        hx = q16(torch.cat([h, feat, uvb], 1))
        z = torch.sigmoid(F.conv2d(hx, W["gru.convz.weight"], W["gru.convz.bias"], padding=2))
        r = torch.sigmoid(F.conv2d(hx, W["gru.convr.weight"], W["gru.convr.bias"], padding=2))
        z = q16(z)
        rhx = torch.cat([q16(r * h), q16(feat), q16(uvb)], 1)
        q = torch.tanh(F.conv2d(rhx, W["gru.convq.weight"], W["gru.convq.bias"], padding=2))
        h = h + z * (q - h)
        hin = q16(torch.cat([h, uvb], 1))
        res = []
        for name, _ in HEADS:
            t = q16(F.relu(F.conv2d(hin, W[f"{name}.0.weight"], W[f"{name}.0.bias"], padding=1)))
            t = q16(F.relu(F.conv2d(t, W[f"{name}.2.weight"], W[f"{name}.2.bias"])))
            res.append(F.conv2d(t, W[f"{name}.4.weight"], W[f"{name}.4.bias"]))
        outs.append(StageOutputs(*res))
    return outs
