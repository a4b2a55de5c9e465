"""Python mirror of the reference's DSINE op interface, over the C ABI.

Each function mirrors one reference entry point, with the same argument
meaning and error behaviour, and runs the corresponding CUDA kernels of
libbvml_dsine.so on the tensors' device and the current torch stream:

  ray_relu            brovisionml::dsine::ray_relu          dsine_ops.h:25-26
  angmf_propagate     brovisionml::dsine::angmf_propagate   dsine_ops.h:47-54
  convex_upsample     brotensor::convex_upsample_forward    dsine_refine.cpp:277-279
  l2_normalize_nchw   brotensor::l2_normalize_nchw_forward  dsine_refine.cpp:280-281
  slice2d             brotensor::slice2d_forward            dsine_refine.cpp:288-292
  refine              the op sequence of Refiner::forward   dsine_refine.cpp:241-292

Tensors may be given in the reference's flat form ((1, C*H*W) with explicit
H, W) or as (B, C, H, W). Storage is float32 or float16 (fp32 arithmetic);
ray maps are float32. Device mismatches raise
``RuntimeError("dsine ops: ...")`` like src/dsine_ops.cpp:180-181,200-202.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from ._capi import BVML_F16, BVML_F32, check, lib


def _code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return BVML_F32
    if t.dtype == torch.float16:
        return BVML_F16
    raise RuntimeError(f"dsine ops: unsupported storage dtype {t.dtype}")


def _cuda(name: str, *ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t.device != dev:
            raise RuntimeError(f"dsine ops: {name}: all inputs must share a device")
    if dev.type != "cuda":
        raise RuntimeError(f"dsine ops: {name}: tensors must be CUDA-resident (this library "
                           "has no CPU path)")
    for t in ts:
        if not t.is_contiguous():
            raise RuntimeError(f"dsine ops: {name}: tensors must be contiguous")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t: torch.Tensor) -> int:
    return t.data_ptr()


def _numel_check(name: str, t: torch.Tensor, n: int, what: str) -> None:
    if t.numel() != n:
        raise RuntimeError(f"dsine ops: {name}: {what} has {t.numel()} elements, expected {n}")


def _frames(t: torch.Tensor, C: int, H: int | None, W: int | None):
    if H is None or W is None:
        if t.dim() != 4:
            raise RuntimeError("dsine ops: pass (B, C, H, W) tensors or explicit H, W")
        return t.shape[0], t.shape[2], t.shape[3]
    HW = H * W
    if HW == 0:
        return 1, H, W
    if t.numel() % (C * HW) != 0:
        raise RuntimeError("dsine ops: tensor size is not a multiple of C*H*W")
    return t.numel() // (C * HW), H, W


def ray_relu(normal: torch.Tensor, ray: torch.Tensor, H: int | None = None,
             W: int | None = None) -> None:
    """RayReLU in place (eps 1e-2). normal: B frames of (3,H,W); ray (3,H,W) fp32."""
    dev = _cuda("ray_relu", normal, ray)
    B, H, W = _frames(normal, 3, H, W)
    _numel_check("ray_relu", ray, 3 * H * W, "ray")
    if ray.dtype != torch.float32:
        raise RuntimeError("dsine ops: ray_relu: ray must be float32")
    with torch.cuda.device(dev):
        check(lib.bvml_ray_relu(_p(normal), _p(ray), B, H, W, _code(normal), _stream(dev)))


def angmf_propagate(pred_norm: torch.Tensor, prob: torch.Tensor, xy: torch.Tensor,
                    angle: torch.Tensor, ray: torch.Tensor, fu: float, cu: float, fv: float,
                    cv: float, H: int | None = None, W: int | None = None,
                    out: torch.Tensor | None = None, *, ps: int = 5, dil: int = 1,
                    logits: bool = False) -> torch.Tensor:
    """Fused AngMF propagate; returns ``out`` (allocated like pred_norm when None,
    as the reference (re)allocates it). With ``logits=True`` prob and angle are
    the prediction heads' raw outputs, activated on load (sigmoid, pi * sigmoid:
    src/dsine_refine.cpp:262-267)."""
    dev = _cuda("angmf_propagate", pred_norm, prob, xy, angle, ray)
    B, H, W = _frames(pred_norm, 3, H, W)
    P = ps * ps
    HW = H * W
    for t, c, nm in ((prob, P, "prob"), (xy, 2 * P, "xy"), (angle, P, "angle")):
        _numel_check("angmf_propagate", t, B * c * HW, nm)
        if t.dtype != pred_norm.dtype:
            raise RuntimeError("dsine ops: angmf_propagate: storage dtypes differ")
    _numel_check("angmf_propagate", ray, 3 * HW, "ray")
    if out is None:
        out = torch.empty_like(pred_norm)
    else:
        _cuda("angmf_propagate", pred_norm, out)
        _numel_check("angmf_propagate", out, pred_norm.numel(), "out")
    fn = lib.bvml_angmf_propagate_logits if logits else lib.bvml_angmf_propagate
    with torch.cuda.device(dev):
        check(fn(_p(pred_norm), _p(prob), _p(xy), _p(angle), _p(ray), float(fu), float(cu),
                 float(fv), float(cv), B, H, W, ps, dil, _code(pred_norm), _p(out),
                 _stream(dev)))
    return out


def convex_upsample(x: torch.Tensor, mask: torch.Tensor, N: int, C: int, H: int, W: int,
                    scale: int = 8, out: torch.Tensor | None = None) -> torch.Tensor:
    """brotensor::convex_upsample_forward(X, mask, N, C, H, W, scale, Y)."""
    dev = _cuda("convex_upsample", x, mask)
    if out is None:
        out = torch.empty((N, C, H * scale, W * scale), device=dev, dtype=x.dtype)
    with torch.cuda.device(dev):
        check(lib.bvml_convex_upsample(_p(x), _p(mask), N, C, H, W, scale, _code(x), _p(out),
                                       _stream(dev)))
    return out


def l2_normalize_nchw(x: torch.Tensor, N: int, C: int, H: int, W: int, eps: float = 1e-12,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """brotensor::l2_normalize_nchw_forward(X, N, C, H, W, eps, Y); out may be x."""
    dev = _cuda("l2_normalize", x)
    if out is None:
        out = torch.empty_like(x)
    with torch.cuda.device(dev):
        check(lib.bvml_l2_normalize_nchw(_p(x), N, C, H, W, float(eps), _code(x), _p(out),
                                         _stream(dev)))
    return out


def slice2d(x: torch.Tensor, N: int, C: int, H: int, W: int, h0: int, w0: int, Ho: int,
            Wo: int) -> torch.Tensor:
    """brotensor::slice2d_forward(X, N, C, H, W, h0, w0, Ho, Wo, Y)."""
    dev = _cuda("slice2d", x)
    out = torch.empty((N, C, Ho, Wo), device=dev, dtype=x.dtype)
    with torch.cuda.device(dev):
        check(lib.bvml_slice2d(_p(x), N, C, H, W, h0, w0, Ho, Wo, _code(x), _p(out),
                               _stream(dev)))
    return out


def refine_workspace_bytes(B: int, h: int, w: int) -> int:
    return int(lib.bvml_refine_workspace_bytes(B, h, w))


def refine(normal0: torch.Tensor, prob: Sequence[torch.Tensor], xy: Sequence[torch.Tensor],
           angle: Sequence[torch.Tensor], mask: torch.Tensor, fu: float, cu: float, fv: float,
           cv: float, *, ray8: torch.Tensor | None = None, ps: int = 5, dil: int = 1,
           full_res_ray_relu: bool = False, crop: tuple[int, int, int, int] | None = None,
           out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
           logits: bool = False) -> torch.Tensor:
    """The refine-ops unit of Refiner::forward for B frames (iters + 1 launches).

    normal0 (B,3,h,w); prob[i] (B,P,h,w); xy[i] (B,2P,h,w); angle[i] (B,P,h,w);
    mask (B,576,h,w); ray8 (3,h,w) fp32 or None (computed on the device);
    crop = (top, left, out_h, out_w) in the 8x output (default: no crop);
    logits=True: prob / angle are the heads' raw outputs (activated on load).
    Returns (B,3,out_h,out_w) in normal0's storage dtype.
    """
    iters = len(prob)
    if len(xy) != iters or len(angle) != iters:
        raise RuntimeError("dsine ops: refine: per-iteration lists differ in length")
    ts = [normal0, mask, *prob, *xy, *angle] + ([ray8] if ray8 is not None else [])
    dev = _cuda("refine", *ts)
    B, _, h, w = normal0.shape
    ct, cl, oh, ow = crop if crop is not None else (0, 0, 8 * h, 8 * w)
    if out is None:
        out = torch.empty((B, 3, oh, ow), device=dev, dtype=normal0.dtype)
    need = refine_workspace_bytes(B, h, w)
    if workspace is None:
        workspace = torch.empty(need, device=dev, dtype=torch.uint8)
    if workspace.numel() * workspace.element_size() < need:
        raise RuntimeError("dsine ops: refine: workspace too small")
    arr = lambda lst: (ctypes.c_void_p * max(1, len(lst)))(*[t.data_ptr() for t in lst])  # noqa
    fn = lib.bvml_refine_logits if logits else lib.bvml_refine
    with torch.cuda.device(dev):
        check(fn(_p(normal0), _p(ray8) if ray8 is not None else None, arr(prob), arr(xy),
                 arr(angle), iters, _p(mask), B, h, w, ps, dil, float(fu), float(cu), float(fv),
                 float(cv), int(bool(full_res_ray_relu)), ct, cl, oh, ow, _code(normal0),
                 _p(workspace), need, _p(out), _stream(dev)))
    return out


# ------------------------------------------------------------ tensor-core conv

ACTIVATIONS = {"none": 0, "relu": 1, "sigmoid": 2, "tanh": 3}


def pad64(c: int) -> int:
    return (c + 63) // 64 * 64


def pack_conv_weight(weight: torch.Tensor, cin_pad: int | None = None,
                     cout_pad: int | None = None) -> torch.Tensor:
    """(C_out, C_in, k, k) conv weights -> the (k*k, C_out_pad, C_in_pad) fp16
    K-major layout conv2d_nhwc takes (zero padded)."""
    cout, cin, k, _ = weight.shape
    cin_pad = cin_pad or pad64(cin)
    cout_pad = cout_pad or pad64(cout)
    w = torch.zeros((k * k, cout_pad, cin_pad), device=weight.device, dtype=torch.float16)
    w[:, :cout, :cin] = weight.permute(2, 3, 0, 1).reshape(k * k, cout, cin).to(torch.float16)
    return w


def conv2d_nhwc(x: torch.Tensor, w_packed: torch.Tensor, bias: torch.Tensor, cout: int, *,
                ks: int, act: str = "none", out: torch.Tensor | None = None,
                err: torch.Tensor | None = None) -> torch.Tensor:
    """Stride-1 "same" conv on the tensor cores: x (B,H,W,cin_pad) fp16,
    w_packed from pack_conv_weight, bias (cout) fp32; returns
    (B,H,W,cout_pad) fp16 (pad channels zero). Raises if the kernel's pipeline
    reported a failure (checked when ``err`` is None: one device sync)."""
    dev = _cuda("conv2d", x, w_packed, bias)
    B, H, W, cin_pad = x.shape
    cout_pad = w_packed.shape[1]
    if x.dtype != torch.float16 or w_packed.dtype != torch.float16:
        raise RuntimeError("dsine ops: conv2d: x and weights must be fp16")
    if bias.dtype != torch.float32 or bias.numel() < cout:
        raise RuntimeError("dsine ops: conv2d: bias must be fp32 with cout entries")
    if w_packed.shape != (ks * ks, cout_pad, cin_pad):
        raise RuntimeError("dsine ops: conv2d: packed weights do not match x / ks")
    if out is None:
        out = torch.empty((B, H, W, cout_pad), device=dev, dtype=torch.float16)
    own_err = err is None
    if own_err:
        err = torch.zeros(1, device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        check(lib.bvml_conv2d_nhwc_f16(_p(x.contiguous()), _p(w_packed), _p(bias), B, H, W,
                                        cin_pad, cout, cout_pad, ks, ACTIVATIONS[act], _p(out),
                                        _p(err), _stream(dev)))
    if own_err and int(err.item()) != 0:
        raise RuntimeError(f"dsine cuda: conv2d: pipeline gave up (code {int(err.item())})")
    return out
