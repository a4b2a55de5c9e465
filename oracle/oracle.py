"""TEST INFRASTRUCTURE ONLY -- Python handle on the CPU oracle.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and its ``--impl reference`` arm) may import this module,
and only as the checker or the timed CPU baseline. The product
(``brovisionml_b200`` and the CUDA library behind ``include/bvml_dsine.h``)
never imports it.

Two native libraries sit behind it, both built by ``oracle/Makefile``:

* ``oracle/_ref/libbvml_ref.so`` -- the reference's own CPU twin
  (``src/dsine_ops.cpp`` of wlejon/brovisionml, compiled in place). It is the
  5x5 / dilation-1 / fp32 / single-frame truth.
* ``oracle/_build/libbvml_oracle.so`` -- ``dsine_oracle.c``, the fp64
  restatement generalised to (ps, dilation), batches, and the convex upsample
  / L2 / crop / full-res RayReLU steps that the reference delegates to the
  absent brotensor library.

It also holds the seeded synthetic input generators for the benchmark
configurations (``gen_unit``), the fp16 rounding used for the fp16-storage
oracle, and the comparison metrics.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(_HERE, "_build", "libbvml_oracle.so")
_REF_SO = os.path.join(_HERE, "_ref", "libbvml_ref.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_libs: dict = {}


def build() -> None:
    """Compile the oracle libraries (needs gcc; the reference tree is optional)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load(path: str, key: str):
    if key not in _libs:
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run `make -C oracle`)")
        _libs[key] = ctypes.CDLL(path)
    return _libs[key]


def oracle_lib():
    lib = _load(_ORACLE_SO, "oracle")
    if not getattr(lib, "_typed", False):
        d, i, l = ctypes.c_double, ctypes.c_int, ctypes.c_long
        lib.bb_ray_relu.argtypes = [_f32p, _f32p, l]
        lib.bb_angmf.argtypes = [_f32p] * 5 + [d] * 4 + [i] * 4 + [_f32p]
        lib.bb_angmf_neighbor.argtypes = [d, d, d, i, i, d, d, d, d, d, d, d, d, d, d, d,
                                          ctypes.POINTER(ctypes.c_double)]
        lib.bb_convex_upsample.argtypes = [_f32p, _f32p, i, i, i, i, _f32p]
        lib.bb_l2_normalize.argtypes = [_f32p, i, l, d, _f32p]
        lib.bb_crop.argtypes = [_f32p, i, i, i, i, i, i, i, _f32p]
        lib.bb_build_ray.argtypes = [d, d, d, d, i, i, i, i, _f32p]
        lib.bb_build_ray_scaled.argtypes = [d, d, d, d, i, i, _f32p]
        lib.bb_refine_unit.argtypes = ([_f32p, _f32p, ctypes.POINTER(_f32p),
                                        ctypes.POINTER(_f32p), ctypes.POINTER(_f32p), _f32p]
                                       + [i] * 5 + [d] * 4 + [i] * 6 + [_f32p])
        lib.bb_refine_unit.restype = i
        lib._typed = True
    return lib


def ref_available() -> bool:
    return os.path.exists(_REF_SO)


def ref_lib():
    lib = _load(_REF_SO, "ref")
    if not getattr(lib, "_typed", False):
        d, i = ctypes.c_double, ctypes.c_int
        lib.bvml_ref_ray_relu.argtypes = [_f32p, _f32p, i, i]
        lib.bvml_ref_ray_relu.restype = i
        lib.bvml_ref_angmf.argtypes = [_f32p] * 5 + [d] * 4 + [i, i, _f32p]
        lib.bvml_ref_angmf.restype = i
        lib.bvml_ref_unit_mt.argtypes = ([_f32p, _f32p, ctypes.POINTER(_f32p),
                                          ctypes.POINTER(_f32p), ctypes.POINTER(_f32p), _f32p]
                                         + [i] * 5 + [d] * 4 + [i] * 5 + [_f32p, i])
        lib.bvml_ref_unit_mt.restype = i
        lib._typed = True
    return lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def _c32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- single ops

def ray_relu(normal: np.ndarray, ray: np.ndarray, *, use_ref: bool = False) -> np.ndarray:
    """RayReLU of (3,H,W) (or (B,3,H,W)) normals against a (3,H,W) ray. Returns a copy."""
    n = _c32(normal).copy()
    r = _c32(ray)
    H, W = n.shape[-2:]
    frames = n.reshape(-1, 3, H, W)
    for b in range(frames.shape[0]):
        fb = np.ascontiguousarray(frames[b])
        if use_ref:
            rc = ref_lib().bvml_ref_ray_relu(_p(fb), _p(r), H, W)
            if rc != 0:
                raise RuntimeError("reference ray_relu failed")
        else:
            oracle_lib().bb_ray_relu(_p(fb), _p(r), H * W)
        frames[b] = fb
    return frames.reshape(n.shape)


def angmf(pred_norm, prob, xy, angle, ray, fu, cu, fv, cv, *, ps: int = 5, dil: int = 1,
          use_ref: bool = False) -> np.ndarray:
    """AngMF propagate. pred_norm (B,3,H,W) or (3,H,W); prob/angle (.., P,H,W);
    xy (.., 2P,H,W); ray (3,H,W) shared by all frames. Returns float32 like pred_norm."""
    pn = _c32(pred_norm)
    H, W = pn.shape[-2:]
    P = ps * ps
    pnb = pn.reshape(-1, 3, H, W)
    B = pnb.shape[0]
    prb = _c32(prob).reshape(B, P, H, W)
    xyb = _c32(xy).reshape(B, 2 * P, H, W)
    anb = _c32(angle).reshape(B, P, H, W)
    r = _c32(ray).reshape(3, H, W)
    out = np.empty_like(pnb)
    for b in range(B):
        o = np.empty((3, H, W), np.float32)
        args = [np.ascontiguousarray(pnb[b]), np.ascontiguousarray(prb[b]),
                np.ascontiguousarray(xyb[b]), np.ascontiguousarray(anb[b]), r]
        if use_ref:
            if ps != 5 or dil != 1:
                raise ValueError("the reference twin is 5x5 / dilation 1 only")
            rc = ref_lib().bvml_ref_angmf(*[_p(a) for a in args], fu, cu, fv, cv, H, W, _p(o))
            if rc != 0:
                raise RuntimeError("reference angmf failed")
        else:
            oracle_lib().bb_angmf(*[_p(a) for a in args], fu, cu, fv, cv, H, W, ps, dil, _p(o))
        out[b] = o
    return out.reshape(pn.shape)


def angmf_neighbor(nx, ny, nz, sx, sy, xs, ys, theta, w, rx, ry, rz, fu, cu, fv, cv):
    o = (ctypes.c_double * 3)()
    oracle_lib().bb_angmf_neighbor(nx, ny, nz, sx, sy, xs, ys, theta, w, rx, ry, rz,
                                   fu, cu, fv, cv, o)
    return np.array(o[:], np.float64)


def convex_upsample(x, mask, scale: int = 8) -> np.ndarray:
    """(B,C,H,W) x (B,9*s*s,H,W) -> (B,C,sH,sW), softmax over the 9 taps."""
    xx = _c32(x)
    C, H, W = xx.shape[-3:]
    xb = xx.reshape(-1, C, H, W)
    mb = _c32(mask).reshape(xb.shape[0], 9 * scale * scale, H, W)
    out = np.empty((xb.shape[0], C, H * scale, W * scale), np.float32)
    for b in range(xb.shape[0]):
        o = np.empty((C, H * scale, W * scale), np.float32)
        oracle_lib().bb_convex_upsample(_p(np.ascontiguousarray(xb[b])),
                                        _p(np.ascontiguousarray(mb[b])), C, H, W, scale, _p(o))
        out[b] = o
    return out.reshape(xx.shape[:-3] + (C, H * scale, W * scale))


def l2_normalize(x, eps: float = 1e-12) -> np.ndarray:
    xx = _c32(x).copy()
    C, H, W = xx.shape[-3:]
    xb = xx.reshape(-1, C, H, W)
    for b in range(xb.shape[0]):
        f = np.ascontiguousarray(xb[b])
        oracle_lib().bb_l2_normalize(_p(f), C, H * W, eps, _p(f))
        xb[b] = f
    return xb.reshape(xx.shape)


def build_ray(fx, fy, cx, cy, Hf, Wf, origH, origW) -> np.ndarray:
    r = np.empty((3, Hf, Wf), np.float32)
    oracle_lib().bb_build_ray(fx, fy, cx, cy, Hf, Wf, origH, origW, _p(r))
    return r


def build_ray_scaled(fu, cu, fv, cv, Hf, Wf) -> np.ndarray:
    r = np.empty((3, Hf, Wf), np.float32)
    oracle_lib().bb_build_ray_scaled(fu, cu, fv, cv, Hf, Wf, _p(r))
    return r


# kPi of src/dsine_refine.cpp:26 (a float constant)
KPI_F32 = np.float32(3.14159265358979323846)


def head_activation(prob_logits, angle_logits):
    """The head activations of Refiner::forward (src/dsine_refine.cpp:262-267):
    prob = sigmoid(prob_logits); angle = sigmoid(angle_logits) * kPi, as the
    fp32 tensors the reference produces. brotensor's sigmoid_forward is not in
    the reference tree (parity unpinned): it is taken as the correctly rounded
    fp32 logistic (fp64 evaluation, one rounding), and scale_inplace as an fp32
    product."""
    def sig(x):
        with np.errstate(over="ignore"):
            return (1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))).astype(np.float32)

    return sig(prob_logits), (sig(angle_logits) * KPI_F32).astype(np.float32)


# ---------------------------------------------------------------- fp16 storage

def f16_round(a: np.ndarray) -> np.ndarray:
    """Round to IEEE binary16 (nearest-even) and back: the fp16-storage oracle input."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------- generators

@dataclass
class UnitInputs:
    """Seeded synthetic inputs of one refine-ops unit (all frames).

    normal0 (B,3,h,w)  ray8 (3,h,w)  prob[i] (B,P,h,w)  xy[i] (B,2P,h,w)
    angle[i] (B,P,h,w)  mask (B,576,h,w) or None; intrinsics already scaled to
    the /8 grid (fu, cu, fv, cv) plus the full-resolution pre-"+0.5" ones.
    """
    B: int
    H: int
    W: int
    h: int
    w: int
    ps: int
    dil: int
    iters: int
    fu: float
    cu: float
    fv: float
    cv: float
    fx: float
    fy: float
    cx: float
    cy: float
    normal0: np.ndarray
    ray8: np.ndarray
    prob: list = field(default_factory=list)
    xy: list = field(default_factory=list)
    angle: list = field(default_factory=list)
    mask: np.ndarray | None = None


def _rng(seed: int, frame: int, stream: int) -> np.random.Generator:
    return np.random.default_rng([int(seed), int(frame), int(stream)])


def gen_unit(H: int, W: int, B: int = 1, *, ps: int = 5, dil: int = 1, iters: int = 5,
             seed: int = 0, upsample: bool = True, face_camera: bool = True,
             angle_max: float = 0.3) -> UnitInputs:
    """Seeded synthetic inputs with the benchmark configurations' distributions.

    Full-res intrinsics fx = fy = 0.8 W, cx = W/2, cy = H/2 (pre-"+0.5"); the /8
    grid ray is build_ray8's; normals are N(0,1)^3 normalised and flipped to
    face the camera (n.ray > 0; ``face_camera=False`` flips them away, the
    clamp-heavy stress case); xy ~ N(0,1); angle ~ U(0, angle_max); prob is a
    softmax over the P window slots of N(0,1) logits; mask logits ~ N(0,1).
    Every frame b draws from its own streams of seed (seed, b, k).
    """
    h, w = H // 8, W // 8
    P = ps * ps
    fx = fy = 0.8 * W
    cx, cy = W / 2.0, H / 2.0
    sw, sh = w / W, h / H
    fu, cu = fx * sw, (cx + 0.5) * sw
    fv, cv = fy * sh, (cy + 0.5) * sh
    ray8 = build_ray(fx, fy, cx, cy, h, w, H, W)
    normal0 = np.empty((B, 3, h, w), np.float32)
    prob = [np.empty((B, P, h, w), np.float32) for _ in range(iters)]
    xy = [np.empty((B, 2 * P, h, w), np.float32) for _ in range(iters)]
    angle = [np.empty((B, P, h, w), np.float32) for _ in range(iters)]
    mask = np.empty((B, 576, h, w), np.float32) if upsample else None
    for b in range(B):
        g = _rng(seed, b, 0)
        n = g.standard_normal((3, h, w))
        n /= np.maximum(np.sqrt((n * n).sum(0, keepdims=True)), 1e-12)
        s = np.sign((n * ray8.astype(np.float64)).sum(0, keepdims=True))
        s[s == 0] = 1.0
        n *= s if face_camera else -s
        normal0[b] = n
        for i in range(iters):
            g = _rng(seed, b, 1 + i)
            xy[i][b] = g.standard_normal((2 * P, h, w))
            angle[i][b] = g.uniform(0.0, angle_max, (P, h, w))
            lg = g.standard_normal((P, h, w))
            lg -= lg.max(0, keepdims=True)
            e = np.exp(lg)
            prob[i][b] = e / e.sum(0, keepdims=True)
        if upsample:
            mask[b] = _rng(seed, b, 99).standard_normal((576, h, w))
    return UnitInputs(B=B, H=H, W=W, h=h, w=w, ps=ps, dil=dil, iters=iters, fu=fu, cu=cu,
                      fv=fv, cv=cv, fx=fx, fy=fy, cx=cx, cy=cy, normal0=normal0, ray8=ray8,
                      prob=prob, xy=xy, angle=angle, mask=mask)


def to_f16_storage(u: UnitInputs) -> UnitInputs:
    """The fp16-storage variant: every stored input rounded to binary16."""
    return UnitInputs(**{**u.__dict__,
                         "normal0": f16_round(u.normal0),
                         "prob": [f16_round(a) for a in u.prob],
                         "xy": [f16_round(a) for a in u.xy],
                         "angle": [f16_round(a) for a in u.angle],
                         "mask": None if u.mask is None else f16_round(u.mask)})


# ---------------------------------------------------------------- whole unit

def refine_unit(u: UnitInputs, *, full_res_ray_relu: bool = False, crop=None) -> np.ndarray:
    """The oracle for the fused device path: ray_relu, iters x AngMF, convex
    upsample, L2, optional full-res RayReLU, crop. Returns (B,3,out_h,out_w)."""
    lib = oracle_lib()
    s = 8
    crop_t, crop_l, out_h, out_w = crop if crop is not None else (0, 0, u.h * s, u.w * s)
    out = np.empty((u.B, 3, out_h, out_w), np.float32)
    for b in range(u.B):
        n0 = np.ascontiguousarray(u.normal0[b])
        pr = [np.ascontiguousarray(a[b]) for a in u.prob]
        xy = [np.ascontiguousarray(a[b]) for a in u.xy]
        an = [np.ascontiguousarray(a[b]) for a in u.angle]
        mk = np.ascontiguousarray(u.mask[b])
        o = np.empty((3, out_h, out_w), np.float32)
        arr = lambda lst: (_f32p * len(lst))(*[_p(a) for a in lst])  # noqa: E731
        rc = lib.bb_refine_unit(_p(n0), _p(u.ray8), arr(pr), arr(xy), arr(an), _p(mk),
                                u.h, u.w, u.iters, u.ps, u.dil, u.fu, u.cu, u.fv, u.cv, s,
                                int(full_res_ray_relu), crop_t, crop_l, out_h, out_w, _p(o))
        if rc != 0:
            raise MemoryError("oracle refine_unit: allocation failed")
        out[b] = o
    return out


def ref_unit_mt(u: UnitInputs, threads: int = 0, *, full_res_ray_relu: bool = False,
                frames: int | None = None, out: np.ndarray | None = None):
    """The unit through the reference twin (5x5, d=1), frames over host threads.
    ``frames`` (default u.B) output frames are computed, frame b from input
    frame b % u.B. Returns (out, threads_used)."""
    if u.ps != 5 or u.dil != 1:
        raise ValueError("the reference twin is 5x5 / dilation 1 only")
    lib = ref_lib()
    out_h, out_w = u.h * 8, u.w * 8
    frames = u.B if frames is None else frames
    if out is None:
        out = np.empty((frames, 3, out_h, out_w), np.float32)
    arr = lambda lst: (_f32p * len(lst))(*[_p(_c32(a)) for a in lst])  # noqa: E731
    keep = [_c32(a) for a in u.prob + u.xy + u.angle]
    n = lib.bvml_ref_unit_mt(_p(_c32(u.normal0)), _p(u.ray8), arr(keep[:u.iters]),
                             arr(keep[u.iters:2 * u.iters]), arr(keep[2 * u.iters:]),
                             _p(_c32(u.mask)), frames, u.B, u.h, u.w, u.iters, u.fu, u.cu, u.fv,
                             u.cv,
                             int(full_res_ray_relu), 0, 0, out_h, out_w, _p(out), threads)
    if n < 0:
        raise RuntimeError("reference unit failed")
    return out, n


# ---------------------------------------------------------------- metrics

def compare(got: np.ndarray, want: np.ndarray) -> dict:
    """max-abs / mean-abs per component plus angular error (degrees) over pixels."""
    g = np.asarray(got, np.float64)
    wv = np.asarray(want, np.float64)
    d = np.abs(g - wv)
    gc = np.moveaxis(g, -3, -1).reshape(-1, 3)
    wc = np.moveaxis(wv, -3, -1).reshape(-1, 3)
    gn = gc / np.maximum(np.linalg.norm(gc, axis=1, keepdims=True), 1e-300)
    wn = wc / np.maximum(np.linalg.norm(wc, axis=1, keepdims=True), 1e-300)
    ang = np.degrees(np.arccos(np.clip((gn * wn).sum(1), -1.0, 1.0)))
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "mean_abs": float(d.mean()) if d.size else 0.0,
        "ang_mean_deg": float(ang.mean()) if ang.size else 0.0,
        "ang_p99_deg": float(np.percentile(ang, 99)) if ang.size else 0.0,
        "ang_max_deg": float(ang.max()) if ang.size else 0.0,
        "nonfinite": int((~np.isfinite(g)).sum()),
    }


TOL_F32 = 1e-5
TOL_F16 = 2e-3

