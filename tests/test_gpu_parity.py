"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Tolerances (per component): max-abs 1e-5 with fp32 storage, 2e-3 with fp16
storage (the fp16 oracle is the fp32 oracle fed fp16-rounded inputs).
The reference twin (oracle/_ref) is the oracle for its own 5x5 / dilation-1 /
fp32 / single-frame case; the pinned restatement covers the rest.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL32 = O.TOL_F32
TOL16 = O.TOL_F16


def lib():
    import brovisionml_b200 as b

    return b


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda:0", dtype)


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def report(name, got, want, tol):
    m = O.compare(got, want)
    print(f"{name}: max_abs {m['max_abs']:.3e} mean_abs {m['mean_abs']:.3e} "
          f"ang_mean {m['ang_mean_deg']:.2e} ang_p99 {m['ang_p99_deg']:.2e} "
          f"ang_max {m['ang_max_deg']:.2e} deg")
    assert m["nonfinite"] == 0
    assert m["max_abs"] <= tol, m
    return m


# ------------------------------------------------------------------ ray_relu

@pytest.mark.parametrize("seed,face", [(0, True), (1, False)])
def test_ray_relu_vs_reference(seed, face):
    b = lib()
    u = O.gen_unit(480, 640, 1, iters=0, seed=seed, upsample=False, face_camera=face)
    want = O.ray_relu(u.normal0[0], u.ray8, use_ref=O.ref_available())
    n = dev(u.normal0)
    b.ray_relu(n, dev(u.ray8))
    report("ray_relu", host(n)[0], want, TOL32)


def test_ray_relu_f16_and_batch():
    b = lib()
    u = O.gen_unit(256, 320, 4, iters=0, seed=5, upsample=False, face_camera=False)
    n16 = O.f16_round(u.normal0)
    want = O.ray_relu(n16, u.ray8)
    n = dev(n16, torch.float16)
    b.ray_relu(n, dev(u.ray8))
    report("ray_relu f16", host(n), want, TOL16)


# ------------------------------------------------------------------ angmf

def _angmf_case(H, W, B, ps, dil, seed, face=True, f16=False, use_ref=False):
    b = lib()
    u = O.gen_unit(H, W, B, ps=ps, dil=dil, iters=1, seed=seed, upsample=False,
                   face_camera=face)
    if f16:
        u = O.to_f16_storage(u)
    n0 = O.ray_relu(u.normal0, u.ray8)
    if f16:
        n0 = O.f16_round(n0)
    want = O.angmf(n0, u.prob[0], u.xy[0], u.angle[0], u.ray8, u.fu, u.cu, u.fv, u.cv, ps=ps,
                   dil=dil, use_ref=use_ref)
    dt = torch.float16 if f16 else torch.float32
    got = b.angmf_propagate(dev(n0, dt), dev(u.prob[0], dt), dev(u.xy[0], dt),
                            dev(u.angle[0], dt), dev(u.ray8), u.fu, u.cu, u.fv, u.cv, ps=ps,
                            dil=dil)
    return host(got), want


@pytest.mark.parametrize("seed,face", [(0, True), (1, True), (2, False), (3, True)])
def test_angmf_cfg0_vs_reference_twin(seed, face):
    got, want = _angmf_case(480, 640, 1, 5, 1, seed, face, use_ref=O.ref_available())
    report(f"angmf cfg0 seed {seed}", got, want, TOL32)


@pytest.mark.parametrize("H,W", [(8, 8), (8, 56), (56, 8), (40, 104), (24, 200), (136, 96)])
def test_angmf_shapes(H, W):
    got, want = _angmf_case(H, W, 1, 5, 1, H + W, use_ref=O.ref_available())
    report(f"angmf {H//8}x{W//8}", got, want, TOL32)


@pytest.mark.parametrize("hw", [(1, 1), (1, 7), (7, 1), (5, 13), (13, 5), (33, 65), (17, 31)])
def test_angmf_odd_grids(hw):
    """Grids that are not /8 of a padded frame (odd widths take the unpaired path)."""
    b = lib()
    h, w = hw
    g = np.random.default_rng(h * 1000 + w)
    n = g.standard_normal((1, 3, h, w)).astype(np.float32)
    n /= np.linalg.norm(n, axis=1, keepdims=True)
    prob = g.random((1, 25, h, w)).astype(np.float32)
    xy = g.standard_normal((1, 50, h, w)).astype(np.float32)
    ang = g.uniform(0, np.pi, (1, 25, h, w)).astype(np.float32)
    fu, cu, fv, cv = 0.8 * w + 0.3, w / 2 + 0.06, 0.8 * h + 0.7, h / 2 + 0.06
    ray = O.build_ray_scaled(fu, cu, fv, cv, h, w)
    want = O.angmf(n, prob, xy, ang, ray, fu, cu, fv, cv)
    got = b.angmf_propagate(dev(n), dev(prob), dev(xy), dev(ang), dev(ray), fu, cu, fv, cv)
    report(f"angmf odd {h}x{w}", host(got), want, TOL32)


@pytest.mark.parametrize("ps,dil", [(3, 1), (5, 2), (7, 1), (7, 2), (3, 4)])
def test_angmf_windows(ps, dil):
    got, want = _angmf_case(256, 320, 2, ps, dil, 40 + ps + dil)
    report(f"angmf ps{ps} d{dil}", got, want, TOL32)


@pytest.mark.parametrize("ps,dil", [(5, 1), (5, 2), (7, 1)])
def test_angmf_f16_storage(ps, dil):
    got, want = _angmf_case(256, 320, 2, ps, dil, 50 + ps + dil, f16=True)
    report(f"angmf f16 ps{ps} d{dil}", got, want, TOL16)


def test_angmf_f16_degenerate_offsets():
    """fp16 storage (no |xy|^2 range test there): zero, signed-zero and
    subnormal xy pairs, theta 0 and fp16(pi), through the staged kernel."""
    b = lib()
    u = O.to_f16_storage(O.gen_unit(512, 768, 1, iters=1, seed=91, upsample=False))
    xy, ang = u.xy[0].copy(), u.angle[0].copy()
    P = ang.shape[1]
    g = np.random.default_rng(17)
    pick = g.random(ang.shape)
    xs, ys = xy[:, :P], xy[:, P:]
    zero = pick < 0.08
    xs[zero], ys[zero] = 0.0, -0.0
    tiny = (pick >= 0.08) & (pick < 0.12)          # binary16 subnormals
    xs[tiny] = np.where(g.random(tiny.sum()) < 0.5, 6e-8, -1.2e-7)
    ys[tiny] = np.where(g.random(tiny.sum()) < 0.5, 0.0, 3e-7)
    ang[(pick >= 0.12) & (pick < 0.15)] = 0.0
    ang[(pick >= 0.15) & (pick < 0.18)] = np.pi
    xy, ang = O.f16_round(xy), O.f16_round(ang)
    n0 = O.f16_round(O.ray_relu(u.normal0, u.ray8))
    want = O.angmf(n0, u.prob[0], xy, ang, u.ray8, u.fu, u.cu, u.fv, u.cv)
    h16 = torch.float16
    got = b.angmf_propagate(dev(n0, h16), dev(u.prob[0], h16), dev(xy, h16), dev(ang, h16),
                            dev(u.ray8), u.fu, u.cu, u.fv, u.cv)
    report("angmf f16 degenerate", host(got), want, TOL16)


def test_angmf_tiny_huge_zero_source_normals():
    """Source normals far from unit length (the reference rotates them raw and
    normalises after): 1e-14, 1e-30, subnormal, 1e25 and exactly zero, with
    rotation angles over the whole (0, pi] range."""
    b = lib()
    u = O.gen_unit(320, 448, 1, iters=1, seed=29, upsample=False, angle_max=float(np.pi))
    n0 = O.ray_relu(u.normal0, u.ray8).copy()
    g = np.random.default_rng(29)
    pick = g.random(n0.shape[2:])
    for lo, scale in ((0.0, 1e-14), (0.05, 1e-30), (0.10, 1e-41), (0.15, 1e25), (0.20, 0.0)):
        sel = (pick >= lo) & (pick < lo + 0.05)
        n0[0][:, sel] *= np.float32(scale)
    want = O.angmf(n0, u.prob[0], u.xy[0], u.angle[0], u.ray8, u.fu, u.cu, u.fv, u.cv)
    got = b.angmf_propagate(dev(n0), dev(u.prob[0]), dev(u.xy[0]), dev(u.angle[0]),
                            dev(u.ray8), u.fu, u.cu, u.fv, u.cv)
    report("angmf tiny/huge/zero sources", host(got), want, TOL32)


def test_angmf_golden_edge_cases():
    """Hand-placed degeneracies (zero xy, |xy| < 1e-12, theta 0 / 1e-7 / pi,
    zero and non-unit normals, (P+d).n ~ 0) against the reference's outputs."""
    import os

    b = lib()
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "edge_9x7.npz"))
    fu, cu, fv, cv = [float(v) for v in d["intr"]]
    args = [dev(d[k][None]) for k in ("prob", "xy", "angle")] + [dev(d["ray8"])]
    got = b.angmf_propagate(dev(d["normal0"][None]), *args, fu, cu, fv, cv)
    report("angmf edge raw", host(got)[0], d["ref_angmf_raw"], TOL32)
    got = b.angmf_propagate(dev(d["ref_ray_relu"][None]), *args, fu, cu, fv, cv)
    report("angmf edge", host(got)[0], d["ref_angmf"], TOL32)


def test_angmf_wide_angles_and_near_singular():
    """theta over the whole (0, pi] range and many grazing normals."""
    b = lib()
    u = O.gen_unit(160, 200, 2, iters=1, seed=77, upsample=False, angle_max=float(np.pi))
    n0 = u.normal0.copy()
    # push a third of the normals close to grazing (n . ray ~ 0)
    r = u.ray8.astype(np.float64)
    t = n0.astype(np.float64) - (n0 * r[None]).sum(1, keepdims=True) * r[None] * 0.999
    t /= np.linalg.norm(t, axis=1, keepdims=True)
    n0[:, :, ::3] = t[:, :, ::3].astype(np.float32)
    want = O.angmf(n0, u.prob[0], u.xy[0], u.angle[0], u.ray8, u.fu, u.cu, u.fv, u.cv)
    got = b.angmf_propagate(dev(n0), dev(u.prob[0]), dev(u.xy[0]), dev(u.angle[0]),
                            dev(u.ray8), u.fu, u.cu, u.fv, u.cv)
    report("angmf wide", host(got), want, TOL32)


def test_angmf_batch_frames_independent_and_stream():
    b = lib()
    u = O.gen_unit(160, 240, 3, iters=1, seed=88, upsample=False)
    args = [dev(u.prob[0]), dev(u.xy[0]), dev(u.angle[0])]
    full = b.angmf_propagate(dev(u.normal0), *args, dev(u.ray8), u.fu, u.cu, u.fv, u.cv)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        one = b.angmf_propagate(dev(u.normal0[1:2]), dev(u.prob[0][1:2]), dev(u.xy[0][1:2]),
                                dev(u.angle[0][1:2]), dev(u.ray8), u.fu, u.cu, u.fv, u.cv)
    s.synchronize()
    assert torch.equal(full[1:2], one)


# ------------------------------------------------------------------ upsample & friends

@pytest.mark.parametrize("h,w,f16", [(60, 80, False), (9, 7, False), (16, 32, True),
                                     (3, 65, False)])
def test_convex_upsample_and_l2(h, w, f16):
    b = lib()
    g = np.random.default_rng(h * w)
    x = g.standard_normal((2, 3, h, w)).astype(np.float32)
    m = (2 * g.standard_normal((2, 576, h, w))).astype(np.float32)
    if f16:
        x, m = O.f16_round(x), O.f16_round(m)
    dt = torch.float16 if f16 else torch.float32
    want = O.convex_upsample(x, m)
    got = b.convex_upsample(dev(x, dt), dev(m, dt), 2, 3, h, w, 8)
    report("convex_upsample", host(got), want, TOL16 * 4 if f16 else TOL32)
    want_n = O.l2_normalize(want)
    got_n = b.l2_normalize_nchw(dev(want), 2, 3, 8 * h, 8 * w, 1e-12)
    report("l2_normalize", host(got_n), want_n, TOL32)
    sl = b.slice2d(dev(want), 2, 3, 8 * h, 8 * w, 3, 5, 8 * h - 4, 8 * w - 6)
    assert np.array_equal(host(sl), want[:, :, 3:8 * h - 1, 5:8 * w - 1])


# ------------------------------------------------------------------ fused unit

def _unit(u, f16=False, full_res_ray_relu=False, crop=None, ray_given=True):
    b = lib()
    if f16:
        u = O.to_f16_storage(u)
    want = O.refine_unit(u, full_res_ray_relu=full_res_ray_relu, crop=crop)
    dt = torch.float16 if f16 else torch.float32
    got = b.refine(dev(u.normal0, dt), [dev(a, dt) for a in u.prob], [dev(a, dt) for a in u.xy],
                   [dev(a, dt) for a in u.angle], dev(u.mask, dt), u.fu, u.cu, u.fv, u.cv,
                   ray8=dev(u.ray8) if ray_given else None, ps=u.ps, dil=u.dil,
                   full_res_ray_relu=full_res_ray_relu, crop=crop)
    return host(got), want


def test_refine_cfg1():
    """Config 1: 480x640, 5 iterations with fresh inputs per iteration, convex
    upsample, full-resolution RayReLU."""
    got, want = _unit(O.gen_unit(480, 640, 1, iters=5, seed=1), full_res_ray_relu=True)
    report("refine cfg1", got, want, TOL32)


def test_refine_cfg1_analytic_ray_and_crop():
    got, want = _unit(O.gen_unit(480, 640, 1, iters=5, seed=2), crop=(4, 6, 470, 628),
                      ray_given=False)
    report("refine cfg1 crop", got, want, TOL32)


@pytest.mark.parametrize("f16", [False, True])
def test_refine_cfg2_like(f16):
    """Config 2 shape class at reduced batch: 1024^2 frames, 5x5 at dilation 2."""
    got, want = _unit(O.gen_unit(1024, 1024, 2, dil=2, iters=5, seed=3), f16=f16)
    report(f"refine cfg2 f16={f16}", got, want, TOL16 if f16 else TOL32)


def test_refine_cfg3_like():
    """Config 3 window (7x7) on a 1024^2 frame."""
    got, want = _unit(O.gen_unit(1024, 1024, 1, ps=7, iters=5, seed=4))
    report("refine cfg3-like", got, want, TOL32)


def test_refine_cfg4_like():
    """Config 4 frames (720x1280, fp16 storage) at reduced batch."""
    got, want = _unit(O.gen_unit(720, 1280, 3, iters=5, seed=5), f16=True)
    report("refine cfg4-like", got, want, TOL16)
