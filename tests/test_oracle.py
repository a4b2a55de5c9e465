"""CPU tests: pin the oracle restatement to the reference and check its
generalisations independently.

* bit-exact against the committed golden fixtures (outputs of the reference's
  own CPU twin, tests/golden/make_golden.py);
* bit-exact against the reference twin library itself (oracle/_ref), when it
  was built, on more seeds and odd shapes;
* the (ps, dilation) generalisation, the convex upsample / L2 / crop
  restatement and the ray builder against independent numpy / torch fp64
  formulations.
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "*_*x*.npz"))))
def test_restatement_matches_reference_goldens(path):
    d = np.load(path)
    fu, cu, fv, cv = d["intr"]
    if "normal0" in d:
        n0, ray = d["normal0"], d["ray8"]
        prob, xy, ang = d["prob"], d["xy"], d["angle"]
    else:  # cfg0: regenerate the seeded inputs and check they are the same inputs
        u = O.gen_unit(480, 640, 1, iters=1, seed=0, upsample=False)
        import hashlib

        h = hashlib.sha256()
        for a in (u.normal0, u.ray8, u.prob[0], u.xy[0], u.angle[0]):
            h.update(np.ascontiguousarray(a, np.float32).tobytes())
        assert h.hexdigest() == str(d["input_sha256"]), "seeded generator drifted"
        n0, ray = u.normal0[0], u.ray8
        prob, xy, ang = u.prob[0][0], u.xy[0][0], u.angle[0][0]
    n = O.ray_relu(n0, ray)
    assert np.array_equal(bits(n), bits(d["ref_ray_relu"]))
    a = O.angmf(n, prob, xy, ang, ray, fu, cu, fv, cv)
    assert np.array_equal(bits(a), bits(d["ref_angmf"]))
    if "ref_angmf_raw" in d:
        a = O.angmf(n0, prob, xy, ang, ray, fu, cu, fv, cv)
        assert np.array_equal(bits(a), bits(d["ref_angmf_raw"]))


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("H,W,seed,face", [(480, 640, 1, True), (96, 136, 2, False),
                                           (8, 8, 3, True), (8, 40, 4, True), (40, 8, 5, True),
                                           (56, 104, 6, True), (16, 16, 7, False)])
def test_restatement_bitexact_vs_reference_twin(H, W, seed, face):
    u = O.gen_unit(H, W, 1, iters=1, seed=seed, upsample=False, face_camera=face)
    n_ref = O.ray_relu(u.normal0, u.ray8, use_ref=True)
    n_or = O.ray_relu(u.normal0, u.ray8)
    assert np.array_equal(bits(n_ref), bits(n_or))
    args = (u.prob[0], u.xy[0], u.angle[0], u.ray8, u.fu, u.cu, u.fv, u.cv)
    a_ref = O.angmf(n_ref, *args, use_ref=True)
    a_or = O.angmf(n_or, *args)
    assert np.array_equal(bits(a_ref), bits(a_or))


@needs_ref
def test_reference_unit_mt_matches_oracle_unit():
    u = O.gen_unit(64, 96, 3, iters=2, seed=11)
    got, nt = O.ref_unit_mt(u, threads=2)
    want = O.refine_unit(u)
    assert nt == 2
    assert np.array_equal(bits(got), bits(want))


def _numpy_angmf_zero_angle(n, prob, ray, ps, dil):
    """Independent formulation for theta = 0 (identity rotation): the update is
    normalise(sum_n w_n RayReLU(n_src, ray_p)) with replicate padding."""
    _, H, W = n.shape
    r = (ps - 1) // 2 * dil
    nn = n.astype(np.float64)
    nn = nn / np.maximum(np.linalg.norm(nn, axis=0, keepdims=True), 1e-12)
    rr = ray.astype(np.float64)
    acc = np.zeros((3, H, W))
    ys, xs = np.mgrid[0:H, 0:W]
    for k in range(ps * ps):
        ky, kx = divmod(k, ps)
        sy = np.clip(ys - r + ky * dil, 0, H - 1)
        sx = np.clip(xs - r + kx * dil, 0, W - 1)
        q = nn[:, sy, sx]
        c = (q * rr).sum(0) / np.maximum(np.linalg.norm(rr, axis=0), 1e-8)
        dc = np.maximum(c - 0.01, 0.0) + 0.01 - c
        m = q + rr * dc
        m = m / np.maximum(np.linalg.norm(m, axis=0, keepdims=True), 1e-12)
        acc += prob[k].astype(np.float64) * m
    return acc / np.maximum(np.linalg.norm(acc, axis=0, keepdims=True), 1e-12)


@pytest.mark.parametrize("ps,dil", [(3, 1), (5, 1), (5, 2), (7, 1), (7, 3)])
def test_generalised_window_indexing(ps, dil):
    u = O.gen_unit(72, 88, 1, ps=ps, dil=dil, iters=1, seed=ps * 10 + dil, upsample=False)
    zero = np.zeros_like(u.angle[0])
    got = O.angmf(u.normal0, u.prob[0], u.xy[0], zero, u.ray8, u.fu, u.cu, u.fv, u.cv,
                  ps=ps, dil=dil)[0]
    want = _numpy_angmf_zero_angle(u.normal0[0], u.prob[0][0], u.ray8, ps, dil)
    assert np.abs(got - want).max() < 1e-6


def _torch_convex_upsample(x, mask, s):
    """Independent fp64 formulation of the header's convex upsample (RAFT style)."""
    xt = torch.from_numpy(x.astype(np.float64))[None]
    mt = torch.from_numpy(mask.astype(np.float64))[None]
    _, C, H, W = xt.shape
    m = torch.softmax(mt.view(1, 1, 9, s, s, H, W), dim=2)
    xp = torch.nn.functional.pad(xt, (1, 1, 1, 1), mode="replicate")
    up = torch.nn.functional.unfold(xp, [3, 3]).view(1, C, 9, 1, 1, H, W)
    o = (m * up).sum(2).permute(0, 1, 4, 2, 5, 3).reshape(1, C, s * H, s * W)
    return o[0].numpy()


@pytest.mark.parametrize("h,w", [(5, 7), (1, 1), (3, 1), (12, 9)])
def test_upsample_restatement_matches_torch_formulation(h, w):
    g = np.random.default_rng(h * 100 + w)
    x = g.standard_normal((3, h, w)).astype(np.float32)
    mask = (3 * g.standard_normal((576, h, w))).astype(np.float32)
    got = O.convex_upsample(x, mask)
    want = _torch_convex_upsample(x, mask, 8)
    assert np.abs(got - want).max() < 2e-6
    l2 = O.l2_normalize(got[None])[0]
    ref = want / np.maximum(np.linalg.norm(want, axis=0, keepdims=True), 1e-12)
    assert np.abs(l2 - ref).max() < 2e-6


def test_build_ray_known_answers():
    # 480x640 image, fx = fy = 512, principal point at the centre (pre "+0.5")
    r = O.build_ray(512.0, 512.0, 320.0, 240.0, 60, 80, 480, 640)
    fu = 512.0 * 80 / 640
    cu = (320.5) * 80 / 640
    fv = 512.0 * 60 / 480
    cv = (240.5) * 60 / 480
    x, y = 13, 41
    v = np.array([((x + 0.5) - cu) / fu, ((y + 0.5) - cv) / fv, 1.0])
    v /= np.linalg.norm(v)
    assert np.abs(r[:, y, x] - v).max() < 1e-7
    assert np.abs(np.linalg.norm(r.astype(np.float64), axis=0) - 1).max() < 1e-6
    rs = O.build_ray_scaled(fu, cu, fv, cv, 60, 80)
    assert np.array_equal(bits(r), bits(rs))


def test_refine_unit_properties():
    u = O.gen_unit(64, 80, 2, iters=2, seed=5)
    out = O.refine_unit(u, full_res_ray_relu=True)
    assert out.shape == (2, 3, 64, 80)
    nrm = np.linalg.norm(out.astype(np.float64), axis=1)
    assert np.abs(nrm - 1).max() < 1e-6
    # full-res RayReLU leaves every normal facing the camera by at least eps
    ray = O.build_ray_scaled(u.fu * 8, u.cu * 8, u.fv * 8, u.cv * 8, 64, 80)
    c = (out.astype(np.float64) * ray[None]).sum(1)
    assert c.min() > 0.01 - 1e-5
    crop = O.refine_unit(u, crop=(3, 5, 40, 50))
    full = O.refine_unit(u)
    assert np.array_equal(crop, full[:, :, 3:43, 5:55])


def test_f16_round_is_ieee_nearest_even():
    a = np.array([1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, 65504.0, 1e-8], np.float32)
    r = O.f16_round(a)
    assert r[0] == 1.0 and r[1] == 1.0 + 2 ** -9 and r[2] == 65504.0
    assert abs(r[3] - 1e-8) < 6e-8


def test_generator_distributions():
    u = O.gen_unit(160, 240, 2, iters=2, seed=9)
    assert abs(u.prob[0].sum(1) - 1).max() < 1e-5
    assert u.angle[1].min() >= 0 and u.angle[1].max() <= 0.3
    c = (u.normal0.astype(np.float64) * u.ray8[None]).sum(1)
    assert c.min() >= 0
    assert abs(np.linalg.norm(u.normal0, axis=1) - 1).max() < 1e-6
    assert u.mask.shape == (2, 576, 20, 30)


def test_head_activation_oracle():
    """sigmoid / pi * sigmoid of src/dsine_refine.cpp:262-267 in the oracle:
    within 2 ulp of torch's fp32 sigmoid, saturating cleanly at the extremes,
    angle never above the float kPi."""
    g = np.random.default_rng(4)
    x = np.concatenate([g.normal(0, 4, 4000), [-1e4, -100.0, -30.0, -0.0, 0.0, 30.0, 100.0,
                                               1e4]]).astype(np.float32)
    p, a = O.head_activation(x, x)
    t = torch.sigmoid(torch.from_numpy(x)).numpy()
    normal = t >= np.finfo(np.float32).tiny  # torch may flush subnormal results
    assert np.all(np.abs(p - t)[normal] <= 2 * np.spacing(t[normal]))
    assert np.all(np.abs(p - t)[~normal] <= 1e-37)
    assert p[-1] == 1.0 and p[-8] == 0.0 and np.all(np.isfinite(a))
    assert a.max() <= O.KPI_F32 and a.min() >= 0.0
    assert a.dtype == np.float32 and np.array_equal(a, (p * O.KPI_F32).astype(np.float32))
