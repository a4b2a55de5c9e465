"""The whole learned refinement (ConvGRU + heads + ops) of one frame as exact
halo row bands (pipeline.refine_frame_banded_full, sharding.refine_halo_rows),
checked on CPU: the stage as its plain fp32 torch restatement
(refine_stage.reference_stage, the reference's formulas) and the ops as the
CPU oracle. The stage runs in float64 here, so that its result does not
depend on the convolutions' summation order (which changes with the band's
size); the ops take its outputs rounded to fp32. Bands with the halo give the
whole-frame result; one row less of halo does not (the formula is tight).
"""
import numpy as np
import pytest
import torch

from brovisionml_b200 import pipeline, sharding
from oracle import oracle as O


def _runner(params, iters):
    from brovisionml_b200.refine_stage import reference_stage
    from brovisionml_b200.refiner import build_uv, grid_intrinsics

    def run_band(normal, feature, hidden, intr, origH, origW, crop):
        _, _, rows, w = normal.shape
        uv = build_uv(intr, rows, w, origH, origW, "cpu")
        outs = reference_stage(params, hidden, feature, uv, iters, emulate_f16=False,
                               dtype=torch.float64)
        fu, cu, fv, cv = grid_intrinsics(intr, rows, w, origH, origW)
        f32 = lambda t: np.ascontiguousarray(t.float().numpy())  # noqa: E731
        act = [O.head_activation(f32(o.prob), f32(o.angle)) for o in outs]
        u = O.UnitInputs(B=1, H=8 * rows, W=8 * w, h=rows, w=w, ps=5, dil=1, iters=iters,
                         fu=fu, cu=cu, fv=fv, cv=cv, fx=intr[0], fy=intr[1], cx=intr[2],
                         cy=intr[3], normal0=np.ascontiguousarray(normal.numpy()),
                         ray8=O.build_ray(intr[0], intr[1], intr[2], intr[3], rows, w, origH,
                                          origW),
                         prob=[a[0] for a in act], xy=[f32(o.xy) for o in outs],
                         angle=[a[1] for a in act], mask=f32(outs[-1].up_mask))
        return torch.from_numpy(O.refine_unit(u, crop=crop))
    return run_band


def _frame(h, w, seed):
    g = torch.Generator().manual_seed(seed)
    normal = torch.nn.functional.normalize(torch.randn((3, h, w), generator=g), dim=0)
    feat = torch.relu(torch.randn((64, h, w), generator=g))
    hid = torch.tanh(torch.randn((64, h, w), generator=g))
    return normal, feat, hid


def test_refine_halo_formula():
    # 5 iterations of 5x5: the hidden state reaches 4 rows per iteration
    assert sharding.refine_halo_rows(5, 5, 1) == 22
    assert sharding.refine_halo_rows(2, 5, 1) == 10
    assert sharding.refine_halo_rows(1, 5, 1) == 6
    # a window wider than the GRU's 4 rows per iteration: the normals decide
    assert sharding.refine_halo_rows(2, 7, 4) == 2 * 12 + 1
    # never narrower than the ops' own halo
    for it in range(1, 7):
        for ps, dil in ((3, 1), (5, 1), (5, 2), (7, 1), (7, 2)):
            assert sharding.refine_halo_rows(it, ps, dil) >= sharding.halo_rows(it, ps, dil)


@pytest.mark.parametrize("iters", [1, 2, 3])
def test_banded_refinement_equals_whole_frame(iters, monkeypatch):
    from brovisionml_b200.refine_stage import random_params

    params = random_params("cpu", seed=50 + iters)
    h, w = 44, 12
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2 - 1.0, H / 2 + 3.0)
    normal, feat, hid = _frame(h, w, seed=7)
    run = _runner(params, iters)
    whole = run(normal[None], feat[None], hid[None], intr, H, W, (0, 0, H, W))[0]
    out = torch.empty_like(whole)
    pipeline.refine_frame_banded_full(normal, feat, hid, intr, H, W, out, n_bands=3,
                                      run_band=run, iters=iters)
    err = (out - whole).abs().max().item()
    assert err <= 1e-6, err  # observed: exactly 0
    # one row less of halo changes the result (by little after several
    # iterations: the last row of the cone reaches the output through the
    # GRU's gates)
    full = sharding.refine_halo_rows
    monkeypatch.setattr(sharding, "refine_halo_rows", lambda *a, **k: full(*a, **k) - 1)
    short = torch.empty_like(whole)
    pipeline.refine_frame_banded_full(normal, feat, hid, intr, H, W, short, n_bands=3,
                                      run_band=run, iters=iters)
    assert (short - whole).abs().max().item() > 0


def test_c_halo_rows_match_the_python_formula():
    """bvml_refine_halo_rows (the C entry a C++ host plans its bands with) is
    the same formula, and rejects what the kernels do not take."""
    from brovisionml_b200._capi import lib

    for it in range(0, 9):
        for ps in (3, 5, 7):
            for dil in (1, 2, 3, 4):
                assert lib.bvml_refine_halo_rows(it, ps, dil) == \
                    sharding.refine_halo_rows(it, ps, dil), (it, ps, dil)
    for bad in ((-1, 5, 1), (65, 5, 1), (5, 4, 1), (5, 5, 0), (5, 5, 5)):
        assert lib.bvml_refine_halo_rows(*bad) == 1   # BVML_EINVAL
        assert b"refine_halo_rows" in lib.bvml_last_error()


def test_c_banded_forward_rejects_bad_arguments():
    """Argument checks of bvml_refiner_forward_banded run before any CUDA call."""
    import ctypes

    from brovisionml_b200._capi import lib

    handles = (ctypes.c_void_p * 1)(ctypes.c_void_p(1))   # never dereferenced here
    fi = (ctypes.c_float * 4)(100.0, 100.0, 50.0, 40.0)
    buf = (ctypes.c_float * 16)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    ok = dict(n=1, h=10, w=12, H=80, W=96, it=5, nb=2, ct=0, cl=0, oh=80, ow=96, dt=0)

    def call(**kw):
        a = dict(ok, **kw)
        return lib.bvml_refiner_forward_banded(handles, a["n"], p, p, p, a["h"], a["w"], fi,
                                               a["H"], a["W"], a["it"], a["nb"], a["ct"],
                                               a["cl"], a["oh"], a["ow"], a["dt"], p)
    assert call(n=0) == 1
    assert call(h=0) == 1
    assert call(it=0) == 1
    assert call(nb=0) == 1
    assert call(dt=7) == 1
    assert call(oh=81) == 1 and b"crop window" in lib.bvml_last_error()
    assert call(ct=1, oh=80) == 1
    null = (ctypes.c_void_p * 1)(None)
    assert lib.bvml_refiner_forward_banded(null, 1, p, p, p, 10, 12, fi, 80, 96, 5, 2, 0, 0, 80,
                                           96, 0, p) == 1
    assert b"null handle" in lib.bvml_last_error()
