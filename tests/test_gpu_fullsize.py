"""GPU tests at the benchmark configurations' full sizes, where the CPU
oracle would take too long: size-independent properties instead.

* every output is finite and unit length (fp32: 1e-5, fp16 storage: 2e-3);
* the frame dimension is independent: a batch computed at once equals the
  same frames computed in smaller batches, bit for bit;
* row bands (config 3's multi-GPU split) stitched together equal the whole
  frame (exact halo, see brovisionml_b200.sharding);
* full-res RayReLU leaves every output facing the camera.

Config 3 (one 4096^2 frame, 7x7, 5 iterations, fp32) is also compared with
the CPU oracle at its full size: the oracle runs as exact halo row bands
(proven equal to its whole-frame result in tests/test_sharding.py) over the
host's cores, so the whole frame is checked within the fp32 tolerance.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

import bench
from brovisionml_b200.sharding import Band, band_intrinsics, halo_rows, plan_bands
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def run(inp, cfg, **kw):
    import brovisionml_b200 as bv

    return bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"],
                     inp["fu"], inp["cu"], inp["fv"], inp["cv"], ray8=inp["ray8"], ps=cfg["ps"],
                     dil=cfg["dil"], full_res_ray_relu=cfg["rr"], **kw)


def check_unit(out, tol):
    o = out.float()
    assert torch.isfinite(o).all()
    err = (o.norm(dim=1) - 1).abs().max().item()
    assert err <= tol, err


@pytest.mark.parametrize("name", ["cfg2", "cfg2h", "cfg4"])
def test_fullsize_unit_norm_and_batch_split(name):
    cfg = dict(bench.CONFIGS[name])
    dev = torch.device("cuda", 0)
    inp = bench.make_device_inputs(cfg, cfg["B"], 5, dev, torch)
    out = run(inp, cfg)
    torch.cuda.synchronize()
    check_unit(out, 2e-3 if cfg["f16"] else 1e-5)
    # the same frames in two halves
    B = cfg["B"]
    half = B // 2
    parts = []
    for sl in (slice(0, half), slice(half, B)):
        sub = dict(inp, normal0=inp["normal0"][sl].contiguous(),
                   prob=[t[sl].contiguous() for t in inp["prob"]],
                   xy=[t[sl].contiguous() for t in inp["xy"]],
                   angle=[t[sl].contiguous() for t in inp["angle"]],
                   mask=inp["mask"][sl].contiguous())
        parts.append(run(sub, cfg))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts), out)


def test_fullsize_cfg3_bands_match_whole_frame():
    """Config 3: one 4096^2 frame (grid 512^2, 7x7, 5 iterations) computed whole
    and as 8 exact halo bands (what 8 GPUs would each compute)."""
    cfg = dict(bench.CONFIGS["cfg3"])
    dev = torch.device("cuda", 0)
    inp = bench.make_device_inputs(cfg, 1, 9, dev, torch)
    whole = run(inp, cfg)
    check_unit(whole, 1e-5)
    h = inp["h"]
    bands = plan_bands(h, 8, halo_rows(cfg["iters"], cfg["ps"], cfg["dil"]))
    rows = []
    for b in bands:
        sl = slice(b.comp0, b.comp1)
        sub = dict(inp, normal0=inp["normal0"][:, :, sl].contiguous(),
                   prob=[t[:, :, sl].contiguous() for t in inp["prob"]],
                   xy=[t[:, :, sl].contiguous() for t in inp["xy"]],
                   angle=[t[:, :, sl].contiguous() for t in inp["angle"]],
                   mask=inp["mask"][:, :, sl].contiguous(),
                   ray8=inp["ray8"][:, sl].contiguous(), cv=band_intrinsics(inp["cv"], b))
        out = run(sub, cfg, crop=(8 * b.crop_top, 0, 8 * (b.own1 - b.own0), 8 * inp["w"]))
        rows.append(out)
    stitched = torch.cat(rows, dim=2)
    torch.cuda.synchronize()
    assert stitched.shape == whole.shape
    err = (stitched - whole).abs().max().item()
    assert err <= 1e-5, err


def test_fullsize_cfg1_full_res_ray_relu_faces_camera():
    cfg = dict(bench.CONFIGS["cfg1"])
    dev = torch.device("cuda", 0)
    inp = bench.make_device_inputs(cfg, 1, 3, dev, torch)
    out = run(inp, cfg)[0].double()
    H, W = cfg["H"], cfg["W"]
    fu, cu, fv, cv = 8 * inp["fu"], 8 * inp["cu"], 8 * inp["fv"], 8 * inp["cv"]
    ys, xs = torch.meshgrid(torch.arange(H, device=dev, dtype=torch.float64),
                            torch.arange(W, device=dev, dtype=torch.float64), indexing="ij")
    r = torch.stack([((xs + 0.5) - cu) / fu, ((ys + 0.5) - cv) / fv, torch.ones_like(xs)])
    r = r / r.norm(dim=0, keepdim=True)
    c = (out * r).sum(0)
    assert c.min().item() >= 0.01 - 1e-5
    check_unit(out[None], 1e-5)


@pytest.mark.parametrize("name,n_bands,given_ray", [("cfg2", 5, False), ("cfg1", 3, True)])
def test_large_frame_driver_matches_whole_frame(name, n_bands, given_ray):
    """brovisionml_b200.pipeline.refine_frame_banded (host inputs of one
    frame, exact-halo row bands, crop-stitch into a host buffer) equals the
    whole-frame refine of the same frame."""
    import brovisionml_b200 as bv
    from brovisionml_b200.pipeline import HostFrame, refine_frame_banded

    cfg = dict(bench.CONFIGS[name])
    cfg["B"] = 1
    dev = torch.device("cuda", 0)
    inp = bench.make_device_inputs(cfg, 1, 17, dev, torch)
    ray = inp["ray8"] if given_ray else None
    want = bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"],
                     inp["fu"], inp["cu"], inp["fv"], inp["cv"], ray8=ray, ps=cfg["ps"],
                     dil=cfg["dil"], full_res_ray_relu=cfg["rr"])[0].float().cpu()
    host = lambda t: t[0].cpu()  # noqa: E731
    frame = HostFrame(host(inp["normal0"]), [host(t) for t in inp["prob"]],
                      [host(t) for t in inp["xy"]], [host(t) for t in inp["angle"]],
                      host(inp["mask"]), ray.cpu() if given_ray else None)
    out = torch.empty_like(want, dtype=inp["dt"])
    refine_frame_banded(frame, out, inp["fu"], inp["cu"], inp["fv"], inp["cv"],
                        n_bands=n_bands, ps=cfg["ps"], dil=cfg["dil"],
                        full_res_ray_relu=cfg["rr"])
    err = (out.float() - want).abs().max().item()
    assert err <= (2e-3 if cfg["f16"] else 1e-5), err


def _oracle_band(u: O.UnitInputs, b: Band) -> np.ndarray:
    """The oracle's unit on one exact-halo band of frame u, owned rows only."""
    sl = slice(b.comp0, b.comp1)
    ub = O.UnitInputs(**{**u.__dict__, "h": b.rows, "H": 8 * b.rows,
                         "cv": band_intrinsics(u.cv, b),
                         "normal0": np.ascontiguousarray(u.normal0[:, :, sl]),
                         "ray8": np.ascontiguousarray(u.ray8[:, sl]),
                         "prob": [np.ascontiguousarray(a[:, :, sl]) for a in u.prob],
                         "xy": [np.ascontiguousarray(a[:, :, sl]) for a in u.xy],
                         "angle": [np.ascontiguousarray(a[:, :, sl]) for a in u.angle],
                         "mask": np.ascontiguousarray(u.mask[:, :, sl])})
    return O.refine_unit(ub, crop=(8 * b.crop_top, 0, 8 * (b.own1 - b.own0), 8 * u.w))


def test_fullsize_cfg3_matches_oracle():
    """Config 3 at full size against the oracle: the whole 4096^2 frame
    refined on the GPU in one call, the fp64 C restatement run as exact halo
    bands on every host core (its ctypes calls release the GIL)."""
    import brovisionml_b200 as bv

    cfg = bench.CONFIGS["cfg3"]
    u = O.gen_unit(cfg["H"], cfg["W"], 1, ps=cfg["ps"], dil=cfg["dil"], iters=cfg["iters"],
                   seed=303)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    got = bv.refine(t(u.normal0), [t(a) for a in u.prob], [t(a) for a in u.xy],
                    [t(a) for a in u.angle], t(u.mask), u.fu, u.cu, u.fv, u.cv,
                    ray8=t(u.ray8), ps=cfg["ps"], dil=cfg["dil"])
    got = got.cpu().numpy()
    n = max(1, min(64, os.cpu_count() or 1))
    bands = plan_bands(u.h, n, halo_rows(cfg["iters"], cfg["ps"], cfg["dil"]))
    with ThreadPoolExecutor(n) as ex:
        parts = list(ex.map(lambda b: _oracle_band(u, b), bands))
    want = np.concatenate(parts, axis=2)
    assert want.shape == got.shape == (1, 3, cfg["H"], cfg["W"])
    m = O.compare(got, want)
    print(f"cfg3 full frame vs oracle ({n} bands): max-abs {m['max_abs']:.2e} mean-abs "
          f"{m['mean_abs']:.2e}; angular error mean {m['ang_mean_deg']:.2e} p99 "
          f"{m['ang_p99_deg']:.2e} max {m['ang_max_deg']:.2e} deg")
    assert m["nonfinite"] == 0
    assert m["max_abs"] <= O.TOL_F32, m


def test_persistent_and_per_iteration_paths_agree():
    """bvml_refine runs all AngMF iterations in one persistent launch when an
    iteration is at most a few waves of tiles (32 frames of 720p) and one
    launch per iteration otherwise (256 frames). The two paths compute the
    same arithmetic, so the first 32 frames of a 256-frame batch equal the
    same 32 frames refined alone, bit for bit; the persistent launch's
    dependency waits all completed (bvml_refine_status)."""
    import ctypes

    import brovisionml_b200 as bv

    cfg = dict(bench.CONFIGS["cfg4"])
    dev = torch.device("cuda", 0)
    inp = bench.make_device_inputs(cfg, 256, 23, dev, torch)
    whole = run(inp, cfg)
    sub = bench.frames_slice(inp, 0, 32)
    ws = torch.empty(bv.refine_workspace_bytes(32, inp["h"], inp["w"]), device=dev,
                     dtype=torch.uint8)
    part = run(sub, cfg, workspace=ws)
    torch.cuda.synchronize()
    assert bv.lib.bvml_refine_status(ctypes.c_void_p(ws.data_ptr()), None) == 0
    assert torch.equal(whole[:32], part)
