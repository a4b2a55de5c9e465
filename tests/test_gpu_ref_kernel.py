"""The reference's own CUDA kernels on the B200, beside this repository's.

oracle/_ref/libbvml_refgpu.so is the reference's src/dsine_ops.cu compiled
unchanged for sm_100a (test infrastructure, built by oracle/Makefile). This
file checks its results against the CPU oracle and the repository's kernels,
and times the reference's GPU path -- one frame at a time, ray_relu then
5 x angmf_propagate with the output re-allocated per call, on the default
stream, as Refiner::forward drives it (src/dsine_refine.cpp:241-272) --
beside the repository's fused unit on the same frames: config 4's frame
size (720p, grid 90 x 160), fp32 storage (the reference's only precision),
5x5 window, 5 iterations. The repository's time covers more work (the
convex upsample with L2 as well). Numbers are printed; with BVML_REFGPU_JSON
set they are also written to that file.
"""
import ctypes
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle",
                   "_ref", "libbvml_refgpu.so")


def _lib():
    if not os.path.exists(LIB):
        pytest.skip("reference GPU library not built (needs the reference tree at build time)")
    lib = ctypes.CDLL(LIB)
    lib.bvml_refgpu_unit.restype = ctypes.c_int
    lib.bvml_refgpu_unit.argtypes = ([ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 +
                                     [ctypes.c_double] * 4 + [ctypes.c_void_p])
    return lib


def _arr(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _ref_gpu(lib, u, dev):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    n0, ray = t(u.normal0), t(u.ray8)
    prob, xy, ang = [t(a) for a in u.prob], [t(a) for a in u.xy], [t(a) for a in u.angle]
    out = torch.empty((u.B, 3, u.h, u.w), device=dev)

    def run():
        rc = lib.bvml_refgpu_unit(n0.data_ptr(), ray.data_ptr(), _arr(prob), _arr(xy), _arr(ang),
                                  u.iters, u.B, u.h, u.w, u.fu, u.cu, u.fv, u.cv, out.data_ptr())
        assert rc == 0
    return run, out, (n0, ray, prob, xy, ang)


def _ours_grid(u, dev, tensors):
    """The repository's ray_relu + iters x angmf_propagate (grid normals)."""
    import brovisionml_b200 as bv

    n0, ray, prob, xy, ang = tensors
    n = n0.clone()
    bv.ray_relu(n, ray)
    for i in range(u.iters):
        n = bv.angmf_propagate(n, prob[i], xy[i], ang[i], ray, u.fu, u.cu, u.fv, u.cv)
    return n


def test_reference_gpu_kernels_match_oracle_and_ours():
    lib = _lib()
    dev = torch.device("cuda", 0)
    u = O.gen_unit(480, 640, 2, iters=3, seed=61)
    run, out, ts = _ref_gpu(lib, u, dev)
    run()
    torch.cuda.synchronize()
    # the CPU oracle on the grid: ray_relu, then the iterations
    want = []
    for b in range(u.B):
        n = O.ray_relu(u.normal0[b], u.ray8)
        for i in range(u.iters):
            n = O.angmf(n, u.prob[i][b], u.xy[i][b], u.angle[i][b], u.ray8, u.fu, u.cu, u.fv,
                        u.cv)
        want.append(n)
    want = np.stack(want)
    m_ref = O.compare(out.cpu().numpy(), want)
    ours = _ours_grid(u, dev, ts)
    torch.cuda.synchronize()
    m_ours = O.compare(ours.cpu().numpy(), want)
    print(f"reference CUDA kernels vs oracle: max-abs {m_ref['max_abs']:.2e}; "
          f"repository kernels vs oracle: max-abs {m_ours['max_abs']:.2e}")
    assert m_ref["max_abs"] <= O.TOL_F32 and m_ours["max_abs"] <= O.TOL_F32


def test_time_reference_gpu_kernels():
    import brovisionml_b200 as bv

    lib = _lib()
    dev = torch.device("cuda", 0)
    frames = 16
    u = O.gen_unit(720, 1280, frames, iters=5, seed=62)
    run, out, ts = _ref_gpu(lib, u, dev)
    n0, ray, prob, xy, ang = ts
    mask = torch.from_numpy(u.mask).to(dev)
    ws = torch.empty(bv.refine_workspace_bytes(frames, u.h, u.w), device=dev, dtype=torch.uint8)
    res = torch.empty((frames, 3, u.H, u.W), device=dev)

    def ours():
        bv.refine(n0, prob, xy, ang, mask, u.fu, u.cu, u.fv, u.cv, ray8=ray, out=res,
                  workspace=ws)

    def ours_grid():
        _ours_grid(u, dev, ts)

    def timed(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(torch.cuda.default_stream(dev))
        for _ in range(reps):
            fn()
        e1.record(torch.cuda.default_stream(dev))
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    with torch.cuda.stream(torch.cuda.default_stream(dev)):
        t_ref = timed(run, 3)
        t_ours = timed(ours, 10)
        t_grid = timed(ours_grid, 10)
    px = frames * u.H * u.W
    rec = {
        "workload": f"{frames} frames of 1280x720 (grid 160x90), fp32 storage, 5x5, d=1, "
                    f"5 iterations",
        "reference_cuda_ms": round(t_ref, 4),
        "reference_cuda_mpx_s": round(px / (t_ref * 1e-3) / 1e6, 1),
        "ours_unit_ms": round(t_ours, 4),
        "ours_unit_mpx_s": round(px / (t_ours * 1e-3) / 1e6, 1),
        "ours_ops_only_ms": round(t_grid, 4),
        "speedup_unit": round(t_ref / t_ours, 1),
        "speedup_same_ops": round(t_ref / t_grid, 1),
        "what": "reference: ray_relu + 5 x angmf_propagate per frame (src/dsine_ops.cu, "
                "one thread per pixel, fp64); ours (unit): bvml_refine incl. the convex "
                "upsample + L2; ours (same ops): ray_relu + 5 x bvml_angmf_propagate",
    }
    print(json.dumps(rec))
    path = os.environ.get("BVML_REFGPU_JSON")
    if path:
        with open(path, "w") as f:
            json.dump(rec, f, indent=1)
    assert t_ours > 0 and t_ref > 0
