"""GPU test of bvml_refine_noalloc, the allocation-free variant of bvml_refine.

Callers that may not allocate device memory (a plugin inside another
application's inference or render loop that owns the GPU memory budget, or a
loop that cannot take cudaMalloc's implicit synchronisation) get the fused
refine with its scratch in a fixed array built into the library. This test
calls it through the C ABI and checks it against bvml_refine with a caller
workspace, on two calls in a row with different inputs (the shared scratch
keeps the previous call's contents, which must not leak into the next
result). Both entry points run the same kernels on the same inputs, so the
results must be bit-identical, not merely within the parity tolerance. It
also runs the largest batch the built-in scratch accepts and checks that one
frame more is refused.

The file name makes pytest collect it last; it also passes alone in a fresh
process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _call(lib, fn, u, dt, out, extra):
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0", dt)  # noqa: E731
    n0, mask = d(u.normal0), d(u.mask)
    prob, xy, ang = [d(a) for a in u.prob], [d(a) for a in u.xy], [d(a) for a in u.angle]
    ray = torch.from_numpy(u.ray8).to("cuda:0")
    code = 1 if dt == torch.float16 else 0
    args = [n0.data_ptr(), ray.data_ptr(), _ptrs(prob), _ptrs(xy), _ptrs(ang), u.iters,
            mask.data_ptr(), u.B, u.h, u.w, u.ps, u.dil, u.fu, u.cu, u.fv, u.cv, 1, 0, 0,
            8 * u.h, 8 * u.w, code] + extra + [out.data_ptr(), None]
    rc = fn(*args)
    torch.cuda.synchronize()
    return rc


@pytest.mark.parametrize("f16", [False, True])
def test_refine_noalloc_matches_refine_twice(f16):
    from brovisionml_b200 import _capi

    lib = _capi.lib
    dt = torch.float16 if f16 else torch.float32
    tol = O.TOL_F16 if f16 else O.TOL_F32
    for call, seed in enumerate((41, 42)):
        u = O.gen_unit(480, 640, 3, iters=5, seed=seed)
        if f16:
            u = O.to_f16_storage(u)
        want = torch.empty((u.B, 3, 8 * u.h, 8 * u.w), device="cuda:0", dtype=dt)
        need = lib.bvml_refine_workspace_bytes(u.B, u.h, u.w)
        ws = torch.empty(need, device="cuda:0", dtype=torch.uint8)
        assert _call(lib, lib.bvml_refine, u, dt, want, [ws.data_ptr(), need]) == 0
        got = torch.full_like(want, float("nan"))
        rc = _call(lib, lib.bvml_refine_noalloc, u, dt, got, [])
        assert rc == 0, lib.bvml_last_error().decode()
        err = (got.float() - want.float()).abs().max().item()
        assert err <= tol, (call, err)
        # same kernels, same inputs: a partial scratch leak would show here
        assert torch.equal(got, want), (call, err)
        assert torch.isfinite(got.float()).all()


def test_refine_noalloc_largest_accepted_batch():
    """96 frames of a 90x160 grid: the scratch regions reach the end of the
    built-in array. Device-generated inputs (the CPU oracle is not needed:
    the check is bit-equality with bvml_refine over a caller workspace)."""
    from brovisionml_b200 import _capi

    lib = _capi.lib
    B, h, w, iters, P = 96, 90, 160, 2, 25
    need = lib.bvml_refine_workspace_bytes(B, h, w)
    assert need <= _capi.REFINE_NOALLOC_MAX_BYTES
    assert lib.bvml_refine_workspace_bytes(B + 1, h, w) > _capi.REFINE_NOALLOC_MAX_BYTES
    dev, dt = "cuda:0", torch.float16
    g = torch.Generator(device=dev).manual_seed(5)
    n0 = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device=dev, generator=g),
                                       dim=1)
    n0[:, 2] = n0[:, 2].abs()  # roughly camera-facing
    n0 = n0.to(dt)
    prob = [torch.softmax(torch.randn((B, P, h, w), device=dev, generator=g), 1).to(dt)
            for _ in range(iters)]
    xy = [torch.randn((B, 2 * P, h, w), device=dev, generator=g).to(dt) for _ in range(iters)]
    ang = [(0.3 * torch.rand((B, P, h, w), device=dev, generator=g)).to(dt)
           for _ in range(iters)]
    mask = torch.randn((B, 576, h, w), device=dev, generator=g).to(dt)
    fu, cu, fv, cv = 0.8 * w, w / 2 + 0.0625, 0.8 * w, h / 2 + 0.0625
    outs = []
    for fn, extra in ((lib.bvml_refine, "ws"), (lib.bvml_refine_noalloc, None)):
        out = torch.full((B, 3, 8 * h, 8 * w), float("nan"), device=dev, dtype=dt)
        args = [n0.data_ptr(), None, _ptrs(prob), _ptrs(xy), _ptrs(ang), iters,
                mask.data_ptr(), B, h, w, 5, 1, fu, cu, fv, cv, 0, 0, 0, 8 * h, 8 * w, 1]
        if extra:
            ws = torch.empty(need, device=dev, dtype=torch.uint8)
            args += [ws.data_ptr(), need]
        rc = fn(*(args + [out.data_ptr(), None]))
        torch.cuda.synchronize()
        assert rc == 0, lib.bvml_last_error().decode()
        outs.append(out)
    assert torch.isfinite(outs[1].float()).all()
    assert torch.equal(outs[0], outs[1])


def test_refine_noalloc_rejects_oversize():
    from brovisionml_b200 import _capi

    lib = _capi.lib
    B, h, w = 97, 90, 160  # one frame more than the 32 MiB scratch holds
    assert lib.bvml_refine_workspace_bytes(B, h, w) > _capi.REFINE_NOALLOC_MAX_BYTES
    assert lib.bvml_refine_workspace_bytes(96, h, w) <= _capi.REFINE_NOALLOC_MAX_BYTES
    fake = ctypes.c_void_p(0x1000)
    arr = (ctypes.c_void_p * 1)(0x1000)
    rc = lib.bvml_refine_noalloc(fake, None, arr, arr, arr, 1, fake, B, h, w, 5, 1, 1.0, 0.0,
                                 1.0, 0.0, 0, 0, 0, 8 * h, 8 * w, 0, fake, None)
    assert rc == 1
    msg = lib.bvml_last_error().decode()
    assert "refine_noalloc" in msg and "scratch" in msg
