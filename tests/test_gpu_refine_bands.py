"""The whole learned refinement of one large frame as exact-halo row bands on
the GPU (pipeline.refine_frame_banded_full over Refiner instances, one per
visible device, bands dealt in turn) against Refiner.forward on the whole
frame. Every output pixel's arithmetic -- the fp16 tensor-core convolutions'
fixed channel x tap order, the elementwise GRU and head epilogues, the fused
ops -- depends only on its own neighbourhood, and the halo rows carry the
neighbourhood's real data, so the stitched frame is expected to be
bit-identical; the bound allows 1e-6 and the result is printed.
"""
import pytest
import torch

from brovisionml_b200 import pipeline, sharding

pytestmark = pytest.mark.gpu


def _frame(h, w, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    normal = torch.nn.functional.normalize(torch.randn((3, h, w), device="cuda", generator=g),
                                           dim=0)
    feat = torch.relu(torch.randn((64, h, w), device="cuda", generator=g))
    hid = torch.tanh(torch.randn((64, h, w), device="cuda", generator=g))
    return normal, feat, hid


@pytest.mark.parametrize("n_bands", [2, 5])
def test_banded_refiner_equals_whole_frame(n_bands):
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import ITERS, Refiner

    params = random_params("cpu", seed=71)
    devices = list(range(torch.cuda.device_count()))
    refiners = []
    for d in devices:
        r = Refiner()
        r.load_params(params)
        refiners.append(r.to(d))
    h, w = 135, 240  # a 1920x1080 frame's grid
    H, W = 8 * h, 8 * w
    intr = (1500.0, 1500.0, 959.5, 543.25)
    normal, feat, hid = _frame(h, w, seed=72)
    whole = refiners[0].forward(normal[None], feat[None], hid[None], intr, H, W,
                                out_dtype=torch.float32)[0]
    out = torch.empty_like(whole)
    pipeline.refine_frame_banded_full(normal, feat, hid, intr, H, W, out, n_bands=n_bands,
                                      run_band=pipeline.banded_refiner(refiners, torch.float32),
                                      iters=ITERS)
    torch.cuda.synchronize()
    err = (out - whole).abs().max().item()
    bands = pipeline.plan_refine_bands(h, n_bands, ITERS)
    print(f"{len(bands)} bands over {len(devices)} device(s), halo "
          f"{sharding.refine_halo_rows(ITERS)} grid rows: max |banded - whole| = {err:.3e}")
    assert err <= 1e-6, err


@pytest.mark.parametrize("n_bands,crop", [(2, None), (5, (4, 8, 1072, 1904))])
def test_c_banded_forward_equals_whole_frame(n_bands, crop):
    """bvml_refiner_forward_banded -- the C entry a C++ host uses for large
    frames, host buffers in and out, bands over two handles (on two devices
    where there are two, else both on device 0) -- against
    bvml_refiner_forward on the whole frame with the same crop."""
    import ctypes

    import numpy as np

    from brovisionml_b200._capi import check, lib
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import ITERS
    from test_gpu_refiner_capi import _weights

    params = random_params("cpu", seed=73)
    keep, wptrs = _weights(params)
    n_dev = torch.cuda.device_count()
    handles = []
    for k in range(2):
        hnd = ctypes.c_void_p()
        check(lib.bvml_refiner_create(wptrs, k % n_dev, ctypes.byref(hnd)))
        handles.append(hnd)
    try:
        h, w = 135, 240
        H, W = 8 * h, 8 * w
        ct, cl, oh, ow = crop if crop is not None else (0, 0, H, W)
        intr = (1500.0, 1500.0, 959.5, 543.25)
        fi = (ctypes.c_float * 4)(*intr)
        normal, feat, hid = _frame(h, w, seed=74)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        whole = torch.empty((1, 3, oh, ow), device="cuda", dtype=torch.float32)
        check(lib.bvml_refiner_forward(handles[0], normal.data_ptr(), feat.data_ptr(),
                                       hid.data_ptr(), 1, h, w, fi, H, W, ITERS, ct, cl, oh, ow,
                                       0, whole.data_ptr(), stream))
        check(lib.bvml_refiner_status(handles[0], stream))
        host = [np.ascontiguousarray(t.cpu().numpy()) for t in (normal, feat, hid)]
        out = np.zeros((3, oh, ow), np.float32)
        arr = (ctypes.c_void_p * 2)(*[hd.value for hd in handles])
        check(lib.bvml_refiner_forward_banded(
            arr, 2, host[0].ctypes.data, host[1].ctypes.data, host[2].ctypes.data, h, w, fi, H,
            W, ITERS, n_bands, ct, cl, oh, ow, 0, out.ctypes.data))
        err = float(np.abs(out - whole[0].cpu().numpy()).max())
        print(f"C banded ({n_bands} bands, crop {crop}): max |banded - whole| = {err:.3e}")
        assert err <= 1e-6, err
    finally:
        for hnd in handles:
            lib.bvml_refiner_destroy(hnd)
