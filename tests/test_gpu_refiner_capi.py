"""bvml_refiner_*: the whole learned refinement (ConvGRU + heads on the
tensor cores, then the fused ops) behind the C ABI, for C / C++ hosts without
Python. It runs the same sequence and packing as the Python
brovisionml_b200.refiner.Refiner, so its output must equal Refiner.forward's
bit for bit -- through ctypes, and from a C++ program that uses only the C
header (tests/refiner_driver.cpp). The weight table (names and shapes) is
checked against the reference's on CPU.
"""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "brovisionml_b200", "_lib")


def test_weight_table_matches_reference_names_and_shapes():
    from brovisionml_b200._capi import REFINER_WEIGHTS, lib
    from brovisionml_b200.refine_stage import param_shapes

    want = param_shapes()
    names = [lib.bvml_refiner_weight_name(i).decode() for i in range(REFINER_WEIGHTS)]
    assert lib.bvml_refiner_weight_name(REFINER_WEIGHTS) is None
    assert sorted(names) == sorted(want)
    for i, n in enumerate(names):
        s = (ctypes.c_int * 4)()
        assert lib.bvml_refiner_weight_shape(i, s) == 0
        shape = tuple(v for v in s if v)
        assert shape == tuple(want[n]), (n, shape, want[n])


def _inputs(B, h, w, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    normal = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device="cuda",
                                                       generator=g), dim=1)
    feat = torch.relu(torch.randn((B, 64, h, w), device="cuda", generator=g))
    hid = torch.tanh(torch.randn((B, 64, h, w), device="cuda", generator=g))
    return normal, feat, hid


def _weights(params):
    from brovisionml_b200._capi import REFINER_WEIGHTS, lib

    arrs = [np.ascontiguousarray(params[lib.bvml_refiner_weight_name(i).decode()].float()
                                 .cpu().numpy()) for i in range(REFINER_WEIGHTS)]
    return arrs, (ctypes.c_void_p * REFINER_WEIGHTS)(*[a.ctypes.data for a in arrs])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_refiner_capi_equals_python_refiner(dtype):
    from brovisionml_b200._capi import check, lib
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import Refiner

    B, h, w = 2, 44, 64          # the reference's 500 x 348 golden size, padded: 512 x 352
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2 - 3.0, H / 2 + 2.0)
    crop = (2, 6, 348, 500)
    normal, feat, hid = _inputs(B, h, w, seed=31)
    params = random_params("cpu", seed=32)
    r = Refiner()
    r.load_params(params)
    r.to(0)
    want = r.forward(normal, feat, hid, intr, H, W, crop=crop, out_dtype=dtype)

    keep, wptrs = _weights(params)
    handle = ctypes.c_void_p()
    check(lib.bvml_refiner_create(wptrs, 0, ctypes.byref(handle)))
    try:
        out = torch.empty((B, 3, crop[2], crop[3]), device="cuda", dtype=dtype)
        fi = (ctypes.c_float * 4)(*intr)
        code = 1 if dtype == torch.float16 else 0
        stream = torch.cuda.current_stream().cuda_stream
        check(lib.bvml_refiner_forward(handle, normal.data_ptr(), feat.data_ptr(), hid.data_ptr(),
                                       B, h, w, fi, H, W, 5, *crop, code, out.data_ptr(),
                                       ctypes.c_void_p(stream)))
        check(lib.bvml_refiner_status(handle, ctypes.c_void_p(stream)))
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    finally:
        lib.bvml_refiner_destroy(handle)


@pytest.mark.gpu
def test_refiner_from_a_cpp_program(tmp_path):
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import Refiner

    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cuda = os.path.dirname(os.path.dirname(nvcc))
    exe = str(tmp_path / "refiner_driver")
    cmd = [shutil.which("g++") or "g++", "-O1", "-std=c++17", "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(cuda, "include"), os.path.join(ROOT, "tests", "refiner_driver.cpp"),
           "-o", exe, "-L" + LIB_DIR, "-lbvml_dsine", "-Wl,-rpath," + LIB_DIR,
           "-L" + os.path.join(cuda, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(cuda, "lib64")]
    b = subprocess.run(cmd, capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    B, h, w = 1, 24, 40
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2, H / 2)
    normal, feat, hid = _inputs(B, h, w, seed=41)
    params = random_params("cpu", seed=42)
    keep, _ = _weights(params)
    for i, a in enumerate(keep):
        a.astype(np.float32).tofile(tmp_path / f"w{i}.f32")
    for name, t in (("normal", normal), ("feature", feat), ("hidden", hid)):
        t.float().cpu().numpy().tofile(tmp_path / f"{name}.f32")
    np.asarray(intr, np.float32).tofile(tmp_path / "intrins.f32")
    run = subprocess.run([exe, str(tmp_path), str(B), str(h), str(w), str(H), str(W), "1"],
                         capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr
    got = np.fromfile(tmp_path / "out.f32", np.float32).reshape(B, 3, H, W)
    r = Refiner()
    r.load_params(params)
    r.to(0)
    want = r.forward(normal, feat, hid, intr, H, W, out_dtype=torch.float16).float().cpu().numpy()
    assert np.array_equal(got, want)


@pytest.mark.gpu
def test_refiner_allocation_failure_is_reported_and_the_handle_recovers():
    """Failure injection through the allocator, with no GPU fault: a forward
    for 200 000 frames of 90 x 160 asks for a 369 GB first buffer, which
    cudaMalloc refuses. The call must fail with BVML_ECUDA naming the allocation, and the
    next forward on the same handle (a normal shape) must run and equal the
    Python Refiner -- the refused allocation must not resurface in its launch
    checks."""
    from brovisionml_b200._capi import check, lib
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import Refiner

    B, h, w = 1, 24, 40
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2, H / 2)
    normal, feat, hid = _inputs(B, h, w, seed=51)
    params = random_params("cpu", seed=52)
    keep, wptrs = _weights(params)
    handle = ctypes.c_void_p()
    check(lib.bvml_refiner_create(wptrs, 0, ctypes.byref(handle)))
    try:
        fi = (ctypes.c_float * 4)(*intr)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        out = torch.empty((B, 3, H, W), device="cuda", dtype=torch.float16)
        big = 200_000
        rc = lib.bvml_refiner_forward(handle, normal.data_ptr(), feat.data_ptr(), hid.data_ptr(),
                                      big, 90, 160, fi, 720, 1280, 5, 0, 0, 720, 1280, 1,
                                      out.data_ptr(), stream)
        assert rc != 0
        assert b"buffer allocation" in lib.bvml_last_error()
        check(lib.bvml_refiner_forward(handle, normal.data_ptr(), feat.data_ptr(), hid.data_ptr(),
                                       B, h, w, fi, H, W, 5, 0, 0, H, W, 1, out.data_ptr(),
                                       stream))
        check(lib.bvml_refiner_status(handle, stream))
        torch.cuda.synchronize()
        r = Refiner()
        r.load_params(params)
        r.to(0)
        assert torch.equal(out, r.forward(normal, feat, hid, intr, H, W,
                                          out_dtype=torch.float16))
    finally:
        lib.bvml_refiner_destroy(handle)
