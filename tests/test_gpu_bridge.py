"""The reference-facing C++ bridge (brovisionml_b200/csrc/dsine_ops_b200.cpp,
libbvml_dsine_bridge.so) driven through brotensor-shaped tensors by a small
C++ program (tests/bridge_driver.cpp), as brovisionml's own dispatch would
call it, against the oracle. The build check runs on CPU; the runs need a GPU.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "brovisionml_b200", "_lib")


def build_driver(dest_dir):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cuda = os.path.dirname(os.path.dirname(nvcc))
    exe = os.path.join(dest_dir, "bridge_driver")
    cmd = [shutil.which("g++") or "g++", "-O1", "-std=c++20", "-DBVML_SHIM_CUDA",
           "-I" + os.path.join(ROOT, "brovisionml_b200", "csrc", "brotensor_shim"),
           "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(cuda, "include"),
           os.path.join(ROOT, "tests", "bridge_driver.cpp"), "-o", exe,
           "-L" + LIB_DIR, "-lbvml_dsine_bridge", "-lbvml_dsine", "-Wl,-rpath," + LIB_DIR,
           "-L" + os.path.join(cuda, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(cuda, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_bridge_driver_builds(tmp_path):
    assert os.access(build_driver(str(tmp_path)), os.X_OK)


def run_driver(tmp_path, op, u, arrays, iters=1):
    exe = build_driver(str(tmp_path))
    np.asarray([u.fu, u.cu, u.fv, u.cv], np.float64).tofile(tmp_path / "intr.f64")
    for name, a in arrays.items():
        np.ascontiguousarray(a, np.float32).tofile(tmp_path / f"{name}.f32")
    r = subprocess.run([exe, op, str(tmp_path), str(u.h), str(u.w), str(iters)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return np.fromfile(tmp_path / "out.f32", np.float32)


def check(name, got, want, tol=O.TOL_F32):
    m = O.compare(got.reshape(want.shape), want)
    print(f"bridge {name}: max_abs {m['max_abs']:.3e} ang_max {m['ang_max_deg']:.2e} deg")
    assert m["nonfinite"] == 0 and m["max_abs"] <= tol, m


@pytest.mark.gpu
def test_bridge_ray_relu_and_angmf(tmp_path):
    u = O.gen_unit(480, 640, 1, iters=1, seed=11, upsample=False, face_camera=False)
    base = {"normal": u.normal0[0], "ray": u.ray8}
    check("ray_relu", run_driver(tmp_path, "ray_relu", u, base),
          O.ray_relu(u.normal0, u.ray8)[0])
    n0 = O.ray_relu(u.normal0, u.ray8)
    arrs = {"normal": n0[0], "ray": u.ray8, "prob0": u.prob[0][0], "xy0": u.xy[0][0],
            "angle0": u.angle[0][0]}
    want = O.angmf(n0, u.prob[0], u.xy[0], u.angle[0], u.ray8, u.fu, u.cu, u.fv, u.cv,
                   use_ref=O.ref_available())[0]
    check("angmf", run_driver(tmp_path, "angmf", u, arrs), want)


@pytest.mark.gpu
def test_bridge_angmf_logits(tmp_path):
    u = O.gen_unit(480, 640, 1, iters=1, seed=12, upsample=False)
    g = np.random.default_rng(12)
    pl = g.normal(0, 2.5, u.prob[0].shape).astype(np.float32)
    al = g.normal(-2.5, 1.5, u.angle[0].shape).astype(np.float32)
    prob, ang = O.head_activation(pl, al)
    n0 = O.ray_relu(u.normal0, u.ray8)
    want = O.angmf(n0, prob, u.xy[0], ang, u.ray8, u.fu, u.cu, u.fv, u.cv)[0]
    arrs = {"normal": n0[0], "ray": u.ray8, "prob0": pl[0], "xy0": u.xy[0][0], "angle0": al[0]}
    check("angmf_logits", run_driver(tmp_path, "angmf_logits", u, arrs), want)


@pytest.mark.gpu
def test_bridge_refine_ops(tmp_path):
    u = O.gen_unit(480, 640, 1, iters=3, seed=13)
    arrs = {"normal": u.normal0[0], "ray": u.ray8, "mask": u.mask[0]}
    for i in range(3):
        arrs[f"prob{i}"], arrs[f"xy{i}"], arrs[f"angle{i}"] = u.prob[i][0], u.xy[i][0], u.angle[i][0]
    check("refine_ops", run_driver(tmp_path, "refine", u, arrs, iters=3), O.refine_unit(u)[0])
