"""The reference's BROVISIONML_PROFILE marks (src/profile.cpp): with the
variable set, Refiner.forward and bvml_refiner_forward each print the
refinement's stage and ops intervals to stderr; without it, nothing.
Run in child processes because the switch is read once per process."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import ctypes, numpy as np, torch
from brovisionml_b200._capi import REFINER_WEIGHTS, check, lib
from brovisionml_b200.refine_stage import random_params
from brovisionml_b200.refiner import Refiner
B, h, w = 1, 16, 24
H, W = 8 * h, 8 * w
g = torch.Generator(device="cuda").manual_seed(3)
n = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device="cuda", generator=g), dim=1)
f = torch.relu(torch.randn((B, 64, h, w), device="cuda", generator=g))
hd = torch.tanh(torch.randn((B, 64, h, w), device="cuda", generator=g))
intr = (0.8 * W, 0.8 * W, W / 2, H / 2)
params = random_params("cpu", seed=4)
r = Refiner(); r.load_params(params); r.to(0)
r.forward(n, f, hd, intr, H, W)
arrs = [np.ascontiguousarray(params[lib.bvml_refiner_weight_name(i).decode()].float().numpy())
        for i in range(REFINER_WEIGHTS)]
ptrs = (ctypes.c_void_p * REFINER_WEIGHTS)(*[a.ctypes.data for a in arrs])
hnd = ctypes.c_void_p()
check(lib.bvml_refiner_create(ptrs, 0, ctypes.byref(hnd)))
out = torch.empty((B, 3, H, W), device="cuda", dtype=torch.float16)
fi = (ctypes.c_float * 4)(*intr)
check(lib.bvml_refiner_forward(hnd, n.data_ptr(), f.data_ptr(), hd.data_ptr(), B, h, w, fi, H, W,
                               5, 0, 0, H, W, 1, out.data_ptr(), None))
check(lib.bvml_refiner_status(hnd, None))
lib.bvml_refiner_destroy(hnd)
print("done")
"""


def _run(flag):
    env = dict(os.environ)
    env.pop("BROVISIONML_PROFILE", None)
    if flag is not None:
        env["BROVISIONML_PROFILE"] = flag
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "done" in r.stdout
    return [ln for ln in r.stderr.splitlines() if ln.startswith("[brovisionml-prof]")]


@pytest.mark.gpu
def test_profile_marks_python_and_c():
    lines = _run("1")
    names = [ln.split()[1] for ln in lines]
    # one pair from Refiner.forward, one from bvml_refiner_forward
    assert names == ["refine.stage", "refine.ops", "refine.stage", "refine.ops"], lines
    for ln in lines:
        assert ln.endswith(" ms") and float(ln.split()[2]) >= 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("flag", [None, "0"])
def test_profile_marks_off(flag):
    assert _run(flag) == []


def test_profile_switch_parsing(monkeypatch):
    from brovisionml_b200.refiner import profile_enabled

    for v, want in ((None, False), ("", False), ("0", False), ("1", True), ("yes", True)):
        if v is None:
            monkeypatch.delenv("BROVISIONML_PROFILE", raising=False)
        else:
            monkeypatch.setenv("BROVISIONML_PROFILE", v)
        assert profile_enabled() is want
