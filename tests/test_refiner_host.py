"""Host side of brovisionml_b200.refiner (the reference's Refiner,
include/brovisionml/dsine_refine.h): grid intrinsics and uv exactly as the
reference computes them (src/dsine_decoder.cpp:242-275,
src/dsine_refine.cpp:230-237), and the load / to / forward order errors."""
import numpy as np
import pytest
import torch


def test_uv_matches_reference_formula():
    from brovisionml_b200.refiner import build_uv, grid_intrinsics

    intr = (517.3, 516.9, 318.6, 255.3)
    h8, w8, H, W = 60, 80, 480, 640
    uv = build_uv(intr, h8, w8, H, W, "cpu").numpy()
    fx, fy, cx, cy = (float(np.float32(v)) for v in intr)
    sw, sh = w8 / W, h8 / H
    fu, cu, fv, cv = fx * sw, (cx + 0.5) * sw, fy * sh, (cy + 0.5) * sh
    want_u = np.array([((x + 0.5) - cu) / fu for x in range(w8)], dtype=np.float64)
    want_v = np.array([((y + 0.5) - cv) / fv for y in range(h8)], dtype=np.float64)
    assert np.array_equal(uv[0], np.broadcast_to(want_u.astype(np.float32), (h8, w8)))
    assert np.array_equal(uv[1], np.broadcast_to(want_v.astype(np.float32)[:, None], (h8, w8)))
    assert grid_intrinsics(intr, h8, w8, H, W) == pytest.approx((fu, cu, fv, cv), rel=1e-6)


def test_refiner_order_errors():
    from brovisionml_b200.refiner import Refiner
    from brovisionml_b200.refine_stage import random_params

    r = Refiner()
    z = torch.zeros(1, 3, 8, 8)
    f = torch.zeros(1, 64, 8, 8)
    with pytest.raises(RuntimeError, match="before load"):
        r.forward(z, f, f, (1, 1, 1, 1), 64, 64)
    r.load_params(random_params("cpu"))
    with pytest.raises(RuntimeError, match="before to"):
        r.forward(z, f, f, (1, 1, 1, 1), 64, 64)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        r.to("cpu")
