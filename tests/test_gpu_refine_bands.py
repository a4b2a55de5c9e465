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
