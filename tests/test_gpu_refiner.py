"""brovisionml_b200.refiner.Refiner.forward on the GPU: the whole refinement
(stage + ops) equals its parts composed by hand, crops like slicing the
uncropped result (src/dsine_refine.cpp:286-292), and gives unit normals."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_refiner_forward_composes_stage_and_ops():
    import brovisionml_b200 as bv
    from brovisionml_b200.refine_stage import RefineStage, random_params
    from brovisionml_b200.refiner import Refiner, build_uv, grid_intrinsics

    B, h, w = 2, 44, 64          # the reference's 500 x 348 golden size, padded: 512 x 352
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2 - 3.0, H / 2 + 2.0)
    g = torch.Generator(device="cuda").manual_seed(5)
    normal = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device="cuda",
                                                       generator=g), dim=1)
    feat = torch.relu(torch.randn((B, 64, h, w), device="cuda", generator=g))
    hid = torch.tanh(torch.randn((B, 64, h, w), device="cuda", generator=g))
    params = random_params("cpu", seed=4)
    r = Refiner()
    r.load_params(params)
    r.to(0)
    got = r.forward(normal, feat, hid, intr, H, W)
    crop = (2, 6, 348, 500)  # (pad_t, pad_l, orig_h, orig_w)
    got_c = r.forward(normal, feat, hid, intr, H, W, crop=crop)
    torch.cuda.synchronize()
    assert got.shape == (B, 3, H, W) and got_c.shape == (B, 3, 348, 500)
    assert torch.equal(got_c, got[:, :, 2:2 + 348, 6:6 + 500])
    assert (got.float().norm(dim=1) - 1).abs().max().item() <= 2e-3

    st = RefineStage(params, B, h, w, out_dtype=torch.float16)
    st.start(hid, feat, build_uv(intr, h, w, H, W, "cuda"))
    outs = [st.step() for _ in range(5)]
    fu, cu, fv, cv = grid_intrinsics(intr, h, w, H, W)
    want = bv.refine(normal.half(), [o.prob for o in outs], [o.xy for o in outs],
                     [o.angle for o in outs], outs[-1].up_mask, fu, cu, fv, cv, logits=True)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_refiner_graph_replay_matches_eager():
    """forward(graph=True): a CUDA graph of the whole refinement, captured
    once per shape / intrinsics / crop, replayed with new inputs, equals the
    eager call."""
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import Refiner

    B, h, w = 1, 24, 40
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2, H / 2)
    r = Refiner()
    r.load_params(random_params("cpu", seed=6))
    r.to(0)
    for seed in (1, 2):
        g = torch.Generator(device="cuda").manual_seed(seed)
        normal = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device="cuda",
                                                           generator=g), dim=1)
        feat = torch.relu(torch.randn((B, 64, h, w), device="cuda", generator=g))
        hid = torch.tanh(torch.randn((B, 64, h, w), device="cuda", generator=g))
        eager = r.forward(normal, feat, hid, intr, H, W, crop=(4, 8, 180, 300))
        replay = r.forward(normal, feat, hid, intr, H, W, crop=(4, 8, 180, 300), graph=True)
        torch.cuda.synchronize()
        assert torch.equal(eager, replay), seed
    assert len(r._graphs) == 1
