"""ConvGRU + prediction heads on the tensor cores (brovisionml_b200.
refine_stage, src/dsine_refine.cpp:95-158 and 253-276) against a plain
PyTorch fp32 restatement of the same formulas, with weights and the
activations between layers rounded to fp16 at the same points
(refine_stage.reference_stage), so the two differ only in summation order
and the rare fp16 rounding flip that order causes.

Tolerances: per head output, max |d| <= 3e-2 and mean |d| <= 1e-3 after one
iteration (outputs are O(1)); after three iterations of feedback through
the GRU state, max |d| <= 6e-2 and mean |d| <= 3e-3. The unrounded fp32
model's distance is printed for information.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def make_inputs(B, h, w, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h0 = torch.tanh(torch.randn((B, 64, h, w), device="cuda", generator=g))
    feat = torch.relu(torch.randn((B, 64, h, w), device="cuda", generator=g))
    ys, xs = torch.meshgrid(torch.arange(h, device="cuda"), torch.arange(w, device="cuda"),
                            indexing="ij")
    uv = torch.stack([((xs + 0.5) - w / 2) / (0.8 * w), ((ys + 0.5) - h / 2) / (0.8 * w)]).float()
    return h0, feat, uv


@pytest.mark.parametrize("B,h,w,iters,out_dtype", [(2, 24, 40, 1, torch.float32),
                                                   (1, 45, 80, 3, torch.float16),
                                                   # the reference's 500 x 348 golden case
                                                   # padded to 512 x 352: fp16 planar rows
                                                   # of 88 bytes (plain stores, no TMA)
                                                   (1, 44, 64, 1, torch.float16),
                                                   (1, 64, 44, 1, torch.float16)])
def test_refine_stage_matches_torch(B, h, w, iters, out_dtype):
    from brovisionml_b200.refine_stage import RefineStage, random_params, reference_stage

    params = random_params("cuda", seed=B + h)
    h0, feat, uv = make_inputs(B, h, w, seed=w)
    st = RefineStage(params, B, h, w, out_dtype=out_dtype)
    st.start(h0, feat, uv)
    outs = [st.step() for _ in range(iters)]
    torch.cuda.synchronize()
    st.check_pipeline()
    want = reference_stage(params, h0, feat, uv, iters)
    exact = reference_stage(params, h0, feat, uv, iters, emulate_f16=False)
    lim_max, lim_mean = (3e-2, 1e-3) if iters == 1 else (6e-2, 3e-3)
    for name in ("prob", "xy", "angle", "up_mask"):
        got = getattr(outs[-1], name).float()
        ref = getattr(want[-1], name)
        d = (got - ref).abs()
        de = (got - getattr(exact[-1], name)).abs()
        print(f"stage {name} it{iters}: max {d.max().item():.2e} mean {d.mean().item():.2e} "
              f"(vs unrounded fp32: max {de.max().item():.2e} mean {de.mean().item():.2e})")
        assert torch.isfinite(got).all()
        assert d.max().item() <= lim_max and d.mean().item() <= lim_mean


def test_refine_stage_feeds_the_ops():
    """Five iterations of the stage straight into the fused ops unit on the
    raw head outputs (refine(..., logits=True)): unit, finite normals."""
    import brovisionml_b200 as bv
    from brovisionml_b200.refine_stage import RefineStage, random_params

    B, h, w = 2, 60, 80
    params = random_params("cuda", seed=3)
    h0, feat, uv = make_inputs(B, h, w, seed=5)
    st = RefineStage(params, B, h, w, out_dtype=torch.float16)
    st.start(h0, feat, uv)
    outs = [st.step() for _ in range(5)]
    g = torch.Generator(device="cuda").manual_seed(1)
    n0 = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device="cuda", generator=g),
                                       dim=1)
    fu, cu, fv, cv = 0.8 * w, w / 2 + 0.06, 0.8 * w, h / 2 + 0.06
    res = bv.refine(n0.half(), [o.prob for o in outs], [o.xy for o in outs],
                    [o.angle for o in outs], outs[-1].up_mask, fu, cu, fv, cv, logits=True)
    torch.cuda.synchronize()
    st.check_pipeline()
    r = res.float()
    assert torch.isfinite(r).all()
    assert (r.norm(dim=1) - 1).abs().max().item() <= 2e-3


def test_refine_stage_skip_up_mask():
    """up_mask=False skips the up-mask head (only the last iteration's
    upsample reaches the output, src/dsine_refine.cpp:270-282) and leaves
    the other heads and the GRU state unchanged."""
    from brovisionml_b200.refine_stage import RefineStage, random_params

    B, h, w = 1, 24, 40
    params = random_params("cuda", seed=9)
    h0, feat, uv = make_inputs(B, h, w, seed=2)
    outs = {}
    for skip in (False, True):
        st = RefineStage(params, B, h, w, out_dtype=torch.float32)
        st.start(h0, feat, uv)
        res = [st.step(up_mask=not skip or i == 2) for i in range(3)]
        torch.cuda.synchronize()
        st.check_pipeline()
        outs[skip] = res
    for i in range(3):
        for name in ("prob", "xy", "angle"):
            assert torch.equal(getattr(outs[False][i], name), getattr(outs[True][i], name))
    assert outs[True][0].up_mask is None and outs[True][1].up_mask is None
    assert torch.equal(outs[False][2].up_mask, outs[True][2].up_mask)


def test_stage_inputs_layouts():
    """bvml_stage_inputs: planar fp32 h0 / feat -> h32 (C4 fp32), hx and fx
    (NHWC fp16), against torch's own permutes; odd sizes."""
    from brovisionml_b200._capi import check, lib
    from brovisionml_b200.ops import _p, _stream

    B, H, W = 3, 7, 13
    g = torch.Generator(device="cuda").manual_seed(4)
    h0 = torch.randn((B, 64, H, W), device="cuda", generator=g)
    feat = torch.randn((B, 64, H, W), device="cuda", generator=g)
    h32 = torch.full((B, 16, H, W, 4), float("nan"), device="cuda")
    hx = torch.empty((B, H, W, 64), device="cuda", dtype=torch.float16)
    fx = torch.empty((B, H, W, 64), device="cuda", dtype=torch.float16)
    check(lib.bvml_stage_inputs(_p(h0), _p(feat), B, H, W, _p(h32), _p(hx), _p(fx),
                                _stream(torch.device("cuda"))))
    torch.cuda.synchronize()
    assert torch.equal(h32, h0.reshape(B, 16, 4, H, W).permute(0, 1, 3, 4, 2))
    assert torch.equal(hx, h0.permute(0, 2, 3, 1).to(torch.float16))
    assert torch.equal(fx, feat.permute(0, 2, 3, 1).to(torch.float16))
