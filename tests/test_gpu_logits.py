"""GPU parity of the head-activation fusion: AngMF and the fused unit given
the prediction heads' raw prob / angle outputs, activated on load
(src/dsine_refine.cpp:262-267), against the oracle fed
oracle.head_activation of the same logits.

Tolerances as the other parity tests: max-abs 1e-5 with fp32 storage, 2e-3
with fp16 storage (fp16 logits; the activations stay fp32 in both paths).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda:0", dtype)


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def report(name, got, want, tol):
    m = O.compare(got, want)
    print(f"{name}: max_abs {m['max_abs']:.3e} ang_p99 {m['ang_p99_deg']:.2e} "
          f"ang_max {m['ang_max_deg']:.2e} deg")
    assert m["nonfinite"] == 0
    assert m["max_abs"] <= tol, m


def head_logits(shape, seed):
    """Raw head outputs: spread logits plus saturated ones at both ends."""
    g = np.random.default_rng(seed)
    pl = g.normal(0.0, 2.5, shape).astype(np.float32)
    al = g.normal(-2.5, 1.5, shape).astype(np.float32)
    pick = g.random(shape)
    pl[pick < 0.02] = 40.0
    pl[(pick >= 0.02) & (pick < 0.04)] = -40.0
    al[(pick >= 0.04) & (pick < 0.06)] = 20.0     # angle -> kPi
    al[(pick >= 0.06) & (pick < 0.08)] = -60.0    # angle -> 0
    pl[..., 3, 5] = -60.0                         # every weight of a pixel vanishes
    pl[..., 4, 6] = -100.0
    return pl, al


@pytest.mark.parametrize("H,W,B,f16", [(480, 640, 1, False), (200, 328, 2, False),
                                       (512, 768, 2, True)])
def test_angmf_logits(H, W, B, f16):
    import brovisionml_b200 as b

    u = O.gen_unit(H, W, B, iters=1, seed=H + W, upsample=False)
    pl, al = head_logits(u.prob[0].shape, H * W)
    n0 = O.ray_relu(u.normal0, u.ray8)
    xy = u.xy[0]
    if f16:
        pl, al, xy, n0 = O.f16_round(pl), O.f16_round(al), O.f16_round(xy), O.f16_round(n0)
    prob, ang = O.head_activation(pl, al)
    want = O.angmf(n0, prob, xy, ang, u.ray8, u.fu, u.cu, u.fv, u.cv)
    dt = torch.float16 if f16 else torch.float32
    got = b.angmf_propagate(dev(n0, dt), dev(pl, dt), dev(xy, dt), dev(al, dt), dev(u.ray8),
                            u.fu, u.cu, u.fv, u.cv, logits=True)
    report(f"angmf logits {H//8}x{W//8} f16={f16}", host(got), want,
           O.TOL_F16 if f16 else O.TOL_F32)


@pytest.mark.parametrize("H,W,B,f16,rr", [(480, 640, 1, False, True), (720, 1280, 2, True, False)])
def test_refine_logits(H, W, B, f16, rr):
    import brovisionml_b200 as b

    u = O.gen_unit(H, W, B, iters=5, seed=W)
    logits = [head_logits(p.shape, 1000 + i) for i, p in enumerate(u.prob)]
    if f16:
        u = O.to_f16_storage(u)
        logits = [(O.f16_round(p), O.f16_round(a)) for p, a in logits]
    acts = [O.head_activation(p, a) for p, a in logits]
    ua = O.UnitInputs(**{**u.__dict__, "prob": [p for p, _ in acts],
                         "angle": [a for _, a in acts]})
    want = O.refine_unit(ua, full_res_ray_relu=rr)
    dt = torch.float16 if f16 else torch.float32
    got = b.refine(dev(u.normal0, dt), [dev(p, dt) for p, _ in logits],
                   [dev(x, dt) for x in u.xy], [dev(a, dt) for _, a in logits],
                   dev(u.mask, dt), u.fu, u.cu, u.fv, u.cv, ray8=dev(u.ray8),
                   full_res_ray_relu=rr, logits=True)
    report(f"refine logits {H}x{W} f16={f16}", host(got), want,
           O.TOL_F16 if f16 else O.TOL_F32)
