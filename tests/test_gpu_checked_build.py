"""The checked build (libbvml_dsine_checked.so: every kernel tests its indices,
shared-memory offsets and TMA coordinates before each access, skips a failing
access and records it) run over the shapes most likely to reach an edge:
odd and single-pixel grids, every window and dilation, crops, full-resolution
RayReLU, the analytic ray, fp16 and fp32, both AngMF paths (persistent and
one launch per iteration), the raw-head-output path, the tensor-core
convolutions and the whole C refiner. Every case must leave the check word
at zero and give the release library's result bit for bit (the tests change
no arithmetic). compute-sanitizer is not available where this is run, so
this is the memory-safety evidence for the kernels.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKED = os.path.join(ROOT, "brovisionml_b200", "_lib", "libbvml_dsine_checked.so")


@pytest.fixture(scope="module")
def checked():
    from brovisionml_b200 import _capi

    if not os.path.exists(CHECKED):
        pytest.fail("libbvml_dsine_checked.so not built (brovisionml_b200/build.py builds it)")
    chk = ctypes.CDLL(CHECKED)
    for name in _capi.EXPORTS:
        f, g = getattr(_capi.lib, name), getattr(chk, name)
        g.restype, g.argtypes = f.restype, f.argtypes
    assert _capi.lib.bvml_check_word(0) == -1  # the release library has no checks
    assert chk.bvml_check_word(1) == 0
    return chk


def _both(checked, monkeypatch, fn):
    """fn() through the release library, then through the checked one."""
    from brovisionml_b200 import _capi, ops, refine_stage

    want = fn()
    torch.cuda.synchronize()
    with monkeypatch.context() as m:
        for mod in (_capi, ops, refine_stage):
            m.setattr(mod, "lib", checked)
        got = fn()
        torch.cuda.synchronize()
    word = checked.bvml_check_word(1)
    assert word == 0, f"check bits {word:#x}"
    return got, want


def _dev(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda:0", dt)


UNIT_CASES = [
    # H, W, B, ps, dil, f16, full-res RayReLU, crop, ray given
    (8, 8, 1, 5, 1, False, False, None, True),
    (8, 56, 2, 3, 1, False, True, None, False),
    (56, 8, 1, 7, 2, False, False, None, True),
    (40, 104, 3, 5, 2, True, False, (3, 5, 30, 90), True),
    (136, 96, 2, 7, 1, True, True, None, False),
    (480, 640, 1, 5, 1, False, True, (4, 6, 470, 628), False),
    (720, 1280, 2, 5, 1, True, False, None, True),
    (256, 320, 2, 3, 4, False, False, None, True),
]


@pytest.mark.parametrize("case", UNIT_CASES, ids=lambda c: f"{c[0]}x{c[1]}b{c[2]}p{c[3]}d{c[4]}")
@pytest.mark.parametrize("logits", [False, True])
def test_checked_refine_unit(checked, monkeypatch, case, logits):
    import brovisionml_b200 as b

    H, W, B, ps, dil, f16, rr, crop, ray_given = case
    u = O.gen_unit(H, W, B, ps=ps, dil=dil, iters=3, seed=H + W + ps, face_camera=True)
    dt = torch.float16 if f16 else torch.float32
    args = ([_dev(a, dt) for a in u.prob], [_dev(a, dt) for a in u.xy],
            [_dev(a, dt) for a in u.angle])
    n0, mask, ray = _dev(u.normal0, dt), _dev(u.mask, dt), _dev(u.ray8)

    def run():
        return b.refine(n0, *args, mask, u.fu, u.cu, u.fv, u.cv,
                        ray8=ray if ray_given else None, ps=ps, dil=dil, full_res_ray_relu=rr,
                        crop=crop, logits=logits)

    got, want = _both(checked, monkeypatch, run)
    assert torch.equal(got, want)


@pytest.mark.parametrize("hw", [(1, 1), (1, 7), (7, 1), (5, 13), (33, 65), (17, 31)])
def test_checked_angmf_odd_grids(checked, monkeypatch, hw):
    import brovisionml_b200 as b

    h, w = hw
    g = np.random.default_rng(h * 1000 + w)
    n = g.standard_normal((2, 3, h, w)).astype(np.float32)
    n /= np.linalg.norm(n, axis=1, keepdims=True)
    prob = _dev(g.random((2, 25, h, w)))
    xy = _dev(g.standard_normal((2, 50, h, w)))
    ang = _dev(g.uniform(0, np.pi, (2, 25, h, w)))
    fu, cu, fv, cv = 0.8 * w + 0.3, w / 2 + 0.06, 0.8 * h + 0.7, h / 2 + 0.06
    ray = _dev(O.build_ray_scaled(fu, cu, fv, cv, h, w))
    nd = _dev(n)
    got, want = _both(checked, monkeypatch,
                      lambda: b.angmf_propagate(nd, prob, xy, ang, ray, fu, cu, fv, cv))
    assert torch.equal(got, want)


@pytest.mark.parametrize("B,H,W,cin,cout,ks", [(1, 4, 32, 64, 64, 1), (2, 23, 37, 130, 64, 5),
                                               (1, 17, 9, 128, 25, 1), (1, 60, 80, 66, 512, 3)])
def test_checked_conv(checked, monkeypatch, B, H, W, cin, cout, ks):
    import brovisionml_b200 as b

    g = torch.Generator(device="cuda").manual_seed(B * H * W + cin)
    cin_pad, cout_pad = b.ops.pad64(cin), b.ops.pad64(cout)
    x = torch.zeros((B, H, W, cin_pad), device="cuda", dtype=torch.float16)
    x[..., :cin] = torch.randn((B, H, W, cin), device="cuda", generator=g).to(torch.float16)
    weight = torch.randn((cout, cin, ks, ks), device="cuda", generator=g) * (cin * ks * ks) ** -0.5
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    wp = b.pack_conv_weight(weight, cin_pad, cout_pad)
    got, want = _both(checked, monkeypatch,
                      lambda: b.conv2d_nhwc(x, wp, bias, cout, ks=ks, act="relu"))
    assert torch.equal(got, want)


@pytest.mark.parametrize("shape", [(1, 16, 24, None), (2, 44, 64, (2, 6, 348, 500))])
def test_checked_refiner(checked, monkeypatch, shape):
    """The whole learned refinement (stage inputs, hoisted terms, ConvGRU,
    heads, head tails, the fused ops) through the checked library."""
    from brovisionml_b200.refine_stage import random_params
    from brovisionml_b200.refiner import Refiner

    B, h, w, crop = shape
    H, W = 8 * h, 8 * w
    intr = (0.8 * W, 0.8 * W, W / 2 - 3.0, H / 2 + 2.0)
    g = torch.Generator(device="cuda").manual_seed(h * w)
    normal = torch.nn.functional.normalize(torch.randn((B, 3, h, w), device="cuda", generator=g),
                                           dim=1)
    feat = torch.relu(torch.randn((B, 64, h, w), device="cuda", generator=g))
    hid = torch.tanh(torch.randn((B, 64, h, w), device="cuda", generator=g))
    params = random_params("cpu", seed=h + w)

    def run():
        r = Refiner()
        r.load_params(params)
        r.to(0)
        return r.forward(normal, feat, hid, intr, H, W, crop=crop, out_dtype=torch.float32)

    got, want = _both(checked, monkeypatch, run)
    assert torch.equal(got, want)
