"""Tensor-core (tcgen05) implicit-GEMM convolution against a plain PyTorch fp32
conv2d of the same fp16-rounded inputs and weights: the refine stage's conv
shapes (ConvGRU 5x5 over 130 -> 64 channels, head 3x3 66 -> 128 and 1x1
layers, src/dsine_refine.cpp:95-158) and edge cases (one CTA, odd frames,
output channels that are not a multiple of the tile).

Tolerance: the kernel rounds its output to fp16 (relative 2^-9) and sums in
another order than torch: |y - ref| <= 8e-3 |ref| + 2e-3.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def ref_conv(x_nhwc, weight, bias, ks, act, cin):
    x = x_nhwc[..., :cin].permute(0, 3, 1, 2).float()
    y = torch.nn.functional.conv2d(x, weight.to(torch.float16).float(), bias, padding=ks // 2)
    y = {"none": y, "relu": torch.relu(y), "sigmoid": torch.sigmoid(y),
         "tanh": torch.tanh(y)}[act]
    return y.permute(0, 2, 3, 1)


def run_case(B, H, W, cin, cout, ks, act, seed=0):
    import brovisionml_b200 as b

    g = torch.Generator(device="cuda").manual_seed(seed)
    cin_pad, cout_pad = b.ops.pad64(cin), b.ops.pad64(cout)
    x = torch.zeros((B, H, W, cin_pad), device="cuda", dtype=torch.float16)
    x[..., :cin] = torch.randn((B, H, W, cin), device="cuda", generator=g).to(torch.float16)
    wstd = (cin * ks * ks) ** -0.5
    weight = torch.randn((cout, cin, ks, ks), device="cuda", generator=g) * wstd
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    y = b.conv2d_nhwc(x, b.pack_conv_weight(weight, cin_pad, cout_pad), bias, cout, ks=ks,
                      act=act)
    torch.cuda.synchronize()
    ref = ref_conv(x, weight, bias, ks, act, cin)
    got = y[..., :cout].float()
    err = ((got - ref).abs() - 8e-3 * ref.abs()).max().item()
    print(f"conv B{B} {H}x{W} {cin}->{cout} k{ks} {act}: excess {err:.2e} "
          f"max_abs {(got - ref).abs().max().item():.2e}")
    assert torch.isfinite(got).all()
    assert err <= 2e-3
    if cout_pad > cout:  # pad channels are zeros
        assert (y[..., cout:] == 0).all()


def test_conv_single_cta_1x1():
    run_case(1, 4, 32, 64, 64, 1, "none")


@pytest.mark.parametrize("B,H,W,cin,cout,ks,act", [
    (1, 8, 16, 64, 128, 3, "relu"),
    (2, 23, 37, 130, 64, 5, "tanh"),     # ConvGRU q: odd frame, padded input channels
    (1, 90, 160, 130, 128, 5, "sigmoid"),  # ConvGRU z, r (fused), config 4 grid
    (1, 60, 80, 66, 512, 3, "relu"),     # the four heads' first layers fused
    (2, 45, 67, 128, 576, 1, "none"),    # up_prob head's last layer
    (1, 17, 9, 128, 25, 1, "none"),      # prob head's last layer: 25 of 64 channels
])
def test_conv_shapes(B, H, W, cin, cout, ks, act):
    run_case(B, H, W, cin, cout, ks, act, seed=H + W)


@pytest.mark.parametrize("shared", [False, True])
def test_conv_addend_and_fp32_output(shared):
    """The per-pixel addend (C4 fp32; per frame, or one frame shared by
    all) joins conv + bias before the activation; fp32 C4 output
    (bvml_conv2d_nhwc_f16_ex with BVML_EPI_C4_F32): the refine stage's
    hoisted feature / uv terms."""
    import ctypes

    import brovisionml_b200 as b
    from brovisionml_b200._capi import EPI_C4_F32, ConvEpilogue, check, lib
    from brovisionml_b200.ops import _p, _stream

    B, H, W, cin, cout, ks = 2, 19, 40, 64, 192, 5
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((B, H, W, cin), device="cuda", generator=g).to(torch.float16)
    weight = torch.randn((cout, cin, ks, ks), device="cuda", generator=g) * (cin * ks * ks) ** -0.5
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    add = torch.randn((1 if shared else B, (cout + 8) // 4, H, W, 4), device="cuda", generator=g)
    y = torch.full((B, cout // 4, H, W, 4), float("nan"), device="cuda")
    err = torch.zeros(1, device="cuda", dtype=torch.int32)
    e = ConvEpilogue(mode=EPI_C4_F32, act=1, out=_p(y), out_c=cout, out_off=0,
                     add=_p(add), add_c=cout + 8, add_shared=int(shared))
    check(lib.bvml_conv2d_nhwc_f16_ex(_p(x), cin, 0, cin, _p(b.pack_conv_weight(weight)),
                                       _p(bias), B, H, W, cout, cout, ks, ctypes.byref(e),
                                       _p(err), _stream(torch.device("cuda"))))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c4 = lambda t: t.permute(0, 2, 3, 1, 4).reshape(t.shape[0], H, W, -1)  # noqa: E731
    ref = torch.relu(ref_conv(x, weight, bias, ks, "none", cin) + c4(add)[..., :cout])
    d = (c4(y) - ref).abs().max().item()
    print(f"conv addend shared={shared}: max_abs {d:.2e}")
    assert d <= 1e-3  # fp32 output: summation order only


@pytest.mark.parametrize("B,H,W,cin,cout,ks,f16", [
    (2, 9, 45, 128, 25, 1, True),     # odd width: plain stores
    (1, 16, 44, 64, 50, 3, True),     # 88-byte rows: plain stores
    (1, 12, 40, 128, 576, 1, True),   # 80-byte rows: TMA stores, N = 192 tiles
    (1, 7, 37, 64, 30, 5, False),     # fp32, odd width
])
def test_conv_planar_outputs(B, H, W, cin, cout, ks, f16):
    """Planar (B, cout, H, W) outputs of bvml_conv2d_nhwc_f16_ex (the heads'
    raw outputs), through TMA stores where the rows allow it and plain stores
    otherwise."""
    import ctypes

    import brovisionml_b200 as b
    from brovisionml_b200._capi import EPI_PLANAR_F16, EPI_PLANAR_F32, ConvEpilogue, check, lib
    from brovisionml_b200.ops import _p, _stream

    g = torch.Generator(device="cuda").manual_seed(W + cout)
    cin_pad = b.ops.pad64(cin)
    x = torch.zeros((B, H, W, cin_pad), device="cuda", dtype=torch.float16)
    x[..., :cin] = torch.randn((B, H, W, cin), device="cuda", generator=g).to(torch.float16)
    weight = torch.randn((cout, cin, ks, ks), device="cuda", generator=g) * (cin * ks * ks) ** -0.5
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    dt = torch.float16 if f16 else torch.float32
    y = torch.full((B, cout, H, W), float("nan"), device="cuda", dtype=dt)
    err = torch.zeros(1, device="cuda", dtype=torch.int32)
    e = ConvEpilogue(mode=EPI_PLANAR_F16 if f16 else EPI_PLANAR_F32, out=_p(y))
    wp = b.pack_conv_weight(weight, cin_pad)
    check(lib.bvml_conv2d_nhwc_f16_ex(_p(x), cin_pad, 0, cin_pad, _p(wp), _p(bias), B, H, W,
                                       cout, wp.shape[1], ks, ctypes.byref(e), _p(err),
                                       _stream(torch.device("cuda"))))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = ref_conv(x, weight, bias, ks, "none", cin).permute(0, 3, 1, 2)
    d = ((y.float() - ref).abs() - (1e-3 if f16 else 0.0) * ref.abs()).max().item()
    print(f"planar conv {B}x{H}x{W} {cin}->{cout} k{ks} f16={f16}: excess {d:.2e}")
    assert torch.isfinite(y.float()).all()
    assert d <= 2e-3  # fp16 output rounding (2^-11 relative) or fp32 summation order


def _conv_ex(x, cin, w_packed, bias, cout, ks, **epi):
    import ctypes

    from brovisionml_b200._capi import ConvEpilogue, check, lib
    from brovisionml_b200.ops import _p, _stream

    B, H, W, xc = x.shape
    err = torch.zeros(1, device="cuda", dtype=torch.int32)
    e = ConvEpilogue(**{k: (_p(v) if isinstance(v, torch.Tensor) else v) for k, v in epi.items()})
    check(lib.bvml_conv2d_nhwc_f16_ex(_p(x), xc, 0, cin, _p(w_packed), _p(bias), B, H, W, cout,
                                       w_packed.shape[1], ks, ctypes.byref(e), _p(err),
                                       _stream(torch.device("cuda"))))
    torch.cuda.synchronize()
    assert int(err.item()) == 0


@pytest.mark.parametrize("cout,ks", [(128, 5), (64, 5), (192, 3)])
def test_conv_extra_k_and_split(cout, ks):
    """The extra K block (conv += xin . wx^T per pixel, through the MMA
    pipeline) and the split-fp16 output (hi + lo of the fp32 result): the
    refine stage's hoisted GRU terms, added by the tensor cores."""
    import brovisionml_b200 as b
    from brovisionml_b200._capi import EPI_C4_F32, EPI_SPLIT_F16

    B, H, W, cin, xc = 2, 21, 40, 64, 128
    g = torch.Generator(device="cuda").manual_seed(cout + ks)
    x = torch.randn((B, H, W, cin), device="cuda", generator=g).to(torch.float16)
    weight = torch.randn((cout, cin, ks, ks), device="cuda", generator=g) * (cin * ks * ks) ** -0.5
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    wp = b.pack_conv_weight(weight)
    ref = ref_conv(x, weight, bias, ks, "none", cin)  # (B,H,W,cout) fp32

    # split output, per 64-channel block hi then lo: hi + lo reproduces the
    # fp32 result to ~2^-16
    sp = torch.full((B, H, W, 2 * cout), float("nan"), device="cuda", dtype=torch.float16)
    _conv_ex(x, cin, wp, bias, cout, ks, mode=EPI_SPLIT_F16, out=sp, out_c=2 * cout, out_off=0)
    blk = sp.reshape(B, H, W, cout // 64, 2, 64).float()
    got = (blk[..., 0, :] + blk[..., 1, :]).reshape(B, H, W, cout)
    d = ((got - ref).abs() - 1e-4 * ref.abs()).max().item()
    print(f"split fp16 cout={cout} k{ks}: excess {d:.2e}")
    assert d <= 1e-3

    # extra K: a 1x1 term of another input (the middle 128 of 256 channels per
    # pixel: a strided view), accumulated by the same MMAs
    xfull = torch.randn((B, H, W, 2 * xc), device="cuda", generator=g).to(torch.float16)
    xin = xfull[..., 64:64 + xc]
    wx = (torch.randn((cout, xc), device="cuda", generator=g) * xc ** -0.5).to(torch.float16)
    y = torch.full((B, cout // 4, H, W, 4), float("nan"), device="cuda")
    _conv_ex(x, cin, wp, bias, cout, ks, mode=EPI_C4_F32, out=y, out_c=cout, out_off=0,
             xin=xin, xin_c=xc, xin_stride=2 * xc, wx=wx[None].contiguous())
    c4 = y.permute(0, 2, 3, 1, 4).reshape(B, H, W, cout)
    want = ref + xin.float() @ wx.float().t()
    d = (c4 - want).abs().max().item()
    print(f"extra K cout={cout} k{ks}: max_abs {d:.2e}")
    assert d <= 1e-3  # fp32 output: summation order only


@pytest.mark.parametrize("W,cout,f16", [(40, 25, True), (44, 50, True), (37, 25, False),
                                        (160, 64, True)])
def test_head_tail_matches_two_convolutions(W, cout, f16):
    """bvml_head_tail_1x1 (1x1 -> ReLU -> 1x1 with the intermediate on chip)
    equals the two separate convolutions bit for bit: the same products,
    the same fp16 rounding of the intermediate, the same summation order."""
    import brovisionml_b200 as b
    from brovisionml_b200._capi import EPI_NHWC, EPI_PLANAR_F16, EPI_PLANAR_F32, check, lib
    from brovisionml_b200.ops import _p, _stream

    B, H, k = 2, 19, 1
    g = torch.Generator(device="cuda").manual_seed(W + cout)
    t1 = torch.randn((B, H, W, 512), device="cuda", generator=g).to(torch.float16)
    w2 = torch.randn((128, 128, 1, 1), device="cuda", generator=g) * 128 ** -0.5
    b2 = torch.randn(128, device="cuda", generator=g) * 0.1
    w4 = torch.randn((cout, 128, 1, 1), device="cuda", generator=g) * 128 ** -0.5
    b4 = torch.randn(cout, device="cuda", generator=g) * 0.1
    w2p, w4p = b.pack_conv_weight(w2), b.pack_conv_weight(w4, 128, 64)
    dt = torch.float16 if f16 else torch.float32
    t2 = torch.zeros((B, H, W, 512), device="cuda", dtype=torch.float16)
    _conv_ex(t1[..., k * 128:(k + 1) * 128].contiguous(), 128, w2p, b2, 128, 1, mode=EPI_NHWC,
             act=1, out=t2, out_c=512, out_off=k * 128)
    want = torch.full((B, cout, H, W), float("nan"), device="cuda", dtype=dt)
    _conv_ex(t2[..., k * 128:(k + 1) * 128].contiguous(), 128, w4p, b4, cout, 1,
             mode=EPI_PLANAR_F16 if f16 else EPI_PLANAR_F32, out=want)
    got = torch.full((B, cout, H, W), float("nan"), device="cuda", dtype=dt)
    err = torch.zeros(1, device="cuda", dtype=torch.int32)
    check(lib.bvml_head_tail_1x1(_p(t1), 512, k * 128, _p(w2p), _p(b2), _p(w4p), _p(b4), B, H,
                                 W, cout, 1 if f16 else 0, _p(got), _p(err),
                                 _stream(torch.device("cuda"))))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    d = (got.float() - want.float()).abs().max().item()
    print(f"head tail W={W} cout={cout} f16={f16}: max |d| {d:.2e}")
    assert torch.equal(got, want)


def test_conv_wait_limit_gives_up_then_next_launch_is_normal():
    """bvml_conv_epilogue.wait_limit bounds every pipeline wait between the
    TMA, MMA and epilogue warps. With 1 (a single non-blocking test) the MMA
    lane's first wait for a tile's operands and the epilogue's first wait for
    an accumulator come before any copy can have landed, so every CTA gives
    up: the kernel sets err and ends, after waiting (with the default bound)
    for the copies and MMAs it had in flight and freeing its TMEM. The next
    launches on the same stream, with the default bound, are normal: err 0
    and the same output, bit for bit, as the launch before the failure."""
    import ctypes

    import brovisionml_b200 as b
    from brovisionml_b200._capi import EPI_NHWC, ConvEpilogue, check, lib
    from brovisionml_b200.ops import _p, _stream

    g = torch.Generator(device="cuda").manual_seed(81)
    B, H, W, cin, cout, ks = 2, 64, 96, 128, 128, 5
    x = torch.randn((B, H, W, cin), device="cuda", generator=g).to(torch.float16)
    weight = torch.randn((cout, cin, ks, ks), device="cuda", generator=g) * (cin * ks * ks) ** -0.5
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    wp = b.pack_conv_weight(weight, cin, cout)

    def launch(limit):
        y = torch.full((B, H, W, cout), float("nan"), device="cuda", dtype=torch.float16)
        err = torch.zeros(1, device="cuda", dtype=torch.int32)
        e = ConvEpilogue(mode=EPI_NHWC, act=1, out=_p(y), out_c=cout, out_off=0,
                         wait_limit=limit)
        check(lib.bvml_conv2d_nhwc_f16_ex(_p(x), cin, 0, cin, _p(wp), _p(bias), B, H, W, cout,
                                           cout, ks, ctypes.byref(e), _p(err),
                                           _stream(torch.device("cuda"))))
        torch.cuda.synchronize()
        return y, int(err.item())

    y0, e0 = launch(0)
    assert e0 == 0
    ref = ref_conv(x, weight, bias, ks, "relu", cin)
    assert ((y0.float() - ref).abs() - 8e-3 * ref.abs()).max().item() <= 2e-3
    for _ in range(2):
        _, e1 = launch(1)
        print(f"wait_limit 1: err {e1}")
        assert e1 != 0
        y2, e2 = launch(0)
        assert e2 == 0
        assert torch.equal(y2, y0)
