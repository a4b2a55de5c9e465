"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and rejects bad arguments with the reference's error wording --
all without touching a GPU (every checked call returns before any CUDA call)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bvml_dsine.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bvml_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported():
    import brovisionml_b200 as b
    from brovisionml_b200 import _capi

    syms = declared_symbols()
    assert len(syms) == 29, syms
    assert sorted(_capi.EXPORTS) == syms
    for s in syms:
        assert hasattr(b.lib, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", b.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (bvml_\w+)", out))
    assert exported == set(syms)
    assert b.abi_version() == 9


def test_bridge_library_exports_reference_signatures():
    path = os.path.join(ROOT, "brovisionml_b200", "_lib", "libbvml_dsine_bridge.so")
    out = subprocess.run(["nm", "-DC", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    assert ("brovisionml::dsine::detail::ray_relu_cuda(brotensor::Tensor&, "
            "brotensor::Tensor const&, int, int)") in out
    assert ("brovisionml::dsine::detail::angmf_propagate_cuda(brotensor::Tensor const&, "
            "brotensor::Tensor const&, brotensor::Tensor const&, brotensor::Tensor const&, "
            "brotensor::Tensor const&, double, double, double, double, int, int, "
            "brotensor::Tensor&)") in out
    assert ("brovisionml::dsine::detail::angmf_propagate_logits_cuda(brotensor::Tensor const&, "
            "brotensor::Tensor const&, brotensor::Tensor const&, brotensor::Tensor const&, "
            "brotensor::Tensor const&, double, double, double, double, int, int, "
            "brotensor::Tensor&)") in out
    assert "brovisionml::dsine::detail::refine_ops_cuda(" in out


def test_argument_errors_without_gpu():
    from brovisionml_b200 import _capi

    lib = _capi.lib
    fake = ctypes.c_void_p(0x1000)
    # unknown dtype
    rc = lib.bvml_ray_relu(fake, fake, 1, 4, 4, 7, None)
    assert rc == 1 and lib.bvml_last_error().decode().startswith("dsine ops: ray_relu")
    # bad window / dilation
    rc = lib.bvml_angmf_propagate(fake, fake, fake, fake, fake, 1.0, 0.0, 1.0, 0.0, 1, 4, 4, 4,
                                  1, 0, ctypes.c_void_p(0x2000), None)
    assert rc == 1 and "window" in lib.bvml_last_error().decode()
    rc = lib.bvml_angmf_propagate(fake, fake, fake, fake, fake, 1.0, 0.0, 1.0, 0.0, 1, 4, 4, 5,
                                  0, 0, ctypes.c_void_p(0x2000), None)
    assert rc == 1
    # null tensors
    rc = lib.bvml_angmf_propagate(None, fake, fake, fake, fake, 1.0, 0.0, 1.0, 0.0, 1, 4, 4, 5,
                                  1, 0, fake, None)
    assert rc == 1 and "null" in lib.bvml_last_error().decode()
    # aliasing out == pred_norm
    rc = lib.bvml_angmf_propagate(fake, fake, fake, fake, fake, 1.0, 0.0, 1.0, 0.0, 1, 4, 4, 5,
                                  1, 0, fake, None)
    assert rc == 1 and "alias" in lib.bvml_last_error().decode()
    # zero focal length
    rc = lib.bvml_angmf_propagate(fake, fake, fake, fake, fake, 0.0, 0.0, 1.0, 0.0, 1, 4, 4, 5,
                                  1, 0, ctypes.c_void_p(0x2000), None)
    assert rc == 1
    # negative shapes
    rc = lib.bvml_ray_relu(fake, fake, -1, 4, 4, 0, None)
    assert rc == 1
    # empty work is a successful no-op (the reference returns early on HW == 0)
    assert lib.bvml_ray_relu(None, None, 1, 0, 4, 0, None) == 0
    assert lib.bvml_angmf_propagate(None, None, None, None, None, 1.0, 0.0, 1.0, 0.0, 1, 0, 5,
                                    5, 1, 0, None, None) == 0
    # upsample is C = 3, scale 8 only
    rc = lib.bvml_convex_upsample(fake, fake, 1, 4, 4, 4, 8, 0, fake, None)
    assert rc == 3 and "C = 3" in lib.bvml_last_error().decode()
    rc = lib.bvml_slice2d(fake, 1, 3, 4, 4, 2, 0, 4, 4, 0, fake, None)
    assert rc == 1 and "outside" in lib.bvml_last_error().decode()
    # refine: workspace size and alignment are checked before any launch
    need = lib.bvml_refine_workspace_bytes(2, 8, 8)
    # sync words (64 + one per 32 x 16 tile, 256-byte aligned), two fp32 normal
    # buffers of 2 frames, the ray
    assert need == 512 + 2 * 1536 + 768
    arr = (ctypes.c_void_p * 1)(0x3000)
    rc = lib.bvml_refine(fake, None, arr, arr, arr, 1, fake, 2, 8, 8, 5, 1, 1.0, 0.0, 1.0, 0.0,
                         0, 0, 0, 64, 64, 0, ctypes.c_void_p(0x10000), need - 1, fake, None)
    assert rc == 1 and "workspace" in lib.bvml_last_error().decode()
    rc = lib.bvml_refine(fake, None, arr, arr, arr, 1, fake, 2, 8, 8, 5, 1, 1.0, 0.0, 1.0, 0.0,
                         0, 0, 0, 65, 64, 0, ctypes.c_void_p(0x10000), need, fake, None)
    assert rc == 1 and "crop" in lib.bvml_last_error().decode()
    rc = lib.bvml_refine(fake, None, arr, arr, arr, 1, fake, 2, 8, 8, 5, 1, 1.0, 0.0, 1.0, 0.0,
                         0, 0, 0, 64, 64, 0, ctypes.c_void_p(0x10010), need, fake, None)
    assert rc == 1 and "aligned" in lib.bvml_last_error().decode()
    # the raw-head-output entry points check the same way, under their own names
    rc = lib.bvml_angmf_propagate_logits(fake, fake, fake, fake, fake, 1.0, 0.0, 1.0, 0.0, 1, 4,
                                         4, 4, 1, 0, ctypes.c_void_p(0x2000), None)
    err = lib.bvml_last_error().decode()
    assert rc == 1 and err.startswith("dsine ops: angmf_propagate_logits") and "window" in err
    assert lib.bvml_angmf_propagate_logits(None, None, None, None, None, 1.0, 0.0, 1.0, 0.0, 1,
                                           0, 5, 5, 1, 0, None, None) == 0
    rc = lib.bvml_refine_logits(fake, None, arr, arr, arr, 1, fake, 2, 8, 8, 5, 1, 1.0, 0.0,
                                1.0, 0.0, 0, 0, 0, 64, 64, 0, ctypes.c_void_p(0x10000), need - 1,
                                fake, None)
    assert rc == 1 and "workspace" in lib.bvml_last_error().decode()


def test_conv_argument_errors_without_gpu():
    """bvml_conv2d_nhwc_f16_ex validates before touching the GPU: kernel
    size, the GRU epilogues' refusal of an addend, the extra K block's
    layout and the split output's room."""
    import ctypes

    from brovisionml_b200._capi import (EPI_GRU_ZR, EPI_NHWC, EPI_SPLIT_F16, ConvEpilogue,
                                        lib)

    fake = 0x10000  # aligned, never dereferenced: every call fails validation first

    def call(ks=5, cout=128, cout_pad=128, **epi):
        e = ConvEpilogue(**epi)
        return lib.bvml_conv2d_nhwc_f16_ex(fake, 64, 0, 64, fake, fake, 1, 8, 16, cout,
                                            cout_pad, ks, ctypes.byref(e), fake, None)

    assert call(ks=4, mode=EPI_NHWC, out=fake, out_c=128) == 1
    assert "kernel size" in lib.bvml_last_error().decode()
    assert call(mode=EPI_GRU_ZR, h32=fake, z=fake, rh=fake, rh_c=64, add=fake, add_c=128) == 1
    assert "no addend" in lib.bvml_last_error().decode()
    assert call(mode=EPI_NHWC, out=fake, out_c=128, xin=fake, xin_c=96, wx=fake) == 1
    assert "extra K" in lib.bvml_last_error().decode()
    assert call(mode=EPI_NHWC, out=fake, out_c=128, xin=fake, xin_c=128, xin_stride=64,
                wx=fake) == 1
    assert "xin_stride" in lib.bvml_last_error().decode()
    assert call(mode=EPI_SPLIT_F16, out=fake, out_c=128) == 1
    assert "split" in lib.bvml_last_error().decode()


def test_python_mirror_rejects_cpu_tensors():
    import torch

    import brovisionml_b200 as b

    with pytest.raises(RuntimeError, match="dsine ops"):
        b.angmf_propagate(torch.zeros(1, 3, 4, 4), torch.zeros(1, 25, 4, 4),
                          torch.zeros(1, 50, 4, 4), torch.zeros(1, 25, 4, 4),
                          torch.zeros(3, 4, 4), 1.0, 0.0, 1.0, 0.0)
