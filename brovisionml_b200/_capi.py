"""ctypes binding of libbvml_dsine.so (the C ABI in include/bvml_dsine.h).

The library must have been built in-tree (``python brovisionml_b200/build.py``
or ``__graft_entry__.build()``); a missing library is an ImportError, never a
silent fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libbvml_dsine.so")

BVML_F32 = 0
BVML_F16 = 1
BVML_OK = 0

# Every symbol include/bvml_dsine.h declares (checked by the CPU test suite).
EXPORTS = ("bvml_last_error", "bvml_abi_version", "bvml_ray_relu", "bvml_angmf_propagate",
           "bvml_convex_upsample", "bvml_l2_normalize_nchw", "bvml_slice2d",
           "bvml_refine_workspace_bytes", "bvml_refine", "bvml_probe_events",
           "bvml_refine_noalloc", "bvml_angmf_propagate_logits", "bvml_refine_logits",
           "bvml_conv2d_nhwc_f16", "bvml_conv2d_nhwc_f16_ex", "bvml_stage_inputs",
           "bvml_head_tail_1x1", "bvml_refine_status", "bvml_probe_recorded",
           "bvml_refiner_weight_name", "bvml_refiner_weight_shape", "bvml_refiner_create",
           "bvml_refiner_forward", "bvml_refiner_status", "bvml_refiner_destroy", "bvml_check_word",
           "bvml_refine_halo_rows", "bvml_refiner_forward_banded", "bvml_upsample_wait_limit")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"brovisionml_b200: CUDA library not built ({LIB_PATH} missing); run "
        "`python brovisionml_b200/build.py` (nvcc for sm_100a)")

lib = ctypes.CDLL(LIB_PATH)

_vp = ctypes.c_void_p
_i = ctypes.c_int
_d = ctypes.c_double
_sz = ctypes.c_size_t

lib.bvml_last_error.restype = ctypes.c_char_p
lib.bvml_last_error.argtypes = []
lib.bvml_abi_version.restype = _i
lib.bvml_abi_version.argtypes = []
lib.bvml_ray_relu.restype = _i
lib.bvml_ray_relu.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp]
lib.bvml_angmf_propagate.restype = _i
lib.bvml_angmf_propagate.argtypes = [_vp, _vp, _vp, _vp, _vp, _d, _d, _d, _d, _i, _i, _i, _i, _i,
                                     _i, _vp, _vp]
lib.bvml_angmf_propagate_logits.restype = _i
lib.bvml_angmf_propagate_logits.argtypes = lib.bvml_angmf_propagate.argtypes
lib.bvml_convex_upsample.restype = _i
lib.bvml_convex_upsample.argtypes = [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]
lib.bvml_l2_normalize_nchw.restype = _i
lib.bvml_l2_normalize_nchw.argtypes = [_vp, _i, _i, _i, _i, ctypes.c_float, _i, _vp, _vp]
lib.bvml_slice2d.restype = _i
lib.bvml_slice2d.argtypes = [_vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp]
lib.bvml_refine_workspace_bytes.restype = _sz
lib.bvml_refine_workspace_bytes.argtypes = [_i, _i, _i]
lib.bvml_refine.restype = _i
lib.bvml_refine.argtypes = ([_vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                             ctypes.POINTER(_vp), _i, _vp] + [_i] * 5 + [_d] * 4 + [_i] * 6
                            + [_vp, _sz, _vp, _vp])
lib.bvml_refine_logits.restype = _i
lib.bvml_refine_logits.argtypes = lib.bvml_refine.argtypes
lib.bvml_refine_noalloc.restype = _i
lib.bvml_refine_noalloc.argtypes = ([_vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                     ctypes.POINTER(_vp), _i, _vp] + [_i] * 5 + [_d] * 4
                                    + [_i] * 6 + [_vp, _vp])
REFINE_NOALLOC_MAX_BYTES = 32 * 1024 * 1024
lib.bvml_conv2d_nhwc_f16.restype = _i
lib.bvml_conv2d_nhwc_f16.argtypes = [_vp, _vp, _vp] + [_i] * 8 + [_vp, _vp, _vp]


class ConvEpilogue(ctypes.Structure):
    """bvml_conv_epilogue (include/bvml_dsine.h)."""
    _fields_ = [("mode", _i), ("act", _i), ("out", _vp), ("out_c", _i), ("out_off", _i),
                ("h32", _vp), ("z", _vp), ("rh", _vp), ("rh_c", _i), ("hx", _vp), ("hx_c", _i),
                ("hin", _vp), ("hin_c", _i), ("add", _vp), ("add_c", _i), ("add_shared", _i),
                ("xin", _vp), ("xin_c", _i), ("wx", _vp), ("xin_stride", _i),
                ("wait_limit", ctypes.c_uint)]


EPI_NHWC, EPI_PLANAR_F16, EPI_PLANAR_F32, EPI_GRU_ZR, EPI_GRU_Q, EPI_C4_F32, EPI_SPLIT_F16 = \
    range(7)
lib.bvml_conv2d_nhwc_f16_ex.restype = _i
lib.bvml_conv2d_nhwc_f16_ex.argtypes = ([_vp, _i, _i, _i, _vp, _vp] + [_i] * 6
                                          + [ctypes.POINTER(ConvEpilogue), _vp, _vp])
lib.bvml_head_tail_1x1.restype = _i
lib.bvml_head_tail_1x1.argtypes = [_vp, _i, _i, _vp, _vp, _vp, _vp] + [_i] * 5 + [_vp, _vp, _vp]
lib.bvml_stage_inputs.restype = _i
lib.bvml_stage_inputs.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp]
lib.bvml_probe_events.restype = _i
lib.bvml_probe_events.argtypes = [ctypes.POINTER(_vp), _i]
lib.bvml_probe_recorded.restype = _i
lib.bvml_probe_recorded.argtypes = []
lib.bvml_check_word.restype = _i
lib.bvml_check_word.argtypes = [_i]
lib.bvml_refine_status.restype = _i
lib.bvml_refine_status.argtypes = [_vp, _vp]
REFINER_WEIGHTS = 30
lib.bvml_refiner_weight_name.restype = ctypes.c_char_p
lib.bvml_refiner_weight_name.argtypes = [_i]
lib.bvml_refiner_weight_shape.restype = _i
lib.bvml_refiner_weight_shape.argtypes = [_i, ctypes.POINTER(_i)]
lib.bvml_refiner_create.restype = _i
lib.bvml_refiner_create.argtypes = [ctypes.POINTER(_vp), _i, ctypes.POINTER(_vp)]
lib.bvml_refiner_forward.restype = _i
lib.bvml_refiner_forward.argtypes = ([_vp, _vp, _vp, _vp] + [_i] * 3 + [ctypes.POINTER(ctypes.c_float)]
                                     + [_i] * 8 + [_vp, _vp])
lib.bvml_refiner_status.restype = _i
lib.bvml_refiner_status.argtypes = [_vp, _vp]
lib.bvml_refiner_destroy.restype = None
lib.bvml_refiner_destroy.argtypes = [_vp]
lib.bvml_upsample_wait_limit.restype = ctypes.c_uint
lib.bvml_upsample_wait_limit.argtypes = [ctypes.c_uint]
lib.bvml_refine_halo_rows.restype = _i
lib.bvml_refine_halo_rows.argtypes = [_i, _i, _i]
lib.bvml_refiner_forward_banded.restype = _i
lib.bvml_refiner_forward_banded.argtypes = ([ctypes.POINTER(_vp), _i, _vp, _vp, _vp, _i, _i,
                                             ctypes.POINTER(ctypes.c_float)] + [_i] * 9 + [_vp])


def abi_version() -> int:
    return int(lib.bvml_abi_version())


def loaded_library() -> str:
    return LIB_PATH


def check(rc: int) -> None:
    if rc != BVML_OK:
        msg = lib.bvml_last_error().decode("utf-8", "replace")
        raise RuntimeError(msg or f"dsine ops: failed with status {rc}")
