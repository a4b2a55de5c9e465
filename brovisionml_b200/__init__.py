"""brovisionml_b200 -- B200-native (sm_100a) DSINE refine ops.

The product is the CUDA library ``_lib/libbvml_dsine.so`` and its C ABI
(``include/bvml_dsine.h``). This package loads that library and mirrors the
reference's op interface (``brovisionml::dsine::ray_relu`` /
``angmf_propagate`` in include/brovisionml/dsine_ops.h:25-54, plus the
brotensor convex-upsample / L2-normalise / slice calls of
src/dsine_refine.cpp:277-292) for Python callers, with torch tensors as the
device-memory carrier. Every op runs in the CUDA library; there is no CPU or
PyTorch fallback, and importing the package fails loudly when the library is
missing.

Errors raise ``RuntimeError`` carrying the library's message, worded like the
reference's exceptions ("dsine ops: ..." / "dsine cuda: ...").
"""
from __future__ import annotations

from ._capi import (BVML_F16, BVML_F32, LIB_PATH, abi_version, check, lib,  # noqa: F401
                    loaded_library)
from .ops import (angmf_propagate, conv2d_nhwc, convex_upsample, l2_normalize_nchw,  # noqa: F401
                  pack_conv_weight, ray_relu, refine, refine_workspace_bytes, slice2d)

__all__ = ["ray_relu", "angmf_propagate", "convex_upsample", "l2_normalize_nchw", "slice2d",
           "conv2d_nhwc", "pack_conv_weight",
           "refine", "refine_workspace_bytes", "lib", "abi_version", "loaded_library",
           "LIB_PATH", "BVML_F32", "BVML_F16"]
