"""Failure detection without a GPU fault: the fused upsample's TMA staging
waits are bounded, and bvml_upsample_wait_limit(0) makes every one of them
give up at once, as if a copy were stuck. The call must still return, the
unit's status must report the upsample wait (bvml_refine_status), and -- with
the default bound restored -- the next call on the same stream must equal a
normal run bit for bit: the warps that gave up issued no further copies and
waited for the ones in flight before their CTA exited, so nothing of theirs
lands later and the context stays usable.
"""
import ctypes
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B", [2, 64])  # persistent AngMF path / one launch per iteration
def test_upsample_wait_that_gives_up_is_reported_and_the_next_call_is_normal(B):
    import bench
    import brovisionml_b200 as bv
    from brovisionml_b200._capi import lib

    dev = torch.device("cuda", 0)
    inp = bench.make_device_inputs(bench.CONFIGS["cfg4"], B, 907, dev, torch)
    h, w = inp["h"], inp["w"]
    ws = torch.empty(bv.refine_workspace_bytes(B, h, w), device=dev, dtype=torch.uint8)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def unit(out):
        bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"], inp["fu"],
                  inp["cu"], inp["fv"], inp["cv"], ray8=inp["ray8"], out=out, workspace=ws)
        return lib.bvml_refine_status(ctypes.c_void_p(ws.data_ptr()), stream)

    mk = lambda: torch.empty((B, 3, 8 * h, 8 * w), device=dev, dtype=inp["dt"])  # noqa: E731
    ref, bad, again = mk(), mk(), mk()
    assert unit(ref) == 0, lib.bvml_last_error()
    prev = lib.bvml_upsample_wait_limit(0)
    try:
        rc = unit(bad)
        msg = lib.bvml_last_error()
    finally:
        lib.bvml_upsample_wait_limit(prev)
    assert prev == 4194304
    assert rc != 0 and b"upsample staging wait gave up" in msg, (rc, msg)
    assert unit(again) == 0, lib.bvml_last_error()
    torch.cuda.synchronize()
    assert torch.equal(again, ref)
