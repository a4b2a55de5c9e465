"""The fused unit's AngMF launches after the first, and its upsample, are
programmatic dependent launches: their CTAs may start during the previous
launch's last wave, issue what does not depend on it (their own per-neighbour
inputs, the mask) and wait (griddepcontrol.wait) before they read its normals.
A CUDA event recorded between two launches -- bvml_probe_events armed --
removes that overlap, so the same unit with probes armed runs fully
serialised. Both must give bit-identical results, on the per-iteration path
(64 frames of a 720p grid: 4.3 waves of tiles per iteration) and on the
persistent path (8 frames), back to back on one stream so that each unit's
first launch also follows the previous unit's upsample.
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


@pytest.mark.parametrize("B,launches", [(64, 6), (8, 2)])
def test_overlapped_launches_equal_serialised(B, launches):
    import bench
    import brovisionml_b200 as bv

    dev = torch.device("cuda", 0)
    cfg = bench.CONFIGS["cfg4"]
    inp = bench.make_device_inputs(cfg, B, 811, dev, torch)
    h, w = inp["h"], inp["w"]

    def unit(out):
        bv.refine(inp["normal0"], inp["prob"], inp["xy"], inp["angle"], inp["mask"], inp["fu"],
                  inp["cu"], inp["fv"], inp["cv"], ray8=inp["ray8"], out=out)

    outs = [torch.empty((B, 3, 8 * h, 8 * w), device=dev, dtype=inp["dt"]) for _ in range(4)]
    unit(outs[0])           # overlapped
    unit(outs[1])           # overlapped, right after the previous unit
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(launches + 1)]
    for e in evs:           # torch creates the CUDA event at its first record
        e.record()
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * len(evs))(*[ctypes.c_void_p(e.cuda_event) for e in evs])
    bv.check(bv.lib.bvml_probe_events(arr, len(evs)))
    try:
        unit(outs[2])       # serialised: an event between every two launches
        recorded = int(bv.lib.bvml_probe_recorded())
    finally:
        bv.lib.bvml_probe_events(None, 0)
    unit(outs[3])
    torch.cuda.synchronize()
    assert recorded == launches + 1, recorded
    for k in (1, 2, 3):
        assert torch.equal(outs[0], outs[k]), k
