"""Failure detection on the host, without a GPU fault.

* refine_frame_banded: a band whose work raises is reported with its band
  index, grid rows and device, every worker thread is joined, and the other
  devices stop taking new bands; a band that never finishes makes the call
  raise TimeoutError naming the device, within the given timeout. The band
  work is replaced by a host-only fake, so nothing touches a GPU.
* the gather: ranks check each other in through the key-value store before
  the collective. A rank that fails between steps posts why and leaves; a
  rank that simply leaves posts nothing. In both cases the surviving rank
  raises RankFailure naming the rank within the timeout instead of hanging
  in the collective (two gloo ranks on 127.0.0.1).
"""
import os
import socket
import threading
import time

import pytest
import torch
import torch.multiprocessing as mp

from brovisionml_b200 import pipeline
from brovisionml_b200.sharding import RankFailure, gather_frames, report_failure


def _frame(h=64, w=16, iters=2, ps=5):
    P = ps * ps
    z = lambda c: torch.zeros((c, h, w))  # noqa: E731
    return pipeline.HostFrame(z(3), [z(P)] * iters, [z(2 * P)] * iters, [z(P)] * iters,
                              z(576), None)


def test_band_failure_names_band_and_device(monkeypatch):
    seen = []

    def fake(frame, out, d, j, *a):
        seen.append((d, j.own0))
        if j.own0 == 32:  # band 2 of eight 16-row bands, on device 0
            raise RuntimeError("simulated launch failure")
        if d == 1:
            time.sleep(0.05)
        out[:, 8 * j.own0:8 * j.own1] = 1.0

    monkeypatch.setattr(pipeline, "_refine_band", fake)
    fr = _frame(h=128)
    out = torch.zeros((3, 8 * 128, 8 * 16))
    before = set(threading.enumerate())
    with pytest.raises(pipeline.BandFailure) as ei:
        pipeline.refine_frame_banded(fr, out, 10.0, 8.0, 10.0, 64.0, n_bands=8, devices=(0, 1))
    msg = str(ei.value)
    assert "band 2" in msg and "cuda:0" in msg and "simulated launch failure" in msg
    assert "grid rows 32..47" in msg
    assert [f[0] for f in ei.value.failures] == [2]
    # every worker joined: no new thread is left running
    assert not [t for t in threading.enumerate() if t not in before and t.is_alive()]
    # device 0 took no band after its failing one, device 1 none after it saw the flag
    assert (0, 64) not in seen and (0, 96) not in seen
    assert len([1 for d, _ in seen if d == 1]) < 4


def test_band_timeout_names_device(monkeypatch):
    release = threading.Event()

    def fake(frame, out, d, j, *a):
        if d == 1:
            release.wait(30)  # a device that stops answering

    monkeypatch.setattr(pipeline, "_refine_band", fake)
    fr = _frame()
    out = torch.zeros((3, 8 * 64, 8 * 16))
    t0 = time.monotonic()
    with pytest.raises(TimeoutError) as ei:
        pipeline.refine_frame_banded(fr, out, 10.0, 8.0, 10.0, 32.0, n_bands=4, devices=(0, 1),
                                     timeout=0.5)
    assert time.monotonic() - t0 < 5
    assert "devices [1]" in str(ei.value) and "bands not finished" in str(ei.value)
    release.set()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, mode, q):
    import torch.distributed as dist
    from datetime import timedelta

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        local = torch.full((2, 3), float(rank))
        if rank == 1:
            if mode == "reports":
                report_failure(store, 7, rank, RuntimeError("band kernel failed on cuda:1"))
            q.put((rank, "left"))
            return  # leaves between steps, nothing in flight (os._exit below)
        t0 = time.monotonic()
        try:
            gather_frames(local, [2, 2], store=store, step=7, timeout=2.0)
            q.put((rank, "no error"))
        except RankFailure as e:
            q.put((rank, f"{type(e).__name__}: {e} after {time.monotonic() - t0:.1f}s"))
    finally:
        q.close()
        q.join_thread()  # the result is delivered before the process leaves
        # leave without tearing the group down: the other rank is already gone
        os._exit(0)


@pytest.mark.parametrize("mode", ["reports", "vanishes"])
def test_gather_reports_a_failed_rank(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    r0 = res[0]
    assert r0.startswith("RankFailure"), r0
    assert "rank 1" in r0
    if mode == "reports":
        assert "band kernel failed on cuda:1" in r0
    else:
        assert "did not arrive" in r0
    assert float(r0.rsplit("after ", 1)[1].rstrip("s")) < 10
