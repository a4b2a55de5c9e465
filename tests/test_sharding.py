"""CPU tests of the multi-GPU partitioning host logic.

The exactness of halo row-bands is checked with the CPU oracle (bands
computed separately and stitched == the whole frame), and the gather is run
as a real 2-rank torch.distributed job over gloo on 127.0.0.1.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from brovisionml_b200.sharding import (Band, band_intrinsics, gather_bands, gather_frames,
                                       halo_rows, plan_bands, plan_frames, plan_tiles)
from oracle import oracle as O


def test_plan_frames_balanced_and_covering():
    for B in (0, 1, 7, 16, 256):
        for world in (1, 2, 3, 8):
            p = plan_frames(B, world)
            assert len(p) == world
            assert sum(n for _, n in p) == B
            assert max(n for _, n in p) - min(n for _, n in p) <= 1
            s = 0
            for st, n in p:
                assert st == s
                s += n


def test_halo_rows_formula():
    assert halo_rows(5, 7, 1) == 16          # the 4096^2 / 7x7 case: 128 full-res px
    assert halo_rows(5, 5, 2) == 21
    assert halo_rows(1, 5, 1, upsample=False) == 2


def test_plan_bands():
    bands = plan_bands(512, 8, 16)
    assert bands[0] == Band(0, 64, 0, 80)
    assert bands[3] == Band(192, 256, 176, 272)
    assert bands[-1] == Band(448, 512, 432, 512)
    owned = np.zeros(512, int)
    for b in bands:
        owned[b.own0:b.own1] += 1
        assert b.crop_top == b.own0 - b.comp0
    assert (owned == 1).all()


def test_plan_tiles_reference_cases():
    # the 4096^2 frame as 1024 tiles with 128 overlap: 5 x 5 tiles, last snapped
    t = plan_tiles(4096, 4096, 1024, 128)
    assert len(t) == 25
    xs = sorted({r.x for r in t})
    assert xs == [0, 896, 1792, 2688, 3072]
    assert all(r.w == 1024 and r.h == 1024 for r in t)
    corner = [r for r in t if r.x == 0 and r.y == 0][0]
    assert corner.ov_l == 0 and corner.ov_t == 0 and corner.ov_r == 128 and corner.ov_b == 128
    # disabled / fits in one tile -> empty plan; overlap clamped below the tile
    assert plan_tiles(100, 100, 0, 0) == [] and plan_tiles(100, 100, 128, 8) == []
    t = plan_tiles(300, 50, 100, 500)
    assert all(r.ov_l in (0, 99) for r in t)
    cover = np.zeros((50, 300), int)
    for r in t:
        cover[r.y:r.y + r.h, r.x:r.x + r.w] = 1
    assert cover.all()


def _band_inputs(u: O.UnitInputs, b: Band) -> O.UnitInputs:
    sl = slice(b.comp0, b.comp1)
    return O.UnitInputs(**{**u.__dict__, "h": b.rows, "H": 8 * b.rows,
                           "cv": band_intrinsics(u.cv, b),
                           "normal0": np.ascontiguousarray(u.normal0[:, :, sl]),
                           "ray8": np.ascontiguousarray(u.ray8[:, sl]),
                           "prob": [np.ascontiguousarray(a[:, :, sl]) for a in u.prob],
                           "xy": [np.ascontiguousarray(a[:, :, sl]) for a in u.xy],
                           "angle": [np.ascontiguousarray(a[:, :, sl]) for a in u.angle],
                           "mask": np.ascontiguousarray(u.mask[:, :, sl])})


def _run_band(u, b):
    ub = _band_inputs(u, b)
    out = O.refine_unit(ub, crop=(8 * b.crop_top, 0, 8 * (b.own1 - b.own0), 8 * u.w))
    return out


@pytest.mark.parametrize("ps,dil,iters", [(5, 1, 2), (7, 1, 1), (5, 2, 1)])
def test_halo_bands_are_exact_with_oracle(ps, dil, iters):
    u = O.gen_unit(8 * 40, 8 * 12, 1, ps=ps, dil=dil, iters=iters, seed=21)
    full = O.refine_unit(u)
    bands = plan_bands(u.h, 3, halo_rows(iters, ps, dil))
    parts = [_run_band(u, b) for b in bands]
    stitched = np.concatenate(parts, axis=2)
    assert stitched.shape == full.shape
    assert np.abs(stitched - full).max() < 1e-5
    # one row less of halo is NOT enough (the formula is tight)
    short = plan_bands(u.h, 3, halo_rows(iters, ps, dil) - 1)
    parts = [_run_band(u, b) for b in short]
    assert np.abs(np.concatenate(parts, axis=2) - full).max() > 1e-4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # frames: each rank "computes" its frames (oracle) and rank 0 gathers
        u = O.gen_unit(64, 48, 5, iters=1, seed=31)
        plan = plan_frames(u.B, world)
        st, n = plan[rank]
        sub = O.UnitInputs(**{**u.__dict__, "B": n,
                              "normal0": u.normal0[st:st + n],
                              "prob": [a[st:st + n] for a in u.prob],
                              "xy": [a[st:st + n] for a in u.xy],
                              "angle": [a[st:st + n] for a in u.angle],
                              "mask": u.mask[st:st + n]})
        local = torch.from_numpy(O.refine_unit(sub))
        got = gather_frames(local, [c for _, c in plan])
        # bands of one frame
        u1 = O.gen_unit(8 * 24, 8 * 10, 1, iters=2, seed=32)
        bands = plan_bands(u1.h, world, halo_rows(2, 5, 1))
        part = torch.from_numpy(_run_band(u1, bands[rank]))
        frame = gather_bands(part, bands)
        if rank == 0:
            e1 = float(np.abs(got.numpy() - O.refine_unit(u)).max())
            e2 = float(np.abs(frame.numpy() - O.refine_unit(u1)).max())
            q.put((e1, e2))
    finally:
        dist.destroy_process_group()


def test_gather_with_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    e1, e2 = q.get(timeout=5)
    assert e1 == 0.0
    assert e2 < 1e-5


@pytest.mark.parametrize("h,n,iters,ps,dil", [(90, 4, 5, 5, 1), (128, 8, 5, 5, 2), (512, 3, 5, 7, 1),
                                              (7, 16, 2, 3, 1), (1, 1, 5, 5, 1)])
def test_band_jobs_tile_the_frame(h, n, iters, ps, dil):
    """The large-frame driver's jobs: owned rows tile the grid exactly, each
    band computes its owned rows plus the exact halo (clipped at the frame),
    and its crop selects exactly the owned 8x output rows."""
    from brovisionml_b200.pipeline import plan_band_jobs
    from brovisionml_b200.sharding import halo_rows

    jobs = plan_band_jobs(h, n, iters, ps, dil)
    halo = halo_rows(iters, ps, dil)
    assert jobs[0].own0 == 0 and jobs[-1].own1 == h
    for a, b in zip(jobs, jobs[1:]):
        assert a.own1 == b.own0
    for j in jobs:
        assert j.own1 > j.own0
        assert j.comp0 == max(0, j.own0 - halo) and j.comp1 == min(h, j.own1 + halo)
        assert j.crop_t == 8 * (j.own0 - j.comp0) and j.out_h == 8 * (j.own1 - j.own0)
        assert j.crop_t + j.out_h <= 8 * (j.comp1 - j.comp0)
    assert len(jobs) == min(n, h)
