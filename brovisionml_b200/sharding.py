"""Work partitioning for the refine ops across the GPUs of one node.

The path has no data exchange between pixels of different frames, and a
frame's result at a pixel depends only on a bounded neighbourhood, so it
shards without any collective:

* frames   -- ``plan_frames``: contiguous, balanced frame ranges per rank
  (image-parallel batches);
* row-bands -- ``plan_bands``: one large frame cut into balanced bands of
  owned grid rows, each computed with a halo of
  ``halo_rows(iters, ps, dil) = iters * (ps // 2) * dil + 1`` extra rows per
  side (each AngMF iteration widens the dependency cone by the window radius
  times the dilation, the 3x3 upsample by one more row). Replicate padding is
  applied only at true image edges; interior band edges see real halo rows,
  and the rows the band edge contaminates are exactly the halo that is
  cropped away, so the stitched result equals the whole-frame result (up to
  fp32 rounding of the band-shifted principal point).
* ``plan_tiles`` restates the reference's tile planner
  (src/tile_runner.cpp:18-60) so a caller can report the reference's 2-D tile
  plan for a frame; the balanced bands are what the GPUs run, since 25 tiles
  of a 4096^2 frame cannot split evenly over 8 GPUs and tiles need
  feathering, while exact bands need none.

The only cross-GPU step is the final gather (``gather_frames`` /
``gather_bands``): each rank's owned output goes to rank 0 (torch.distributed
gather, NCCL over NVLink on GPUs, gloo on CPU) or is copied to host by each
rank.

Failure detection is on the host, between steps: before a collective, every
rank posts its status for that step in the process group's key-value store
(``check_ranks``), a rank that fails posts why (``report_failure``), and the
others learn of it -- or of a rank that never arrives -- from the store within
a timeout, before they enter the collective, and raise RankFailure naming the
rank. No GPU kernel waits on another rank.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence


def plan_frames(B: int, world: int) -> list[tuple[int, int]]:
    """Balanced contiguous (start, count) frame ranges, one per rank."""
    if world <= 0:
        raise ValueError("world must be positive")
    base, extra = divmod(max(B, 0), world)
    out, s = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((s, n))
        s += n
    return out


def halo_rows(iters: int, ps: int, dil: int, upsample: bool = True) -> int:
    """Grid rows of halo a band needs per side for an exact result of the
    refine OPS (given head outputs)."""
    return iters * (ps // 2) * dil + (1 if upsample else 0)


def refine_halo_rows(iters: int, ps: int = 5, dil: int = 1, upsample: bool = True) -> int:
    """Grid rows of halo a band needs per side for an exact result of the
    WHOLE learned refinement (ConvGRU + heads + ops), from the decoder's
    normal, feature and hidden state.

    With R = (ps // 2) * dil and n = 1 (the upsample's 3x3) or 0: iteration
    i's normals are needed n + (I - i) R rows out; AngMF reads the iteration's
    head outputs at its own pixel only, and the heads' 3x3 reads the hidden
    state h_i one row further; h_i at a row reads h_(i-1) four rows out (z and
    r: 5x5 over h; q: 5x5 over r * h), so
        need(h_I) = n + 1,  need(h_i) = max(n + (I - i) R + 1, need(h_(i+1)) + 4);
    the decoder's hidden state and feature (through the hoisted 5x5 terms of
    z, r and q) are read need(h_1) + 4 rows out, its normal n + I R rows out."""
    n = 1 if upsample else 0
    R = (ps // 2) * dil
    if iters <= 0:
        return n
    need = n + 1
    for i in range(iters - 1, 0, -1):
        need = max(n + (iters - i) * R + 1, need + 4)
    return max(need + 4, n + iters * R)


@dataclass(frozen=True)
class Band:
    own0: int    # first owned grid row
    own1: int    # one past the last owned grid row
    comp0: int   # first computed grid row (own0 - halo, clipped)
    comp1: int   # one past the last computed grid row (own1 + halo, clipped)

    @property
    def rows(self) -> int:
        return self.comp1 - self.comp0

    @property
    def crop_top(self) -> int:
        """Owned rows start this many grid rows into the computed band."""
        return self.own0 - self.comp0


def plan_bands(h: int, world: int, halo: int) -> list[Band]:
    """Balanced owned row-bands of an h-row grid, with halos clipped to the frame."""
    bands = []
    for own0, n in plan_frames(h, world):
        own1 = own0 + n
        bands.append(Band(own0, own1, max(0, own0 - halo), min(h, own1 + halo)))
    return bands


@dataclass(frozen=True)
class TileRect:
    x: int
    y: int
    w: int
    h: int
    ov_l: int = 0
    ov_r: int = 0
    ov_t: int = 0
    ov_b: int = 0


def _axis_starts(extent: int, tile: int, step: int) -> list[int]:
    if extent <= tile:
        return [0]
    starts, p = [], 0
    while True:
        if p + tile >= extent:
            starts.append(extent - tile)
            return starts
        starts.append(p)
        p += step


def plan_tiles(W: int, H: int, tile: int, overlap: int) -> list[TileRect]:
    """The reference's overlapping-tile plan (src/tile_runner.cpp:33-60):
    empty when tiling is off or the frame fits one tile; trailing tiles snap
    to the edge at full size; feather overlap only toward a neighbour."""
    if tile <= 0 or W <= 0 or H <= 0:
        return []
    if W <= tile and H <= tile:
        return []
    ov = min(max(overlap, 0), tile - 1)
    step = max(1, tile - ov)
    xs, ys = _axis_starts(W, tile, step), _axis_starts(H, tile, step)
    out = []
    for y in ys:
        th = min(tile, H - y)
        for x in xs:
            tw = min(tile, W - x)
            out.append(TileRect(x, y, tw, th, ov if x > 0 else 0, ov if x + tw < W else 0,
                                ov if y > 0 else 0, ov if y + th < H else 0))
    return out


def band_intrinsics(cv: float, band: Band) -> float:
    """Principal point v of a band: rows are re-indexed from comp0."""
    return cv - band.comp0


def gather_frames(local, counts: Sequence[int], group=None, *, store=None, step=None,
                  timeout: float = 60.0):
    """Gather each rank's (count_r, ...) output to rank 0 (torch.distributed).

    Returns the concatenated tensor on rank 0 and None elsewhere. Every rank
    must call it (a collective). Without an initialised process group (one
    process) the local part is the whole result. With a key-value ``store``,
    the ranks first check each other in for ``step`` (check_ranks, bounded by
    ``timeout`` seconds): a rank that failed or left is reported as
    RankFailure on every other rank instead of a hang in the collective."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        if len(counts) != 1:
            raise RuntimeError("gather_frames: several ranks' counts but no process group")
        return local[: counts[0]]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if store is not None:
        check_ranks(store, step, rank, world, timeout)
    mx = max(counts)
    pad_shape = (mx,) + tuple(local.shape[1:])
    send = torch.zeros(pad_shape, dtype=local.dtype, device=local.device)
    if local.shape[0]:
        send[: local.shape[0]].copy_(local)
    recv = [torch.empty_like(send) for _ in range(world)] if rank == 0 else None
    dist.gather(send, recv, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([recv[r][: counts[r]] for r in range(world)], dim=0)


def gather_bands(local_rows, bands: Sequence[Band], group=None, row_dim: int = -2,
                 scale: int = 8, **check):
    """Gather owned output rows (scale x grid rows) of every band to rank 0 and
    stitch them along ``row_dim``. Returns the frame on rank 0, None elsewhere.
    ``check`` (store, step, timeout) as for gather_frames."""
    counts = [scale * (b.own1 - b.own0) for b in bands]
    moved = local_rows.movedim(row_dim, 0).contiguous()
    full = gather_frames(moved, counts, group, **check)
    return None if full is None else full.movedim(0, row_dim).contiguous()


class RankFailure(RuntimeError):
    """Ranks that reported a failure, or did not arrive in time, for a step."""

    def __init__(self, step, failed: dict, missing: list):
        self.step, self.failed, self.missing = step, failed, missing
        parts = [f"rank {r} failed: {m}" for r, m in sorted(failed.items())]
        parts += [f"rank {r} did not arrive" for r in missing]
        super().__init__(f"dsine ops: step {step}: " + "; ".join(parts))


def _key(step, rank: int) -> str:
    return f"bvml/step/{step}/rank/{rank}"


def report_failure(store, step, rank: int, exc: BaseException | str) -> None:
    """A rank that cannot take part in `step` posts why (then leaves)."""
    store.set(_key(step, rank), ("failed: " + str(exc)).encode())


def check_ranks(store, step, rank: int, world: int, timeout: float) -> None:
    """Post this rank's arrival for `step` and wait (up to `timeout` seconds)
    until every rank has posted; raise RankFailure if any rank reported a
    failure or did not arrive. Call it before each collective of the step."""
    import time

    store.set(_key(step, rank), b"ok")
    deadline = time.monotonic() + timeout
    failed, pending = {}, [r for r in range(world) if r != rank]
    while pending:
        still = []
        for r in pending:
            k = _key(step, r)
            if store.check([k]):
                v = store.get(k).decode()
                if v != "ok":
                    failed[r] = v[len("failed: "):] if v.startswith("failed: ") else v
            else:
                still.append(r)
        pending = still
        if failed:
            break
        if pending and time.monotonic() > deadline:
            break
        if pending:
            time.sleep(0.01)
    if failed or pending:
        raise RankFailure(step, failed, [] if failed else pending)
