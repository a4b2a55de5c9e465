"""Generate the golden fixtures of tests/golden/ from the reference itself.

Runs the reference's own CPU twin (src/dsine_ops.cpp of wlejon/brovisionml,
compiled in place by oracle/Makefile into oracle/_ref/libbvml_ref.so) on
small seeded inputs and stores inputs and outputs, so that the oracle
restatement can be pinned to the reference on machines without the
reference tree:

    make -C oracle && python tests/golden/make_golden.py

Cases (all 5x5 window, dilation 1, fp32, single frame -- the reference's
only shape):
  rand_12x16   seeded generator inputs (camera-facing normals), 12x16 grid
  away_12x16   normals flipped to face away (RayReLU clamps almost all)
  edge_9x7     odd grid with hand-placed degeneracies: zero xy pairs, tiny
               and zero angles, angle pi, a zero normal, a neighbour with
               (P+d).n ~ 0 (ref_angmf_raw runs AngMF on the raw normals so
               these reach the propagate unclamped)
  cfg0_60x80   config 0 (480x640 image, seed 0): outputs only, plus the
               SHA-256 of the regenerated inputs
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402


def input_digest(u: O.UnitInputs, it: int = 0) -> str:
    h = hashlib.sha256()
    for a in (u.normal0, u.ray8, u.prob[it], u.xy[it], u.angle[it]):
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def run_ref(u: O.UnitInputs):
    n = O.ray_relu(u.normal0[0], u.ray8, use_ref=True)
    a = O.angmf(n, u.prob[0][0], u.xy[0][0], u.angle[0][0], u.ray8, u.fu, u.cu, u.fv, u.cv,
                use_ref=True)
    return n, a


def run_ref_raw(u: O.UnitInputs):
    """AngMF straight on normal0 (no RayReLU first), so hand-placed normals
    (zero, non-unit, (P+d).n ~ 0) reach the propagate unchanged."""
    return O.angmf(u.normal0[0], u.prob[0][0], u.xy[0][0], u.angle[0][0], u.ray8, u.fu, u.cu,
                   u.fv, u.cv, use_ref=True)


def edge_case() -> O.UnitInputs:
    u = O.gen_unit(72, 56, 1, iters=1, seed=7, upsample=False)  # grid 9x7
    xy, ang, nrm = u.xy[0][0], u.angle[0][0], u.normal0[0]
    xy[0, 0, 0] = xy[25, 0, 0] = 0.0          # zero xy pair
    xy[3, 4, 4] = 1e-30                        # |xy| below the 1e-12 clamp
    xy[28, 4, 4] = 0.0
    ang[5, 2, 3] = 0.0
    ang[6, 2, 3] = 1e-7                        # Taylor branch
    ang[7, 2, 3] = np.float32(np.pi)
    ang[8, 8, 6] = 3.0
    nrm[:, 5, 1] = 0.0                         # zero normal (not renormalised)
    nrm[:, 6, 2] = [0.3, -0.2, 0.5]            # non-unit normal
    # make neighbour slot 12 (centre) of pixel (3,3) have (P + d).n ~ 0:
    # pick n orthogonal to P + d for the pixel's own xy offset
    y, x = 3, 3
    xs, ys = xy[12, y, x], xy[37, y, x]
    r = 1.0 / max(np.hypot(xs, ys), 1e-12)
    tu = (x + 0.5 + xs * r - u.cu) / u.fu
    tv = (y + 0.5 + ys * r - u.cv) / u.fv
    q = np.array([tu, tv, 1.0])
    n = np.cross(q, [0.0, 1.0, 0.0])
    n /= np.linalg.norm(n)
    nrm[:, y, x] = n
    return u


def main() -> None:
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libbvml_ref.so missing: run `make -C oracle` with the "
                         "reference tree present")
    cases = {
        "rand_12x16": O.gen_unit(96, 128, 1, iters=1, seed=3, upsample=False),
        "away_12x16": O.gen_unit(96, 128, 1, iters=1, seed=4, upsample=False,
                                 face_camera=False),
        "edge_9x7": edge_case(),
    }
    for name, u in cases.items():
        n, a = run_ref(u)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"), normal0=u.normal0[0], ray8=u.ray8,
            prob=u.prob[0][0], xy=u.xy[0][0], angle=u.angle[0][0],
            intr=np.array([u.fu, u.cu, u.fv, u.cv], np.float64), ref_ray_relu=n, ref_angmf=a,
            ref_angmf_raw=run_ref_raw(u))
        print(name, a.shape)
    u = O.gen_unit(480, 640, 1, iters=1, seed=0, upsample=False)
    n, a = run_ref(u)
    np.savez_compressed(os.path.join(HERE, "cfg0_60x80.npz"), ref_ray_relu=n, ref_angmf=a,
                        intr=np.array([u.fu, u.cu, u.fv, u.cv], np.float64),
                        input_sha256=np.array(input_digest(u)))
    print("cfg0_60x80", a.shape, input_digest(u)[:16])


if __name__ == "__main__":
    main()
