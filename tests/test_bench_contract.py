"""bench.py's reference arm on the host (no GPU needed): one JSON line with
the contract's keys, the reference CPU path timed on a bounded sample, and
the reference-CUDA leg reporting itself unavailable when there is no GPU;
under a multi-rank launch only rank 0 prints."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    env.pop("MASTER_ADDR", None)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libbvml_ref.so")),
                    reason="reference twin not built")
def test_reference_arm_line():
    lines = _run({"CUDA_VISIBLE_DEVICES": ""})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["value"] > 0 and d["unit"] == "Mpixel/s" and d["higher_is_better"] is True
    assert d["config"]["workload"] == "cfg4"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "Mpixel/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert "unavailable" in d["reference_cuda"]


def test_reference_arm_other_ranks_print_nothing():
    assert _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
