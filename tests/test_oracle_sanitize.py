"""Host-side sanitizers on the oracle (compute-sanitizer is closed on this
pool, and the oracle is the checker every GPU result is measured against):
oracle/dsine_oracle.c built with AddressSanitizer and UndefinedBehavior-
Sanitizer and run over odd shapes, every window / dilation, crops and the
full-resolution RayReLU (tests/oracle_sanitize_main.c)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_oracle_under_asan_ubsan(tmp_path):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    exe = str(tmp_path / "oracle_sanitize")
    cmd = [cc, "-O1", "-g", "-ffp-contract=off", "-fno-omit-frame-pointer",
           "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
           os.path.join(ROOT, "oracle", "dsine_oracle.c"),
           os.path.join(ROOT, "tests", "oracle_sanitize_main.c"), "-o", exe, "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0",
               UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count("case ") == 36 and "rc=-1" not in r.stdout
