"""Build libbvml_dsine.so (the CUDA kernels + C ABI) for sm_100a, in-tree.

    python brovisionml_b200/build.py [--ptxas]

(Run it by path: importing the package loads the library, which may be stale
or missing before this script has run.)

Compiles each brovisionml_b200/csrc/*.cu with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` (B200 only) and links them into
``brovisionml_b200/_lib/libbvml_dsine.so``. The C++ drop-in bridge
(csrc/dsine_ops_b200.cpp) is compiled into ``_lib/libbvml_dsine_bridge.so``
against the stand-in brotensor header, to prove that it builds.
Rebuilds only what changed (source / header mtimes).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "_lib")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(LIB_DIR, "libbvml_dsine.so")
# The same sources with -DBVML_CHECKED: every kernel tests its indices and TMA
# coordinates before each access and records failures (bvml_check_word); the
# GPU tests run the odd shapes through it.
CHECKED_LIB = os.path.join(LIB_DIR, "libbvml_dsine_checked.so")
BRIDGE = os.path.join(LIB_DIR, "libbvml_dsine_bridge.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build brovisionml_b200")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile (if stale) and return the path of libbvml_dsine.so."""
    nvcc = _nvcc()
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    headers = (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
               + glob.glob(os.path.join(ROOT, "include", "*.h")))
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = []
    objs = []
    cobjs = []
    for src in sources:
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if _stale(obj, [src] + headers) or ptxas_info:
            cmd = [nvcc] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + \
                  ["-c", src, "-o", obj]
            jobs.append(cmd)
        cobj = os.path.join(OBJ_DIR, "checked_" + os.path.basename(src)[:-3] + ".o")
        cobjs.append(cobj)
        if _stale(cobj, [src] + headers):
            jobs.append([nvcc] + ARCH + NVCC_FLAGS + ["-DBVML_CHECKED", "-c", src, "-o", cobj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for out in ex.map(run, jobs):
            if verbose or ptxas_info:
                sys.stdout.write(out)
    if _stale(LIB, objs + [__file__]):
        # Shared cudart: callers (torch, or a brotensor runtime) hand in stream
        # handles created by THEIR CUDA runtime; one shared runtime instance
        # per process is what makes those handles valid here too.
        run([nvcc] + ARCH + ["-shared", "-cudart", "shared", "-o", LIB] + objs +
            ["-Xlinker", "-rpath,/usr/local/cuda/lib64"])
    if _stale(CHECKED_LIB, cobjs + [__file__]):
        run([nvcc] + ARCH + ["-shared", "-cudart", "shared", "-o", CHECKED_LIB] + cobjs +
            ["-Xlinker", "-rpath,/usr/local/cuda/lib64"])

    bridge_src = os.path.join(CSRC, "dsine_ops_b200.cpp")
    if os.path.exists(bridge_src):
        deps = [bridge_src, LIB] + headers + glob.glob(os.path.join(CSRC, "brotensor_shim", "*", "*.h"))
        if _stale(BRIDGE, deps):
            cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
            cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc)), "include")
            cmd = [cxx, "-O2", "-std=c++20", "-fPIC", "-shared", "-Wall", "-Wextra",
                   "-I" + os.path.join(CSRC, "brotensor_shim"), "-I" + os.path.join(ROOT, "include"),
                   "-I" + cuda_inc, "-DBVML_SHIM_CUDA", bridge_src, "-o", BRIDGE,
                   "-L" + LIB_DIR, "-lbvml_dsine", "-Wl,-rpath,$ORIGIN",
                   "-L" + os.path.join(os.path.dirname(os.path.dirname(nvcc)), "lib64"), "-lcudart", "-Wl,--exclude-libs,ALL"]
            run(cmd)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))
