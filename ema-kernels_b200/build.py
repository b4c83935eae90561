"""Build libema_ssd_b200.so (sm_100a) in-tree.

Each ``csrc/*.cu`` compiles to an object in ``_build/`` (in parallel), then the
objects link into ``kernels/libema_ssd_b200.so`` next to the Python package
that loads it.  nvcc cross-compiles: no GPU is needed to build.

    python ema-kernels_b200/build.py [--force] [--jobs N]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "kernels", "libema_ssd_b200.so")
# test-only library (tcgen05 operand self-test), kept out of the product library
SELFTEST_SRC = os.path.join(ROOT, "tests", "native", "tc_selftest.cu")
SELFTEST_LIB = os.path.join(ROOT, "tests", "native", "libema_selftest_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def _nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found")
    return exe


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, f)
                                                                for f in os.listdir(INCLUDE)]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj, verbose):
    cmd = [_nvcc(), *ARCH, *CFLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    objs = [os.path.join(BUILD, s[:-3] + ".o") for s in srcs]
    todo = [(os.path.join(CSRC, s), o) for s, o in zip(srcs, objs) if force or _stale(o, deps)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for log in ex.map(lambda so: _compile(so[0], so[1], verbose), todo):
                if verbose and log:
                    sys.stderr.write(log)
    if force or todo or _stale(LIB, objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_selftest(force)
    return LIB


def build_selftest(force: bool = False) -> str:
    """tests/native/libema_selftest_b200.so: the tcgen05 operand self-test the GPU
    tests run (not part of the product library)."""
    deps = _deps() + [SELFTEST_SRC, os.path.join(os.path.dirname(SELFTEST_SRC), "ema_selftest_b200.h")]
    if force or _stale(SELFTEST_LIB, deps):
        cmd = [_nvcc(), *ARCH, *CFLAGS, "-I", os.path.dirname(SELFTEST_SRC), "-shared", "-o", SELFTEST_LIB,
               SELFTEST_SRC, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {SELFTEST_SRC}:\n{r.stdout}\n{r.stderr}")
    return SELFTEST_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
