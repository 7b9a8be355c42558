"""Build liblsrm_sparse.so (sm_100a) in-tree with nvcc.

    python large-sparse-reconstruction-model_b200/build.py [--jobs N] [--force] [--device-checks]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (skipped when up to
date), then all objects link into ``lsrm_sparse/liblsrm_sparse.so``.  The
library links the CUDA runtime statically and resolves the driver's tensor-map
encoder at run time, so it loads next to any PyTorch build.

``--device-checks`` builds a debug copy, ``lsrm_sparse/liblsrm_sparse_checked.so``
(objects under ``_build_checked/``), with -DLSRM_DEVICE_CHECKS: the kernels
test their data-dependent indices before use and report a failed test as
LSRM_ERR_BAD_INDEX plus a site bit in the error word instead of making the
access.  Load it by pointing ``lsrm_sparse._lib.LIB_PATH`` at it before the
first call.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(PKG_ROOT, "_build")
LIB = os.path.join(PKG_ROOT, "lsrm_sparse", "liblsrm_sparse.so")
BUILD_CHECKED = os.path.join(PKG_ROOT, "_build_checked")
LIB_CHECKED = os.path.join(PKG_ROOT, "lsrm_sparse", "liblsrm_sparse_checked.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I" + INCLUDE,
    "-I" + CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime(src: str) -> float:
    m = os.path.getmtime(src)
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".cuh", ".h")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def compile_one(src: str, force: bool, verbose_ptxas: bool, checked: bool = False) -> str:
    obj = os.path.join(BUILD_CHECKED if checked else BUILD, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= _deps_mtime(src):
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + (["-DLSRM_DEVICE_CHECKS"] if checked else []) + ["-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False, checked: bool = False) -> str:
    lib = LIB_CHECKED if checked else LIB
    os.makedirs(BUILD_CHECKED if checked else BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, verbose_ptxas, checked), srcs))
    if force or not os.path.exists(lib) or os.path.getmtime(lib) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", lib] + objs + ["-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--ptxas-v", action="store_true", help="print register / shared-memory usage")
    ap.add_argument("--device-checks", action="store_true", help="debug copy with device-side index checks")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.ptxas_v, a.device_checks))
