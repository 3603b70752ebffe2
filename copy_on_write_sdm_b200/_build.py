"""Build the in-tree sm_100a shared library ``libcowsdm.so`` with nvcc.

Each ``csrc/*.cu`` translation unit compiles in its own nvcc process (in
parallel), then nvcc links them into ``copy_on_write_sdm_b200/libcowsdm.so``.
A unit is rebuilt only when it, ``cow_common.cuh`` or the public header is
newer than its object file.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libcowsdm.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + CSRC]


def _nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libcowsdm.so")
    return path


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps_mtime() -> float:
    deps = [os.path.join(CSRC, "cow_common.cuh"), os.path.join(INCLUDE, "cow_sdm.h")]
    return max(os.path.getmtime(d) for d in deps if os.path.exists(d))


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [_nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr}")
    return res.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile (if stale) and link ``libcowsdm.so``; returns its path."""
    os.makedirs(OBJ, exist_ok=True)
    deps = _deps_mtime()
    jobs = []
    objs = []
    for src in _sources():
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), deps)
        if stale:
            jobs.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for log in ex.map(lambda j: _compile(j[0], j[1], verbose), jobs):
            if verbose and log:
                sys.stderr.write(log)
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        res = subprocess.run([_nvcc(), *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
