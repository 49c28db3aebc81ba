"""Builds ``tikun_b200/lib/libtikun_cuda.so`` from ``tikun_b200/csrc`` with nvcc.

sm_100a only.  The library links the CUDA runtime statically and exports only
the ``tk_*`` C-ABI symbols declared in ``include/tikun_cuda.h``.  Objects are
rebuilt when a source or header is newer than the library.

    python -m tikun_b200.build [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "lib")
OBJ_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(LIB_DIR, "libtikun_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the tikun_b200 CUDA library cannot be built")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _deps() -> list[str]:
    return _sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(
        os.path.join(CSRC, "*.cuh")) + [os.path.join(REPO, "include", "tikun_cuda.h"),
                                        os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def _compile(src: str) -> str:
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    cmd = [nvcc(), "-c", src, "-o", obj, "-O3", "-std=c++17", *ARCH, "-lineinfo",
           "-I", os.path.join(REPO, "include"), "-I", CSRC,
           "-Xcompiler", "-fPIC,-fvisibility=hidden,-ffp-contract=off",
           "-Xptxas", "-warn-spills"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = True) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(_compile, srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-shared", "-o", tmp, *objs, *ARCH, "-cudart", "static",
           "-Xcompiler", "-fPIC", "-Xlinker", "--exclude-libs,ALL"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
