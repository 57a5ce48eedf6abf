"""Builds the in-tree shared libraries.

* ``libsf_b200.so``            -- every CUDA kernel plus the C ABI (include/splatforge_b200.h),
                                  compiled for sm_100a only.
* ``libsf_b200_hostcheck.so``  -- the same arithmetic headers compiled for the host, used
                                  only by the CPU test-suite.

``python -m splatforge_b200.build`` rebuilds what is out of date (a digest of the
sources is kept next to each library).
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libsf_b200.so"
HOSTCHECK = PKG / "libsf_b200_hostcheck.so"
CUDA_SOURCES = ("preprocess.cu", "binning.cu", "raster.cu", "composite.cu", "opacity_field.cu", "geometry.cu", "meshing.cu", "training.cu", "capi.cu",
                "binning_static.cu")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _digest(paths, extra=""):
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def sources_digest():
    files = [CSRC / s for s in CUDA_SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    files += sorted(INCLUDE.glob("*.h"))
    return _digest(files, " ".join(ARCH))


def _stale(lib, digest):
    stamp = lib.with_suffix(".sha256")
    return not lib.exists() or not stamp.exists() or stamp.read_text().strip() != digest


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsf_b200.so")


def build_library(force=False, verbose=False):
    digest = sources_digest()
    if not force and not _stale(LIB, digest):
        return LIB
    build = PKG / "_build"
    build.mkdir(exist_ok=True)
    objs = []
    cmd_base = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                "-I", str(INCLUDE), "-I", str(CSRC)]
    for src in CUDA_SOURCES:
        obj = build / (Path(src).stem + ".o")
        cmd = cmd_base + ["-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs], check=True)
    os.replace(tmp, LIB)
    LIB.with_suffix(".sha256").write_text(digest)
    return LIB


def build_hostcheck(force=False):
    files = [CSRC / "hostcheck.cpp"] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    digest = _digest(files, "hostcheck")
    if not force and not _stale(HOSTCHECK, digest):
        return HOSTCHECK
    cxx = os.environ.get("CXX", "g++")
    tmp = HOSTCHECK.with_suffix(".so.tmp")
    subprocess.run(
        [cxx, "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
         "-I", str(INCLUDE), "-I", str(CSRC), str(CSRC / "hostcheck.cpp"), "-o", str(tmp)],
        check=True,
    )
    os.replace(tmp, HOSTCHECK)
    HOSTCHECK.with_suffix(".sha256").write_text(digest)
    return HOSTCHECK


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_library(force=force, verbose="-v" in sys.argv))
    print(build_hostcheck(force=force))
