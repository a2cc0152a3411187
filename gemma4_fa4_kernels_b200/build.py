"""Build ``libgemma4_b200.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m gemma4_fa4_kernels_b200.build`` (or ``build_library()``).
Objects go to ``<repo>/_build`` and the shared library next to this file, so
it travels with the source tree.  The CUDA runtime is linked statically; the
driver's TMA encoder is fetched at run time, so no ``-lcuda`` is needed.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
ROOT = os.path.dirname(PKG_DIR)
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_NAME = "libgemma4_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; install the CUDA toolkit (12.8+)")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    lib_mtime = os.path.getmtime(LIB_PATH)
    deps = _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return all(os.path.getmtime(d) <= lib_mtime for d in deps)


def _compile(nvcc: str, src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile every kernel source and link the shared library; returns its path."""
    if not force and _up_to_date():
        return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), _sources()))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
