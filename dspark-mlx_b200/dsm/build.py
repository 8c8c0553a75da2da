"""Build ``libdsm.so`` (all CUDA sources under ``csrc/``) for sm_100a, in-tree.

    python -m dsm.build [--force] [--jobs N]

Each ``.cu`` is compiled separately (relocatable device code) in parallel, then nvcc
device-links and links the shared library next to this file. The CUDA runtime is linked
statically so the library does not depend on which ``libcudart`` the host process loaded.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include")
BUILD_DIR = os.path.join(os.path.dirname(PKG_DIR), "_build")
LIB_PATH = os.path.join(PKG_DIR, "libdsm.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(SRC_DIR, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(SRC_DIR, "*.cuh")) + glob.glob(os.path.join(INCLUDE_DIR, "*.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def _compile(src: str, verbose_ptxas: bool) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    cmd = [_nvcc(), *ARCH, *FLAGS, "-I", INCLUDE_DIR, "-I", SRC_DIR, "-dc", src, "-o", obj]
    if verbose_ptxas:
        cmd[cmd.index("-warn-spills")] = "-v"
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False) -> str:
    if not force and not _stale():
        return LIB_PATH
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose_ptxas=a.ptxas_verbose))


if __name__ == "__main__":
    main()
