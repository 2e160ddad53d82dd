"""Build libasdsl_b200.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed), and beside it
libasdsl_b200_timeline.so, the same sources with the per-CTA timeline records compiled in
(ASDSL_B200_TIMELINE=1; loaded instead of the default library when ASDSL_B200_TIMELINE=1 is set).

    python -m asdsl_b200.build [--force] [--timeline | --all]
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(ROOT, "csrc")
REPO = os.path.dirname(ROOT)
LIB = os.path.join(PKG, "libasdsl_b200.so")
LIB_TIMELINE = os.path.join(PKG, "libasdsl_b200_timeline.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(REPO, "include", "*.h")))


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(s) <= t for s in sources())


def _command(lib: str, verbose: bool) -> list[str]:
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", lib + ".tmp", os.path.join(CSRC, "asdsl_b200.cu")]
    if lib == LIB_TIMELINE:
        cmd.insert(1, "-DASDSL_B200_TIMELINE=1")
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    return cmd


def build_library(force: bool = False, verbose: bool = False, timeline: bool = False) -> str:
    lib = LIB_TIMELINE if timeline else LIB
    if not force and up_to_date(lib):
        return lib
    subprocess.run(_command(lib, verbose), check=True)
    os.replace(lib + ".tmp", lib)
    return lib


def build_all(force: bool = False) -> list[str]:
    """Both libraries, compiled concurrently."""
    todo = [lib for lib in (LIB, LIB_TIMELINE) if force or not up_to_date(lib)]
    procs = [(lib, subprocess.Popen(_command(lib, False))) for lib in todo]
    failed = [lib for lib, p in procs if p.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    for lib in todo:
        os.replace(lib + ".tmp", lib)
    return [LIB, LIB_TIMELINE]


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--timeline", action="store_true", help="only the timeline build")
    ap.add_argument("--all", action="store_true", help="both libraries")
    a = ap.parse_args()
    print(build_all(a.force) if a.all else build_library(a.force, a.verbose, a.timeline))
