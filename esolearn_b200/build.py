"""Builds libscryb200.so (all CUDA sources in csrc/) for sm_100a with nvcc.

The library is built in-tree (esolearn_b200/libscryb200.so) so that it travels
with the repository to the GPU host.  Usage: ``python -m esolearn_b200.build``.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libscryb200.so")
OBJ = os.path.join(PKG, "_build")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
# SB_STEP_TIMELINE=1: the profiling build, with the persistent step's phase
# timeline compiled in (sb_llama_set_timeline); the default build has none.
if os.environ.get("SB_STEP_TIMELINE") == "1":
    FLAGS.append("-DSB_STEP_TIMELINE")


def _needs(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(ROOT, "include", "sb_api.h")]
    objs, cmds = [], []
    for src in sources:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or ptxas_info or _needs(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            cmds.append(cmd)
    # Translation units compile independently; the persistent decode step's
    # instantiation units dominate, so they run side by side.
    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        return subprocess.run(cmd, capture_output=True, text=True)
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        results = list(ex.map(run, cmds))
    for cmd, r in zip(cmds, results):
        if r.stdout or r.stderr:
            sys.stdout.write(r.stdout)
            sys.stderr.write(r.stderr)
        if r.returncode != 0:
            raise subprocess.CalledProcessError(r.returncode, cmd)
    if force or _needs(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas" in sys.argv, force="--force" in sys.argv)
    print(LIB)
