"""Builds the native libraries in-tree.

* ``libmlb200.so``   — the sm_100a kernels, the decode runtime and the C ABI of
  include/mlb200.h (nvcc, ``-gencode arch=compute_100a,code=sm_100a``), linked
  against NCCL for tensor parallelism.
* ``libmlb_synth.so`` — the CPU side of the seeded synthetic-weight generator
  (g++, no CUDA).

Both land next to this file so they travel with the source tree.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libmlb200.so")
SYNTH_LIB = os.path.join(HERE, "libmlb_synth.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_dirs():
    """NCCL headers and library: the pip package torch uses, else the system one."""
    purelib = sysconfig.get_paths()["purelib"]
    pkg = os.path.join(purelib, "nvidia", "nccl")
    inc, lib = os.path.join(pkg, "include"), os.path.join(pkg, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _stale(target: str, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [
        os.path.join(ROOT, "include", "mlb200.h")]
    if not force and not _stale(LIB, deps):
        return LIB
    inc, lib = _nccl_dirs()
    # one nvcc per translation unit, in parallel, then one link
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
             "--expt-relaxed-constexpr", "-I", inc, "-I", os.path.join(ROOT, "include")]
    if verbose:
        flags.insert(0, "-Xptxas=-v")
    objs = [os.path.join(objdir, os.path.basename(s) + ".o") for s in srcs]

    def compile_one(pair):
        src, obj = pair
        subprocess.run([NVCC, *flags, "-c", "-o", obj, src], check=True)

    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        list(ex.map(compile_one, zip(srcs, objs)))
    subprocess.run([NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-L", lib,
                    "-l:libnccl.so.2", "-Xlinker", "-rpath=" + lib], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_synth(force: bool = False) -> str:
    src = os.path.join(CSRC, "synth_host.cc")
    deps = [src, os.path.join(CSRC, "synth.h")]
    if not force and not _stale(SYNTH_LIB, deps):
        return SYNTH_LIB
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-pthread",
           "-o", SYNTH_LIB + ".tmp", src]
    subprocess.run(cmd, check=True)
    os.replace(SYNTH_LIB + ".tmp", SYNTH_LIB)
    return SYNTH_LIB


def build(force: bool = False, verbose: bool = False) -> None:
    build_synth(force)
    build_cuda(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
