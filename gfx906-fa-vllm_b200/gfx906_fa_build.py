"""Build the sm_100a library and the `gfx906_fa` torch extension in-tree.

  libgfx906fa_b200.so  -- every CUDA kernel plus the C ABI of
                          include/gfx906_fa_b200.h (nvcc, -gencode
                          arch=compute_100a,code=sm_100a); depends on the CUDA
                          runtime only, so it loads without torch.
  gfx906_fa.so         -- the pybind/torch operator module (g++ against the
                          torch headers), linked to libgfx906fa_b200.so with an
                          $ORIGIN rpath.

Both land next to this file.  Rebuilds are incremental on file mtimes.
Run:  python gfx906_fa_build.py  [--force]
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgfx906fa_b200.so")
EXT = os.path.join(HERE, "gfx906_fa.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    # IEEE division / reciprocal / sqrt and no flush-to-zero: the Q8_0
    # quantiser must reproduce the reference's fp32 arithmetic bit for bit.
    "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def _headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def build_lib(force: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = _headers()
    objs, procs = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            cmd = [NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o]
            print("+", " ".join(cmd), flush=True)
            procs.append(subprocess.Popen(cmd))
            if len(procs) >= jobs:
                for p in procs:
                    if p.wait() != 0:
                        raise RuntimeError("nvcc failed")
                procs = []
    for p in procs:
        if p.wait() != 0:
            raise RuntimeError("nvcc failed")
    if force or _newer(LIB, objs):
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB + ".tmp", *objs])
        os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ext(force: bool = False) -> str:
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_ops.cpp")
    if not (force or _newer(EXT, [src, LIB] + _headers())):
        return EXT
    inc = ce.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE,
                                sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths()
    import torch
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=gfx906_fa", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in inc], src, "-o", EXT + ".tmp",
           *[f"-L{p}" for p in libdirs], f"-L{HERE}", "-lgfx906fa_b200",
           "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
           "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in libdirs]]
    _run(cmd)
    os.replace(EXT + ".tmp", EXT)
    return EXT


def build(force: bool = False) -> None:
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
