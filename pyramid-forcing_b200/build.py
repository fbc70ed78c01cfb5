"""Build the B200 MegaCache library in-tree.

* ``pyramidkv/lib/libpkv.so``    -- the CUDA kernels and the C ABI of
  ``include/pkv.h`` (nvcc, sm_100a, static cudart);
* ``pyramidkv/lib/_adahead.so``  -- the torch glue that registers the
  ``adahead`` op library and ``PyramidKVCacheManager`` class on top of it.

Objects go to ``_build/`` next to this file.  Rebuilds only what changed.

    python pyramid-forcing_b200/build.py [-j N] [--force]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INC = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "pyramidkv", "lib")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

CU_SOURCES = ["pkv_update.cu", "pkv_merge.cu", "pkv_plan.cu", "pkv_pack.cu", "pkv_attn.cu",
              "pkv_attend.cu", "pkv_legacy.cu", "pkv_rope.cu", "pkv_exchange.cu"]
HEADERS = ["pkv_common.cuh", "pkv_internal.h", "pkv_plan.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
           "--ptxas-options=-v"] + ARCH


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], log: str | None = None) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        with open(log, "w") as f:
            f.write(r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")


def torch_paths():
    import torch
    root = os.path.dirname(torch.__file__)
    return ([os.path.join(root, "include"), os.path.join(root, "include", "torch", "csrc",
                                                         "api", "include")],
            os.path.join(root, "lib"), int(torch._C._GLIBCXX_USE_CXX11_ABI))


def build(jobs: int = 8, force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INC, "pkv.h")]

    def compile_cu(src: str) -> str:
        obj = os.path.join(BUILD, src + ".o")
        path = os.path.join(CSRC, src)
        if force or _stale(obj, [path] + hdrs):
            _run([NVCC] + NVFLAGS + ["-I", INC, "-I", CSRC, "-c", path, "-o", obj],
                 log=os.path.join(BUILD, src + ".log"))
            if verbose:
                print("compiled", src)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_cu, CU_SOURCES))
    libpkv = os.path.join(LIB, "libpkv.so")
    if force or _stale(libpkv, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", libpkv] + objs)

    incs, tlib, abi = torch_paths()
    bind_src = os.path.join(CSRC, "adahead_bind.cpp")
    bind_obj = os.path.join(BUILD, "adahead_bind.o")
    if force or _stale(bind_obj, [bind_src, os.path.join(INC, "pkv.h")]):
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               "-I", INC, "-I", os.path.join(CUDA, "include"),
               "-I", sysconfig.get_paths()["include"]]
        for i in incs:
            cmd += ["-I", i]
        _run(cmd + ["-c", bind_src, "-o", bind_obj])
    glue = os.path.join(LIB, "_adahead.so")
    if force or _stale(glue, [bind_obj, libpkv]):
        _run(["g++", "-shared", "-o", glue, bind_obj, "-L", LIB, "-lpkv", "-L", tlib,
              "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
              "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + tlib])
    return glue


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.force, verbose=True))
