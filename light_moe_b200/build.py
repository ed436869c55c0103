"""Build the sm_100a library and the `_C` operator module in-tree.

    python -m light_moe_b200.build            # incremental
    python -m light_moe_b200.build --force    # rebuild everything

Produces
  light_moe_b200/lib/liblmoe_b200.so   C ABI (include/lmoe_b200.h), nvcc, sm_100a only
  light_moe_b200/_C.<abi>.so           pybind11 operator module linked against it

nvcc cross-compiles without a GPU, so this runs on a CPU-only machine as well.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "liblmoe_b200.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["host_util.cu", "router.cu", "quant.cu", "grouped_gemm.cu", "decode_gemm.cu", "simt_gemm.cu",
              "layer.cu", "dispatch.cu", "ep_p2p.cu"]
HEADERS = ["ptx.cuh", "lmoe_math.cuh", "host_util.h", "w4_layout.cuh", "w4_dequant.cuh", "grouped_gemm.h",
           "decode_gemm.h"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-I", INCLUDE,
]


def ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def ext_path() -> str:
    return os.path.join(PKG, "_C" + ext_suffix())


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build_library(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "lmoe_b200.h")]
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or not _newer(o, [s] + hdrs):
            jobs.append([NVCC, *NVCC_FLAGS, "-c", s, "-o", o])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for r in ex.map(_run, jobs):
                if verbose and r.stderr:
                    print(r.stderr, file=sys.stderr)
    if force or jobs or not _newer(LIB, objs):
        _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
              "-o", LIB, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"])
    return LIB


def build_extension(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    out = ext_path()
    src = os.path.join(CSRC, "bindings.cpp")
    deps = [src, os.path.join(INCLUDE, "lmoe_b200.h"), LIB]
    if not force and _newer(out, deps):
        return out
    inc = cpp_extension.include_paths(device_type="cuda") + [INCLUDE, os.path.join(CUDA_HOME, "include"),
                                                            sysconfig.get_paths()["include"]]
    import pybind11
    inc.append(pybind11.get_include())
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", src, "-o", out,
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in inc], *[f"-L{p}" for p in libdirs], f"-L{LIBDIR}",
           "-llmoe_b200", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda",
           "-Wl,-rpath,$ORIGIN/lib", *[f"-Wl,-rpath,{p}" for p in libdirs]]
    _run(cmd)
    return out


def build(force: bool = False, verbose: bool = False):
    lib = build_library(force=force, verbose=verbose)
    ext = build_extension(force=force)
    return lib, ext


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
