"""Build recipe for the native parts of xsimgs_b200 (run once per checkout).

1. libxsimgs_b200.so — every CUDA kernel plus the C ABI declared in
   include/xsimgs_b200.h, compiled by nvcc for sm_100a only
   (-gencode arch=compute_100a,code=sm_100a), cudart linked statically.
2. _C*.so — the PyTorch extension exposing the reference's `xsimgs._C`
   operator names; host C++ only, linked against libxsimgs_b200.so with an
   $ORIGIN rpath so both load from this directory.

Objects are cached under xsimgs_b200/_build/ and rebuilt when a source or
header is newer.  `python xsimgs_b200/build.py` builds everything (run it as
a script: importing the package needs the extension already built).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libxsimgs_b200.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", os.path.join(ROOT, "include")]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "xsimgs_b200.h")]
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if ptxas_info or _newer(obj, [src] + headers):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            _run([NVCC, *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj], verbose)
        objs.append(obj)
    if _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs], verbose)
        os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ext(verbose: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "ext", "xsimgs_ext.cpp")
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = os.path.join(PKG, "_C" + suffix)
    deps = [src, os.path.join(ROOT, "include", "xsimgs_b200.h"), LIB]
    if not _newer(out, deps):
        return out
    inc = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], os.path.join(ROOT, "include"),
                                           os.path.join(CUDA_HOME, "include")]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-DTORCH_EXTENSION_NAME=_C",
           "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-fvisibility=hidden"]
    for d in inc:
        cmd += ["-I", d]
    cmd += [src, "-o", out + ".tmp", "-L", torch_lib, "-Wl,-rpath," + torch_lib, "-lc10", "-ltorch",
            "-ltorch_cpu", "-ltorch_python", "-L", PKG, "-lxsimgs_b200", "-Wl,-rpath,$ORIGIN"]
    # c10_cuda provides the current CUDA stream
    if os.path.exists(os.path.join(torch_lib, "libc10_cuda.so")):
        cmd += ["-lc10_cuda"]
    _run(cmd, verbose)
    os.replace(out + ".tmp", out)
    return out


def build(verbose: bool = False) -> None:
    build_lib(verbose)
    build_ext(verbose)


if __name__ == "__main__":
    v = "-v" in sys.argv
    if "--ptxas" in sys.argv:
        build_lib(True, ptxas_info=True)
    else:
        build(v)
    print(LIB)
