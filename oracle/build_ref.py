"""Build recipe for the GPU test oracle compiled from the reference's OWN
CUDA sources (test infrastructure, never part of the shipped library).

The reference's kernels need two header trees its checkout lacks: the GLM
submodule (`third_party/glm` is empty) and pytoast's `toast/utils/*.h` and
`toast/math/{quat,motion,scalar}.h` (not installed, no pinned version).
`oracle/ref_compat/` holds this project's own minimal stand-ins for exactly
what those sources use (vector and matrix arithmetic, quaternions, the motion
model, launch and argument-check helpers); see the header comments there for
the semantics assumed.  The reference sources are compiled where they lie,
unmodified, with the reference's own nvcc flags (setup.py:12-24: -O3, FMA
contraction on, no fast math) for sm_100a, plus -maxrregcount=64 for the
camera and range-tiling sources: the reference launches some of their
kernels with 1024-thread blocks (its block reductions require it,
include/utils/reduce_helpers.cuh:5-6), which only fit the SM's register file
at 64 registers a thread (register allocation changes no arithmetic).
`oracle/ref_module.cpp` binds the reference's bind_* functions into the
module `_xsimgs_ref`.

Compiled (paths within the reference project):
    csrc/rasterization/eval3d_fwd.cu, eval3d_bwd.cu, eval3d_dynamic_fwd.cu,
        eval3d_dynamic_bwd.cu, eval3d_bind.cpp
    csrc/tiling/regular_tiling.cu, tiling_common.cu, mask_radii.cu
    csrc/color/sh_fwd.cu, sh_bwd.cu, sh_bind.cpp
    csrc/cameras/perspective.cu, distorted_perspective.cu, fisheye_opencv.cu,
        spherical.cu (every camera class with pack, rays, pixel times,
        projection and the UT projections, include/cameras/*.h)
    csrc/tiling/phm_lidar_tiling.cu, phm_spherical_tiling.cu
Output: oracle/_ref/_xsimgs_ref<EXT_SUFFIX>.so (git-ignored; it travels to
the GPU box with the working tree, where the reference checkout is absent).

What the stand-ins cannot pin: pytoast's quaternion and motion primitives
(std(), to_matrix, apply, slerp and their backwards) are written from the
conventions the CPU oracle assumes, so the camera-side results are pinned to
the reference's own code everywhere except inside those primitives.

Not compiled: the SMPL / scene-assembly sources (csrc/nodes, which need
pytoast's SE3 headers) and everything outside the render path.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
# the reference checkout: $XSG_REFERENCE_ROOT, else the folder `reference`
# beside this repository's root
REF = os.environ.get("XSG_REFERENCE_ROOT",
                     os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
OUT_DIR = os.path.join(HERE, "_ref")
# object files stay in the git- and gpurun-ignored build folder; only the
# module travels
OBJ_DIR = os.path.join(HERE, "_build", "ref_obj")
NAME = "_xsimgs_ref"
COMPAT = os.path.join(HERE, "ref_compat")
MODULE_SRC = os.path.join(HERE, "ref_module.cpp")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

# Link order matters: eval3d_fwd.cu and eval3d_dynamic_fwd.cu each define a
# different struct named TileSharedMemoryFwd (and the two backward files two
# TileSharedMemoryBwd), so the linker keeps one instantiation of
# set_max_shared_mem<TileSharedMemoryFwd> for both kernels.  With the static
# file first, the dynamic kernel's shared-memory limit is set below what its
# launch asks for and the launch fails (cudaErrorInvalidValue); with the
# dynamic (larger) layouts first, both launches are valid.
REF_SOURCES = [
    "csrc/rasterization/eval3d_dynamic_fwd.cu",
    "csrc/rasterization/eval3d_dynamic_bwd.cu",
    "csrc/rasterization/eval3d_fwd.cu",
    "csrc/rasterization/eval3d_bwd.cu",
    "csrc/rasterization/eval3d_bind.cpp",
    "csrc/tiling/regular_tiling.cu",
    "csrc/tiling/tiling_common.cu",
    "csrc/tiling/mask_radii.cu",
    "csrc/color/sh_fwd.cu",
    "csrc/color/sh_bwd.cu",
    "csrc/color/sh_bind.cpp",
    "csrc/cameras/perspective.cu",
    "csrc/cameras/distorted_perspective.cu",
    "csrc/cameras/fisheye_opencv.cu",
    "csrc/cameras/spherical.cu",
    "csrc/tiling/phm_lidar_tiling.cu",
    "csrc/tiling/phm_spherical_tiling.cu",
]


def out_path() -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(OUT_DIR, NAME + suffix)


def available() -> bool:
    return os.path.isdir(os.path.join(REF, "csrc", "rasterization"))


def _flags():
    import torch
    from torch.utils import cpp_extension
    inc = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], os.path.join(CUDA_HOME, "include"),
                                           COMPAT, os.path.join(REF, "include")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    common = ["-DTORCH_API_INCLUDE_EXTENSION_H", f"-DTORCH_EXTENSION_NAME={NAME}", f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    for d in inc:
        common += ["-I", d]
    nvcc = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
            "-DCUDA_HAS_FP16=1", "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
            "-D__CUDA_NO_HALF2_OPERATORS__", "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "--extended-lambda",
            "--expt-relaxed-constexpr", "-diag-suppress", "186,177,550", *common]
    cxx = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", *common]
    return nvcc, cxx


def _compile(args):
    cmd, src = args
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiling {src} failed:\n{r.stderr[-6000:]}")
    return src


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str | None:
    """Compile the reference oracle; returns the module path, or None when
    the reference checkout is absent (then a previously built module, if any,
    is kept as it is)."""
    out = out_path()
    if not available():
        return out if os.path.exists(out) else None
    import torch
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc, cxx = _flags()
    compat_headers = [os.path.join(dp, f) for dp, _, fs in os.walk(COMPAT) for f in fs]
    jobs_list, objs = [], []
    for rel in REF_SOURCES + [MODULE_SRC]:
        src = rel if os.path.isabs(rel) else os.path.join(REF, rel)
        obj = os.path.join(OBJ_DIR, rel.replace("/", "_").lstrip("_") + ".o")
        objs.append(obj)
        deps = [src] + compat_headers
        if not force and not _newer(obj, deps):
            continue
        if src.endswith(".cu"):
            extra = ["-maxrregcount=64"] if ("/cameras/" in rel or "/phm_" in rel) else []
            cmd = [NVCC, *nvcc, *extra, "-c", src, "-o", obj]
        else:
            cmd = ["g++", *cxx, "-c", src, "-o", obj]
        jobs_list.append((cmd, src))
    if jobs_list:
        n = jobs or max(1, min(len(jobs_list), os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(n) as ex:
            for src in ex.map(_compile, jobs_list):
                if verbose:
                    print("built", src, flush=True)
    if force or _newer(out, objs + [os.path.abspath(__file__)]):
        torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
        cmd = ["g++", "-shared", "-o", out + ".tmp", *objs, "-L", torch_lib, "-Wl,-rpath," + torch_lib,
               "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-L", os.path.join(CUDA_HOME, "lib64"),
               "-lcudart"]
        if os.path.exists(os.path.join(torch_lib, "libc10_cuda.so")):
            cmd += ["-lc10_cuda", "-ltorch_cuda"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


def load():
    """Import the prebuilt module (raises ImportError when it was never built)."""
    import importlib.machinery
    import importlib.util
    path = out_path()
    if not os.path.exists(path):
        raise ImportError(f"reference oracle not built: {path} (run oracle/build_ref.py where the reference "
                          f"checkout is present)")
    import torch  # noqa: F401  (libtorch must be loaded first)
    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
