"""Loads the in-tree native extension (``_C*.so`` + ``libxsimgs_b200.so``).

There is no fallback: if the extension was not built (``python
xsimgs_b200/build.py``) importing the package raises ImportError naming the
missing file, so no CPU or eager-PyTorch path can silently stand in for the
CUDA kernels.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys

_PKG = os.path.dirname(os.path.abspath(__file__))


def lib_path() -> str:
    return os.path.join(_PKG, "libxsimgs_b200.so")


def _load_ext():
    import torch  # noqa: F401  (libtorch symbols must be loaded first)

    hits = sorted(glob.glob(os.path.join(_PKG, "_C*.so")))
    if not hits or not os.path.exists(lib_path()):
        raise ImportError(
            "xsimgs_b200 native extension not built: expected _C*.so and "
            f"libxsimgs_b200.so in {_PKG}; run `python xsimgs_b200/build.py`")
    name = "xsimgs_b200._C"
    if name in sys.modules:
        return sys.modules[name]
    loader = importlib.machinery.ExtensionFileLoader(name, hits[0])
    spec = importlib.util.spec_from_file_location(name, hits[0], loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


_C = _load_ext()
