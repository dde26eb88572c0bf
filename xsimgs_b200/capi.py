"""ctypes binding of the C ABI in include/xsimgs_b200.h (libxsimgs_b200.so).

The PyTorch extension `_C` is the normal way in; this module is the plain
C-ABI route (raw device pointers and sizes), used for the instrumentation
calls and by tests that exercise the boundary directly.
"""
from __future__ import annotations

import ctypes as C
import os
import re

from ._native import lib_path

_lib = None
_HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "xsimgs_b200.h")


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = C.CDLL(lib_path())
        _lib.xsg_last_error.restype = C.c_char_p
        _lib.xsg_version.restype = C.c_char_p
        _lib.xsg_launch_count.restype = C.c_longlong
        _lib.xsg_isect_workspace_size.restype = C.c_size_t
        _lib.xsg_isect_workspace_size.argtypes = [C.c_int64, C.c_int64]
        _lib.xsg_rasterize_workspace_size.restype = C.c_size_t
        _lib.xsg_rasterize_workspace_size.argtypes = [C.c_int64, C.c_int, C.c_int64, C.c_int64, C.c_int]
        _lib.xsg_sh_bwd_workspace_size.restype = C.c_size_t
        _lib.xsg_sh_bwd_workspace_size.argtypes = [C.c_int64]
        _lib.xsg_timing_query.argtypes = [C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_longlong)]
        _lib.xsg_fp32_probe.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_double)]
        _lib.xsg_set_pair_counters.argtypes = [C.c_void_p]
    return _lib


def declared_symbols() -> list[str]:
    """Names of all functions declared in include/xsimgs_b200.h."""
    text = open(_HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(xsg_[a-z0-9_]+)\s*\(", text)))


def check(rc: int):
    if rc != 0:
        raise RuntimeError(lib().xsg_last_error().decode())


def launch_count() -> int:
    return int(lib().xsg_launch_count())


def timing_enable(on: bool):
    lib().xsg_timing_enable(C.c_int(1 if on else 0))


def timing_reset():
    lib().xsg_timing_reset()


def timing_query(name: str) -> tuple[float, int]:
    ms, cnt = C.c_double(0.0), C.c_longlong(0)
    check(lib().xsg_timing_query(name.encode(), C.byref(ms), C.byref(cnt)))
    return ms.value, cnt.value


def set_pair_counters(ptr: int | None):
    lib().xsg_set_pair_counters(C.c_void_p(ptr) if ptr else None)


def fp32_probe(scratch_ptr: int, iters: int, blocks: int, stream_ptr: int) -> float:
    flops = C.c_double(0.0)
    check(lib().xsg_fp32_probe(C.c_void_p(scratch_ptr), iters, blocks, C.c_void_p(stream_ptr), C.byref(flops)))
    return flops.value
