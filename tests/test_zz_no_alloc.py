"""The allocation-free spherical-harmonics backward (xsg_sh_bwd_noalloc).

Some callers of this library cannot allocate device memory: a host runtime
that only lends the library the buffers it already owns, or code that must
not call cudaMalloc on its hot path.  For them the library keeps its scratch
(per-block partial sums of the origin gradient) in a fixed device array.
This test calls that entry point through the C ABI several times in a row
and checks each result against the regular xsg_sh_bwd, which takes a caller
workspace.  Both run the same kernels with the same block partition and the
same summation order, so every output must agree bit for bit.  Later calls
are smaller than the first (fewer blocks, a size that is not a multiple of
the block), one with a Gaussian mask, so anything a call read from an earlier
call's leftovers would show up as a wrong origin gradient.

It lives in its own file named to be collected last, so a run that stops at
the first failure has run every other test before it.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from tests.helpers import to_np

pytestmark = pytest.mark.gpu


def _lib():
    from xsimgs_b200 import capi
    lib = capi.lib()
    lib.xsg_sh_bwd_noalloc_max_gaussians.restype = C.c_int64
    f = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int,
         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.xsg_sh_bwd_noalloc.argtypes = f + [C.c_void_p]
    lib.xsg_sh_bwd.argtypes = f + [C.c_void_p, C.c_size_t, C.c_void_p]
    return lib


def _case(seed, n, degree, dev, masked=False):
    rng = np.random.default_rng(seed)
    k = (degree + 1) ** 2
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)
    mask = None
    if masked:
        bits = np.packbits(rng.random(n) < 0.7, bitorder="little")
        bits = np.concatenate([bits, np.zeros((-len(bits)) % 4, np.uint8)])
        mask = torch.from_numpy(bits.view(np.uint32).astype(np.int64).astype(np.int32)).to(dev)
    return dict(pos=t(rng.normal(size=(n, 3)) * 10), origin=t([0.3, -0.7, 1.1]),
                coeffs=t(rng.normal(size=(n, k, 3))), d_out=t(rng.normal(size=(n, 3))), n=n, k=k, degree=degree,
                mask=mask)


def _outputs(c):
    return (torch.zeros_like(c["coeffs"]), torch.zeros_like(c["pos"]), torch.zeros(3, device=c["pos"].device))


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _run(lib, c, noalloc):
    d_coeffs, d_pos, d_origin = _outputs(c)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    mask = _ptr(c["mask"]) if c["mask"] is not None else None
    args = [c["degree"], _ptr(c["origin"]), _ptr(c["pos"]), _ptr(c["coeffs"]), None, mask, 0, c["n"], c["k"],
            _ptr(c["d_out"]), _ptr(d_coeffs), None, _ptr(d_pos), _ptr(d_origin)]
    if noalloc:
        rc = lib.xsg_sh_bwd_noalloc(*args, stream)
    else:
        ws_bytes = lib.xsg_sh_bwd_workspace_size(C.c_int64(c["n"]))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=c["pos"].device)
        rc = lib.xsg_sh_bwd(*args, _ptr(ws), ws_bytes, stream)
    assert rc == 0, lib.xsg_last_error().decode()
    torch.cuda.synchronize()
    return d_coeffs, d_pos, d_origin


def test_sh_backward_without_allocation_matches_workspace_version(cuda):
    lib = _lib()
    cases = [_case(1, 300_000, 3, cuda),                # many blocks
             _case(2, 70_001, 2, cuda),                 # fewer blocks, ragged last block
             _case(3, 12_345, 3, cuda, masked=True),    # fewer still, masked Gaussians
             _case(4, 300_000, 1, cuda, masked=True)]   # back to many blocks
    for c in cases:
        got = _run(lib, c, noalloc=True)
        ref = _run(lib, c, noalloc=False)
        for name, a, b in zip(("d_coeffs", "d_positions", "d_origin"), got, ref):
            np.testing.assert_array_equal(to_np(a), to_np(b), err_msg=f"{name} (n={c['n']})")


def test_sh_backward_without_allocation_rejects_oversize(cuda):
    lib = _lib()
    limit = lib.xsg_sh_bwd_noalloc_max_gaussians()
    assert limit == 1 << 23
    dummy = torch.zeros(4, device=cuda)
    p = _ptr(dummy)
    rc = lib.xsg_sh_bwd_noalloc(0, p, p, p, None, None, 0, limit + 1, 1, p, p, None, p, p,
                                C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc != 0
    assert b"exceed the maximum" in lib.xsg_last_error()
