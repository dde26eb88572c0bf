"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every symbol include/xsimgs_b200.h declares, and the extension module carries
the reference's operator names and signatures (no GPU calls)."""
import ctypes
import inspect

import pytest


def test_c_abi_exports_every_declared_symbol():
    from xsimgs_b200 import capi
    lib = capi.lib()
    names = capi.declared_symbols()
    assert len(names) > 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert b"sm_100a" in lib.xsg_version()


def test_c_abi_rejects_bad_arguments_without_gpu():
    from xsimgs_b200 import capi
    lib = capi.lib()
    # argument validation happens before any CUDA call
    rc = lib.xsg_rasterize_fwd(*([None] * 7), 7, *([None] * 18))  # unsupported channel count first
    assert rc != 0
    rc = lib.xsg_mask_radii(None, None, ctypes.c_int64(4), None, None)
    assert rc == 1 and b"exactly one mask" in lib.xsg_last_error()
    assert lib.xsg_camera_pack_words(0) == 22 and lib.xsg_camera_pack_words(3) == 24
    assert lib.xsg_camera_pack_words(9) == -1


REFERENCE_OPS = [
    "rasterize_eval3d_fwd", "rasterize_eval3d_bwd", "rasterize_eval3d_dynamic_fwd",
    "rasterize_eval3d_dynamic_bwd", "eval3d_supported_ndims", "isect_regular_tiles", "isect_lidar_tiles",
    "isect_spherical_tiles", "isect_offset_encode", "mask_radii", "mask_radii_packed",
    "spherical_harmonics_fused_fwd", "spherical_harmonics_fused_bwd",
    "PerspectiveCamera", "OpenCVFisheyeCamera", "SphericalCamera", "LidarCamera", "ProjectionMode",
]
CAMERA_METHODS = ["pack", "camera_rays", "pixel_time", "pixel_time_delta", "pixel_time_from_uv",
                  "pixel_time_delta_from_uv", "projection", "projection_nojac", "projection_utgs"]


def test_extension_carries_reference_op_names():
    from xsimgs_b200 import _C
    missing = [n for n in REFERENCE_OPS if not hasattr(_C, n)]
    assert not missing, missing
    for cls in ("PerspectiveCamera", "OpenCVFisheyeCamera", "SphericalCamera", "LidarCamera"):
        for m in CAMERA_METHODS:
            assert hasattr(getattr(_C, cls), m), (cls, m)
    assert hasattr(_C.SphericalCamera, "projection_utgs_phm") and hasattr(_C.LidarCamera, "projection_utgs_phm")
    assert not hasattr(_C.PerspectiveCamera, "projection_utgs_phm")
    assert _C.eval3d_supported_ndims() == [0, 1, 2, 3, 4, 5, 8, 9, 16, 17, 32, 33, 64, 65, 128, 129, 256,
                                           257, 512, 513]


def test_keyword_signatures_match_reference():
    from xsimgs_b200 import _C
    doc = _C.rasterize_eval3d_fwd.__doc__
    for kw in ("means", "quats", "scales", "colors", "opacities", "image_width", "image_height",
               "tile_size_width", "tile_size_height", "ray_origs", "ray_dirs", "tile_offsets", "flatten_ids"):
        assert kw in doc, kw
    doc = _C.isect_regular_tiles.__doc__
    for kw in ("means2d", "radii", "depth", "img_width", "img_height", "tile_size_x", "tile_size_y",
               "sort: bool = True", "double_buffer: bool = True"):
        assert kw in doc, kw
    doc = _C.spherical_harmonics_fused_fwd.__doc__
    for kw in ("degree_to_use", "origin", "positions", "coeffs", "mask", "layout_3kn", "coeffs_dc", "output"):
        assert kw in doc, kw


def test_camera_pack_layout_on_cpu():
    import torch
    from xsimgs_b200 import _C
    t = lambda *v: torch.tensor(v, dtype=torch.float32)
    pack = _C.PerspectiveCamera.pack([t(1, 0, 0, 0), t(1, 2, 3), t(4, 5, 6), t(7, 8, 9), t(0.1, 0.2), t(0.5),
                                      t(0.25), t(0.6, 0.7, 0.5, 0.4)])
    assert pack.shape == (1, 22)
    assert pack.view(-1).tolist()[:14] == [1, 0, 0, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 0]
    got = pack.view(-1)[14:].tolist()
    assert got == pytest.approx([0.1, 0.2, 0.5, 0.25, 0.6, 0.7, 0.5, 0.4])
    with pytest.raises(RuntimeError, match="Tensor list size mismatch"):
        _C.PerspectiveCamera.pack([t(1, 0, 0, 0)])
    # gradients flow through the pack to the camera tensors
    f = t(0.6, 0.7, 0.5, 0.4).requires_grad_(True)
    p = _C.PerspectiveCamera.pack([t(1, 0, 0, 0), t(0, 0, 0), t(0, 0, 0), t(0, 0, 0), t(0, 0), t(0), t(0), f])
    p.sum().backward()
    assert f.grad.tolist() == [1, 1, 1, 1]
