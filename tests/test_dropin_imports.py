"""The reference's own import statements resolve against this package
(src/xsimgs/rendering/rasterize.py:4, rasterize_dynamic.py:4,
render.py:3, sh.py:3-6, cameras/ext/*.py, nodes/*.py), so code written
against the reference runs unchanged.  No GPU needed: importing loads the
extension but calls no kernel."""


def test_reference_import_statements_resolve():
    from xsimgs._C import rasterize_eval3d_fwd, rasterize_eval3d_bwd  # rasterize.py:4
    from xsimgs._C import rasterize_eval3d_dynamic_fwd, rasterize_eval3d_dynamic_bwd  # rasterize_dynamic.py:4
    from xsimgs._C import mask_radii, isect_offset_encode, eval3d_supported_ndims  # render.py:3
    from xsimgs._C import spherical_harmonics_fused_fwd, spherical_harmonics_fused_bwd  # sh.py:3-6
    from xsimgs._C import isect_regular_tiles, isect_lidar_tiles, isect_spherical_tiles  # ext_camera.py, lidar.py
    from xsimgs._C import (PerspectiveCamera, OpenCVFisheyeCamera, SphericalCamera, LidarCamera,  # noqa: F401
                           DistortedPerspectiveCamera)
    from xsimgs._C import image_to_hwc_rgb_byte, image_to_hwc_rgba_byte, image_to_chw_rgb_byte  # noqa: F401
    from xsimgs.rendering import ut_gs_render, ut_gs_tiling, ut_gs_rasterize  # noqa: F401
    from xsimgs.rendering.sh import spherical_harmonics_fused, rgb_to_sh0, sh0_to_rgb  # noqa: F401
    from xsimgs.rendering.render import ut_gs_render as r2
    from xsimgs.cameras.ext import PerspectiveCamera as P, FisheyeCamera, SphericalCamera as S, LidarCamera as L  # noqa
    from xsimgs.cameras.ext.ext_camera import FusedRSCamera  # noqa: F401
    from xsimgs.nodes import (smpl_lbs_skinning, smpl_local_to_global_pose, interpolate_smpl_poses,  # noqa: F401
                              rigid_transform_and_put, packed_mask_from_instances, valid_instances_indices)
    import xsimgs
    import xsimgs_b200
    assert xsimgs._C is xsimgs_b200._C
    assert rasterize_eval3d_fwd is xsimgs_b200._C.rasterize_eval3d_fwd
    assert r2 is ut_gs_render is xsimgs_b200.ut_gs_render
    for f in (rasterize_eval3d_bwd, mask_radii, isect_offset_encode, eval3d_supported_ndims,
              spherical_harmonics_fused_fwd, spherical_harmonics_fused_bwd, isect_regular_tiles, isect_lidar_tiles,
              isect_spherical_tiles, rasterize_eval3d_dynamic_fwd, rasterize_eval3d_dynamic_bwd):
        assert callable(f)
    assert sorted(eval3d_supported_ndims()) == [0, 1, 2, 3, 4, 5, 8, 9, 16, 17, 32, 33, 64, 65, 128, 129, 256,
                                                257, 512, 513]
