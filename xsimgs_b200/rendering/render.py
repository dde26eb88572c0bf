"""Public render API: `ut_gs_tiling` and `ut_gs_render`, with the reference's
signatures and behaviour (src/xsimgs/rendering/render.py:10-187).

`ut_gs_render` on a regular-tile camera does not wait for the intersection
count on the host between the tile count and the compositing (the reference
sizes its lists from a host copy of the count, tiling/regular_tiling.cu:
101-103): the lists are allocated for a per-view capacity remembered from
earlier renders of the same view shape, the tiler writes the count on the
device and the compositor reads the list length from there.  The host reads
the count once the forward is enqueued; if it exceeded the capacity, the view
is rendered again with exact lists and the capacity grows.  The first render
of a view shape, and every render with XSIMGS_B200_SYNC_TILING=1, uses the
exact lists directly."""
import os
from collections import OrderedDict

import torch

from .._native import _C
from .rasterize import ut_gs_rasterize
from .rasterize_dynamic import ut_gs_dynamic_rasterize

# capacity headroom over the largest count seen for a view shape
_CAP_GROWTH = 1.25
_CAP_SLACK = 4096
_CAP_ENTRIES = 256
_capacity: "OrderedDict[tuple, int]" = OrderedDict()


def _capacity_key(camera, points, width, height, tile_size_x, tile_size_y):
    return (points.device, type(camera).__name__, getattr(camera, "camera_name", None), int(width), int(height),
            int(tile_size_x), int(tile_size_y), int(points.shape[0]))


def _remember_count(key, total: int):
    want = int(total * _CAP_GROWTH) + _CAP_SLACK
    if _capacity.get(key, 0) < want:
        _capacity[key] = want
    _capacity.move_to_end(key)
    while len(_capacity) > _CAP_ENTRIES:
        _capacity.popitem(last=False)


def _sync_free_tiling_applies(camera) -> bool:
    if os.environ.get("XSIMGS_B200_SYNC_TILING", "0") not in ("", "0"):
        return False
    # regular tiles only: range-image cameras bring their own tilers
    return type(camera).isect_gs_tiles is _regular_isect_gs_tiles()


def _regular_isect_gs_tiles():
    from ..cameras.ext_camera import FusedRSCamera
    return FusedRSCamera.isect_gs_tiles


def ut_gs_tiling(camera, points, scale, rotation, width: int, height: int, points_velocity=None,
                 opacity=None, packed_particle_mask=None, tile_size_x: int = 16, tile_size_y: int = 16,
                 ut_alpha: float = 0.1, ut_beta: float = 2.0, ut_kappa: float = 0.0, use_phm=None):
    """UT projection -> optional radius mask -> tile intersection and sort ->
    per-tile offsets (render.py:10-81)."""
    with camera._freeze_ctx():
        flags, radii, means2d, depth = camera.ut_gs_projection(
            points=points, points_velocity=points_velocity, scale=scale, rotation=rotation,
            opacity=opacity, width=width, height=height, ut_alpha=ut_alpha, ut_beta=ut_beta,
            ut_kappa=ut_kappa, use_phm=use_phm)
        if packed_particle_mask is not None:
            _C.mask_radii_packed(packed_particle_mask, radii)
        tiles_per_gs, isect_ids, flatten_ids = camera.isect_gs_tiles(
            points=points, points_velocity=points_velocity, scale=scale, rotation=rotation,
            opacity=opacity, flags=flags, means2d=means2d, radii=radii, depths=depth, width=width,
            height=height, ut_alpha=ut_alpha, ut_beta=ut_beta, ut_kappa=ut_kappa,
            tile_size_x=tile_size_x, tile_size_y=tile_size_y, sort=True, double_buffer=True)
        n_tiles_width = (width + tile_size_x - 1) // tile_size_x
        n_tiles_height = (height + tile_size_y - 1) // tile_size_y
        tile_gs_offsets = _C.isect_offset_encode(isect_ids, tile_width=n_tiles_width,
                                                 tile_height=n_tiles_height)
    return dict(means2d=means2d, radii=radii, depth=depth, isect_offsets=tile_gs_offsets,
                flatten_ids=flatten_ids)


def _tiling_capacity(camera, points, scale, rotation, width, height, points_velocity, opacity,
                     packed_particle_mask, tile_size_x, tile_size_y, ut_alpha, ut_beta, ut_kappa, use_phm,
                     capacity):
    """ut_gs_tiling with capacity-sized lists and the count on the device:
    (tile data, device counts {total, written})."""
    flags, radii, means2d, depth = camera.ut_gs_projection(
        points=points, points_velocity=points_velocity, scale=scale, rotation=rotation, opacity=opacity,
        width=width, height=height, ut_alpha=ut_alpha, ut_beta=ut_beta, ut_kappa=ut_kappa, use_phm=use_phm)
    if packed_particle_mask is not None:
        _C.mask_radii_packed(packed_particle_mask, radii)
    _, _, flatten_ids, offsets, counts = _C.isect_regular_tiles_async(
        means2d, radii, depth, img_width=width, img_height=height, tile_size_x=tile_size_x,
        tile_size_y=tile_size_y, capacity=capacity)
    return dict(means2d=means2d, radii=radii, depth=depth, isect_offsets=offsets, flatten_ids=flatten_ids), counts


def ut_gs_render(camera, points, scale, rotation, opacity, width: int, height: int, colors=None,
                 points_velocity=None, packed_particle_mask=None, tile_size_x: int = 16,
                 tile_size_y: int = 16, ut_alpha: float = 0.1, ut_beta: float = 2.0,
                 ut_kappa: float = 0.0, use_phm=None, ray_o=None, ray_d=None, ray_time_delta=None):
    """Render colour [H, W, C], depth [H, W] and alpha [H, W] of Gaussians
    seen by `camera`, differentiable w.r.t. the Gaussian parameters
    (render.py:85-187).  Returns (color, depth, alpha, meta)."""
    return _render(camera, points, scale, rotation, opacity, width, height, colors, points_velocity,
                   packed_particle_mask, tile_size_x, tile_size_y, ut_alpha, ut_beta, ut_kappa, use_phm, ray_o,
                   ray_d, ray_time_delta, sync_tiling=False)


def _render(camera, points, scale, rotation, opacity, width, height, colors, points_velocity,
            packed_particle_mask, tile_size_x, tile_size_y, ut_alpha, ut_beta, ut_kappa, use_phm, ray_o, ray_d,
            ray_time_delta, sync_tiling):
    assert camera.device == points.device, (
        "Camera must be on the same device as gaussian tensors. "
        "Given camera on {}, points on {}".format(camera.device, points.device))
    if colors is not None:
        assert colors.shape[-1] in _C.eval3d_supported_ndims(), (
            "Color feature dimension = {} is not supported. Supported CDIMs=[{}].".format(
                colors.shape[-1], ", ".join(str(v) for v in _C.eval3d_supported_ndims())))
    with camera._freeze_ctx():
        points = points.contiguous()
        scale = scale.contiguous()
        rotation = rotation.contiguous()
        opacity = opacity.contiguous()
        colors = colors.contiguous() if colors is not None else None
        points_velocity = points_velocity.contiguous() if points_velocity is not None else None

        key = counts = None
        if not sync_tiling and points.is_cuda and _sync_free_tiling_applies(camera):
            key = _capacity_key(camera, points, width, height, tile_size_x, tile_size_y)
        capacity = _capacity.get(key) if key is not None else None
        if capacity is not None:
            tile_data, counts = _tiling_capacity(
                camera, points, scale, rotation, width, height, points_velocity, opacity, packed_particle_mask,
                tile_size_x, tile_size_y, ut_alpha, ut_beta, ut_kappa, use_phm, capacity)
            counts_host = torch.empty(2, dtype=torch.int64, pin_memory=True)
            counts_host.copy_(counts, non_blocking=True)
            counted = torch.cuda.Event()
            counted.record()
        else:
            tile_data = ut_gs_tiling(
                camera=camera, points=points, scale=scale, rotation=rotation, width=width, height=height,
                points_velocity=points_velocity, opacity=opacity, packed_particle_mask=packed_particle_mask,
                tile_size_x=tile_size_x, tile_size_y=tile_size_y, ut_alpha=ut_alpha, ut_beta=ut_beta,
                ut_kappa=ut_kappa, use_phm=use_phm)
            if key is not None:
                _remember_count(key, tile_data["flatten_ids"].numel())

        is_scene_static = points_velocity is None
        if ray_o is None or ray_d is None:
            ray_o, ray_d = camera.camera_rays(width=width, height=height, normalized_rays=True,
                                              return_origins=True, world_space=True)
        kwargs = dict(positions=points, rotation=rotation, scale=scale, density=opacity, colors=colors,
                      ray_o=ray_o, ray_d=ray_d, isect_offsets=tile_data["isect_offsets"],
                      flatten_ids=tile_data["flatten_ids"], tile_size_x=tile_size_x,
                      tile_size_y=tile_size_y)
        if counts is not None:
            kwargs["n_isects"] = counts[1:]
        if is_scene_static:
            color, depth, alpha = ut_gs_rasterize(**kwargs)
        else:
            if ray_time_delta is None:
                ray_time_delta = camera.image_time_delta(ray_o)
            color, depth, alpha = ut_gs_dynamic_rasterize(**kwargs, velocity=points_velocity,
                                                          ray_time_delta=ray_time_delta)
        if counts is not None:
            # the whole forward is enqueued: wait for the count alone
            counted.synchronize()
            total = int(counts_host[0])
            _remember_count(key, total)
            if total > capacity:
                return _render(camera, points, scale, rotation, opacity, width, height, colors, points_velocity,
                               packed_particle_mask, tile_size_x, tile_size_y, ut_alpha, ut_beta, ut_kappa,
                               use_phm, ray_o, ray_d, ray_time_delta, sync_tiling=True)
    meta = dict(radii=tile_data["radii"], width=width, height=height)
    return color, depth, alpha, meta
