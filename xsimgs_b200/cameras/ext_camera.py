"""Rolling-shutter camera objects for `ut_gs_render` without `pytoast`.

The reference builds its cameras (src/xsimgs/cameras/ext/*.py) on toast's
LinearMotion / RollingShutter objects.  These classes keep the interface
`ut_gs_render` relies on (`pack`, `device`, `_freeze_ctx`, `use_phm`,
`supports_phm`, `ut_gs_projection`, `isect_gs_tiles`, `camera_rays`,
`image_time_delta`, ...; ext_camera.py:8-210) but take plain tensors:

    q0            [4]  camera->world rotation at pose_time, (w, x, y, z)
    t0            [3]  camera centre at pose_time
    v, w          [3]  linear / angular velocity (world frame)
    rolling_time  [2]  shutter duration along u and v (RollingShutter.duration)
    trigger_time  [1]  capture time of uv = (0, 0) (RollingShutter.offset_time)
    pose_time     [1]  time of the pose (q0, t0)

Camera axes: +Z forward, +X right (image u), +Y down (image v).
"""
from __future__ import annotations

from contextlib import contextmanager

import numpy as np
import torch

from .._native import _C


def _vec(x, n, device, default=0.0):
    if x is None:
        return torch.full((n,), float(default), dtype=torch.float32, device=device)
    t = torch.as_tensor(x, dtype=torch.float32, device=device).reshape(n)
    return t.contiguous()


class FusedRSCamera:
    ext_cls = None
    use_phm: bool = False

    N_ROLLING_ITERATIONS: int = 5
    residual_thr_early_stop: float = 1e-4
    residual_max_valid: float = 0.002
    max_margin: float = 1.0

    def __init__(self, q0, t0, v=None, w=None, rolling_time=None, trigger_time=0.0, pose_time=0.0,
                 device=None, camera_name=None):
        device = torch.device(device) if device is not None else torch.as_tensor(q0).device
        self.q0 = _vec(q0, 4, device)
        self.t0 = _vec(t0, 3, device)
        self.v = _vec(v, 3, device)
        self.w = _vec(w, 3, device)
        self.rolling_time = _vec(rolling_time, 2, device)
        self.trigger_time = _vec(trigger_time, 1, device)
        self.pose_time = _vec(pose_time, 1, device)
        self.camera_name = camera_name
        self._pack = None
        self._freeze_flag = False

    # ------------------------------------------------------------- pack --
    @property
    def device(self):
        return self.q0.device

    @property
    def _pack_data(self) -> list[torch.Tensor]:
        return [self.q0, self.t0, self.v, self.w, self.rolling_time, self.trigger_time,
                self.pose_time]

    def _set_freeze(self, value: bool):
        self._freeze_flag = value
        self._pack = None

    @contextmanager
    def _freeze_ctx(self):
        needed = not self._freeze_flag
        if needed:
            self._set_freeze(True)
        try:
            yield
        finally:
            if needed:
                self._set_freeze(False)

    @classmethod
    def supports_phm(cls) -> bool:
        return hasattr(cls.ext_cls, "projection_utgs_phm")

    @property
    def pack(self):
        if self._freeze_flag and self._pack is not None:
            return self._pack
        self._pack = self.ext_cls.pack(self._pack_data)
        return self._pack

    def to(self, device):
        for name in ("q0", "t0", "v", "w", "rolling_time", "trigger_time", "pose_time"):
            setattr(self, name, getattr(self, name).to(device))
        self._pack = None
        return self

    # ---------------------------------------------------------- queries --
    def world_to_uv(self, points, points_velocity=None, points_time=None):
        if points_time is not None and points_velocity is not None:
            points = points + (points_time - self.pose_time) * points_velocity
        return self.ext_cls.projection(
            self.pack, points.contiguous(),
            points_velocity.contiguous() if points_velocity is not None else None,
            residual_thr_early_stop=self.residual_thr_early_stop,
            max_residual=self.residual_max_valid, max_margin=self.max_margin)

    def camera_rays(self, width: int, height: int, normalized_rays: bool = True,
                    world_space: bool = True, return_origins: bool = True, return_valid: bool = False):
        out = self.ext_cls.camera_rays(self.pack, width=width, height=height, world_space=world_space,
                                       normalized=normalized_rays, return_valid=return_valid)
        ray_o = out[0] if return_origins else None
        if return_valid:
            return ray_o, out[1], out[2]
        return ray_o, out[1]

    def uv_time(self, uv):
        return self.ext_cls.pixel_time_from_uv(self.pack, uv.contiguous()).unsqueeze(-1)

    def uv_time_delta(self, uv):
        return self.ext_cls.pixel_time_delta_from_uv(self.pack, uv.contiguous()).unsqueeze(-1)

    def image_time(self, image):
        return self.ext_cls.pixel_time(self.pack, width=image.shape[1], height=image.shape[0]).unsqueeze(-1)

    def image_time_delta(self, image):
        return self.ext_cls.pixel_time_delta(self.pack, width=image.shape[1],
                                             height=image.shape[0]).unsqueeze(-1)

    def ut_gs_projection(self, points, scale, rotation, width, height, points_velocity=None, opacity=None,
                         ut_alpha=0.1, ut_beta=2.0, ut_kappa=0.0, use_phm=None):
        if use_phm is None:
            use_phm = self.use_phm
        proj_fn = (self.ext_cls.projection_utgs_phm if use_phm and self.supports_phm()
                   else self.ext_cls.projection_utgs)
        return proj_fn(self.pack, points.contiguous(),
                       points_velocity.contiguous() if points_velocity is not None else None,
                       scale.contiguous(), rotation.contiguous(),
                       opacity.contiguous() if opacity is not None else None,
                       width=width, height=height, ut_alpha=ut_alpha, ut_beta=ut_beta, ut_kappa=ut_kappa,
                       residual_thr_early_stop=self.residual_thr_early_stop,
                       max_residual=self.residual_max_valid, max_margin=self.max_margin)

    def isect_gs_tiles(self, points, scale, rotation, width, height, flags, radii, means2d, depths,
                       points_velocity=None, opacity=None, tile_size_x=16, tile_size_y=16,
                       ut_alpha=0.1, ut_beta=2.0, ut_kappa=0.0, sort=True, double_buffer=True):
        return _C.isect_regular_tiles(means2d, radii, depths, img_width=width, img_height=height,
                                      tile_size_x=tile_size_x, tile_size_y=tile_size_y, sort=sort,
                                      double_buffer=double_buffer)


class PerspectiveCamera(FusedRSCamera):
    """Pinhole; intrinsics [fx, fy, cx, cy] normalised by the image size."""
    ext_cls = _C.PerspectiveCamera

    def __init__(self, q0, t0, normalized_intrinsics, **kw):
        super().__init__(q0, t0, **kw)
        self.normalized_intrinsics = _vec(normalized_intrinsics, 4, self.device)

    @staticmethod
    def intrinsics_from_sized(fx, fy, cx, cy, width, height):
        return torch.tensor([fx / width, fy / height, cx / width, cy / height], dtype=torch.float32)

    @property
    def _pack_data(self):
        return super()._pack_data + [self.normalized_intrinsics]

    def to(self, device):
        super().to(device)
        self.normalized_intrinsics = self.normalized_intrinsics.to(device)
        return self


class FisheyeCamera(FusedRSCamera):
    """OpenCV (Kannala-Brandt) fisheye; intrinsics normalised, k1..k4."""
    ext_cls = _C.OpenCVFisheyeCamera

    def __init__(self, q0, t0, normalized_intrinsics, distortion, **kw):
        super().__init__(q0, t0, **kw)
        self.normalized_intrinsics = _vec(normalized_intrinsics, 4, self.device)
        self.distortion = _vec(distortion, 4, self.device)

    @property
    def _pack_data(self):
        return super()._pack_data + [self.normalized_intrinsics, self.distortion]

    def to(self, device):
        super().to(device)
        self.normalized_intrinsics = self.normalized_intrinsics.to(device)
        self.distortion = self.distortion.to(device)
        return self


def max_valid_radius(normalized_intrinsics, distortion, margin: float = 1.5, search_limit: float = 16.0,
                     num_samples: int = 8192) -> torch.Tensor:
    """Largest camera-space radius r = |xy| / z at which an 8-coefficient
    calibration is trusted (cameras/torch/distortion_utils.py:96-164): the
    smaller of the first r where the radial map rho(r) = r * scale(r) stops
    increasing (past it two ray angles share an image point) and `margin`
    times the radius of the farthest image corner, found by inverting rho on
    its running maximum.  Both are read off the same grid of `num_samples`
    radii in [0, search_limit].  Returns a [..., 1] tensor."""
    dist = distortion.reshape(-1, 8)
    intr = normalized_intrinsics.reshape(-1, 4)
    r = torch.linspace(0.0, search_limit, num_samples, device=dist.device, dtype=dist.dtype)
    r2 = (r * r)[None, :]
    k = [dist[:, i:i + 1] for i in range(8)]  # k1 k2 p1 p2 k3 k4 k5 k6
    rho = r[None, :] * ((1.0 + r2 * (k[0] + r2 * (k[1] + r2 * k[4]))) /
                        (1.0 + r2 * (k[5] + r2 * (k[6] + r2 * k[7]))))
    falls = rho[:, 1:] < rho[:, :-1]
    first_fall = torch.where(falls.any(dim=-1), falls.to(torch.uint8).argmax(dim=-1),
                             torch.full((dist.shape[0],), num_samples - 1, dtype=torch.long, device=dist.device))
    corners = torch.tensor([[0.0, 0.0], [1.0, 0.0], [0.0, 1.0], [1.0, 1.0]], device=dist.device, dtype=dist.dtype)
    reach = ((corners[None] - intr[:, None, 2:]) / intr[:, None, :2]).norm(dim=-1).amax(dim=-1)
    at_corner = torch.searchsorted(rho.cummax(dim=-1).values.contiguous(), reach[:, None])[:, 0]
    at_corner = at_corner.clamp(max=num_samples - 1)
    radius = torch.minimum(r[first_fall], margin * r[at_corner])
    return radius.reshape(*distortion.shape[:-1], 1)


class DistortedPerspectiveCamera(PerspectiveCamera):
    """Pinhole with the OpenCV 8-coefficient model: `distortion` =
    (k1, k2, p1, p2, k3, k4, k5, k6); intrinsics normalised by the image size
    (cameras/ext/distorted_perspective.py, cameras/torch/distorted_perspective.py).
    The pack also carries max_radius^2 (`max_radius`, derived from the
    coefficients and intrinsics, `max_radius_margin` past the image corner):
    points beyond it do not project, rays beyond it are not valid."""
    ext_cls = _C.DistortedPerspectiveCamera
    max_radius_margin: float = 1.5

    def __init__(self, q0, t0, normalized_intrinsics, distortion, **kw):
        super().__init__(q0, t0, normalized_intrinsics, **kw)
        self.distortion = _vec(distortion, 8, self.device)
        self._max_radius = None

    @property
    def max_radius(self) -> torch.Tensor:
        if self._max_radius is None:
            self._max_radius = max_valid_radius(self.normalized_intrinsics.detach(), self.distortion.detach(),
                                                margin=self.max_radius_margin)
        return self._max_radius

    @property
    def _pack_data(self):
        return super()._pack_data + [self.distortion, self.max_radius.reshape(1).square().contiguous()]

    def undistort_map(self, width: int, height: int, normalized_range: bool = False):
        return self.ext_cls.undistort_map(self.pack, width=width, height=height, normalized_range=normalized_range)

    def undistort(self) -> PerspectiveCamera:
        """The same camera without distortion."""
        return PerspectiveCamera(self.q0, self.t0, self.normalized_intrinsics, v=self.v, w=self.w,
                                 rolling_time=self.rolling_time, trigger_time=self.trigger_time,
                                 pose_time=self.pose_time, camera_name=self.camera_name)

    def to(self, device):
        super().to(device)
        self.distortion = self.distortion.to(device)
        self._max_radius = None
        return self


class SphericalCamera(FusedRSCamera):
    """Equirectangular range image; limits [phi_min, phi_range, theta_min, theta_range]."""
    ext_cls = _C.SphericalCamera

    def __init__(self, q0, t0, limits=None, **kw):
        super().__init__(q0, t0, **kw)
        if limits is None:
            limits = [0.0, 2 * np.pi, -np.pi / 2.0, np.pi]
        self.limits = _vec(limits, 4, self.device)

    @property
    def _pack_data(self):
        return super()._pack_data + [self.limits]

    def to(self, device):
        super().to(device)
        self.limits = self.limits.to(device)
        return self

    def isect_gs_tiles(self, points, scale, rotation, width, height, flags, radii, means2d, depths,
                       points_velocity=None, opacity=None, tile_size_x=16, tile_size_y=16,
                       ut_alpha=0.1, ut_beta=2.0, ut_kappa=0.0, sort=True, double_buffer=True):
        return _C.isect_spherical_tiles(
            camera_pack=self.pack, points=points, points_velocity=points_velocity, scale=scale,
            quat=rotation, opacity=opacity, flag=flags, means2d=means2d, radii=radii, depths=depths,
            tile_size_x=tile_size_x, tile_size_y=tile_size_y, img_width=width, img_height=height,
            ut_alpha=ut_alpha, ut_beta=ut_beta, ut_kappa=ut_kappa, sort=sort, double_buffer=double_buffer)


def data_addr_tensor(src: torch.Tensor) -> torch.Tensor:
    """The 64-bit device address of `src` as two float32 words (low, high),
    the form the lidar pack carries it in (ext/lidar.py:14-19)."""
    ptr = src.data_ptr()
    arr = np.array([ptr & 0xFFFFFFFF, ptr >> 32], dtype=np.uint32).view(np.float32)
    return torch.tensor(arr, device=src.device)


def cornering_values_from_pixel_values(vmin, vmax, img_size: int):
    """Angle limits at the image borders from the first/last pixel-centre
    angles (cameras/torch/lidar.py:9-18)."""
    rescale = 0.5 / (img_size - 0.5)
    b = (vmin - vmax * rescale) / (1 - rescale)
    a = 2 * (vmin - b)
    return b, a * img_size + b


class LidarCamera(SphericalCamera):
    """Spinning lidar: per-row elevation table `beam_v` (normalised v of each
    beam) and azimuth/elevation limits.  The pack holds beam_v's device
    address, so the camera keeps beam_v alive."""
    ext_cls = _C.LidarCamera

    def __init__(self, q0, t0, limits, beam_v, **kw):
        super().__init__(q0, t0, limits=limits, **kw)
        self.beam_v = torch.as_tensor(beam_v, dtype=torch.float32, device=self.device).contiguous()

    @classmethod
    def create(cls, q0, t0, beam_angles, phi_min, phi_range, **kw):
        """Limits and beam table from beam elevation angles (radians), as
        LidarCameraTorch.create (cameras/torch/lidar.py:26-57)."""
        beam_angles = torch.as_tensor(beam_angles, dtype=torch.float32)
        num_beams = beam_angles.shape[-1]
        theta_min, theta_max = cornering_values_from_pixel_values(
            vmin=beam_angles.amax(dim=-1), vmax=beam_angles.amin(dim=-1), img_size=num_beams)
        theta_min = theta_min.clamp(-np.pi / 2, np.pi / 2)
        theta_max = theta_max.clamp(-np.pi / 2, np.pi / 2)
        theta_range = theta_max - theta_min
        limits = torch.stack([torch.as_tensor(float(phi_min)), torch.as_tensor(float(phi_range)),
                              theta_min, theta_range])
        beam_v = (beam_angles.contiguous() - theta_min) / theta_range
        return cls(q0, t0, limits=limits, beam_v=beam_v, **kw)

    @property
    def num_beams(self):
        return self.beam_v.shape[-1]

    @property
    def _pack_data(self):
        return super()._pack_data + [data_addr_tensor(self.beam_v)]

    def to(self, device):
        super().to(device)
        self.beam_v = self.beam_v.to(device).contiguous()
        return self

    def isect_gs_tiles(self, points, scale, rotation, width, height, flags, radii, means2d, depths,
                       points_velocity=None, opacity=None, tile_size_x=16, tile_size_y=16,
                       ut_alpha=0.1, ut_beta=2.0, ut_kappa=0.0, sort=True, double_buffer=True):
        elev_boundaries = self.beam_v[::tile_size_y].contiguous()
        return _C.isect_lidar_tiles(
            camera_pack=self.pack, points=points, points_velocity=points_velocity, scale=scale,
            quat=rotation, opacity=opacity, flag=flags, means2d=means2d, radii=radii, depths=depths,
            elev_boundaries=elev_boundaries, tile_size_x=tile_size_x, img_width=width, img_height=height,
            ut_alpha=ut_alpha, ut_beta=ut_beta, ut_kappa=ut_kappa, sort=sort, double_buffer=double_buffer)


def look_at_quat(eye, target, up=(0.0, 0.0, 1.0)) -> np.ndarray:
    """Camera->world rotation (w, x, y, z) of a camera at `eye` looking at
    `target`, camera +Z forward, +X right, +Y down (world +Z up)."""
    eye, target, up = (np.asarray(a, dtype=np.float64) for a in (eye, target, up))
    z = target - eye
    z /= np.linalg.norm(z)
    x = np.cross(z, up)
    if np.linalg.norm(x) < 1e-9:
        x = np.cross(z, np.array([0.0, 1.0, 0.0]))
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    R = np.stack([x, y, z], axis=1)  # columns = camera axes in world
    return rotmat_to_quat(R)


def rotmat_to_quat(R: np.ndarray) -> np.ndarray:
    """Rotation matrix -> unit quaternion (w, x, y, z), w >= 0."""
    m = R
    tr = m[0, 0] + m[1, 1] + m[2, 2]
    if tr > 0:
        s = np.sqrt(tr + 1.0) * 2
        q = [0.25 * s, (m[2, 1] - m[1, 2]) / s, (m[0, 2] - m[2, 0]) / s, (m[1, 0] - m[0, 1]) / s]
    elif m[0, 0] > m[1, 1] and m[0, 0] > m[2, 2]:
        s = np.sqrt(1.0 + m[0, 0] - m[1, 1] - m[2, 2]) * 2
        q = [(m[2, 1] - m[1, 2]) / s, 0.25 * s, (m[0, 1] + m[1, 0]) / s, (m[0, 2] + m[2, 0]) / s]
    elif m[1, 1] > m[2, 2]:
        s = np.sqrt(1.0 + m[1, 1] - m[0, 0] - m[2, 2]) * 2
        q = [(m[0, 2] - m[2, 0]) / s, (m[0, 1] + m[1, 0]) / s, 0.25 * s, (m[1, 2] + m[2, 1]) / s]
    else:
        s = np.sqrt(1.0 + m[2, 2] - m[0, 0] - m[1, 1]) * 2
        q = [(m[1, 0] - m[0, 1]) / s, (m[0, 2] + m[2, 0]) / s, (m[1, 2] + m[2, 1]) / s, 0.25 * s]
    q = np.asarray(q)
    q /= np.linalg.norm(q)
    if q[0] < 0:
        q = -q
    return q.astype(np.float32)
