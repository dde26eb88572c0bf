"""Seeded synthetic scenes with the shapes and value distributions of the
benchmark configurations (no datasets or checkpoints are needed).

C1  10k Gaussians in front of one 256x256 pinhole (fx = fy = 256), SH degree 0.
C2  1M Gaussians in a 100 x 100 x 20 m street-like box (70 % on a ground
    plane z ~ N(0, 0.2), 30 % uniform), SH degree 3 (DC ~ U(0,1) as SH,
    higher bands ~ N(0, 0.05)), one 1920x1080 pinhole (fx = fy = 1200) at
    (-55, 0, 1.6) looking +X.
C3  the C2 recipe at 2M Gaussians seen by a 6-camera rig at (0, 0, 1.6):
    pinholes 1920x1080 at yaw 0/120/240 deg, KB fisheyes 1280x960
    (fx = fy = 400 px, k1..k4 ~ U(-0.05, 0.05)) at yaw 60/180/300 deg.
C4  a 128-beam x 2048-column lidar (elevations uniform in [-25, 15] deg) at
    (0, 0, 1.8) over the C2 recipe; one intensity channel.

Everything is generated on the CPU with torch.Generator(seed) and returned as
CPU float32 tensors; move them with .to(device).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .rendering.sh import rgb_to_sh0
from .cameras.ext_camera import look_at_quat


@dataclass
class GaussianScene:
    means: torch.Tensor      # [N, 3]
    quats: torch.Tensor      # [N, 4] wxyz, unit
    scales: torch.Tensor     # [N, 3] activated (exp of log-scale)
    opacities: torch.Tensor  # [N] activated (sigmoid)
    sh: torch.Tensor         # [N, K, 3]
    sh_degree: int

    @property
    def n(self) -> int:
        return self.means.shape[0]

    def to(self, device) -> "GaussianScene":
        return GaussianScene(*(t.to(device) for t in (self.means, self.quats, self.scales,
                                                      self.opacities, self.sh)), self.sh_degree)

    def params(self):
        return dict(means=self.means, quats=self.quats, scales=self.scales,
                    opacities=self.opacities, sh=self.sh)


def _quats(g, n):
    q = torch.randn(n, 4, generator=g)
    return q / q.norm(dim=-1, keepdim=True)


def _sh(g, n, degree, dc_rgb=None):
    k = (degree + 1) ** 2
    sh = torch.randn(n, k, 3, generator=g) * 0.05
    rgb = torch.rand(n, 3, generator=g) if dc_rgb is None else dc_rgb
    sh[:, 0, :] = rgb_to_sh0(rgb)
    return sh


def c1_scene(n: int = 10_000, seed: int = 0) -> GaussianScene:
    g = torch.Generator().manual_seed(seed)
    means = torch.rand(n, 3, generator=g) * 10.0 - 5.0
    means[:, 2] += 10.0  # z in [5, 15] in front of the camera
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.5 - 2.0)
    quats = _quats(g, n)
    opac = torch.sigmoid(torch.randn(n, generator=g))
    rgb = torch.rand(n, 3, generator=g)
    sh = rgb_to_sh0(rgb).view(n, 1, 3)
    return GaussianScene(means, quats, scales, opac, sh, 0)


def street_scene(n: int = 1_000_000, seed: int = 0, sh_degree: int = 3) -> GaussianScene:
    g = torch.Generator().manual_seed(seed)
    n_ground = int(round(0.7 * n))
    xy = torch.rand(n, 2, generator=g) * 100.0 - 50.0
    z = torch.empty(n)
    z[:n_ground] = torch.randn(n_ground, generator=g) * 0.2
    z[n_ground:] = torch.rand(n - n_ground, generator=g) * 20.0
    means = torch.cat([xy, z[:, None]], dim=1)
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.7 - 3.0)
    quats = _quats(g, n)
    opac = torch.sigmoid(torch.randn(n, generator=g) * 1.5)
    sh = _sh(g, n, sh_degree)
    return GaussianScene(means, quats, scales, opac, sh, sh_degree)


@dataclass
class CameraSpec:
    kind: str            # "pinhole" | "fisheye" | "distorted" | "lidar" | "spherical"
    width: int
    height: int
    q0: np.ndarray       # camera->world wxyz
    t0: np.ndarray
    intrinsics: np.ndarray | None = None   # normalised fx, fy, cx, cy
    distortion: np.ndarray | None = None
    beam_angles: np.ndarray | None = None  # lidar, radians
    phi_min: float = 0.0
    phi_range: float = 2 * math.pi
    rolling_time: tuple = (0.0, 0.0)
    trigger_time: float = 0.0
    pose_time: float = 0.0
    v: tuple = (0.0, 0.0, 0.0)
    w: tuple = (0.0, 0.0, 0.0)

    def make(self, device):
        from .cameras import DistortedPerspectiveCamera, PerspectiveCamera, FisheyeCamera, LidarCamera, SphericalCamera
        kw = dict(v=self.v, w=self.w, rolling_time=self.rolling_time, trigger_time=self.trigger_time,
                  pose_time=self.pose_time, device=device)
        q0 = torch.as_tensor(self.q0, dtype=torch.float32, device=device)
        t0 = torch.as_tensor(self.t0, dtype=torch.float32, device=device)
        if self.kind == "pinhole":
            return PerspectiveCamera(q0, t0, self.intrinsics, **kw)
        if self.kind == "fisheye":
            return FisheyeCamera(q0, t0, self.intrinsics, self.distortion, **kw)
        if self.kind == "distorted":
            return DistortedPerspectiveCamera(q0, t0, self.intrinsics, self.distortion, **kw)
        if self.kind == "lidar":
            cam = LidarCamera.create(q0, t0, torch.as_tensor(self.beam_angles, dtype=torch.float32),
                                     self.phi_min, self.phi_range, **kw)
            return cam.to(device)
        return SphericalCamera(q0, t0, **kw)


def pinhole(width, height, fx, fy, eye, target, **kw) -> CameraSpec:
    intr = np.array([fx / width, fy / height, 0.5, 0.5], dtype=np.float32)
    return CameraSpec("pinhole", width, height, look_at_quat(eye, target), np.asarray(eye, np.float32),
                      intrinsics=intr, **kw)


def c1_camera() -> CameraSpec:
    # camera at the origin looking +Z: the identity rotation
    return CameraSpec("pinhole", 256, 256, np.array([1, 0, 0, 0], np.float32), np.zeros(3, np.float32),
                      intrinsics=np.array([1.0, 1.0, 0.5, 0.5], np.float32))


def c2_camera() -> CameraSpec:
    return pinhole(1920, 1080, 1200.0, 1200.0, eye=(-55.0, 0.0, 1.6), target=(0.0, 0.0, 1.6))


def _yaw_target(eye, yaw_deg):
    a = math.radians(yaw_deg)
    return (eye[0] + math.cos(a), eye[1] + math.sin(a), eye[2])


def c3_rig(seed: int = 0, eight: bool = False) -> list[CameraSpec]:
    """6-camera rig (C3); eight=True adds pinholes at yaw 30/210 (C3-8)."""
    rng = np.random.default_rng(seed)
    eye = (0.0, 0.0, 1.6)
    cams = []
    for i, yaw in enumerate(range(0, 360, 60)):
        if i % 2 == 0:
            cams.append(pinhole(1920, 1080, 1200.0, 1200.0, eye, _yaw_target(eye, yaw)))
        else:
            intr = np.array([400.0 / 1280, 400.0 / 960, 0.5, 0.5], np.float32)
            dist = rng.uniform(-0.05, 0.05, size=4).astype(np.float32)
            cams.append(CameraSpec("fisheye", 1280, 960, look_at_quat(eye, _yaw_target(eye, yaw)),
                                   np.asarray(eye, np.float32), intrinsics=intr, distortion=dist))
    if eight:
        for yaw in (30, 210):
            cams.append(pinhole(1920, 1080, 1200.0, 1200.0, eye, _yaw_target(eye, yaw)))
    return cams


def c4_lidar(beams: int = 128, columns: int = 2048) -> CameraSpec:
    # beam 0 is the highest elevation (row 0 at the top), as spinning lidars index them
    ang = np.radians(np.linspace(15.0, -25.0, beams)).astype(np.float32)
    # identity rotation: the lidar frame is the world frame (z up); azimuth
    # 0 at -y, increasing towards -x (cartesian_to_spherical of the reference)
    return CameraSpec("lidar", columns, beams, np.array([1, 0, 0, 0], np.float32),
                      np.array([0.0, 0.0, 1.8], np.float32), beam_angles=ang)


def upstream_grads(height: int, width: int, channels: int, seed: int = 1):
    """N(0, 1) gradients of the colour, depth and alpha images."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(height, width, channels, generator=g), torch.randn(height, width, generator=g),
            torch.randn(height, width, generator=g))


# ------------------------------------------------------------------ C5 --
SMPL_PARENTS = (-1, 0, 0, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 9, 9, 12, 13, 14, 16, 17, 18, 19, 20, 21)


def axis_angle_to_quat(aa: torch.Tensor) -> torch.Tensor:
    """Rotation vectors [..., 3] -> unit quaternions [..., 4] (w, x, y, z)."""
    theta = aa.norm(dim=-1, keepdim=True)
    half = 0.5 * theta
    k = torch.where(theta > 1e-8, torch.sin(half) / theta.clamp_min(1e-8), 0.5 - theta ** 2 / 48.0)
    return torch.cat([torch.cos(half), aa * k], dim=-1)


def c5_smpl(n_bodies: int = 8, gauss_per_body: int = 20_000, template_verts: int = 6890, seed: int = 0,
            pose_sigma: float = 0.3):
    """Synthetic SMPL-style bodies (no model assets are needed): a template
    of `template_verts` vertices ~ N(0, 0.3), 24 joints at the means of the
    vertices nearest to 24 seed vertices, per-vertex LBS weights
    Dirichlet(0.5) over the 4 nearest joints, axis-angle pose ~ N(0,
    pose_sigma) per joint, a0_inv = identity.  Each body carries
    `gauss_per_body` Gaussians bound to random template vertices (rest
    position = vertex + N(0, 0.01), inheriting its weights), so V =
    gauss_per_body.  Bodies stand on the ground 6..14 m in front of the
    origin (+X), one instance per body.

    Returns a dict of CPU tensors with the reference's layouts (quaternions
    w, x, y, z; ids uint32 stored as int32)."""
    g = torch.Generator().manual_seed(seed)
    tv = torch.randn(template_verts, 3, generator=g) * 0.3
    seeds = tv[torch.randperm(template_verts, generator=g)[:24]]
    d = torch.cdist(seeds, tv)                                   # [24, T]
    near = d.topk(64, dim=1, largest=False).indices               # [24, 64]
    joints0 = tv[near].mean(dim=1)                                # [24, 3]
    dj = torch.cdist(tv, joints0)                                 # [T, 24]
    nn4 = dj.topk(4, dim=1, largest=False).indices                # [T, 4]
    conc = torch.full((template_verts, 4), 0.5)
    w4 = _dirichlet(g, conc)
    tw = torch.zeros(template_verts, 24)
    tw.scatter_(1, nn4, w4)
    V = gauss_per_body
    bind = torch.randint(0, template_verts, (n_bodies, V), generator=g)
    vertices = tv[bind] + torch.randn(n_bodies, V, 3, generator=g) * 0.01
    weights = tw[bind].permute(0, 2, 1).contiguous()               # [N, 24, V]
    quats = torch.randn(n_bodies, V, 4, generator=g)
    quats = quats / quats.norm(dim=-1, keepdim=True)
    local_q = axis_angle_to_quat(torch.randn(n_bodies, 24, 3, generator=g) * pose_sigma)
    joints = joints0.expand(n_bodies, 24, 3).contiguous()
    a0_inv_q = torch.zeros(n_bodies, 24, 4)
    a0_inv_q[..., 0] = 1.0
    a0_inv_t = torch.zeros(n_bodies, 24, 3)
    instance_t = torch.stack([6.0 + 8.0 * torch.rand(n_bodies, generator=g),
                              -4.0 + 8.0 * torch.rand(n_bodies, generator=g), torch.full((n_bodies,), 0.9)], dim=1)
    instance_v = torch.randn(n_bodies, 3, generator=g) * 0.5
    instance_ids = torch.arange(n_bodies, dtype=torch.int32)
    return dict(local_q=local_q, joints=joints, a0_inv_q=a0_inv_q, a0_inv_t=a0_inv_t, vertices=vertices,
                quats=quats, weights=weights, instance_ids=instance_ids, instance_t=instance_t,
                instance_v=instance_v, valid_ids=torch.arange(n_bodies, dtype=torch.int32))


def _dirichlet(g, conc):
    """Dirichlet samples from gamma draws (Marsaglia-Tsang for shape >= 1,
    boosted for shape < 1) with the given generator."""
    a = conc + 1.0
    d = a - 1.0 / 3.0
    c = 1.0 / torch.sqrt(9.0 * d)
    out = torch.empty_like(conc)
    todo = torch.ones_like(conc, dtype=torch.bool)
    while todo.any():
        x = torch.randn(conc.shape, generator=g)
        v = (1.0 + c * x) ** 3
        u = torch.rand(conc.shape, generator=g)
        ok = (v > 0) & (torch.log(u.clamp_min(1e-30)) < 0.5 * x * x + d - d * v + d * torch.log(v.clamp_min(1e-30)))
        take = todo & ok
        out[take] = (d * v)[take]
        todo &= ~ok
    u = torch.rand(conc.shape, generator=g)
    gam = out * u ** (1.0 / conc)
    return gam / gam.sum(dim=-1, keepdim=True)
