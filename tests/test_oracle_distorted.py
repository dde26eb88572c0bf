"""The OpenCV 8-coefficient pinhole of the CPU oracle (the
DistortedPerspectiveCamera of csrc/cameras/distorted_perspective.cu) checked
by properties that need no reference output: its camera rays invert its
projection (distort(undistort(x)) = x, and a world point on a pixel's ray
projects back onto that pixel), the undistort map is the distortion of the
pixel grid, rays past the trusted radius are invalid and points past it do
not project, and max_valid_radius finds the fold of a known model."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_oracle_camgrad import DIST8, camera_pack


def distort_np(x, y, k):
    k1, k2, p1, p2, k3, k4, k5, k6 = (float(v) for v in k)
    r2 = x * x + y * y
    sc = (1 + r2 * (k1 + r2 * (k2 + r2 * k3))) / (1 + r2 * (k4 + r2 * (k5 + r2 * k6)))
    return x * sc + 2 * p1 * x * y + p2 * (r2 + 2 * x * x), y * sc + p1 * (r2 + 2 * y * y) + 2 * p2 * x * y


def _grid(W, H, pack):
    u = (np.arange(W, dtype=np.float32) + np.float32(0.5)) / np.float32(W)
    v = (np.arange(H, dtype=np.float32) + np.float32(0.5)) / np.float32(H)
    U, V = np.meshgrid(u, v)
    return U.astype(np.float64), V.astype(np.float64)


def test_rays_invert_the_distortion():
    W, H = 64, 48
    pack = camera_pack("distorted")
    _, rd, valid = O.camera_rays("distorted", pack, W, H, world_space=False, normalized=False)
    assert valid.all()
    np.testing.assert_array_equal(rd[..., 2], 1.0)
    U, V = _grid(W, H, pack)
    xd, yd = distort_np(rd[..., 0].astype(np.float64), rd[..., 1].astype(np.float64), pack[24:32])
    np.testing.assert_allclose(xd * pack[20] + pack[22], U, atol=2e-6)
    np.testing.assert_allclose(yd * pack[21] + pack[23], V, atol=2e-6)


def test_projection_round_trip():
    """World points on the pixels' rays (static camera) project back onto the
    pixel centres, with the point's depth along +z."""
    W, H = 40, 30
    pack = camera_pack("distorted")
    pack[0:4] /= np.linalg.norm(pack[0:4])  # the projection takes q0 as a unit quaternion
    pack[7:13] = 0.0  # no motion: the projection's time solve is trivial
    pack[14:16] = 0.0
    ro, rd, _ = O.camera_rays("distorted", pack, W, H, world_space=True, normalized=True)
    rng = np.random.default_rng(0)
    depth = rng.uniform(2.0, 20.0, size=(H, W, 1)).astype(np.float32)
    pts = (ro + rd * depth).reshape(-1, 3)
    uvdt, mask = O.projection("distorted", pack, pts)
    assert mask.all()
    U, V = _grid(W, H, pack)
    np.testing.assert_allclose(uvdt[:, 0], U.reshape(-1), atol=5e-6)
    np.testing.assert_allclose(uvdt[:, 1], V.reshape(-1), atol=5e-6)
    _, rc, _ = O.camera_rays("distorted", pack, W, H, world_space=False, normalized=True)
    np.testing.assert_allclose(uvdt[:, 2], (depth * rc[..., 2:3]).reshape(-1), rtol=1e-5)


def test_trusted_radius():
    W, H = 32, 24
    pack = camera_pack("distorted")
    _, rc, valid = O.camera_rays("distorted", pack, W, H, world_space=False, normalized=False)
    r2 = (rc[..., :2].astype(np.float64) ** 2).sum(-1)
    pack[32] = np.float32(np.median(r2))
    _, _, valid = O.camera_rays("distorted", pack, W, H, world_space=False, normalized=False)
    np.testing.assert_array_equal(valid, r2 <= pack[32])
    pts = np.concatenate([rc.reshape(-1, 3) * 5.0], 0).astype(np.float32)
    pack[0:4] = (1, 0, 0, 0)
    pack[4:13] = 0.0
    pack[14:16] = 0.0
    uvdt, mask = O.projection("distorted", pack, pts)
    np.testing.assert_array_equal(mask, (r2 <= pack[32]).reshape(-1))


@pytest.mark.parametrize("normalized_range", [False, True])
def test_undistort_map_is_the_distorted_grid(normalized_range):
    W, H = 48, 32
    pack = camera_pack("distorted")
    got = O.undistort_map(pack, W, H, normalized_range)
    U, V = _grid(W, H, pack)
    xd, yd = distort_np((U - pack[22]) / pack[20], (V - pack[23]) / pack[21], pack[24:32])
    want = np.stack([xd * pack[20] + pack[22], yd * pack[21] + pack[23]], -1)
    if not normalized_range:
        want = want * 2 - 1
    np.testing.assert_allclose(got, want, atol=3e-6)


def test_max_valid_radius():
    from xsimgs_b200.cameras import max_valid_radius
    step = 16.0 / 8191
    # rho(r) = r (1 - 0.3 r^2) turns over at r = 1 / sqrt(0.9)
    d = torch.tensor([-0.3, 0, 0, 0, 0, 0, 0, 0], dtype=torch.float64)
    wide = torch.tensor([0.05, 0.05, 0.5, 0.5], dtype=torch.float64)  # corner far past the fold
    r = float(max_valid_radius(wide, d))
    assert abs(r - 1 / np.sqrt(0.9)) <= step
    # a long lens reaches margin x its corner first: the corner's rho is
    # |(1,1) - c| / f and r maps through the (here undistorted) rho = r
    d0 = torch.zeros(8, dtype=torch.float64)
    tele = torch.tensor([2.0, 3.0, 0.5, 0.5], dtype=torch.float64)
    r = float(max_valid_radius(tele, d0, margin=1.5))
    corner = float(np.hypot(0.5 / 2.0, 0.5 / 3.0))
    assert abs(r - 1.5 * corner) <= 1.5 * step
    # batched: one radius per camera
    out = max_valid_radius(torch.stack([wide, tele]), torch.stack([d, d0]))
    assert out.shape == (2, 1)
    # the test camera of the distorted checks stays inside its trusted radius
    p = camera_pack("distorted")
    r = float(max_valid_radius(torch.tensor(p[18:22]), torch.tensor(np.array(DIST8, np.float32))))
    assert r > 1.0
