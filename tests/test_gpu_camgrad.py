"""Camera-parameter gradients on the GPU against the CPU oracle: the
backward of camera_rays (every camera model; world / camera space;
normalised / raw rays; with and without ray origins), of pixel_time(_delta)
and of pixel_time(_delta)_from_uv (pack and uv gradients), through the
reference's `_C.<Camera>.camera_rays / pixel_time*` autograd surface and
through the camera objects' own tensors (q0, t0, ... -> pack -> rays).

Tolerance: per camera tensor, |gpu - oracle| <= 1e-3 (|oracle| + max|oracle|
of that tensor) — float32 per-pixel terms summed in a different order than
the oracle's float64 sums; words without a gradient must be exactly zero and
d_uv (one float32 product) bit-exact."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import camera_inputs, to_np
from tests.test_gpu_cameras import KINDS, _specs

pytestmark = pytest.mark.gpu

GROUPS = [(0, 4), (4, 7), (7, 10), (10, 13), (14, 16), (16, 17), (17, 18), (18, 20), (20, 22), (22, 24),
          (24, 28), (28, 32), (32, 36)]


@pytest.fixture(scope="module")
def specs(cuda):
    return _specs()


def check_pack_grad(got, want, what, rtol=1e-3):
    got = to_np(got).reshape(-1).astype(np.float64)
    assert got.shape == want.shape, f"{what}: {got.shape} vs {want.shape}"
    for a, b in GROUPS:
        if a >= len(want):
            break
        g, w = got[a:b], want[a:b]
        bound = rtol * (np.abs(w) + np.abs(w).max()) + 1e-30
        assert (np.abs(g - w) <= bound).all(), f"{what} words {a}:{b}: gpu {g} vs oracle {w}"
    assert got[13] == 0.0, f"{what}: padding word got a gradient"


def _upstream(H, W, seed, kind=None, pack=None):
    """Upstream ray gradients (non-zero mean, so the sums do not cancel).  For
    the fisheye they are zero at ill-conditioned pixels: where the forward's
    float32 solve did not converge (those rays are whatever the last Newton
    step left, on either side), and near the distortion's turning point
    (d theta_d / d theta < 0.05), where theta = theta(delta) amplifies the
    float32 rounding of the solve by 1/theta_d' — any float32 implementation,
    the reference's included, lands a different gradient there."""
    rng = np.random.default_rng(seed)
    go = (rng.normal(size=(H, W, 3)) + 0.3).astype(np.float32)
    gd = (rng.normal(size=(H, W, 3)) + 0.3).astype(np.float32)
    if kind == "fisheye":
        _, rc, valid = O.camera_rays("fisheye", pack, W, H, world_space=False, normalized=True)
        th = np.arccos(np.clip(rc[..., 2].astype(np.float64), -1.0, 1.0))
        k1, k2, k3, k4 = (float(x) for x in pack[24:28])
        t2 = th * th
        der = 1 + t2 * (3 * k1 + t2 * (5 * k2 + t2 * (7 * k3 + t2 * 9 * k4)))
        keep = valid & (der > 0.05)
        assert keep.mean() > 0.5, keep.mean()
        go *= keep[..., None]
        gd *= keep[..., None]
    return go, gd


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("world,normalized", [(True, True), (False, True), (True, False)])
def test_ray_gradients_match_oracle(specs, cuda, kind, world, normalized):
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    go, gd = _upstream(H, W, 11, kind, pack)
    p = cam.pack.detach().clone().requires_grad_(True)
    ro, rd = cam.ext_cls.camera_rays(p, width=W, height=H, world_space=world, normalized=normalized)
    loss = (ro * torch.from_numpy(go).to(cuda)).sum() + (rd * torch.from_numpy(gd).to(cuda)).sum()
    loss.backward()
    want = O.camera_rays_bwd(kind, pack, W, H, go, gd, world, normalized, elev=elev)
    check_pack_grad(p.grad, want, f"{kind} world={world} normalized={normalized}")
    if kind in ("spherical", "lidar"):
        assert not to_np(p.grad).reshape(-1)[18:].any(), "range-image limits / table address got a gradient"
    # deterministic: the same backward twice gives the same bits
    g1 = p.grad.clone()
    p.grad = None
    ro, rd = cam.ext_cls.camera_rays(p, width=W, height=H, world_space=world, normalized=normalized)
    ((ro * torch.from_numpy(go).to(cuda)).sum() + (rd * torch.from_numpy(gd).to(cuda)).sum()).backward()
    assert torch.equal(g1, p.grad)


def test_ray_gradients_full_hd(cuda):
    """1920 x 1080 moving pinhole (more pixels than the reduction grid has
    threads, so every thread strides over many pixels)."""
    from xsimgs_b200 import scenes
    spec = scenes.pinhole(1920, 1080, 1400.0, 1400.0, (0.0, 0.0, 1.6), (5.0, 1.0, 1.4), rolling_time=(0.0, 0.03),
                          v=(8.0, 0.2, 0.0), w=(0.0, 0.01, 0.4), trigger_time=0.0, pose_time=0.015)
    cam, pack, _ = camera_inputs(spec, cuda)
    go, gd = _upstream(1080, 1920, 12)
    p = cam.pack.detach().clone().requires_grad_(True)
    ro, rd = cam.ext_cls.camera_rays(p, width=1920, height=1080)
    ((ro * torch.from_numpy(go).to(cuda)).sum() + (rd * torch.from_numpy(gd).to(cuda)).sum()).backward()
    check_pack_grad(p.grad, O.camera_rays_bwd("pinhole", pack, 1920, 1080, go, gd), "pinhole 1080p")


@pytest.mark.parametrize("kind", ["pinhole", "fisheye", "distorted"])
def test_camera_tensors_receive_gradients(specs, cuda, kind):
    """Leaf camera tensors -> differentiable pack -> rays; also with the
    origins not returned (ray_d gradient only)."""
    spec = specs[kind]
    cam, pack, _ = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    leaves = [cam.q0, cam.t0, cam.v, cam.w, cam.rolling_time, cam.trigger_time, cam.pose_time,
              cam.normalized_intrinsics] + ([cam.distortion] if kind != "pinhole" else [])
    for t in leaves:
        t.requires_grad_(True)
    go, gd = _upstream(H, W, 13, kind, pack)
    for return_origins in (True, False):
        for t in leaves:
            t.grad = None
        ro, rd = cam.camera_rays(W, H, return_origins=return_origins)
        loss = (rd * torch.from_numpy(gd).to(cuda)).sum()
        if return_origins:
            loss = loss + (ro * torch.from_numpy(go).to(cuda)).sum()
        else:
            assert ro is None
        loss.backward()
        want = O.camera_rays_bwd(kind, pack, W, H, go if return_origins else None, gd)
        # the leaves' gradients laid out as pack words: padding words 13 and
        # (16-byte aligned impls) 18..19 get none, nor does max_radius^2 (32)
        # or the distorted pack's tail padding (33..35)
        aligned = kind in ("fisheye", "distorted")
        got = np.concatenate([to_np(t.grad).reshape(-1) for t in leaves[:4]] + [[0.0]] +
                             [to_np(t.grad).reshape(-1) for t in leaves[4:7]] +
                             ([[0.0, 0.0]] if aligned else []) +
                             [to_np(t.grad).reshape(-1) for t in leaves[7:]] +
                             ([[0.0] * 4] if kind == "distorted" else []))
        check_pack_grad(got, want, f"{kind} leaves origins={return_origins}")
        if aligned:
            assert not want[18:20].any()
        if kind == "distorted":
            assert not want[32:].any()


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("delta", [False, True])
def test_pixel_time_gradients_match_oracle(specs, cuda, kind, delta):
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    rng = np.random.default_rng(14)
    g = (rng.normal(size=(H, W)) + 0.2).astype(np.float32)
    p = cam.pack.detach().clone().requires_grad_(True)
    fn = cam.ext_cls.pixel_time_delta if delta else cam.ext_cls.pixel_time
    (fn(p, width=W, height=H) * torch.from_numpy(g).to(cuda)).sum().backward()
    want, _ = O.pixel_time_bwd(kind, pack, g, delta, W=W, H=H, elev=elev)
    check_pack_grad(p.grad, want, f"{kind} pixel_time delta={delta}")
    assert not to_np(p.grad).reshape(-1)[:14].any() and not to_np(p.grad).reshape(-1)[18:].any()

    uv = rng.uniform(0, 1, size=(3, 1001, 2)).astype(np.float32)  # batched leading dims
    gu = (rng.normal(size=(3, 1001)) + 0.2).astype(np.float32)
    p.grad = None
    tuv = torch.from_numpy(uv).to(cuda).requires_grad_(True)
    fn = cam.ext_cls.pixel_time_delta_from_uv if delta else cam.ext_cls.pixel_time_from_uv
    (fn(p, tuv) * torch.from_numpy(gu).to(cuda)).sum().backward()
    want, d_uv = O.pixel_time_bwd(kind, pack, gu, delta, uv=uv)
    check_pack_grad(p.grad, want, f"{kind} pixel_time_from_uv delta={delta}")
    np.testing.assert_array_equal(to_np(tuv.grad).reshape(-1, 2), d_uv)


def test_empty_inputs(specs, cuda):
    """Zero uv / points: every entry point returns empty outputs (and a zero
    pack gradient) instead of rejecting the empty tensors."""
    from xsimgs_b200 import _C
    cam, _, _ = camera_inputs(specs["pinhole"], cuda)
    p = cam.pack.detach().clone().requires_grad_(True)
    tuv = torch.zeros(0, 2, device=cuda, requires_grad=True)
    cam.ext_cls.pixel_time_from_uv(p, tuv).sum().backward()
    assert not p.grad.any() and tuv.grad.shape == (0, 2)
    pts = torch.zeros(0, 3, device=cuda)
    uvdt, mask = cam.ext_cls.projection(cam.pack, pts)
    assert uvdt.shape == (0, 4) and mask.shape == (0,)
    q = torch.zeros(0, 4, device=cuda)
    flags, radii, means2d, depths = cam.ext_cls.projection_utgs(cam.pack, pts, None, pts, q, None, width=64, height=48)
    assert flags.shape == (0,) and radii.shape == (0, 2) and depths.shape == (0,)
    _C.mask_radii(torch.zeros(0, dtype=torch.bool, device=cuda), radii)


@pytest.mark.parametrize("dynamic", [False, True])
def test_render_gradient_reaches_camera(specs, cuda, dynamic):
    """ut_gs_render with camera tensors that require grad: the camera
    gradient equals the oracle's ray (and, for a dynamic scene, pixel-time)
    backward applied to the ray gradients the compositing backward produces
    for the same render with the rays passed in as leaves."""
    from xsimgs_b200.rendering import ut_gs_render
    spec = specs["pinhole"]
    cam, pack, _ = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    g = torch.Generator().manual_seed(5)
    n = 20_000
    d = torch.randn(n, 3, generator=g)
    d = d / d.norm(dim=1, keepdim=True)
    means = (d * (3.0 + 20.0 * torch.rand(n, 1, generator=g)) + torch.tensor((0.0, 0.0, 1.6))).to(cuda)
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.4 - 1.8).to(cuda)
    quats = torch.nn.functional.normalize(torch.randn(n, 4, generator=g), dim=1).to(cuda)
    opac = torch.sigmoid(torch.randn(n, generator=g)).to(cuda)
    colors = torch.rand(n, 3, generator=g).to(cuda)
    vel = (torch.randn(n, 3, generator=g) * 0.5).to(cuda) if dynamic else None
    w_img = torch.randn(H, W, 3, generator=g).to(cuda)
    leaves = [cam.q0, cam.t0, cam.v, cam.w, cam.rolling_time, cam.trigger_time, cam.pose_time,
              cam.normalized_intrinsics]
    for t in leaves:
        t.requires_grad_(True)
    color, _, _, _ = ut_gs_render(cam, means, scales, quats, opac, W, H, colors=colors, points_velocity=vel)
    (color * w_img).sum().backward()
    got = np.concatenate([to_np(t.grad).reshape(-1) for t in leaves[:4]] + [[0.0]] +
                         [to_np(t.grad).reshape(-1) for t in leaves[4:]])
    for t in leaves:
        t.requires_grad_(False)
    with torch.no_grad():
        ro, rd = cam.camera_rays(W, H)
        rt = cam.image_time_delta(ro) if dynamic else None
    ro.requires_grad_(True)
    rd.requires_grad_(True)
    if dynamic:
        rt.requires_grad_(True)
    color, _, _, _ = ut_gs_render(cam, means, scales, quats, opac, W, H, colors=colors, points_velocity=vel,
                                  ray_o=ro, ray_d=rd, ray_time_delta=rt)
    (color * w_img).sum().backward()
    want = O.camera_rays_bwd("pinhole", pack, W, H, to_np(ro.grad), to_np(rd.grad))
    if dynamic:
        want += O.pixel_time_bwd("pinhole", pack, to_np(rt.grad), True, W=W, H=H)[0]
    assert np.abs(want).max() > 0
    check_pack_grad(got, want, f"render -> camera dynamic={dynamic}")
