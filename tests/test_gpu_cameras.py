"""Every camera model on the GPU against the CPU oracle, stage by stage:
rays, pixel times, the rolling-shutter point projection (all three modes),
the UT projection (with the PHM variant of the range-image cameras), regular /
spherical / lidar tiling and compositing forward + backward over each camera's
own rays and tiles, plus the dynamic (per-Gaussian velocity) compositing.

Cameras move during the exposure (linear and angular velocity, rolling
shutter), so the Newton solve of the projection and the flag-2 split of the
range-image tilers are exercised.  Tolerances: tests/helpers.py; the
projection's time output may differ by the solver's early-stop threshold
(1e-4 s), because CPU and GPU libm can stop one iteration apart."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_grads_close, assert_images_close, camera_inputs, to_np, zero_at

pytestmark = pytest.mark.gpu

DEPTH_ATOL_CPU = 2e-4

EYE = (0.0, 0.0, 1.6)


def _specs():
    from xsimgs_b200 import scenes
    from xsimgs_b200.cameras.ext_camera import look_at_quat
    motion = dict(v=(3.0, 0.5, 0.0), w=(0.01, -0.02, 0.3), trigger_time=0.01, pose_time=0.02)
    ph = scenes.pinhole(480, 272, 300.0, 300.0, EYE, (1.0, 0.2, 1.5), rolling_time=(0.0, 0.03), **motion)
    fe = scenes.CameraSpec("fisheye", 400, 300, look_at_quat(EYE, (0.3, 1.0, 1.6)), np.asarray(EYE, np.float32),
                           intrinsics=np.array([120.0 / 400, 120.0 / 300, 0.5, 0.5], np.float32),
                           distortion=np.array([0.03, -0.02, 0.01, -0.004], np.float32),
                           rolling_time=(0.02, 0.0), **motion)
    di = scenes.CameraSpec("distorted", 480, 272, look_at_quat(EYE, (1.0, -0.4, 1.4)), np.asarray(EYE, np.float32),
                           intrinsics=np.array([300.0 / 480, 300.0 / 272, 0.52, 0.48], np.float32),
                           distortion=np.array([-0.25, 0.07, 3e-4, -2e-4, -0.008, 0.03, 0.002, 0.0005], np.float32),
                           rolling_time=(0.0, 0.03), **motion)
    sp = scenes.CameraSpec("spherical", 512, 256, np.array([1, 0, 0, 0], np.float32), np.asarray(EYE, np.float32),
                           rolling_time=(0.1, 0.0), **motion)
    li = scenes.c4_lidar(beams=64, columns=512)
    li.rolling_time, li.trigger_time, li.pose_time = (0.1, 0.0), 0.0, 0.05
    li.v, li.w = (4.0, 0.0, 0.0), (0.0, 0.0, 0.2)
    return {"pinhole": ph, "fisheye": fe, "distorted": di, "spherical": sp, "lidar": li}


KINDS = ["pinhole", "fisheye", "distorted", "spherical", "lidar"]


@pytest.fixture(scope="module")
def specs(cuda):
    return _specs()


@pytest.fixture(scope="module")
def shell():
    """Gaussians in a shell 3..30 m around the sensor, seen by every camera."""
    g = torch.Generator().manual_seed(21)
    n = 20_000
    d = torch.randn(n, 3, generator=g)
    d = d / d.norm(dim=1, keepdim=True)
    d[:, 2] *= 0.35
    r = 3.0 + 27.0 * torch.rand(n, 1, generator=g)
    means = d * r + torch.tensor(EYE)
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.5 - 2.1)
    quats = torch.randn(n, 4, generator=g)
    quats = quats / quats.norm(dim=1, keepdim=True)
    opac = torch.sigmoid(torch.randn(n, generator=g) * 1.5)
    vel = torch.randn(n, 3, generator=g) * 0.5
    rgb = torch.rand(n, 3, generator=g)
    return dict(means=means, scales=scales, quats=quats, opac=opac, vel=vel, colors=rgb)


@pytest.mark.parametrize("kind", KINDS)
def test_camera_rays_and_pixel_time(specs, cuda, kind):
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    for world, norm in [(True, True), (False, True), (True, False)]:
        ro, rd, valid = cam.ext_cls.camera_rays(cam.pack, width=W, height=H, world_space=world, normalized=norm,
                                                return_valid=True)
        oo, od, ov = O.camera_rays(kind, pack, W, H, world_space=world, normalized=norm, elev=elev)
        agree = to_np(valid).astype(bool) == ov
        assert agree.mean() > 0.999, f"{kind}: valid masks agree on {agree.mean()}"
        both = to_np(valid).astype(bool) & ov
        np.testing.assert_allclose(to_np(ro)[both], oo[both], atol=2e-5, rtol=1e-6)
        np.testing.assert_allclose(to_np(rd)[both], od[both], atol=2e-5, rtol=2e-5)
    for delta in (False, True):
        fn = cam.ext_cls.pixel_time_delta if delta else cam.ext_cls.pixel_time
        t = to_np(fn(cam.pack, width=W, height=H))
        np.testing.assert_allclose(t, O.pixel_time(kind, pack, W, H, delta, elev=elev), atol=1e-7, rtol=1e-6)
    uv = np.random.default_rng(2).uniform(0, 1, size=(1000, 2)).astype(np.float32)
    for delta in (False, True):
        fn = cam.ext_cls.pixel_time_delta_from_uv if delta else cam.ext_cls.pixel_time_from_uv
        t = to_np(fn(cam.pack, torch.from_numpy(uv).to(cuda)))
        want = _pixel_time_from_uv(kind, pack, uv, delta)
        np.testing.assert_allclose(t, want, atol=1e-7, rtol=1e-6)


@pytest.mark.parametrize("normalized_range", [False, True])
def test_undistort_map(specs, cuda, normalized_range):
    spec = specs["distorted"]
    cam, pack, _ = camera_inputs(spec, cuda)
    got = to_np(cam.undistort_map(spec.width, spec.height, normalized_range=normalized_range))
    np.testing.assert_allclose(got, O.undistort_map(pack, spec.width, spec.height, normalized_range), atol=2e-6)
    from xsimgs_b200 import _C
    assert not hasattr(_C.PerspectiveCamera, "undistort_map")  # only the distorted camera has one


def _pixel_time_from_uv(kind, pack, uv, delta):
    import ctypes as C
    pack = np.ascontiguousarray(pack, np.float32)
    out = np.zeros(uv.shape[0], np.float32)
    O.lib().xsgo_pixel_time_from_uv(C.c_int(O.CAM[kind]), pack.ctypes.data_as(C.c_void_p),
                                    uv.ctypes.data_as(C.c_void_p), C.c_int64(uv.shape[0]), C.c_int(int(delta)),
                                    out.ctypes.data_as(C.c_void_p))
    return out


@pytest.mark.parametrize("kind", KINDS)
def test_point_projection_all_modes(specs, shell, cuda, kind):
    from xsimgs_b200 import _C
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    pts, vel = shell["means"], shell["vel"]
    modes = [(_C.ProjectionMode.Central, 0), (_C.ProjectionMode.NegativeDelta, 1),
             (_C.ProjectionMode.PositiveDelta, 2)]
    for nojac in (False, True):
        fn = cam.ext_cls.projection_nojac if nojac else cam.ext_cls.projection
        for mode, mi in modes:
            for v in (None, vel):
                uvdt, mask = fn(cam.pack, pts.to(cuda), None if v is None else v.to(cuda), projection_mode=mode)
                ruv, rmask = O.projection(kind, pack, pts.numpy(), None if v is None else v.numpy(), mode=mi,
                                          nojac=nojac, elev=elev)
                uvdt, mask = to_np(uvdt), to_np(mask).astype(bool)
                agree = mask == rmask
                assert agree.mean() > 0.999, f"{kind} mode {mi} nojac {nojac}: masks agree on {agree.mean()}"
                both = mask & rmask
                du = uvdt[both, 0] - ruv[both, 0]
                if kind in ("spherical", "lidar"):
                    du = (du + 0.5) % 1.0 - 0.5  # azimuth wraps at the seam
                assert np.abs(du).max(initial=0) < 2e-5
                np.testing.assert_allclose(uvdt[both, 1], ruv[both, 1], atol=2e-5)
                np.testing.assert_allclose(uvdt[both, 2], ruv[both, 2], rtol=1e-4, atol=1e-4)
                np.testing.assert_allclose(uvdt[both, 3], ruv[both, 3], atol=1.5e-4)


def _project(cam, spec, shell, cuda, phm=False, with_vel=False):
    W, H = spec.width, spec.height
    fn = cam.ext_cls.projection_utgs_phm if phm else cam.ext_cls.projection_utgs
    g = lambda t: t.to(cuda).contiguous()
    return fn(cam.pack, g(shell["means"]), g(shell["vel"]) if with_vel else None, g(shell["scales"]),
              g(shell["quats"]), g(shell["opac"]), width=W, height=H)


@pytest.mark.parametrize("kind,phm,with_vel", [("pinhole", False, False), ("pinhole", False, True),
                                               ("fisheye", False, True), ("distorted", False, True),
                                               ("spherical", False, True),
                                               ("spherical", True, True), ("lidar", False, True),
                                               ("lidar", True, False)])
def test_ut_projection(specs, shell, cuda, kind, phm, with_vel):
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    flags, radii, m2, dep = map(to_np, _project(cam, spec, shell, cuda, phm, with_vel))
    rf, rr, rm, rd = O.projection_utgs(kind, pack, shell["means"].numpy(),
                                       shell["vel"].numpy() if with_vel else None, shell["scales"].numpy(),
                                       shell["quats"].numpy(), shell["opac"].numpy(), spec.width, spec.height,
                                       phm=phm, elev=elev)
    agree = flags == rf
    assert agree.mean() > 0.999, f"flags agree on {agree.mean()}"
    assert (flags > 0).sum() > 500, "too few visible Gaussians for a meaningful check"
    both = (flags > 0) & (rf > 0) & agree
    du = m2[both, 0] - rm[both, 0]
    if kind in ("spherical", "lidar"):
        du = (du + spec.width / 2) % spec.width - spec.width / 2
    assert np.abs(du).max(initial=0) < 5e-2
    np.testing.assert_allclose(m2[both, 1], rm[both, 1], rtol=1e-5, atol=5e-2)
    # radii come from the spread of seven sigma-point projections, each a
    # Newton solve that may stop one iteration apart on CPU and GPU
    np.testing.assert_allclose(radii[both], rr[both], rtol=1e-3, atol=5e-2)
    np.testing.assert_allclose(dep[both], rd[both], rtol=1e-5, atol=1e-5)
    assert (radii[flags == 0] == 0).all()


def _tiles(cam, kind, spec, shell, cuda, proj, with_vel, tsx=16, tsy=16):
    from xsimgs_b200 import _C
    flags, radii, m2, dep = proj
    W, H = spec.width, spec.height
    g = lambda t: t.to(cuda).contiguous()
    if kind in ("pinhole", "fisheye", "distorted"):
        return _C.isect_regular_tiles(m2, radii, dep, W, H, tsx, tsy), None
    kw = dict(camera_pack=cam.pack, points=g(shell["means"]), points_velocity=g(shell["vel"]) if with_vel else None,
              scale=g(shell["scales"]), quat=g(shell["quats"]), opacity=g(shell["opac"]), flag=flags,
              means2d=m2, radii=radii, depths=dep, tile_size_x=tsx, img_width=W, img_height=H)
    if kind == "lidar":
        eb = cam.beam_v[::tsy].contiguous()
        return _C.isect_lidar_tiles(elev_boundaries=eb, **kw), to_np(eb)
    return _C.isect_spherical_tiles(tile_size_y=tsy, **kw), None


def _oracle_tiles(kind, pack, elev, spec, shell, proj, eb, with_vel, tsx=16, tsy=16):
    flags, radii, m2, dep = map(to_np, proj)
    if kind in ("pinhole", "fisheye", "distorted"):
        return O.isect_regular(m2, radii, dep, spec.width, spec.height, tsx, tsy)
    return O.isect_spherical(kind == "lidar", pack, elev, shell["means"].numpy(),
                             shell["vel"].numpy() if with_vel else None, shell["scales"].numpy(),
                             shell["quats"].numpy(), shell["opac"].numpy(), flags, m2, radii, dep, eb, tsx, tsy,
                             spec.width, spec.height)


def _assert_tiles_match(got, ref, flags):
    """Bit-exact for every Gaussian the tiler does not re-project; a flag-2
    Gaussian's second rectangle comes from a UT projection run inside the
    tiler, whose float results may differ by an ulp between CPU and GPU."""
    tpg, ids, flat = map(to_np, got)
    rt, ri, rfl = ref
    fixed = flags != 2
    np.testing.assert_array_equal(tpg[fixed], rt[fixed])
    if (~fixed).any():
        kg, kr = fixed[flat], fixed[rfl]
        np.testing.assert_array_equal(ids[kg], ri[kr])
        np.testing.assert_array_equal(flat[kg], rfl[kr])
        assert abs(len(ids) - len(ri)) <= max(4, len(ri) // 1000)
    else:
        np.testing.assert_array_equal(ids, ri)
        np.testing.assert_array_equal(flat, rfl)


@pytest.mark.parametrize("kind,phm", [("pinhole", False), ("fisheye", False), ("distorted", False),
                                      ("spherical", False),
                                      ("spherical", True), ("lidar", False), ("lidar", True)])
def test_tiling_matches_oracle(specs, shell, cuda, kind, phm):
    """With PHM the range-image projection marks Gaussians that straddle the
    start/end seam of the spin (flag 2); the tilers then emit two rectangles."""
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    proj = _project(cam, spec, shell, cuda, phm=phm, with_vel=True)
    if phm:
        assert int((proj[0] == 2).sum()) > 0, "no seam-straddling Gaussians: the flag-2 path is not exercised"
    (got, eb) = _tiles(cam, kind, spec, shell, cuda, proj, True)
    ref = _oracle_tiles(kind, pack, elev, spec, shell, proj, eb, True)
    _assert_tiles_match(got, ref, to_np(proj[0]))
    assert len(ref[1]) > 1000


def _offsets(kind, spec, ids, eb, tsx=16, tsy=16):
    from xsimgs_b200 import _C
    tw = (spec.width + tsx - 1) // tsx
    th = len(eb) if kind == "lidar" else (spec.height + tsy - 1) // tsy
    return _C.isect_offset_encode(ids, tw, th)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("dynamic", [False, True])
def test_composite_fwd_bwd_per_camera(specs, shell, cuda, kind, dynamic):
    """Compositing over each camera's own rays and tile layout; the dynamic
    variant moves each Gaussian by velocity x the ray's time offset."""
    from xsimgs_b200 import _C, scenes
    spec = specs[kind]
    cam, pack, elev = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    proj = _project(cam, spec, shell, cuda, phm=(kind == "lidar"), with_vel=dynamic)
    (tpg, ids, flat), eb = _tiles(cam, kind, spec, shell, cuda, proj, dynamic)
    off = _offsets(kind, spec, ids, eb if eb is not None else [])
    ro, rd = cam.ext_cls.camera_rays(cam.pack, width=W, height=H)[:2]
    g = lambda t: t.to(cuda).contiguous()
    cols = shell["colors"]
    n = cols.shape[0]
    args = dict(means=g(shell["means"]), quats=g(shell["quats"]), scales=g(shell["scales"]),
                colors=g(cols).unsqueeze(0), opacities=g(shell["opac"]).view(1, -1), image_width=W, image_height=H,
                tile_size_width=16, tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=off,
                flatten_ids=flat)
    rt = None
    if dynamic:
        rt = cam.ext_cls.pixel_time_delta(cam.pack, width=W, height=H).unsqueeze(-1).contiguous()
        rgb, depth, alpha, last = _C.rasterize_eval3d_dynamic_fwd(velocity=g(shell["vel"]), ray_time_delta=rt,
                                                                  **args)
    else:
        rgb, depth, alpha, last = _C.rasterize_eval3d_fwd(**args)
    np_in = (shell["means"].numpy(), shell["quats"].numpy(), shell["scales"].numpy(), cols.numpy(),
             shell["opac"].numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat))
    dyn_kw = dict(velocity=shell["vel"].numpy(), ray_t=to_np(rt)) if dynamic else {}
    rrgb, rdep, ralpha, rlast, near = O.rasterize_fwd(*np_in, **dyn_kw)
    assert float(to_np(alpha).mean()) > 0.05, "too little coverage for a meaningful check"
    assert_images_close(rgb, rrgb, near, what="rgb")
    # absolute, not relative: the CPU restatement rounds every product on its
    # own (no FMA), which puts it up to ~5 ulps of a 30 m depth away from the
    # reference's GPU kernels; against those kernels this package's depth is
    # bit-exact (test_gpu_ref_parity.py)
    assert_images_close(depth, rdep, near, atol=DEPTH_ATOL_CPU, what="depth")
    assert_images_close(alpha, ralpha, near, what="alpha")
    np.testing.assert_array_equal(to_np(last)[~near], rlast[~near])

    vr, vd, va = zero_at(near, *scenes.upstream_grads(H, W, 3, seed=9))
    bwd_args = [g(shell["means"]), g(shell["scales"]), g(shell["quats"]), g(shell["opac"]), g(cols), ro, rd]
    tail = [off, flat, alpha, last, g(vr), g(vd), g(va)]
    if dynamic:
        out = _C.rasterize_eval3d_dynamic_bwd(bwd_args[0], g(shell["vel"]), *bwd_args[1:], rt, 16, 16, *tail)
        names = ["v_means", "v_velocity", "v_quats", "v_scales", "v_opacities", "v_colors", "v_ray_o", "v_ray_d",
                 "v_ray_t"]
    else:
        out = _C.rasterize_eval3d_bwd(*bwd_args, 16, 16, *tail)
        names = ["v_means", "v_quats", "v_scales", "v_opacities", "v_colors", "v_ray_o", "v_ray_d"]
    ref = O.rasterize_bwd(*np_in, to_np(alpha), to_np(last), vr.numpy(), vd.numpy(), va.numpy(), **dyn_kw)
    for got, key in zip(out, names):
        if key == "v_ray_t":
            got = to_np(got).reshape(H, W)
        assert_grads_close(got, ref[key], f"{kind} {key}")
    # the variant without ray gradients gives the same Gaussian gradients
    if dynamic:
        fast = _C.rasterize_eval3d_dynamic_bwd(bwd_args[0], g(shell["vel"]), *bwd_args[1:], rt, 16, 16, *tail,
                                               ray_grads=False)
        assert fast[6] is None and fast[7] is None and fast[8] is None
    else:
        fast = _C.rasterize_eval3d_bwd(*bwd_args, 16, 16, *tail, ray_grads=False)
        assert fast[5] is None and fast[6] is None
    for got, key in zip(fast, names):
        if not key.startswith("v_ray"):
            assert_grads_close(got, ref[key], f"{kind} {key} (no ray grads)")
    assert n == to_np(out[0]).shape[0]
    # the forward's workspace handed to the backward: records, tile order and
    # contributor masks reused (the backward visits only composited entries)
    ws = torch.empty(_C.rasterize_workspace_size(n, 3, n_isects=flat.numel(), n_tiles=off.numel(), tile_pixels=256),
                     dtype=torch.uint8, device=cuda)
    if dynamic:
        _C.rasterize_eval3d_dynamic_fwd(velocity=g(shell["vel"]), ray_time_delta=rt, workspace=ws, **args)
    else:
        _C.rasterize_eval3d_fwd(workspace=ws, **args)
    for rg in (True, False):
        if dynamic:
            reused = _C.rasterize_eval3d_dynamic_bwd(bwd_args[0], g(shell["vel"]), *bwd_args[1:], rt, 16, 16, *tail,
                                                     ray_grads=rg, forward_workspace=ws)
        else:
            reused = _C.rasterize_eval3d_bwd(*bwd_args, 16, 16, *tail, ray_grads=rg, forward_workspace=ws)
        for got, key in zip(reused, names):
            if rg or not key.startswith("v_ray"):
                if key == "v_ray_t":
                    got = to_np(got).reshape(H, W)
                assert_grads_close(got, ref[key], f"{kind} {key} (forward workspace, ray grads {rg})")


def test_mask_radii_match_oracle(cuda):
    from xsimgs_b200 import _C
    from xsimgs_b200.utils import pack_bits
    rng = np.random.default_rng(4)
    n = 10_001
    radii = rng.uniform(0, 5, size=(n, 2)).astype(np.float32)
    mask = rng.random(n) < 0.6
    r1 = torch.from_numpy(radii.copy()).to(cuda)
    _C.mask_radii(torch.from_numpy(mask).to(cuda), r1)
    np.testing.assert_array_equal(to_np(r1), O.mask_radii(radii, mask=mask))
    r2 = torch.from_numpy(radii.copy()).to(cuda)
    pm = pack_bits(torch.from_numpy(mask)).to(cuda)
    _C.mask_radii_packed(pm, r2)
    np.testing.assert_array_equal(to_np(r2), O.mask_radii(radii, packed=to_np(pm.view(torch.int32)).view(np.uint32)))
    assert math.isclose(float((to_np(r2) == 0).all(axis=1).mean()), float((~mask).mean()), abs_tol=0.02)
