"""GPU kernels vs the CPU oracle on identical seeded inputs (C1 and small
variants), stage by stage, through the package's `_C` ops (which call the
C ABI of libxsimgs_b200.so).  Tolerances: see tests/helpers.py."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import (assert_grads_close, assert_images_close, camera_inputs, sh_colors, to_np,
                           zero_at)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c1(cuda):
    from xsimgs_b200 import scenes
    sc = scenes.c1_scene()
    spec = scenes.c1_camera()
    return sc, spec


def _project(sc, cam, W, H, device):
    from xsimgs_b200 import _C
    return cam.ext_cls.projection_utgs(cam.pack, sc.means.to(device), None, sc.scales.to(device),
                                       sc.quats.to(device), sc.opacities.to(device), width=W, height=H)


def test_projection_utgs_matches_oracle(c1, cuda):
    sc, spec = c1
    cam, pack, _ = camera_inputs(spec, cuda)
    flags, radii, m2, dep = _project(sc, cam, spec.width, spec.height, cuda)
    rf, rr, rm, rd = O.projection_utgs("pinhole", pack, sc.means.numpy(), None, sc.scales.numpy(),
                                       sc.quats.numpy(), sc.opacities.numpy(), spec.width, spec.height)
    flags, radii, m2, dep = map(to_np, (flags, radii, m2, dep))
    agree = flags == rf
    assert agree.mean() > 0.999, f"visibility flags agree on {agree.mean()}"
    both = (flags > 0) & (rf > 0)
    np.testing.assert_allclose(m2[both], rm[both], rtol=1e-5, atol=5e-2)
    np.testing.assert_allclose(radii[both], rr[both], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(dep[both], rd[both], rtol=1e-6, atol=1e-5)
    # invisible Gaussians are fully zeroed, like the reference's zero-initialised outputs
    assert (radii[flags == 0] == 0).all() and (m2[flags == 0] == 0).all() and (dep[flags == 0] == 0).all()


@pytest.mark.parametrize("sort", [True, False])
def test_isect_regular_bit_exact(c1, cuda, sort):
    from xsimgs_b200 import _C
    sc, spec = c1
    cam, pack, _ = camera_inputs(spec, cuda)
    flags, radii, m2, dep = _project(sc, cam, spec.width, spec.height, cuda)
    tpg, ids, flat = _C.isect_regular_tiles(m2, radii, dep, spec.width, spec.height, 16, 16, sort=sort)
    rt, ri, rfl = O.isect_regular(to_np(m2), to_np(radii), to_np(dep), spec.width, spec.height, 16, 16, sort=sort)
    np.testing.assert_array_equal(to_np(tpg), rt)
    np.testing.assert_array_equal(to_np(ids), ri)
    np.testing.assert_array_equal(to_np(flat), rfl)
    if sort:
        off = _C.isect_offset_encode(ids, 16, 16)
        np.testing.assert_array_equal(to_np(off), O.isect_offset_encode(ri, 16, 16))


@pytest.mark.parametrize("tile", [(16, 16), (8, 8), (32, 8)])
def test_isect_tile_sizes_and_odd_image(cuda, tile):
    """Ragged image (not a multiple of the tile) and other tile shapes."""
    from xsimgs_b200 import _C
    rng = np.random.default_rng(3)
    n, W, H = 5000, 203, 117
    m2 = rng.uniform(-20, W + 20, size=(n, 2)).astype(np.float32)
    m2[:, 1] = rng.uniform(-20, H + 20, size=n)
    radii = rng.exponential(6.0, size=(n, 2)).astype(np.float32)
    radii[rng.random(n) < 0.1] = 0.0
    dep = rng.uniform(0.5, 50, size=n).astype(np.float32)
    dep[:50] = dep[50:100]  # equal depths: ties broken by Gaussian index
    tsx, tsy = tile
    t = lambda a: torch.from_numpy(a).to(cuda)
    tpg, ids, flat = _C.isect_regular_tiles(t(m2), t(radii), t(dep), W, H, tsx, tsy)
    rt, ri, rfl = O.isect_regular(m2, radii, dep, W, H, tsx, tsy)
    np.testing.assert_array_equal(to_np(tpg), rt)
    np.testing.assert_array_equal(to_np(ids), ri)
    np.testing.assert_array_equal(to_np(flat), rfl)
    tw, th = (W + tsx - 1) // tsx, (H + tsy - 1) // tsy
    np.testing.assert_array_equal(to_np(_C.isect_offset_encode(ids, tw, th)), O.isect_offset_encode(ri, tw, th))


@pytest.mark.parametrize("n", [1500, 9000, 40000])
def test_isect_crowded_tiles_and_negative_depths(cuda, n):
    """Tiles holding more intersections than each shared-memory bucket sort
    takes (2048 and 16384 per tile, then the global-memory sort), equal
    depths (ties kept in emission order) and negative depths (the reference's
    sign-extended keys collect them in the all-ones bucket)."""
    from xsimgs_b200 import _C
    rng = np.random.default_rng(n)
    W, H = 80, 48
    m2 = rng.uniform(0, W, size=(n, 2)).astype(np.float32)
    m2[:, 1] = rng.uniform(0, H, size=n)
    radii = rng.uniform(20, 90, size=(n, 2)).astype(np.float32)
    dep = rng.uniform(0.5, 50, size=n).astype(np.float32)
    dep[: n // 10] = dep[n // 10: 2 * (n // 10)]
    dep[rng.random(n) < 0.03] *= -1.0
    t = lambda a: torch.from_numpy(a).to(cuda)
    tpg, ids, flat = _C.isect_regular_tiles(t(m2), t(radii), t(dep), W, H, 16, 16)
    rt, ri, rfl = O.isect_regular(m2, radii, dep, W, H, 16, 16)
    counts = np.bincount((ri[ri >= 0] >> 32).astype(np.int64))
    assert counts.max() > {1500: 1000, 9000: 2048, 40000: 16384}[n]
    np.testing.assert_array_equal(to_np(tpg), rt)
    np.testing.assert_array_equal(to_np(ids), ri)
    np.testing.assert_array_equal(to_np(flat), rfl)


def test_isect_empty(cuda):
    from xsimgs_b200 import _C
    z = torch.zeros(10, 2, device=cuda)
    tpg, ids, flat = _C.isect_regular_tiles(z, z, torch.ones(10, device=cuda), 64, 64, 16, 16)
    assert ids.numel() == 0 and flat.numel() == 0 and int(tpg.sum()) == 0
    off = _C.isect_offset_encode(ids, 4, 4)
    assert (off == 0).all()


def test_camera_rays_match_oracle(c1, cuda):
    sc, spec = c1
    cam, pack, _ = camera_inputs(spec, cuda)
    ro, rd = cam.camera_rays(spec.width, spec.height)
    oo, od, _ = O.camera_rays("pinhole", pack, spec.width, spec.height)
    np.testing.assert_allclose(to_np(ro), oo, atol=1e-6)
    np.testing.assert_allclose(to_np(rd), od, atol=2e-6)


def _raster_inputs(sc, spec, cuda):
    from xsimgs_b200 import _C
    cam, pack, _ = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    flags, radii, m2, dep = _project(sc, cam, W, H, cuda)
    tpg, ids, flat = _C.isect_regular_tiles(m2, radii, dep, W, H, 16, 16)
    off = _C.isect_offset_encode(ids, (W + 15) // 16, (H + 15) // 16)
    ro, rd = cam.camera_rays(W, H)
    return cam, off, flat, ro, rd


def test_rasterize_fwd_bwd_match_oracle(c1, cuda):
    from xsimgs_b200 import _C, scenes
    sc, spec = c1
    W, H = spec.width, spec.height
    cam, off, flat, ro, rd = _raster_inputs(sc, spec, cuda)
    colors = sh_colors(sc.sh, 0)
    g = lambda t: t.to(cuda).contiguous()
    rgb, depth, alpha, last = _C.rasterize_eval3d_fwd(
        means=g(sc.means), quats=g(sc.quats), scales=g(sc.scales), colors=g(colors).unsqueeze(0),
        opacities=g(sc.opacities).view(1, -1), image_width=W, image_height=H, tile_size_width=16,
        tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=off, flatten_ids=flat)
    r = O.rasterize_fwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(), colors.numpy(),
                        sc.opacities.numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat))
    rrgb, rdep, ralpha, rlast, near = r
    assert_images_close(rgb, rrgb, near, what="rgb")
    assert_images_close(depth, rdep, near, atol=1e-4, what="depth")
    assert_images_close(alpha, ralpha, near, what="alpha")
    ok = ~near
    np.testing.assert_array_equal(to_np(last)[ok], rlast[ok])

    vr, vd, va = zero_at(near, *scenes.upstream_grads(H, W, 3))
    grads = _C.rasterize_eval3d_bwd(g(sc.means), g(sc.scales), g(sc.quats), g(sc.opacities), g(colors), ro, rd,
                                    16, 16, off, flat, alpha, last, g(vr), g(vd), g(va))
    # the oracle replays from the GPU's forward outputs so both see the same
    # alpha / last-contributor images
    rg = O.rasterize_bwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(), colors.numpy(),
                         sc.opacities.numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat),
                         to_np(alpha), to_np(last), vr.numpy(), vd.numpy(), va.numpy())
    v_means, v_quats, v_scales, v_opac, v_colors, v_ro, v_rd = grads
    assert_grads_close(v_means, rg["v_means"], "v_means")
    assert_grads_close(v_quats, rg["v_quats"], "v_quats")
    assert_grads_close(v_scales, rg["v_scales"], "v_scales")
    assert_grads_close(v_opac, rg["v_opacities"], "v_opacities")
    assert_grads_close(v_colors, rg["v_colors"], "v_colors")
    assert_grads_close(v_ro, rg["v_ray_o"], "v_ray_o")
    assert_grads_close(v_rd, rg["v_ray_d"], "v_ray_d")
    # without ray gradients (the variant that factors the shared ray origin
    # out of the per-pixel sums): same Gaussian gradients, no ray outputs
    fast = _C.rasterize_eval3d_bwd(g(sc.means), g(sc.scales), g(sc.quats), g(sc.opacities), g(colors), ro, rd,
                                   16, 16, off, flat, alpha, last, g(vr), g(vd), g(va), ray_grads=False)
    assert fast[5] is None and fast[6] is None
    for got, key in zip(fast[:5], ["v_means", "v_quats", "v_scales", "v_opacities", "v_colors"]):
        assert_grads_close(got, rg[key], key + " (no ray grads)")


def test_rasterize_mixed_origins_forward_workspace(c1, cuda):
    """An image where some 16 x 4 pixel blocks share pixel 0's ray origin and
    others do not: with the forward's workspace the backward gives the first
    kind to the two-pixels-a-lane kernel and the second to the per-pixel one;
    together they must match the oracle on every Gaussian gradient."""
    from xsimgs_b200 import _C, scenes
    sc, spec = c1
    W, H = spec.width, spec.height
    cam, off, flat, ro, rd = _raster_inputs(sc, spec, cuda)
    shape = ro.shape
    ro = ro.clone().view(H, W, 3)
    ro[20:36, :, 0] += 1e-3          # whole rows of blocks with another origin
    ro[::7, ::13, 1] -= 2e-3         # scattered pixels spoil other blocks
    ro = ro.reshape(shape).contiguous()
    colors = sh_colors(sc.sh, 0)
    g = lambda t: t.to(cuda).contiguous()
    args = dict(means=g(sc.means), quats=g(sc.quats), scales=g(sc.scales), colors=g(colors).unsqueeze(0),
                opacities=g(sc.opacities).view(1, -1), image_width=W, image_height=H, tile_size_width=16,
                tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=off, flatten_ids=flat)
    n = sc.means.shape[0]
    ws = torch.empty(_C.rasterize_workspace_size(n, 3, n_isects=flat.numel(), n_tiles=off.numel(), tile_pixels=256),
                     dtype=torch.uint8, device=cuda)
    rgb, depth, alpha, last = _C.rasterize_eval3d_fwd(workspace=ws, **args)
    r = O.rasterize_fwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(), colors.numpy(),
                        sc.opacities.numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat))
    near = r[4]
    vr, vd, va = zero_at(near, *scenes.upstream_grads(H, W, 3))
    rg = O.rasterize_bwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(), colors.numpy(),
                         sc.opacities.numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat),
                         to_np(alpha), to_np(last), vr.numpy(), vd.numpy(), va.numpy())
    for ray_grads in (False, True):
        out = _C.rasterize_eval3d_bwd(g(sc.means), g(sc.scales), g(sc.quats), g(sc.opacities), g(colors), ro, rd,
                                      16, 16, off, flat, alpha, last, g(vr), g(vd), g(va), ray_grads=ray_grads,
                                      forward_workspace=ws)
        for got, key in zip(out[:5], ["v_means", "v_quats", "v_scales", "v_opacities", "v_colors"]):
            assert_grads_close(got, rg[key], f"{key} (mixed origins, ray grads {ray_grads})")


def test_rasterize_backward_kernel_choice(c1, cuda):
    """The forward counts how far the contributor masks of the two 8 x 4
    blocks of each pair overlap (pair counters 6 and 7); the backward runs two
    pixels a lane when the union is at most 72 % of the sum, else per pixel.
    The C1 scene (large Gaussians) and the same scene shrunk 20-fold land on
    the two sides, and both backward kernels match the oracle."""
    from xsimgs_b200 import _C, capi, scenes
    sc, spec = c1
    W, H = spec.width, spec.height
    ratios = []
    for shrink in (1.0, 0.05):
        sc_s = type(sc)(**{**sc.__dict__, "scales": sc.scales * shrink}) if shrink != 1.0 else sc
        cam, off, flat, ro, rd = _raster_inputs(sc_s, spec, cuda)
        colors = sh_colors(sc_s.sh, 0)
        g = lambda t: t.to(cuda).contiguous()
        n = sc_s.means.shape[0]
        ws = torch.empty(_C.rasterize_workspace_size(n, 3, n_isects=flat.numel(), n_tiles=off.numel(),
                                                     tile_pixels=256), dtype=torch.uint8, device=cuda)
        cnt = torch.zeros(8, dtype=torch.int64, device=cuda)
        capi.set_pair_counters(cnt.data_ptr())
        try:
            rgb, depth, alpha, last = _C.rasterize_eval3d_fwd(
                means=g(sc_s.means), quats=g(sc_s.quats), scales=g(sc_s.scales), colors=g(colors).unsqueeze(0),
                opacities=g(sc_s.opacities).view(1, -1), image_width=W, image_height=H, tile_size_width=16,
                tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=off, flatten_ids=flat, workspace=ws)
            torch.cuda.synchronize()
        finally:
            capi.set_pair_counters(None)
        c = cnt.tolist()
        assert c[7] > 0 and c[7] >= c[6] >= c[7] // 2
        ratios.append(c[6] / c[7])
        args = (sc_s.means.numpy(), sc_s.quats.numpy(), sc_s.scales.numpy(), colors.numpy(),
                sc_s.opacities.numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat))
        near = O.rasterize_fwd(*args)[4]
        vr, vd, va = zero_at(near, *scenes.upstream_grads(H, W, 3))
        rg = O.rasterize_bwd(*args, to_np(alpha), to_np(last), vr.numpy(), vd.numpy(), va.numpy())
        out = _C.rasterize_eval3d_bwd(g(sc_s.means), g(sc_s.scales), g(sc_s.quats), g(sc_s.opacities), g(colors),
                                      ro, rd, 16, 16, off, flat, alpha, last, g(vr), g(vd), g(va), ray_grads=False,
                                      forward_workspace=ws)
        for got, key in zip(out[:5], ["v_means", "v_quats", "v_scales", "v_opacities", "v_colors"]):
            assert_grads_close(got, rg[key], f"{key} (scales x {shrink}, mask overlap {ratios[-1]:.3f})")
    assert ratios[0] <= 0.72 < ratios[1], ratios


@pytest.mark.parametrize("degree", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("layout_3kn", [False, True])
def test_sh_fwd_bwd_match_oracle(cuda, degree, layout_3kn):
    from xsimgs_b200 import _C
    rng = np.random.default_rng(degree)
    n = 3000
    k = (degree + 1) ** 2 + 1  # one spare band: must get zero gradient
    pos = rng.normal(size=(n, 3)).astype(np.float32) * 10
    origin = np.array([0.5, -1.0, 2.0], np.float32)
    coeffs = rng.normal(size=(n, k, 3)).astype(np.float32)
    if layout_3kn:
        coeffs = np.ascontiguousarray(coeffs.transpose(2, 1, 0))
    d_out = rng.normal(size=(n, 3)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    out = _C.spherical_harmonics_fused_fwd(degree, t(origin), t(pos), t(coeffs), None, layout_3kn)
    ref = O.sh_fwd(degree, origin, pos, coeffs, layout_3kn=layout_3kn)
    np.testing.assert_allclose(to_np(out), ref, atol=2e-5, rtol=1e-5)
    d_coeffs, d_dc, d_pos, d_origin = _C.spherical_harmonics_fused_bwd(
        degree, t(origin), t(pos), t(coeffs), None, layout_3kn, t(d_out))
    rc, _, rp, ro = O.sh_bwd(degree, origin, pos, coeffs, d_out, layout_3kn=layout_3kn)
    np.testing.assert_allclose(to_np(d_coeffs), rc, atol=1e-5, rtol=1e-5)
    assert_grads_close(d_pos, rp, "d_positions")
    np.testing.assert_allclose(to_np(d_origin), ro, rtol=1e-3, atol=1e-3 * np.abs(rp).sum())


def test_sh_separate_dc_and_mask(cuda):
    from xsimgs_b200 import _C
    from xsimgs_b200.utils import pack_bits
    rng = np.random.default_rng(7)
    n, degree = 1000, 3
    pos = rng.normal(size=(n, 3)).astype(np.float32)
    origin = np.zeros(3, np.float32)
    coeffs = rng.normal(size=(n, 15, 3)).astype(np.float32)
    dc = rng.normal(size=(n, 1, 3)).astype(np.float32)
    mask = rng.random(n) < 0.7
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    pm = pack_bits(torch.from_numpy(mask)).to(cuda)
    out = _C.spherical_harmonics_fused_fwd(degree, t(origin), t(pos), t(coeffs), pm, False, t(dc))
    ref = O.sh_fwd(degree, origin, pos, coeffs, dc=dc, mask=to_np(pm.view(torch.int32)).view(np.uint32))
    np.testing.assert_allclose(to_np(out), ref, atol=2e-5)
    assert (to_np(out)[~mask] == 0).all()


@pytest.mark.parametrize("spread", [0.5, 1.5])
def test_raster_anisotropic_and_near_camera(cuda, spread):
    """Needles, discs and Gaussians close to the camera stress the exact
    per-warp culling of the compositing kernels: results must still match
    the oracle, which evaluates every pair of every tile list."""
    from xsimgs_b200 import _C, scenes
    sc = scenes.c1_scene(n=6000, seed=11)
    g = torch.Generator().manual_seed(5)
    sc.scales = torch.exp(torch.randn(sc.n, 3, generator=g) * spread - 2.0)
    near = torch.rand(sc.n, generator=g) < 0.05
    sc.means[near, 2] = 0.6 + torch.rand(int(near.sum()), generator=g) * 0.8
    sc.means[near, :2] *= 0.1
    spec = scenes.c1_camera()
    W, H = spec.width, spec.height
    cam, off, flat, ro, rd = _raster_inputs(sc, spec, cuda)
    colors = sh_colors(sc.sh, 0)
    gg = lambda t: t.to(cuda).contiguous()
    rgb, depth, alpha, last = _C.rasterize_eval3d_fwd(
        means=gg(sc.means), quats=gg(sc.quats), scales=gg(sc.scales), colors=gg(colors).unsqueeze(0),
        opacities=gg(sc.opacities).view(1, -1), image_width=W, image_height=H, tile_size_width=16,
        tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=off, flatten_ids=flat)
    rrgb, rdep, ralpha, rlast, nearpx = O.rasterize_fwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(),
                                                       colors.numpy(), sc.opacities.numpy(), W, H, 16, 16, to_np(ro),
                                                       to_np(rd), to_np(off), to_np(flat))
    assert_images_close(rgb, rrgb, nearpx, what="rgb")
    assert_images_close(alpha, ralpha, nearpx, what="alpha")
    np.testing.assert_array_equal(to_np(last)[~nearpx], rlast[~nearpx])
    vr, vd, va = zero_at(nearpx, *scenes.upstream_grads(H, W, 3, seed=4))
    grads = _C.rasterize_eval3d_bwd(gg(sc.means), gg(sc.scales), gg(sc.quats), gg(sc.opacities), gg(colors), ro, rd,
                                    16, 16, off, flat, alpha, last, gg(vr), gg(vd), gg(va))
    rg = O.rasterize_bwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(), colors.numpy(),
                         sc.opacities.numpy(), W, H, 16, 16, to_np(ro), to_np(rd), to_np(off), to_np(flat),
                         to_np(alpha), to_np(last), vr.numpy(), vd.numpy(), va.numpy())
    for got, key in zip(grads, ["v_means", "v_quats", "v_scales", "v_opacities", "v_colors", "v_ray_o", "v_ray_d"]):
        assert_grads_close(got, rg[key], key)
