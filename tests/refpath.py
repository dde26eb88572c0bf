"""The reference's own render path on the GPU, for the parity tests.

`oracle/_ref` holds the reference's CUDA sources compiled for sm_100a
(oracle/build_ref.py).  This module drives them exactly as the reference's
Python layer does (src/xsimgs/rendering/render.py:10-187,
src/xsimgs/cameras/ext/*.py) on the camera objects and scenes of this
package, and compares every stage with this package's kernels on identical
inputs.  Each `compare_*` function returns a dict of measured differences;
the tests assert on them and print them.

Test infrastructure only: nothing in the shipped package imports it.
"""
from __future__ import annotations

import functools

import numpy as np
import torch

REF_CLASS = {"pinhole": "PerspectiveCamera", "fisheye": "OpenCVFisheyeCamera",
             "distorted": "DistortedPerspectiveCamera", "spherical": "SphericalCamera", "lidar": "LidarCamera"}
TILE = 16


@functools.lru_cache(maxsize=1)
def ref_module():
    from oracle import build_ref
    return build_ref.load()


def available() -> bool:
    try:
        ref_module()
        return True
    except ImportError:
        return False


class RefCamera:
    """The reference's static camera ops (include/cameras/bind.h:23-129) on a
    pack the reference builds itself from the camera's tensors."""

    def __init__(self, cam, kind: str):
        self.R = ref_module()
        self.cam = cam
        self.kind = kind
        self.cls = getattr(self.R, REF_CLASS[kind])
        self.pack = self.cls.pack(cam._pack_data)

    def rays(self, W, H):
        return self.cls.camera_rays(self.pack, width=W, height=H, world_space=True, normalized=True,
                                    return_origins=True)

    def project(self, means, scales, quats, opac, W, H, phm=False, velocity=None):
        fn = self.cls.projection_utgs_phm if phm else self.cls.projection_utgs
        return fn(self.pack, means, velocity, scales, quats, opac, width=W, height=H)

    def tiles(self, means, scales, quats, opac, W, H, proj, velocity=None):
        """isect_gs_tiles of the reference's camera class (ext/*.py)."""
        flags, radii, m2, dep = proj
        R = self.R
        if self.kind == "lidar":
            eb = self.cam.beam_v[::TILE].contiguous()
            return R.isect_lidar_tiles(camera_pack=self.pack, points=means, points_velocity=velocity, scale=scales,
                                       quat=quats, opacity=opac, flag=flags, means2d=m2, radii=radii, depths=dep,
                                       elev_boundaries=eb, tile_size_x=TILE, img_width=W, img_height=H)
        if self.kind == "spherical":
            return R.isect_spherical_tiles(camera_pack=self.pack, points=means, points_velocity=velocity,
                                           scale=scales, quat=quats, opacity=opac, flag=flags, means2d=m2,
                                           radii=radii, depths=dep, tile_size_x=TILE, tile_size_y=TILE,
                                           img_width=W, img_height=H)
        return R.isect_regular_tiles(m2, radii, dep, W, H, TILE, TILE)

    def tiling(self, means, scales, quats, opac, W, H, phm=False, velocity=None):
        """render.py:10-81 with the reference's ops: projection, tiles,
        offsets."""
        proj = self.project(means, scales, quats, opac, W, H, phm=phm, velocity=velocity)
        tpg, ids, flat = self.tiles(means, scales, quats, opac, W, H, proj, velocity=velocity)
        off = self.R.isect_offset_encode(ids, (W + TILE - 1) // TILE, (H + TILE - 1) // TILE)
        return dict(proj=proj, tiles_per_gauss=tpg, isect_ids=ids, flatten_ids=flat, offsets=off)


def mine_tiling(cam, means, scales, quats, opac, W, H, phm=False, velocity=None):
    """The same stages through this package's camera object and `_C` ops."""
    from xsimgs_b200 import _C
    with cam._freeze_ctx():
        proj = cam.ut_gs_projection(points=means, scale=scales, rotation=quats, width=W, height=H,
                                    points_velocity=velocity, opacity=opac, use_phm=phm)
        flags, radii, m2, dep = proj
        tpg, ids, flat = cam.isect_gs_tiles(points=means, scale=scales, rotation=quats, width=W, height=H,
                                            flags=flags, radii=radii, means2d=m2, depths=dep,
                                            points_velocity=velocity, opacity=opac)
        off = _C.isect_offset_encode(ids, tile_width=(W + TILE - 1) // TILE, tile_height=(H + TILE - 1) // TILE)
    return dict(proj=proj, tiles_per_gauss=tpg, isect_ids=ids, flatten_ids=flat, offsets=off)


def _np(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def count_diff(a, b) -> int:
    a, b = _np(a), _np(b)
    if a.shape != b.shape:
        return -1
    return int((a != b).sum())


def compare_projection(mine, ref) -> dict:
    """UT outputs (flags, radii, means2d, depths) of two projections."""
    mf, mr, mm, md = (_np(t) for t in mine)
    rf, rr, rm, rd = (_np(t) for t in ref)
    both = (mf > 0) & (rf > 0)
    out = {"n": int(mf.size), "visible_mine": int((mf > 0).sum()), "visible_ref": int((rf > 0).sum()),
           "flags_diff": int((mf != rf).sum()), "radii_bitdiff": int((mr != rr).any(-1).sum()),
           "means2d_bitdiff": int((mm != rm).any(-1).sum()), "depth_bitdiff": int((md != rd).sum())}
    if both.any():
        out["means2d_maxabs_px"] = float(np.abs(mm[both] - rm[both]).max())
        out["radii_maxabs_px"] = float(np.abs(mr[both] - rr[both]).max())
        out["depth_maxrel"] = float((np.abs(md[both] - rd[both]) / np.maximum(np.abs(rd[both]), 1e-30)).max())
    return out


def compare_tiling(mine: dict, ref: dict) -> dict:
    """Integer outputs of two tilings (bit-exact is the target)."""
    mi, ri = _np(mine["isect_ids"]), _np(ref["isect_ids"])
    out = {"tiles_per_gauss_diff": count_diff(mine["tiles_per_gauss"], ref["tiles_per_gauss"]),
           "n_isects_mine": int(mi.size), "n_isects_ref": int(ri.size),
           "offsets_diff": count_diff(mine["offsets"], ref["offsets"])}
    if mi.size == ri.size:
        out["isect_ids_diff"] = count_diff(mi, ri)
        out["flatten_ids_diff"] = count_diff(mine["flatten_ids"], ref["flatten_ids"])
    else:
        # compare as multisets of (key, id) pairs
        a = set(zip(mi.tolist(), _np(mine["flatten_ids"]).tolist()))
        b = set(zip(ri.tolist(), _np(ref["flatten_ids"]).tolist()))
        out["isect_ids_diff"] = len(a ^ b)
        out["flatten_ids_diff"] = len(a ^ b)
    return out


def image_stats(a, b, keep=None) -> dict:
    a, b = _np(a).astype(np.float64), _np(b).astype(np.float64)
    d = np.abs(a - b)
    if d.ndim == 3:
        d = d.max(axis=-1)
    out = {"maxabs_all": float(d.max()) if d.size else 0.0}
    if keep is not None:
        dk = np.where(keep, d, 0.0)
        out["maxabs"] = float(dk.max()) if dk.size else 0.0
    return out


# per-element gradient bound: |got - ref| <= GRAD_RTOL |ref| + GRAD_FLOOR max|ref|
GRAD_RTOL = 1e-3
GRAD_FLOOR = 3e-4


def grad_stats(a, b) -> dict:
    """Element-wise and tensor-wise relative errors of a gradient tensor;
    `bound_ratio` is the largest error over the per-element bound
    GRAD_RTOL |ref| + GRAD_FLOOR max|ref| (<= 1 passes)."""
    a, b = _np(a).astype(np.float64).ravel(), _np(b).astype(np.float64).ravel()
    if b.size == 0:
        return {"rel_l2": 0.0, "bound_ratio": 0.0}
    err = np.abs(a - b)
    scale = np.abs(b).max()
    rms = float(np.sqrt(np.mean(b * b)))
    rel = err / np.maximum(np.abs(b), 1e-30)
    big = np.abs(b) > 1e-2 * scale   # elements of at least 1 % of the largest
    bound = GRAD_RTOL * np.abs(b) + GRAD_FLOOR * scale + 1e-30
    return {"rel_l2": float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)),
            "maxabs_over_max": float(err.max() / max(scale, 1e-30)),
            "maxabs_over_rms": float(err.max() / max(rms, 1e-30)),
            "maxrel_big": float(rel[big].max()) if big.any() else 0.0,
            "bound_ratio": float((err / bound).max()),
            "n_rel_over_1e-3": int((rel > 1e-3).sum()),
            "n": int(b.size)}


def divergent_pixels(mine_last, ref_last, mine_alpha, ref_alpha) -> np.ndarray:
    """Pixels where the two forward passes composited a different set of
    Gaussians: a different last contributor, or an alpha apart by more than
    the 1e-4 image tolerance (a skipped or kept Gaussian mid-list)."""
    ml, rl = _np(mine_last), _np(ref_last)
    ma, ra = _np(mine_alpha), _np(ref_alpha)
    return (ml != rl) | (np.abs(ma.astype(np.float64) - ra) > 1e-4)


def oracle_band(sc_np: dict, colors, W, H, ro, rd, off, flat, velocity=None, ray_t=None) -> np.ndarray:
    """The CPU oracle's threshold-ambiguity band: pixels where one of the
    compositing's threshold tests fell inside the float32 error band of the
    pair's alpha (oracle/xsg_oracle.cpp, alpha_rel_error)."""
    from oracle import oracle as O
    *_, near = O.rasterize_fwd(sc_np["means"], sc_np["quats"], sc_np["scales"], _np(colors), sc_np["opacities"],
                               W, H, TILE, TILE, _np(ro), _np(rd), _np(off), _np(flat),
                               velocity=None if velocity is None else _np(velocity),
                               ray_t=None if ray_t is None else _np(ray_t))
    return near


def tile_start_of_pixels(off, W, H) -> np.ndarray:
    offs = _np(off).reshape(-1)
    tw = (W + TILE - 1) // TILE
    ty = np.arange(H) // TILE
    tx = np.arange(W) // TILE
    return offs[ty[:, None] * tw + tx[None, :]]


def view_parity(sc, spec, device, colors=None, deg=3, cdim=3, phm=False, velocity=None, mutate=None,
                with_autograd=True, band=False) -> dict:
    """Every stage of one view through this package and through the
    reference's kernels on identical inputs.

    Stages compared: camera pack and rays; UT projection; tiling end to end
    (each side from its own projection) and in isolation (the reference's
    tiler fed this package's projection); compositing forward and backward
    on identical tiling, rays and forward outputs; the autograd path (forward
    workspace and kernel choice) against the reference's backward; and the
    whole render end to end.  Pixels are "ambiguous" where the two forward
    passes composited a different set of Gaussians (and, with `band`, where
    the CPU oracle's threshold band flags them); images are compared outside
    them and the upstream gradients are zero there on both sides."""
    import xsimgs_b200 as X
    from xsimgs_b200 import _C, scenes
    R = ref_module()
    cam = spec.make(device)
    if mutate is not None:
        mutate(cam)
    W, H = spec.width, spec.height
    m, s, q, o = (t.to(device).contiguous() for t in (sc.means, sc.scales, sc.quats, sc.opacities))
    vel = None if velocity is None else velocity.to(device).contiguous()
    rc = RefCamera(cam, spec.kind)
    st = {"pack_diff": count_diff(rc.pack, cam.pack)}
    ro, rd = cam.camera_rays(W, H)
    rro, rrd = rc.rays(W, H)
    st["rays_bitdiff"] = int(((ro != rro).any(-1) | (rd != rrd).any(-1)).sum())
    st["rays_maxabs"] = float(torch.maximum((ro - rro).abs().max(), (rd - rrd).abs().max()))
    mt = mine_tiling(cam, m, s, q, o, W, H, phm=phm, velocity=vel)
    rt = rc.tiling(m, s, q, o, W, H, phm=phm, velocity=vel)
    st["projection"] = compare_projection(mt["proj"], rt["proj"])
    st["tiling_e2e"] = compare_tiling(mt, rt)
    rt2 = rc.tiles(m, s, q, o, W, H, mt["proj"], velocity=vel)
    off2 = R.isect_offset_encode(rt2[1], (W + TILE - 1) // TILE, (H + TILE - 1) // TILE)
    st["tiling_isolated"] = compare_tiling(
        mt, dict(tiles_per_gauss=rt2[0], isect_ids=rt2[1], flatten_ids=rt2[2], offsets=off2))

    if colors is None:
        if cdim == 3 and deg is not None:
            colors = X.spherical_harmonics_fused(sc.sh.to(device), m, cam.t0, deg).detach()
        else:
            colors = torch.rand(sc.n, cdim, generator=torch.Generator().manual_seed(5)).to(device)
    colors = colors.contiguous()
    off, flat = mt["offsets"], mt["flatten_ids"]
    dyn = vel is not None
    rt_delta = cam.image_time_delta(ro).contiguous() if dyn else None
    args = dict(means=m, quats=q, scales=s, colors=colors.unsqueeze(0), opacities=o.view(1, -1), image_width=W,
                image_height=H, tile_size_width=TILE, tile_size_height=TILE, ray_origs=ro, ray_dirs=rd,
                tile_offsets=off, flatten_ids=flat)
    if dyn:
        mine_f = _C.rasterize_eval3d_dynamic_fwd(velocity=vel, ray_time_delta=rt_delta, **args)
        ref_f = R.rasterize_eval3d_dynamic_fwd(velocity=vel, ray_time_delta=rt_delta, **args)
    else:
        mine_f = _C.rasterize_eval3d_fwd(**args)
        ref_f = R.rasterize_eval3d_fwd(**args)
    if band:
        sc_np = {k: _np(v) for k, v in sc.params().items()}
        near = oracle_band(sc_np, colors, W, H, ro, rd, off, flat, velocity=vel, ray_t=rt_delta)
    else:
        near = np.zeros((H, W), bool)
    div = divergent_pixels(mine_f[3], ref_f[3], mine_f[2], ref_f[2])
    amb = near | div
    st["fwd"] = {"pixels": W * H, "oracle_band_frac": float(near.mean()), "divergent_px": int(div.sum()),
                 "divergent_outside_band": int((div & ~near).sum()), "ambiguous_frac": float(amb.mean()),
                 "last_ids_diff": count_diff(mine_f[3], ref_f[3]),
                 "last_ids_diff_outside_band": int(((_np(mine_f[3]) != _np(ref_f[3])) & ~near).sum()),
                 "rgb": image_stats(mine_f[0], ref_f[0], ~amb), "depth": image_stats(mine_f[1], ref_f[1], ~amb),
                 "alpha": image_stats(mine_f[2], ref_f[2], ~amb), "depth_max": float(ref_f[1].abs().max())}
    # backward on identical inputs (this package's forward outputs)
    vr, vd, va = (t.to(device) for t in scenes.upstream_grads(H, W, colors.shape[-1]))
    keep = torch.from_numpy(~amb).to(device)
    vr, vd, va = (vr * keep[..., None]).contiguous(), (vd * keep).contiguous(), (va * keep).contiguous()
    a, last = mine_f[2], mine_f[3]
    if dyn:
        gm = _C.rasterize_eval3d_dynamic_bwd(m, vel, s, q, o, colors, ro, rd, rt_delta, TILE, TILE, off, flat, a, last,
                                             vr, vd, va)
        gr = R.rasterize_eval3d_dynamic_bwd(m, vel, s, q, o, colors, ro, rd, rt_delta, TILE, TILE, off, flat, a, last,
                                            vr, vd, va)
        names = ["v_means", "v_velocity", "v_quats", "v_scales", "v_opacities", "v_colors", "v_ray_o", "v_ray_d",
                 "v_time_delta"]
    else:
        gm = _C.rasterize_eval3d_bwd(m, s, q, o, colors, ro, rd, TILE, TILE, off, flat, a, last, vr, vd, va)
        gr = R.rasterize_eval3d_bwd(m, s, q, o, colors, ro, rd, TILE, TILE, off, flat, a, last, vr, vd, va)
        names = ["v_means", "v_quats", "v_scales", "v_opacities", "v_colors", "v_ray_o", "v_ray_d"]
    st["bwd"] = {k: grad_stats(x, y) for k, x, y in zip(names, gm, gr) if x is not None and y is not None}
    # the reference against itself: its float atomics sum in a different
    # order on every run, which sets the scale of agreement to expect
    if dyn:
        gr2 = R.rasterize_eval3d_dynamic_bwd(m, vel, s, q, o, colors, ro, rd, rt_delta, TILE, TILE, off, flat, a, last,
                                             vr, vd, va)
    else:
        gr2 = R.rasterize_eval3d_bwd(m, s, q, o, colors, ro, rd, TILE, TILE, off, flat, a, last, vr, vd, va)
    st["ref_self"] = {k: grad_stats(x, y) for k, x, y in zip(names, gr2, gr) if x is not None and y is not None}
    ref_by_name = dict(zip(names, gr))
    if with_autograd:
        lv = {k: t.clone().requires_grad_(True) for k, t in
              dict(v_means=m, v_quats=q, v_scales=s, v_opacities=o, v_colors=colors).items()}
        if dyn:
            lv["v_velocity"] = vel.clone().requires_grad_(True)
            rgb, dep, al = X.ut_gs_dynamic_rasterize(lv["v_means"], lv["v_velocity"], lv["v_quats"], lv["v_scales"],
                                                     lv["v_opacities"], lv["v_colors"], ro, rd, rt_delta, off, flat,
                                                     TILE, TILE)
        else:
            rgb, dep, al = X.ut_gs_rasterize(lv["v_means"], lv["v_quats"], lv["v_scales"], lv["v_opacities"],
                                             lv["v_colors"], ro, rd, off, flat, TILE, TILE)
        ((rgb * vr).sum() + (dep * vd).sum() + (al * va).sum()).backward()
        st["bwd_autograd"] = {k: grad_stats(t.grad, ref_by_name[k]) for k, t in lv.items()}
    # end to end: each side its own rays, projection, tiling and compositing;
    # last ids are compared relative to each side's tile start
    rargs = dict(args, ray_origs=rro, ray_dirs=rrd, tile_offsets=rt["offsets"], flatten_ids=rt["flatten_ids"])
    rf2 = (R.rasterize_eval3d_dynamic_fwd(velocity=vel, ray_time_delta=rt_delta, **rargs) if dyn
           else R.rasterize_eval3d_fwd(**rargs))
    ml = _np(mine_f[3]) - tile_start_of_pixels(off, W, H)
    rl = _np(rf2[3]) - tile_start_of_pixels(rt["offsets"], W, H)
    d2 = (ml != rl) | (np.abs(_np(mine_f[2]).astype(np.float64) - _np(rf2[2])) > 1e-4)
    amb2 = near | d2
    st["e2e_render"] = {"divergent_px": int(d2.sum()), "divergent_outside_band": int((d2 & ~near).sum()),
                        "rgb": image_stats(mine_f[0], rf2[0], ~amb2), "depth": image_stats(mine_f[1], rf2[1], ~amb2),
                        "alpha": image_stats(mine_f[2], rf2[2], ~amb2)}
    return st


def c5_container(device, n_static: int = 1_000_000, n_bodies: int = 8, gauss_per_body: int = 20_000):
    """The C5 scene assembled on the GPU: the static street scene followed in
    the container by `n_bodies` SMPL bodies skinned by this package's kernels
    (smpl_local_to_global_pose + smpl_lbs_skinning), with the bodies' instance
    velocities (the static part has zero velocity).  Returns a scene object
    for `view_parity`, the velocity [M, 3] and RGB colours [M, 3]."""
    from types import SimpleNamespace
    from xsimgs_b200 import scenes
    from xsimgs_b200.nodes import smpl_lbs_skinning, smpl_local_to_global_pose
    st = scenes.street_scene(n_static)
    s = scenes.c5_smpl(n_bodies=n_bodies, gauss_per_body=gauss_per_body)
    g = lambda t: t.to(device).contiguous()
    valid = g(s["valid_ids"])
    with torch.no_grad():
        gq, gt = smpl_local_to_global_pose(valid, g(s["local_q"]), g(s["joints"]), g(s["a0_inv_q"]), g(s["a0_inv_t"]))
        nb = n_bodies * gauss_per_body
        pos = torch.cat([g(st.means), torch.zeros(nb, 3, device=device)])
        rot = torch.cat([g(st.quats), torch.zeros(nb, 4, device=device)])
        vel = torch.zeros(n_static + nb, 3, device=device)
        pos, rot, vel, _ = smpl_lbs_skinning(valid, gq, gt, g(s["vertices"]), g(s["quats"]), g(s["weights"]),
                                             g(s["instance_ids"]), g(s["instance_t"]), g(s["instance_v"]), n_static,
                                             pos, rot, vel)
    gen = torch.Generator().manual_seed(21)
    scales = torch.cat([st.scales, torch.exp(torch.randn(nb, 3, generator=gen) * 0.3 - 3.5)])
    opac = torch.cat([st.opacities, torch.sigmoid(torch.randn(nb, generator=gen) + 1.0)])
    colors = torch.rand(n_static + nb, 3, generator=gen)
    sc = SimpleNamespace(means=pos, quats=rot, scales=scales, opacities=opac, n=n_static + nb,
                         params=lambda: dict(means=pos, quats=rot, scales=scales, opacities=opac))
    return sc, vel, colors
