"""ctypes front end of the CPU oracle (test infrastructure, never a product
path).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
use it, as the checker / the timed CPU restatement.  Parity status: unpinned
(see oracle/xsg_oracle.cpp).

All functions take and return numpy arrays (float32 unless stated).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.OUT
        if not os.path.exists(path):
            path = _build.build()
        _lib = C.CDLL(path)
        _lib.xsgo_isect_regular.restype = C.c_int64
        _lib.xsgo_isect_spherical.restype = C.c_int64
        _lib.xsgo_num_threads.restype = C.c_int
        _lib.xsgo_smpl_ids_compaction.restype = C.c_int64
    return _lib


CAM = {"pinhole": 0, "fisheye": 1, "spherical": 2, "lidar": 3, "distorted": 4}


def _p(a):
    if a is None:
        return None
    return a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int):
    lib().xsgo_set_num_threads(C.c_int(n))


def num_threads() -> int:
    return int(lib().xsgo_num_threads())


def camera_rays(cam, pack, W, H, world_space=True, normalized=True, elev=None):
    pack = _f32(pack).reshape(-1)
    elev = _f32(elev)
    ro = np.zeros((H, W, 3), np.float32)
    rd = np.zeros((H, W, 3), np.float32)
    valid = np.zeros((H, W), np.uint8)
    lib().xsgo_camera_rays(C.c_int(CAM[cam]), _p(pack), _p(elev), C.c_int(W), C.c_int(H), C.c_int(int(world_space)),
                           C.c_int(int(normalized)), _p(ro), _p(rd), _p(valid))
    return ro, rd, valid.astype(bool)


def pixel_time(cam, pack, W, H, delta, elev=None):
    pack = _f32(pack).reshape(-1)
    out = np.zeros((H, W), np.float32)
    lib().xsgo_pixel_time(C.c_int(CAM[cam]), _p(pack), _p(_f32(elev)), C.c_int(W), C.c_int(H), C.c_int(int(delta)),
                          _p(out))
    return out


def projection(cam, pack, pts, vel=None, thr=1e-4, max_res=0.002, margin=1.0, mode=0, nojac=False, elev=None):
    pack = _f32(pack).reshape(-1)
    pts = _f32(pts)
    vel = _f32(vel)
    n = pts.shape[0]
    uvdt = np.zeros((n, 4), np.float32)
    mask = np.zeros(n, np.uint8)
    lib().xsgo_projection(C.c_int(CAM[cam]), _p(pack), _p(_f32(elev)), _p(pts), _p(vel), C.c_int64(n),
                          C.c_float(thr), C.c_float(max_res), C.c_float(margin), C.c_int(mode), C.c_int(int(nojac)),
                          _p(uvdt), _p(mask))
    return uvdt, mask.astype(bool)


def projection_utgs(cam, pack, pts, vel, scales, quats, opac, W, H, ua=0.1, ub=2.0, uk=0.0, thr=1e-4,
                    max_res=0.002, margin=1.0, phm=False, elev=None):
    pack = _f32(pack).reshape(-1)
    pts, vel, scales, quats, opac = (_f32(a) for a in (pts, vel, scales, quats, opac))
    n = pts.shape[0]
    flags = np.zeros(n, np.uint8)
    radii = np.zeros((n, 2), np.float32)
    means2d = np.zeros((n, 2), np.float32)
    depths = np.zeros(n, np.float32)
    lib().xsgo_projection_utgs(C.c_int(CAM[cam]), _p(pack), _p(_f32(elev)), _p(pts), _p(vel), _p(scales),
                               _p(quats), _p(opac), C.c_int64(n), C.c_float(W), C.c_float(H), C.c_float(ua),
                               C.c_float(ub), C.c_float(uk), C.c_float(thr), C.c_float(max_res),
                               C.c_float(margin), C.c_int(int(phm)), _p(flags), _p(radii), _p(means2d),
                               _p(depths))
    return flags, radii, means2d, depths


def mask_radii(radii, mask=None, packed=None):
    radii = _f32(radii).copy()
    n = radii.shape[0]
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint8)
    pk = None if packed is None else np.ascontiguousarray(packed, dtype=np.uint32)
    lib().xsgo_mask_radii(_p(m), _p(pk), C.c_int64(n), _p(radii))
    return radii


def isect_regular(means2d, radii, depths, W, H, tsx=16, tsy=16, sort=True):
    means2d, radii, depths = _f32(means2d), _f32(radii), _f32(depths)
    n = means2d.shape[0]
    tpg = np.zeros(n, np.int32)
    total = lib().xsgo_isect_regular(_p(means2d), _p(radii), _p(depths), C.c_int64(n), C.c_int(W), C.c_int(H),
                                     C.c_int(tsx), C.c_int(tsy), C.c_int(int(sort)), _p(tpg), None, None)
    ids = np.zeros(total, np.int64)
    flat = np.zeros(total, np.int32)
    lib().xsgo_isect_regular(_p(means2d), _p(radii), _p(depths), C.c_int64(n), C.c_int(W), C.c_int(H), C.c_int(tsx),
                             C.c_int(tsy), C.c_int(int(sort)), _p(tpg), _p(ids), _p(flat))
    return tpg, ids, flat


def isect_spherical(lidar, pack, elev_values, pts, vel, scales, quats, opac, flags, means2d, radii, depths,
                    elev_bounds, tsx, tsy, W, H, ua=0.1, ub=2.0, uk=0.0, sort=True):
    pack = _f32(pack).reshape(-1)
    pts, vel, scales, quats, opac = (_f32(a) for a in (pts, vel, scales, quats, opac))
    means2d, radii, depths = _f32(means2d), _f32(radii), _f32(depths)
    flags = np.ascontiguousarray(flags, dtype=np.uint8)
    eb = _f32(elev_bounds)
    n_eb = 0 if eb is None else eb.shape[0]
    n = means2d.shape[0]
    tpg = np.zeros(n, np.int32)
    args = [C.c_int(int(lidar)), _p(pack), _p(_f32(elev_values)), _p(pts), _p(vel), _p(scales), _p(quats),
            _p(opac), _p(flags), _p(means2d), _p(radii), _p(depths), _p(eb), C.c_int(n_eb), C.c_int64(n),
            C.c_int(tsx), C.c_int(tsy), C.c_float(W), C.c_float(H), C.c_float(ua), C.c_float(ub), C.c_float(uk),
            C.c_int(int(sort)), _p(tpg)]
    total = lib().xsgo_isect_spherical(*args, None, None)
    ids = np.zeros(total, np.int64)
    flat = np.zeros(total, np.int32)
    lib().xsgo_isect_spherical(*args, _p(ids), _p(flat))
    return tpg, ids, flat


def isect_offset_encode(isect_ids, tw, th):
    ids = np.ascontiguousarray(isect_ids, dtype=np.int64)
    out = np.zeros((th, tw), np.int32)
    lib().xsgo_isect_offset_encode(_p(ids), C.c_int64(ids.shape[0]), C.c_int(tw), C.c_int(th), _p(out))
    return out


def rasterize_fwd(means, quats, scales, colors, opac, W, H, tsx, tsy, ray_o, ray_d, offsets, flatten,
                  velocity=None, ray_t=None):
    means, quats, scales, opac = (_f32(a) for a in (means, quats, scales, opac))
    colors = _f32(colors)
    cdim = 0 if colors is None else colors.shape[-1]
    ray_o, ray_d, vel, ray_t = _f32(ray_o), _f32(ray_d), _f32(velocity), _f32(ray_t)
    offsets = np.ascontiguousarray(offsets, dtype=np.int32)
    flatten = np.ascontiguousarray(flatten, dtype=np.int32)
    th, tw = offsets.shape
    rgb = np.zeros((H, W, cdim), np.float32)
    depth = np.zeros((H, W), np.float32)
    alpha = np.zeros((H, W), np.float32)
    last = np.zeros((H, W), np.int32)
    near = np.zeros((H, W), np.uint8)
    lib().xsgo_rasterize_fwd(_p(means), _p(vel), _p(quats), _p(scales), _p(colors), C.c_int(cdim), _p(opac),
                             C.c_int(W), C.c_int(H), C.c_int(tsx), C.c_int(tsy), _p(ray_o), _p(ray_d), _p(ray_t),
                             _p(offsets), C.c_int(tw), C.c_int(th), _p(flatten), C.c_int64(flatten.shape[0]),
                             _p(rgb), _p(depth), _p(alpha), _p(last), _p(near))
    return rgb, depth, alpha, last, near.astype(bool)


def rasterize_bwd(means, quats, scales, colors, opac, W, H, tsx, tsy, ray_o, ray_d, offsets, flatten,
                  render_alpha, last_ids, v_rgb, v_depth, v_alpha, velocity=None, ray_t=None):
    means, quats, scales, opac = (_f32(a) for a in (means, quats, scales, opac))
    colors = _f32(colors)
    cdim = 0 if colors is None else colors.shape[-1]
    ray_o, ray_d, vel, ray_t = _f32(ray_o), _f32(ray_d), _f32(velocity), _f32(ray_t)
    offsets = np.ascontiguousarray(offsets, dtype=np.int32)
    flatten = np.ascontiguousarray(flatten, dtype=np.int32)
    render_alpha, v_rgb, v_depth, v_alpha = (_f32(a) for a in (render_alpha, v_rgb, v_depth, v_alpha))
    last_ids = np.ascontiguousarray(last_ids, dtype=np.int32)
    th, tw = offsets.shape
    n = means.shape[0]
    out = dict(v_means=np.zeros((n, 3), np.float32), v_quats=np.zeros((n, 4), np.float32),
               v_scales=np.zeros((n, 3), np.float32), v_opacities=np.zeros(n, np.float32),
               v_colors=np.zeros((n, cdim), np.float32) if cdim else None,
               v_ray_o=np.zeros((H, W, 3), np.float32), v_ray_d=np.zeros((H, W, 3), np.float32))
    if vel is not None:
        out["v_velocity"] = np.zeros((n, 3), np.float32)
        out["v_ray_t"] = np.zeros((H, W), np.float32)
    lib().xsgo_rasterize_bwd(_p(means), _p(vel), _p(quats), _p(scales), _p(colors), C.c_int(cdim), _p(opac),
                             C.c_int(W), C.c_int(H), C.c_int(tsx), C.c_int(tsy), _p(ray_o), _p(ray_d), _p(ray_t),
                             _p(offsets), C.c_int(tw), C.c_int(th), _p(flatten), C.c_int64(flatten.shape[0]),
                             C.c_int64(n), _p(render_alpha), _p(last_ids), _p(v_rgb), _p(v_depth), _p(v_alpha),
                             _p(out["v_means"]), _p(out.get("v_velocity")), _p(out["v_quats"]),
                             _p(out["v_scales"]), _p(out["v_colors"]), _p(out["v_opacities"]), _p(out["v_ray_o"]),
                             _p(out["v_ray_d"]), _p(out.get("v_ray_t")))
    return out


def _sh_dims(coeffs, layout_3kn):
    n = coeffs.shape[2] if layout_3kn else coeffs.shape[0]
    return n, coeffs.shape[1]


def sh_fwd(degree, origin, pos, coeffs, dc=None, mask=None, layout_3kn=False):
    origin, pos, coeffs, dc = _f32(origin), _f32(pos), _f32(coeffs), _f32(dc)
    mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
    n, dim = _sh_dims(coeffs, layout_3kn)
    out = np.zeros((n, 3), np.float32)
    lib().xsgo_sh_fwd(C.c_int(degree), _p(origin), _p(pos), _p(coeffs), _p(dc), _p(mask), C.c_int(int(layout_3kn)),
                      C.c_int64(n), C.c_int(dim), _p(out))
    return out


def sh_bwd(degree, origin, pos, coeffs, d_out, dc=None, mask=None, layout_3kn=False):
    origin, pos, coeffs, dc, d_out = _f32(origin), _f32(pos), _f32(coeffs), _f32(dc), _f32(d_out)
    mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
    n, dim = _sh_dims(coeffs, layout_3kn)
    d_coeffs = np.zeros_like(coeffs)
    d_dc = None if dc is None else np.zeros_like(dc)
    d_pos = np.zeros((n, 3), np.float32)
    d_origin = np.zeros(3, np.float32)
    lib().xsgo_sh_bwd(C.c_int(degree), _p(origin), _p(pos), _p(coeffs), _p(dc), _p(mask), C.c_int(int(layout_3kn)),
                      C.c_int64(n), C.c_int(dim), _p(d_out), _p(d_coeffs), _p(d_dc), _p(d_pos), _p(d_origin))
    return d_coeffs, d_dc, d_pos, d_origin


# ------------------------------------------------------------------ SMPL --
def _u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def smpl_local_to_global_fwd(ids, local_q, joints, a0q, a0t):
    ids, local_q, joints, a0q, a0t = _u32(ids), _f32(local_q), _f32(joints), _f32(a0q), _f32(a0t)
    b = ids.shape[0]
    out_q = np.zeros((b, 24, 4), np.float32)
    out_t = np.zeros((b, 24, 3), np.float32)
    lib().xsgo_smpl_local_to_global_fwd(C.c_int64(b), _p(ids), _p(local_q), _p(joints), _p(a0q), _p(a0t),
                                        _p(out_q), _p(out_t))
    return out_q, out_t


def smpl_local_to_global_bwd(ids, local_q, joints, a0q, a0t, out_q, out_t, gq, gt):
    ids, local_q, joints, a0q, a0t = _u32(ids), _f32(local_q), _f32(joints), _f32(a0q), _f32(a0t)
    out_q, out_t, gq, gt = _f32(out_q), _f32(out_t), _f32(gq), _f32(gt)
    d_local_q, d_a0q, d_a0t = np.zeros_like(local_q), np.zeros_like(a0q), np.zeros_like(a0t)
    lib().xsgo_smpl_local_to_global_bwd(C.c_int64(ids.shape[0]), _p(ids), _p(local_q), _p(joints), _p(a0q),
                                        _p(a0t), _p(out_q), _p(out_t), _p(gq), _p(gt), _p(d_local_q), _p(d_a0q),
                                        _p(d_a0t))
    return d_local_q, d_a0q, d_a0t


def smpl_lbs_fwd(valid_ids, gq, gt, vertices, quats, weights, inst_ids, inst_t, inst_v, global_offset,
                 container_size, with_vel=True, with_mask=True):
    valid_ids, inst_ids = _u32(valid_ids), _u32(inst_ids)
    gq, gt, vertices, quats, weights, inst_t, inst_v = (_f32(a) for a in (gq, gt, vertices, quats, weights, inst_t,
                                                                         inst_v))
    V = vertices.shape[1]
    pos = np.zeros((container_size, 3), np.float32)
    rot = np.zeros((container_size, 4), np.float32)
    vel = np.zeros((container_size, 3), np.float32) if with_vel else None
    mask = np.zeros(container_size, np.uint8) if with_mask else None
    lib().xsgo_smpl_lbs_fwd(C.c_int64(valid_ids.shape[0]), C.c_int64(V), _p(valid_ids), _p(gq), _p(gt),
                            _p(vertices), _p(quats), _p(weights), _p(inst_ids), _p(inst_t), _p(inst_v),
                            C.c_int64(global_offset), _p(pos), _p(rot), _p(vel), _p(mask))
    return pos, rot, vel, mask


def smpl_lbs_bwd(valid_ids, inst_ids, gq, gt, vertices, quats, weights, global_offset, n_instances, g_pos, g_rot,
                 g_vel=None):
    valid_ids, inst_ids = _u32(valid_ids), _u32(inst_ids)
    gq, gt, vertices, quats, weights = (_f32(a) for a in (gq, gt, vertices, quats, weights))
    g_pos, g_rot, g_vel = _f32(g_pos), _f32(g_rot), _f32(g_vel)
    V = vertices.shape[1]
    d = dict(global_q=np.zeros_like(gq), global_t=np.zeros_like(gt), vertices=np.zeros_like(vertices),
             quats=np.zeros_like(quats), weights=np.zeros_like(weights),
             instance_v=np.zeros((n_instances, 3), np.float32), instance_t=np.zeros((n_instances, 3), np.float32))
    lib().xsgo_smpl_lbs_bwd(C.c_int64(valid_ids.shape[0]), C.c_int64(V), _p(valid_ids), _p(inst_ids), _p(gq),
                            _p(gt), _p(vertices), _p(quats), _p(weights), C.c_int64(global_offset), _p(g_pos),
                            _p(g_rot), _p(g_vel), _p(d["global_q"]), _p(d["global_t"]), _p(d["vertices"]),
                            _p(d["quats"]), _p(d["weights"]), _p(d["instance_v"]), _p(d["instance_t"]))
    return d


def smpl_ids_compaction(instance_ids, instance_mask):
    ids = _u32(instance_ids)
    mask = np.ascontiguousarray(instance_mask, dtype=np.uint8)
    out = np.zeros(ids.shape[0], np.uint32)
    c = lib().xsgo_smpl_ids_compaction(_p(ids), C.c_int64(ids.shape[0]), _p(mask), _p(out))
    return out[:c]


# ---------------------------------------------------------- scene nodes --
def _opt_u32(a):
    return None if a is None else _u32(a)


def rigid_transform_fwd(pos, rot, inst_id, iq, it, iv, iw, imask, offset, size, per_inst=None, gs_off=None):
    pos, rot, iq, it, iv, iw = (_f32(a) for a in (pos, rot, iq, it, iv, iw))
    inst_id, per_inst, gs_off = _u32(inst_id), _opt_u32(per_inst), _opt_u32(gs_off)
    imask = np.ascontiguousarray(imask, dtype=np.uint8)
    out_p = np.zeros((size, 3), np.float32)
    out_r = np.zeros((size, 4), np.float32)
    out_v = np.zeros((size, 3), np.float32)
    out_m = np.zeros(size, np.uint8)
    lib().xsgo_rigid_transform_fwd(C.c_int64(pos.shape[0]), _p(pos), _p(rot), _p(inst_id), _p(iq), _p(it), _p(iv),
                                   _p(iw), _p(imask), C.c_int64(offset), _p(per_inst), _p(gs_off), _p(out_p),
                                   _p(out_r), _p(out_v), _p(out_m))
    return out_p, out_r, out_v, out_m


def rigid_transform_bwd(pos, rot, inst_id, iq, iw, imask, offset, v_pos, v_rot, v_vel=None, per_inst=None,
                        gs_off=None):
    pos, rot, iq, iw, v_pos, v_rot, v_vel = (_f32(a) for a in (pos, rot, iq, iw, v_pos, v_rot, v_vel))
    inst_id, per_inst, gs_off = _u32(inst_id), _opt_u32(per_inst), _opt_u32(gs_off)
    imask = np.ascontiguousarray(imask, dtype=np.uint8)
    g = dict(positions=np.zeros_like(pos), rotations=np.zeros_like(rot), q=np.zeros_like(iq),
             t=np.zeros_like(iw), v=np.zeros_like(iw), w=np.zeros_like(iw))
    lib().xsgo_rigid_transform_bwd(C.c_int64(pos.shape[0]), _p(pos), _p(rot), _p(inst_id), _p(iq), _p(iw),
                                   _p(imask), C.c_int64(offset), _p(per_inst), _p(gs_off), _p(v_pos), _p(v_rot),
                                   _p(v_vel), _p(g["positions"]), _p(g["rotations"]), _p(g["q"]), _p(g["t"]),
                                   _p(g["v"]), _p(g["w"]))
    return g


def packed_mask_from_instances(ids, mask):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    out = np.zeros((ids.shape[0] + 31) // 32, np.uint32)
    lib().xsgo_packed_mask_from_instances(C.c_int64(ids.shape[0]), _p(ids), _p(mask), _p(out))
    return out


def interpolate_smpl_fwd(poses, times, root_q, inst_ids, query):
    poses, times, root_q = _f32(poses), _f32(times), _f32(root_q)
    inst_ids = _u32(inst_ids)
    n, frames, joints, _ = poses.shape
    out = np.zeros((n, joints, 4), np.float32)
    lib().xsgo_interpolate_smpl_fwd(C.c_int64(n), C.c_int(frames), C.c_int(joints), C.c_float(query), _p(poses),
                                    _p(times), _p(root_q), _p(inst_ids), _p(out))
    return out


def interpolate_smpl_bwd(poses, times, inst_ids, query, g_out, n_instances):
    poses, times, g_out = _f32(poses), _f32(times), _f32(g_out)
    inst_ids = _u32(inst_ids)
    n, frames, joints, _ = poses.shape
    d_poses = np.zeros_like(poses)
    d_root = np.zeros((n_instances, 4), np.float32)
    d_q = np.zeros(1, np.float32)
    lib().xsgo_interpolate_smpl_bwd(C.c_int64(n), C.c_int(frames), C.c_int(joints), C.c_float(query), _p(poses),
                                    _p(times), _p(inst_ids), _p(g_out), _p(d_poses), _p(d_root), _p(d_q))
    return d_poses, d_root, float(d_q[0])


# pack words per camera and the first word of its intrinsics (impls holding a
# float4 start 16-byte aligned, at word 20)
WORDS = {"pinhole": 22, "fisheye": 28, "spherical": 22, "lidar": 24, "distorted": 36}
INTR = {"pinhole": 18, "fisheye": 20, "spherical": 18, "lidar": 18, "distorted": 20}


def camera_rays_bwd(cam, pack, W, H, d_ray_o, d_ray_d, world_space=True, normalized=True, elev=None):
    """Gradient (float64, one per pack word) of sum(d_ray_o . ray_o + d_ray_d . ray_d)."""
    pack = _f32(pack).reshape(-1)
    out = np.zeros(WORDS[cam], np.float64)
    lib().xsgo_camera_rays_bwd(C.c_int(CAM[cam]), _p(pack), _p(_f32(elev)), C.c_int(W), C.c_int(H),
                               C.c_int(int(world_space)), C.c_int(int(normalized)), _p(_f32(d_ray_o)),
                               _p(_f32(d_ray_d)), C.c_int(out.size), _p(out))
    return out


def pixel_time_bwd(cam, pack, grad, delta, W=None, H=None, uv=None, elev=None):
    """(d_pack float64, d_uv or None) of sum(grad * pixel_time[_delta]); pixel grid
    when uv is None, else the given uv [n, 2]."""
    pack = _f32(pack).reshape(-1)
    grad = _f32(grad).reshape(-1)
    out = np.zeros(WORDS[cam], np.float64)
    d_uv = None
    if uv is not None:
        uv = _f32(uv).reshape(-1, 2)
        d_uv = np.zeros_like(uv)
        n, W, H = uv.shape[0], 1, 1
    else:
        n = W * H
    lib().xsgo_pixel_time_bwd(C.c_int(CAM[cam]), _p(pack), _p(_f32(elev)), C.c_int(W), C.c_int(H), _p(uv),
                              C.c_int64(n), C.c_int(int(delta)), _p(grad), C.c_int(out.size), _p(out), _p(d_uv))
    return out, d_uv


def undistort_map(pack, W, H, normalized_range=False):
    """Distorted uv of every pixel centre of a "distorted" camera, [H, W, 2]."""
    pack = _f32(pack).reshape(-1)
    out = np.zeros((H, W, 2), np.float32)
    lib().xsgo_undistort_map(_p(pack), C.c_int(W), C.c_int(H), C.c_int(int(normalized_range)), _p(out))
    return out


IMAGE_LAYOUTS = {"hwc_rgb": 0, "hwc_rgba": 1, "chw_rgb": 2}


def image_to_bytes(image, layout):
    """float32 [H, W, 3] -> uint8 [H, W, 3] / [H, W, 4] / [3, H, W]."""
    image = _f32(image)
    H, W = image.shape[:2]
    shape = {"hwc_rgb": (H, W, 3), "hwc_rgba": (H, W, 4), "chw_rgb": (3, H, W)}[layout]
    out = np.zeros(shape, np.uint8)
    lib().xsgo_image_to_bytes(C.c_int(IMAGE_LAYOUTS[layout]), C.c_int64(H * W), _p(image), _p(out))
    return out
