"""SMPL skinning on the GPU against the CPU oracle (C5-style synthetic
bodies), op by op through `_C`, then end to end: joint rotations ->
global joint transforms -> skinned Gaussians in the scene container ->
ut_gs_render -> backward to the joint rotations, checked against the
oracle's chain of the same stages."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_grads_close, assert_images_close, to_np, zero_at

pytestmark = pytest.mark.gpu


def _bodies(n=8, V=3000, seed=0, sigma=0.5):
    from xsimgs_b200 import scenes
    return scenes.c5_smpl(n_bodies=n, gauss_per_body=V, template_verts=2000, seed=seed, pose_sigma=sigma)


def _u32(t):
    return np.ascontiguousarray(to_np(t)).astype(np.uint32)


def test_local_to_global_matches_oracle(cuda):
    from xsimgs_b200 import _C
    s = _bodies()
    rng = np.random.default_rng(3)
    local_q = s["local_q"] * torch.from_numpy(rng.uniform(0.6, 1.8, size=(8, 24, 1)).astype(np.float32))
    local_q[2, 7] *= -1
    a0q = s["local_q"][[3, 1, 0, 7, 6, 5, 4, 2]].contiguous()
    a0t = torch.from_numpy(rng.normal(size=(8, 24, 3)).astype(np.float32) * 0.1)
    ids = torch.tensor([5, 0, 3, 7, 1], dtype=torch.int32)
    g = lambda t: t.to(cuda).contiguous()
    oq, ot = _C.smpl_local_to_global_fwd(g(ids), g(local_q), g(s["joints"]), g(a0q), g(a0t))
    rq, rt = O.smpl_local_to_global_fwd(_u32(ids), local_q.numpy(), s["joints"].numpy(), a0q.numpy(), a0t.numpy())
    np.testing.assert_allclose(to_np(oq), rq, atol=3e-6)
    np.testing.assert_allclose(to_np(ot), rt, atol=3e-6)
    gq = torch.from_numpy(rng.normal(size=rq.shape).astype(np.float32))
    gt = torch.from_numpy(rng.normal(size=rt.shape).astype(np.float32))
    d_local, d_a0q, d_a0t = _C.smpl_local_to_global_bwd(g(ids), g(local_q), g(s["joints"]), g(a0q), g(a0t), oq, ot,
                                                        g(gq), g(gt))
    r_local, r_a0q, r_a0t = O.smpl_local_to_global_bwd(_u32(ids), local_q.numpy(), s["joints"].numpy(), a0q.numpy(),
                                                       a0t.numpy(), rq, rt, gq.numpy(), gt.numpy())
    assert_grads_close(d_local, r_local, "d_local_q", rtol=2e-4)
    assert_grads_close(d_a0q, r_a0q, "d_a0_inv_q", rtol=2e-4)
    assert_grads_close(d_a0t, r_a0t, "d_a0_inv_t", rtol=2e-4)
    # bodies not named in the ids get no gradient
    assert float(d_local[[2, 4, 6]].abs().max()) == 0.0


@pytest.mark.parametrize("V,with_vel", [(3000, True), (20_000, False)])
def test_lbs_skinning_matches_oracle(cuda, V, with_vel):
    from xsimgs_b200 import _C
    s = _bodies(V=V, seed=1)
    valid = torch.tensor([6, 1, 3, 0, 2], dtype=torch.int32)
    g = lambda t: t.to(cuda).contiguous()
    gq, gt = _C.smpl_local_to_global_fwd(g(valid), g(s["local_q"]), g(s["joints"]), g(s["a0_inv_q"]),
                                         g(s["a0_inv_t"]))
    offset = 1234
    size = offset + 8 * V + 77
    pos = torch.full((size, 3), 7.0, device=cuda)
    rot = torch.full((size, 4), 7.0, device=cuda)
    vel = torch.full((size, 3), 7.0, device=cuda) if with_vel else None
    mask = torch.zeros(size, dtype=torch.bool, device=cuda)
    args = [g(s["vertices"]), g(s["quats"]), g(s["weights"]), g(s["instance_ids"]), g(s["instance_t"]),
            g(s["instance_v"])]
    _C.smpl_lbs_skinning(g(valid), gq, gt, *args, offset, pos, rot, vel, mask)
    np_args = [s["vertices"].numpy(), s["quats"].numpy(), s["weights"].numpy(), _u32(s["instance_ids"]),
               s["instance_t"].numpy(), s["instance_v"].numpy()]
    rp, rr, rv, rm = O.smpl_lbs_fwd(_u32(valid), to_np(gq), to_np(gt), *np_args, offset, size, with_vel=with_vel)
    written = rm.astype(bool)
    np.testing.assert_array_equal(to_np(mask), written)
    np.testing.assert_allclose(to_np(pos)[written], rp[written], atol=5e-6)
    np.testing.assert_allclose(to_np(rot)[written], rr[written], atol=5e-6)
    assert (to_np(pos)[~written] == 7.0).all() and (to_np(rot)[~written] == 7.0).all()
    if with_vel:
        np.testing.assert_array_equal(to_np(vel)[written], rv[written])
    rng = np.random.default_rng(5)
    g_pos = rng.normal(size=(size, 3)).astype(np.float32)
    g_rot = rng.normal(size=(size, 4)).astype(np.float32)
    g_vel = rng.normal(size=(size, 3)).astype(np.float32) if with_vel else None
    t = lambda a: None if a is None else torch.from_numpy(a).to(cuda)
    out = _C.smpl_lbs_skinning_bwd(g(valid), g(s["instance_ids"]), gq, gt, *args[:3], offset, 8, t(g_pos), t(g_rot),
                                   t(g_vel))
    ref = O.smpl_lbs_bwd(_u32(valid), _u32(s["instance_ids"]), to_np(gq), to_np(gt), *np_args[:3], offset, 8, g_pos,
                         g_rot, g_vel)
    for got, key in zip(out, ["global_q", "global_t", "vertices", "quats", "weights", "instance_v", "instance_t"]):
        assert_grads_close(got, ref[key], key, rtol=2e-4)


def test_ids_compaction_matches_oracle(cuda):
    from xsimgs_b200 import _C
    from xsimgs_b200.nodes import valid_instances_indices
    rng = np.random.default_rng(2)
    for n, k in [(700, 40), (3000, 300), (1, 1)]:
        ids = rng.integers(0, k, size=n).astype(np.int32)
        mask = rng.random(k) < 0.5
        got = _C.smpl_ids_compaction(torch.from_numpy(ids).to(cuda), torch.from_numpy(mask).to(cuda))
        np.testing.assert_array_equal(to_np(got).astype(np.uint32), O.smpl_ids_compaction(ids, mask))
        alt = valid_instances_indices(torch.from_numpy(ids).to(cuda), torch.from_numpy(mask).to(cuda))
        np.testing.assert_array_equal(to_np(alt).astype(np.uint32), O.smpl_ids_compaction(ids, mask))


def test_skinned_bodies_render_end_to_end(cuda):
    """Pose -> skinning into a container behind a static scene -> render ->
    backward; the joint-rotation gradient matches the oracle's chain."""
    import xsimgs_b200 as X
    from xsimgs_b200 import scenes
    from xsimgs_b200.nodes import smpl_lbs_skinning, smpl_local_to_global_pose
    n_b, V = 3, 2500
    s = _bodies(n=n_b, V=V, seed=4, sigma=0.4)
    s["instance_t"] = torch.tensor([[0.3, 0.0, 4.0], [-0.8, 0.2, 5.0], [1.0, -0.3, 6.0]])
    static = scenes.c1_scene(n=3000, seed=9)
    n_s = static.n
    size = n_s + n_b * V
    spec = scenes.c1_camera()
    W, H = spec.width, spec.height
    cam = spec.make(cuda)
    g = lambda t: t.to(cuda).contiguous()
    local_q = g(s["local_q"]).requires_grad_(True)
    valid = torch.arange(n_b, dtype=torch.int32, device=cuda)
    body_scale = torch.full((n_b * V, 3), 0.03)
    scales = g(torch.cat([static.scales, body_scale]))
    opac = g(torch.cat([static.opacities, torch.full((n_b * V,), 0.7)]))
    colors = g(torch.rand(size, 3, generator=torch.Generator().manual_seed(2)))

    def forward(lq):
        gq, gt = smpl_local_to_global_pose(valid, lq, g(s["joints"]), g(s["a0_inv_q"]), g(s["a0_inv_t"]))
        pos = torch.cat([g(static.means), torch.zeros(n_b * V, 3, device=cuda)])
        rot = torch.cat([g(static.quats), torch.zeros(n_b * V, 4, device=cuda)])
        pos, rot, _, _ = smpl_lbs_skinning(valid, gq, gt, g(s["vertices"]), g(s["quats"]), g(s["weights"]),
                                           g(s["instance_ids"]), g(s["instance_t"]), g(s["instance_v"]), n_s, pos,
                                           rot)
        return gq, gt, pos, rot

    gq, gt, pos, rot = forward(local_q)
    rgb, depth, alpha, meta = X.ut_gs_render(cam, pos, scales, rot, opac, W, H, colors=colors)
    # the oracle replays the compositing on the GPU's container and tiling
    td = X.ut_gs_tiling(cam, pos.detach(), scales, rot.detach(), W, H, opacity=opac)
    ro, rd = cam.camera_rays(W, H)
    np_in = (to_np(pos), to_np(rot), to_np(scales), to_np(colors), to_np(opac), W, H, 16, 16, to_np(ro), to_np(rd),
             to_np(td["isect_offsets"]), to_np(td["flatten_ids"]))
    rrgb, rdep, ralpha, rlast, near = O.rasterize_fwd(*np_in)
    assert_images_close(rgb, rrgb, near, what="rgb")
    body_px = O.rasterize_fwd(*np_in[:4], np.where(np.arange(size) >= n_s, np_in[4], 0), *np_in[5:])[2]
    assert (body_px > 0.05).mean() > 0.02, "the bodies must cover part of the image"
    vr, vd, va = zero_at(near, *scenes.upstream_grads(H, W, 3, seed=6))
    loss = (rgb * g(vr)).sum() + (depth * g(vd)).sum() + (alpha * g(va)).sum()
    loss.backward()

    _, _, _, last = X._C.rasterize_eval3d_fwd(
        means=pos.detach(), quats=rot.detach(), scales=scales, colors=colors.unsqueeze(0), opacities=opac.view(1, -1),
        image_width=W, image_height=H, tile_size_width=16, tile_size_height=16, ray_origs=ro, ray_dirs=rd,
        tile_offsets=td["isect_offsets"], flatten_ids=td["flatten_ids"])
    rg = O.rasterize_bwd(*np_in, to_np(alpha), to_np(last), vr.numpy(), vd.numpy(), va.numpy())
    d = O.smpl_lbs_bwd(_u32(valid), _u32(s["instance_ids"]), to_np(gq), to_np(gt), s["vertices"].numpy(),
                       s["quats"].numpy(), s["weights"].numpy(), n_s, n_b, rg["v_means"], rg["v_quats"])
    d_local, _, _ = O.smpl_local_to_global_bwd(_u32(valid), s["local_q"].numpy(), s["joints"].numpy(),
                                               s["a0_inv_q"].numpy(), s["a0_inv_t"].numpy(), to_np(gq), to_np(gt),
                                               d["global_q"], d["global_t"])
    assert float(np.abs(d_local).max()) > 0
    assert_grads_close(local_q.grad, d_local, "d_local_q (end to end)", rtol=2e-3)
