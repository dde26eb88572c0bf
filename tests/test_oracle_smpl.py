"""The SMPL part of the CPU oracle against float64 autograd of an independent
torch restatement (same conventions: w-first Hamilton quaternions, R(q) as
the quaternion polynomial, std() = unit with w >= 0, Shepperd's
matrix-to-quaternion).  Pins the oracle's hand-written backward passes
(smpl_local_to_global.cu:123-279, smpl_lbs_skinning.cu:137-268 restated) and
its forward values."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

PARENTS = (-1, 0, 0, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 9, 9, 12, 13, 14, 16, 17, 18, 19, 20, 21)


def qmul(a, b):
    aw, av = a[..., :1], a[..., 1:]
    bw, bv = b[..., :1], b[..., 1:]
    return torch.cat([aw * bw - (av * bv).sum(-1, keepdim=True), aw * bv + bw * av + torch.cross(av, bv, dim=-1)],
                     dim=-1)


def rotm(q):
    w, x, y, z = q.unbind(-1)
    return torch.stack([torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
                        torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
                        torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)], -2)


def qstd(q):
    n = q / q.norm(dim=-1, keepdim=True)
    return torch.where(q[..., :1] < 0, -n, n)


def shepperd(m):
    m00, m11, m22 = m[..., 0, 0], m[..., 1, 1], m[..., 2, 2]
    tr = m00 + m11 + m22
    r = lambda v: torch.sqrt(torch.clamp(v, min=1e-6)) * 2
    s0, s1, s2, s3 = r(tr + 1), r(1 + m00 - m11 - m22), r(1 + m11 - m00 - m22), r(1 + m22 - m00 - m11)
    q0 = torch.stack([0.25 * s0, (m[..., 2, 1] - m[..., 1, 2]) / s0, (m[..., 0, 2] - m[..., 2, 0]) / s0,
                      (m[..., 1, 0] - m[..., 0, 1]) / s0], -1)
    q1 = torch.stack([(m[..., 2, 1] - m[..., 1, 2]) / s1, 0.25 * s1, (m[..., 0, 1] + m[..., 1, 0]) / s1,
                      (m[..., 0, 2] + m[..., 2, 0]) / s1], -1)
    q2 = torch.stack([(m[..., 0, 2] - m[..., 2, 0]) / s2, (m[..., 0, 1] + m[..., 1, 0]) / s2, 0.25 * s2,
                      (m[..., 1, 2] + m[..., 2, 1]) / s2], -1)
    q3 = torch.stack([(m[..., 1, 0] - m[..., 0, 1]) / s3, (m[..., 0, 2] + m[..., 2, 0]) / s3,
                      (m[..., 1, 2] + m[..., 2, 1]) / s3, 0.25 * s3], -1)
    b1 = (m00 > m11) & (m00 > m22)
    b2 = m11 > m22
    return torch.where((tr > 0)[..., None], q0, torch.where(b1[..., None], q1, torch.where(b2[..., None], q2, q3)))


def torch_l2g(ids, local_q, joints, a0q, a0t):
    L_q = qstd(local_q)
    rel = joints.clone()
    rel[:, 1:] = joints[:, 1:] - joints[:, list(PARENTS[1:])]
    Gq, Gt = [None] * 24, [None] * 24
    for j in range(24):
        if PARENTS[j] < 0:
            Gq[j], Gt[j] = L_q[:, j], rel[:, j]
        else:
            p = PARENTS[j]
            Gq[j] = qmul(Gq[p], L_q[:, j])
            Gt[j] = (rotm(Gq[p]) @ rel[:, j, :, None])[..., 0] + Gt[p]
    Gq, Gt = torch.stack(Gq, 1), torch.stack(Gt, 1)
    Tt = Gt - (rotm(Gq) @ joints[..., None])[..., 0]
    Oq = qmul(Gq, a0q)
    Ot = (rotm(Gq) @ a0t[..., None])[..., 0] + Tt
    return Oq[ids], Ot[ids]


def torch_lbs(valid_ids, gq, gt, vertices, quats, weights, inst_ids, inst_t, inst_v):
    M = torch.cat([rotm(gq), gt[..., None]], dim=-1)                    # [B, 24, 3, 4]
    w = weights[valid_ids]                                              # [B, 24, V]
    W = (w[..., None, None] * M[:, :, None]).sum(1)                      # [B, V, 3, 4]
    v = vertices[valid_ids]
    P = (W[..., :3] @ v[..., None])[..., 0] + W[..., 3] + inst_t[inst_ids[valid_ids]][:, None]
    R = qmul(qstd(shepperd(W[..., :3])), quats[valid_ids])
    vel = inst_v[inst_ids[valid_ids]][:, None].expand_as(P)
    return P, R, vel


def _small(seed, n=3, V=400):
    from xsimgs_b200 import scenes
    return scenes.c5_smpl(n_bodies=n, gauss_per_body=V, template_verts=800, seed=seed, pose_sigma=0.6)


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_local_to_global_is_autograd(seed):
    s = _small(seed)
    rng = np.random.default_rng(seed)
    ids = np.array([2, 0], np.uint32)
    local_q = s["local_q"].numpy() * rng.uniform(0.5, 2.0, size=(3, 24, 1)).astype(np.float32)  # raw, not unit
    local_q[0, 5] *= -1.0  # a negative real part: std() flips it
    a0q = s["local_q"].numpy()[[1, 2, 0]]
    a0t = rng.normal(size=(3, 24, 3)).astype(np.float32) * 0.1
    oq, ot = O.smpl_local_to_global_fwd(ids, local_q, s["joints"].numpy(), a0q, a0t)
    T = lambda a, g=False: torch.tensor(np.asarray(a), dtype=torch.float64, requires_grad=g)
    tl, ta0q, ta0t = T(local_q, True), T(a0q, True), T(a0t, True)
    rq, rt = torch_l2g(torch.tensor(ids.astype(np.int64)), tl, T(s["joints"].numpy()), ta0q, ta0t)
    np.testing.assert_allclose(oq, rq.detach().numpy(), atol=2e-6)
    np.testing.assert_allclose(ot, rt.detach().numpy(), atol=5e-6)
    gq = rng.normal(size=oq.shape).astype(np.float32)
    gt = rng.normal(size=ot.shape).astype(np.float32)
    ((rq * T(gq)).sum() + (rt * T(gt)).sum()).backward()
    d_local, d_a0q, d_a0t = O.smpl_local_to_global_bwd(ids, local_q, s["joints"].numpy(), a0q, a0t, oq, ot, gq, gt)
    np.testing.assert_allclose(d_local, tl.grad.numpy(), rtol=1e-4, atol=1e-4 * np.abs(tl.grad.numpy()).max())
    np.testing.assert_allclose(d_a0q, ta0q.grad.numpy(), rtol=1e-4, atol=1e-4 * np.abs(ta0q.grad.numpy()).max())
    np.testing.assert_allclose(d_a0t, ta0t.grad.numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_lbs_is_autograd(seed):
    s = _small(seed)
    rng = np.random.default_rng(10 + seed)
    B = 3
    valid = np.array([1, 2, 0], np.uint32)
    # global transforms from the chain (unit quaternions), one per valid object
    gq, gt = O.smpl_local_to_global_fwd(valid, s["local_q"].numpy(), s["joints"].numpy(), s["a0_inv_q"].numpy(),
                                        s["a0_inv_t"].numpy())
    V = s["vertices"].shape[1]
    offset, size = 17, 17 + 3 * V + 5
    args = [s["vertices"].numpy(), s["quats"].numpy(), s["weights"].numpy(), s["instance_ids"].numpy().astype(
        np.uint32), s["instance_t"].numpy(), s["instance_v"].numpy()]
    pos, rot, vel, mask = O.smpl_lbs_fwd(valid, gq, gt, *args, offset, size)
    T = lambda a, g=False: torch.tensor(np.asarray(a), dtype=torch.float64, requires_grad=g)
    tq, tt, tv, tqs, tw, tit, tiv = (T(a, True) for a in (gq, gt, args[0], args[1], args[2], args[4], args[5]))
    vid = torch.tensor(valid.astype(np.int64))
    P, R, Vl = torch_lbs(vid, tq, tt, tv, tqs, tw, torch.tensor(args[3].astype(np.int64)), tit, tiv)
    rows = (offset + vid[:, None] * V + torch.arange(V)[None]).reshape(-1).numpy()
    np.testing.assert_allclose(pos[rows], P.detach().reshape(-1, 3).numpy(), atol=2e-5)
    np.testing.assert_allclose(rot[rows], R.detach().reshape(-1, 4).numpy(), atol=2e-5)
    np.testing.assert_allclose(vel[rows], Vl.detach().reshape(-1, 3).numpy(), atol=0)
    assert mask[rows].all() and mask.sum() == B * V
    g_pos = rng.normal(size=pos.shape).astype(np.float32)
    g_rot = rng.normal(size=rot.shape).astype(np.float32)
    g_vel = rng.normal(size=vel.shape).astype(np.float32)
    loss = ((P.reshape(-1, 3) * T(g_pos[rows])).sum() + (R.reshape(-1, 4) * T(g_rot[rows])).sum()
            + (Vl.reshape(-1, 3) * T(g_vel[rows])).sum())
    loss.backward()
    d = O.smpl_lbs_bwd(valid, args[3], gq, gt, args[0], args[1], args[2], offset, 3, g_pos, g_rot, g_vel)
    for key, t in [("global_q", tq), ("global_t", tt), ("vertices", tv), ("quats", tqs), ("weights", tw),
                   ("instance_t", tit), ("instance_v", tiv)]:
        ref = t.grad.numpy()
        np.testing.assert_allclose(d[key], ref, rtol=2e-4, atol=2e-4 * max(1.0, np.abs(ref).max()), err_msg=key)


def test_oracle_ids_compaction():
    ids = np.array([3, 0, 2, 2, 1, 3], np.uint32)
    mask = np.array([1, 0, 1, 0], np.uint8)
    np.testing.assert_array_equal(O.smpl_ids_compaction(ids, mask), [1, 2, 3])
    assert O.smpl_ids_compaction(ids[:0], mask).size == 0
