"""The scene-assembly part of the CPU oracle (container rigid transform,
packed instance masks, SMPL keyframe interpolation) against float64 autograd
of an independent torch restatement with the same conventions (w-first
Hamilton quaternions, std() = unit with w >= 0, shortest-arc slerp with a
normalised-lerp fallback above cos = 0.9995)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_oracle_smpl import qmul, qstd, rotm


def T(a, g=False):
    return torch.tensor(np.asarray(a), dtype=torch.float64, requires_grad=g)


def _rigid_case(seed, n=300, k=5, offsets=False):
    rng = np.random.default_rng(seed)
    pos = rng.normal(size=(n, 3)).astype(np.float32)
    rot = rng.normal(size=(n, 4)).astype(np.float32)
    inst = rng.integers(0, k, size=n).astype(np.uint32)
    iq = rng.normal(size=(k, 4)).astype(np.float32)
    iq /= np.linalg.norm(iq, axis=1, keepdims=True)
    it, iv, iw = (rng.normal(size=(k, 3)).astype(np.float32) for _ in range(3))
    imask = (np.arange(k) != 2).astype(np.uint8)
    per_inst = gs_off = None
    if offsets:  # instance-major packing: per_inst = start of each instance, gs_off = rank inside it
        counts = np.bincount(inst, minlength=k)
        per_inst = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint32)
        gs_off = np.zeros(n, np.uint32)
        seen = np.zeros(k, np.int64)
        for p in range(n):
            gs_off[p] = seen[inst[p]]
            seen[inst[p]] += 1
    return pos, rot, inst, iq, it, iv, iw, imask, per_inst, gs_off


@pytest.mark.parametrize("offsets", [False, True])
def test_oracle_rigid_transform_is_autograd(offsets):
    pos, rot, inst, iq, it, iv, iw, imask, per_inst, gs_off = _rigid_case(3, offsets=offsets)
    n, off = pos.shape[0], 7
    size = off + n + 4
    op, orr, ov, om = O.rigid_transform_fwd(pos, rot, inst, iq, it, iv, iw, imask, off, size, per_inst, gs_off)
    on = imask[inst].astype(bool)
    rows = (off + per_inst[inst] + gs_off) if offsets else (off + np.arange(n))
    rows_on = rows[on]
    assert om.sum() == on.sum() and om[rows_on].all()
    tp, tr, tq, tt, tv, tw = T(pos, True), T(rot, True), T(iq, True), T(it, True), T(iv, True), T(iw, True)
    ii = torch.tensor(inst.astype(np.int64))
    R = rotm(tq)[ii]
    pr = (R @ tp[..., None])[..., 0]
    P = pr + tt[ii]
    Q = qmul(tq[ii], tr)
    V = tv[ii] + torch.cross(tw[ii], pr, dim=-1)
    np.testing.assert_allclose(op[rows_on], P.detach().numpy()[on], atol=1e-5)
    np.testing.assert_allclose(orr[rows_on], Q.detach().numpy()[on], atol=1e-5)
    np.testing.assert_allclose(ov[rows_on], V.detach().numpy()[on], atol=1e-5)
    rng = np.random.default_rng(4)
    gp, gr, gv = (rng.normal(size=s).astype(np.float32) for s in [(size, 3), (size, 4), (size, 3)])
    m = torch.tensor(on, dtype=torch.float64)[:, None]
    loss = ((P * T(gp[rows])) * m).sum() + ((Q * T(gr[rows])) * m).sum() + ((V * T(gv[rows])) * m).sum()
    loss.backward()
    g = O.rigid_transform_bwd(pos, rot, inst, iq, iw, imask, off, gp, gr, gv, per_inst, gs_off)
    for key, t in [("positions", tp), ("rotations", tr), ("q", tq), ("t", tt), ("v", tv), ("w", tw)]:
        np.testing.assert_allclose(g[key], t.grad.numpy(), rtol=1e-4, atol=1e-4, err_msg=key)


def test_oracle_packed_mask():
    ids = np.array([-1, 0, 1, 2, 1, -1, 3] * 7, np.int32)
    mask = np.array([1, 0, 1, 0], np.uint8)
    got = O.packed_mask_from_instances(ids, mask)
    want = np.where(ids < 0, 1, mask[np.maximum(ids, 0)]).astype(bool)
    bits = np.array([(got[i // 32] >> (i % 32)) & 1 for i in range(ids.size)], bool)
    np.testing.assert_array_equal(bits, want)
    assert got[-1] >> (ids.size % 32) == 0  # bits past the end are clear


def _slerp(a, b, t):
    d = (a * b).sum(-1, keepdim=True)
    b = torch.where(d < 0, -b, b)
    d = d.abs()
    lin = a + t * (b - a)
    lin = lin / lin.norm(dim=-1, keepdim=True)
    th = torch.acos(d.clamp(max=0.9995))
    s = torch.sin(th)
    sl = (torch.sin((1 - t) * th) * a + torch.sin(t * th) * b) / s
    return torch.where(d > 0.9995, lin, sl)


@pytest.mark.parametrize("query", [0.37, -1.0, 5.0, 1.0])
def test_oracle_interpolation_is_autograd(query):
    rng = np.random.default_rng(int(query * 100) % 97)
    n, frames, joints, k = 3, 5, 24, 4
    poses = rng.normal(size=(n, frames, joints, 4)).astype(np.float32)
    poses[0, :, 5] = poses[0, 0, 5]  # identical keyframes: the lerp branch
    times = np.sort(rng.uniform(0, 2, size=(n, frames)), axis=1).astype(np.float32)
    root_q = rng.normal(size=(k, 4)).astype(np.float32)
    inst = np.array([2, 0, 3], np.uint32)
    out = O.interpolate_smpl_fwd(poses, times, root_q, inst, query)
    tp, tr, tqt = T(poses, True), T(root_q, True), T([query], True)
    res = []
    for o in range(n):
        f = next((i for i in range(frames) if times[o, i] >= query), frames)
        l, r = max(f - 1, 0), min(f, frames - 1)
        dt = float(times[o, r] - times[o, l])
        w = ((tqt - float(times[o, l])) / dt).clamp(0, 1) if dt > 0 else torch.zeros(1, dtype=torch.float64)
        rows = [tr[int(inst[o])]]
        for j in range(1, joints):
            rows.append(_slerp(qstd(tp[o, l, j]), qstd(tp[o, r, j]), w))
        res.append(torch.stack(rows))
    R = torch.stack(res)
    np.testing.assert_allclose(out, R.detach().numpy(), atol=2e-5)
    g = rng.normal(size=out.shape).astype(np.float32)
    (R * T(g)).sum().backward()
    d_poses, d_root, d_q = O.interpolate_smpl_bwd(poses, times, inst, query, g, k)
    np.testing.assert_allclose(d_poses, tp.grad.numpy(), rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(d_root, tr.grad.numpy(), atol=1e-6)
    want_q = float(tqt.grad[0]) if tqt.grad is not None else 0.0  # outside every key range: no gradient
    np.testing.assert_allclose(d_q, want_q, rtol=1e-3, atol=1e-3)


def _image_values(rng, shape):
    img = rng.uniform(-0.3, 1.3, size=shape).astype(np.float32)
    flat = img.reshape(-1)
    special = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1.0, 1.0 + 1e-7, 1.0 - 1e-7, 0.5 / 255, 1 / 255,
                        254.9999 / 255, 128 / 255], np.float32)
    k = min(special.size, flat.size)
    flat[:k] = special[:k]
    levels = (np.arange(min(256, flat.size - k)) / 255.0).astype(np.float32)
    flat[k:k + levels.size] = levels
    return img


@pytest.mark.parametrize("layout", ["hwc_rgb", "hwc_rgba", "chw_rgb"])
def test_oracle_image_layouts(layout):
    """Against numpy: saturate (NaN -> 0), times 255 in float32, truncate."""
    img = _image_values(np.random.default_rng(1), (7, 9, 3))
    s = np.where(np.isnan(img), np.float32(0), np.clip(img, np.float32(0), np.float32(1))).astype(np.float32)
    b = (s * np.float32(255)).astype(np.uint8)
    want = {"hwc_rgb": b, "hwc_rgba": np.concatenate([b, np.full((7, 9, 1), 255, np.uint8)], -1),
            "chw_rgb": b.transpose(2, 0, 1)}[layout]
    np.testing.assert_array_equal(O.image_to_bytes(img, layout), want)
