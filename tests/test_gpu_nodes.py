"""Scene assembly on the GPU against the CPU oracle: rigid per-instance
transforms into the container (instance-sorted and shuffled particles, with
and without per-instance offsets), packed instance masks, and SMPL keyframe
interpolation (queries inside, before and after the key range)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_grads_close, to_np
from tests.test_oracle_nodes import _rigid_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("offsets", [False, True])
@pytest.mark.parametrize("sorted_ids", [False, True])
def test_rigid_transform_matches_oracle(cuda, offsets, sorted_ids):
    from xsimgs_b200 import _C
    pos, rot, inst, iq, it, iv, iw, imask, per_inst, gs_off = _rigid_case(8, n=20_000, k=7, offsets=offsets)
    if sorted_ids:  # instances stored together: warp-uniform gradient reduction
        order = np.argsort(inst, kind="stable")
        pos, rot, inst = pos[order], rot[order], inst[order]
        if offsets:
            gs_off = gs_off[order]
    n, off = pos.shape[0], 33
    size = off + n + 5
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    ti = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a).astype(np.int32)).to(cuda)
    out_p = torch.zeros(size, 3, device=cuda)
    out_r = torch.zeros(size, 4, device=cuda)
    out_v = torch.zeros(size, 3, device=cuda)
    out_m = torch.zeros(size, dtype=torch.bool, device=cuda)
    _C.copy_gs_rigid_transform_fwd(t(pos), t(rot), ti(inst), t(iq), t(it), t(iv), t(iw),
                                   torch.from_numpy(imask.astype(bool)).to(cuda), out_p, out_r, out_v, out_m, off,
                                   ti(per_inst), ti(gs_off))
    rp, rr, rv, rm = O.rigid_transform_fwd(pos, rot, inst, iq, it, iv, iw, imask, off, size, per_inst, gs_off)
    np.testing.assert_array_equal(to_np(out_m), rm.astype(bool))
    np.testing.assert_allclose(to_np(out_p), rp, atol=2e-6)
    np.testing.assert_allclose(to_np(out_r), rr, atol=2e-6)
    np.testing.assert_allclose(to_np(out_v), rv, atol=2e-6)
    rng = np.random.default_rng(9)
    gp, gr, gv = (rng.normal(size=s).astype(np.float32) for s in [(size, 3), (size, 4), (size, 3)])
    got = _C.copy_gs_rigid_transform_bwd(t(pos), t(rot), ti(inst), t(iq), t(iw),
                                         torch.from_numpy(imask.astype(bool)).to(cuda), off, ti(per_inst),
                                         ti(gs_off), t(gp), t(gr), t(gv))
    ref = O.rigid_transform_bwd(pos, rot, inst, iq, iw, imask, off, gp, gr, gv, per_inst, gs_off)
    for g, key in zip(got, ["positions", "rotations", "q", "t", "v", "w"]):
        assert_grads_close(g, ref[key], key, rtol=2e-4)


def test_rigid_transform_autograd(cuda):
    from xsimgs_b200.nodes import rigid_transform_and_put
    pos, rot, inst, iq, it, iv, iw, imask, _, _ = _rigid_case(12, n=5000, k=4)
    t = lambda a, g=False: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).requires_grad_(g)
    tq, tt = t(iq, True), t(it, True)
    tp = t(pos, True)
    out_p, out_r, out_v, out_m = rigid_transform_and_put(tp, t(rot), t(inst.astype(np.int32)), tq, tt, t(iv), t(iw),
                                                         t(imask.astype(bool)))
    w = torch.randn_like(out_p)
    (out_p * w).sum().backward()
    ref = O.rigid_transform_bwd(pos, rot, inst, iq, iw, imask, 0, to_np(w), np.zeros_like(to_np(out_r)), None)
    assert_grads_close(tq.grad, ref["q"], "inst_q", rtol=2e-4)
    assert_grads_close(tt.grad, ref["t"], "inst_t", rtol=2e-4)
    assert_grads_close(tp.grad, ref["positions"], "positions", rtol=2e-4)


@pytest.mark.parametrize("n", [1, 31, 1000, 70_001])
def test_packed_mask_matches_oracle(cuda, n):
    from xsimgs_b200 import _C
    rng = np.random.default_rng(n)
    ids = rng.integers(-1, 6, size=n).astype(np.int32)
    mask = rng.random(6) < 0.5
    got = _C.packed_mask_from_instances(torch.from_numpy(ids).to(cuda), torch.from_numpy(mask).to(cuda))
    np.testing.assert_array_equal(to_np(got.view(torch.int32)).view(np.uint32), O.packed_mask_from_instances(ids, mask))


@pytest.mark.parametrize("query", [0.41, -3.0, 9.0])
def test_interpolation_matches_oracle(cuda, query):
    from xsimgs_b200 import _C
    rng = np.random.default_rng(int(abs(query) * 10))
    n, frames, joints, k = 9, 6, 24, 5
    poses = rng.normal(size=(n, frames, joints, 4)).astype(np.float32)
    poses[0, :, 7] = poses[0, 0, 7]  # identical keys: the linear branch
    times = np.sort(rng.uniform(0, 2, size=(n, frames)), axis=1).astype(np.float32)
    root_q = rng.normal(size=(k, 4)).astype(np.float32)
    inst = rng.integers(0, k, size=n).astype(np.uint32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    qt = t(np.array([query], np.float32))
    ti = t(inst.astype(np.int32))
    out = _C.interpolate_smpl_poses_fwd(t(poses), t(times), t(root_q), ti, qt)
    np.testing.assert_allclose(to_np(out), O.interpolate_smpl_fwd(poses, times, root_q, inst, query), atol=3e-6)
    g = rng.normal(size=(n, joints, 4)).astype(np.float32)
    d_poses, d_root, d_q = _C.interpolate_smpl_poses_bwd(t(poses), t(times), t(root_q), ti, qt, t(g))
    r_poses, r_root, r_q = O.interpolate_smpl_bwd(poses, times, inst, query, g, k)
    assert_grads_close(d_poses, r_poses, "d_poses", rtol=2e-4)
    np.testing.assert_allclose(to_np(d_root), r_root, atol=1e-5)
    np.testing.assert_allclose(float(to_np(d_q)[0]), r_q, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("layout", ["hwc_rgb", "hwc_rgba", "chw_rgb"])
@pytest.mark.parametrize("hw", [(1, 1), (7, 5), (48, 64), (1080, 1920), (3, 1)])
def test_image_layouts_match_oracle(cuda, layout, hw):
    """Bit-exact against the oracle, including NaN / inf / out-of-range values
    and exact k/255 levels, for pixel counts that are and are not multiples
    of four (vector and tail kernels)."""
    from tests.test_oracle_nodes import _image_values
    from xsimgs_b200 import nodes
    fn = {"hwc_rgb": nodes.image_to_hwc_rgb_byte, "hwc_rgba": nodes.image_to_hwc_rgba_byte,
          "chw_rgb": nodes.image_to_chw_rgb_byte}[layout]
    img = _image_values(np.random.default_rng(hw[0] * 7 + hw[1]), (*hw, 3))
    got = fn(torch.from_numpy(img).to(cuda))
    assert got.dtype == torch.uint8 and got.is_cuda
    np.testing.assert_array_equal(to_np(got), O.image_to_bytes(img, layout))
    # the reference's host-memory path gives the same bytes on finite values
    fin = np.nan_to_num(img, nan=0.0, posinf=2.0, neginf=-1.0)
    np.testing.assert_array_equal(to_np(fn(torch.from_numpy(fin).to(cuda))), to_np(fn(torch.from_numpy(fin))))


@pytest.mark.parametrize("layout", ["hwc_rgb", "hwc_rgba", "chw_rgb"])
def test_image_layouts_unaligned_and_strided(cuda, layout):
    from xsimgs_b200 import _C
    fn = getattr(_C, f"image_to_{layout}_byte")
    rng = np.random.default_rng(3)
    H, W = 37, 53
    base = torch.from_numpy(rng.uniform(-0.2, 1.2, size=H * W * 3 + 1).astype(np.float32)).to(cuda)
    img = base[1:].view(H, W, 3)  # 4-byte but not 16-byte aligned: the per-pixel kernel
    assert img.data_ptr() % 16 != 0
    np.testing.assert_array_equal(to_np(fn(img)), O.image_to_bytes(to_np(img), layout))
    big = torch.from_numpy(rng.uniform(-0.2, 1.2, size=(H, 2 * W, 3)).astype(np.float32)).to(cuda)
    view = big[:, ::2]  # non-contiguous: made contiguous first
    np.testing.assert_array_equal(to_np(fn(view)), O.image_to_bytes(to_np(view), layout))
    empty = torch.zeros(0, 4, 3, device=cuda)
    assert fn(empty).numel() == 0
    with pytest.raises(RuntimeError, match="must have dimensions"):
        fn(torch.zeros(4, 4, 4, device=cuda))
    with pytest.raises(RuntimeError, match="float32"):
        fn(torch.zeros(4, 4, 3, device=cuda, dtype=torch.float16))
