"""Host-synchronisation-free regular tiling (isect_regular_tiles_async) and
the `ut_gs_render` path built on it.

  * With enough capacity the lists, per-tile offsets and counts equal
    isect_regular_tiles + isect_offset_encode bit for bit; the tail past the
    count is never read.
  * With too little capacity the device counts say so ({total, capacity}),
    nothing is written past the capacity, and `ut_gs_render` renders the view
    again with exact lists: images and gradients equal the exact-list render
    bit for bit (gradients up to the float-atomic summation order of the
    backward: within 8x the spread of two exact-list renders), and the
    remembered capacity grows.
  * Empty views (no Gaussian on a tile) give all-zero offsets.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _view(cuda, n=200_000, seed=3):
    from xsimgs_b200 import scenes
    sc = scenes.street_scene(n, seed=seed).to(cuda)
    spec = scenes.c2_camera()
    cam = spec.make(cuda)
    return sc, cam, spec.width, spec.height


def _exact(m2, radii, dep, W, H):
    from xsimgs_b200 import _C
    tpg, ids, flat = _C.isect_regular_tiles(m2, radii, dep, W, H, 16, 16)
    off = _C.isect_offset_encode(ids, tile_width=(W + 15) // 16, tile_height=(H + 15) // 16)
    return tpg, ids, flat, off


@pytest.mark.parametrize("headroom", [1.0, 1.3])
def test_async_lists_equal_exact_lists(cuda, headroom):
    from xsimgs_b200 import _C
    sc, cam, W, H = _view(cuda)
    flags, radii, m2, dep = cam.ut_gs_projection(sc.means, sc.scales, sc.quats, W, H, opacity=sc.opacities)
    tpg, ids, flat, off = _exact(m2, radii, dep, W, H)
    n = ids.numel()
    assert n > 0
    cap = int(n * headroom)
    tpg2, ids2, flat2, off2, counts = _C.isect_regular_tiles_async(m2, radii, dep, W, H, 16, 16, capacity=cap)
    assert ids2.numel() == cap and flat2.numel() == cap
    assert counts.tolist() == [n, n]
    assert torch.equal(tpg2, tpg)
    assert torch.equal(ids2[:n], ids) and torch.equal(flat2[:n], flat)
    assert torch.equal(off2, off)


def test_async_overflow_reports_total(cuda):
    from xsimgs_b200 import _C
    sc, cam, W, H = _view(cuda)
    flags, radii, m2, dep = cam.ut_gs_projection(sc.means, sc.scales, sc.quats, W, H, opacity=sc.opacities)
    n = int(_C.isect_regular_tiles(m2, radii, dep, W, H, 16, 16)[1].numel())
    cap = n // 3
    _, ids2, flat2, off2, counts = _C.isect_regular_tiles_async(m2, radii, dep, W, H, 16, 16, capacity=cap)
    assert counts.tolist() == [n, cap]
    # what was written is sorted by (tile, depth) and indexes real Gaussians
    ids_np = ids2.cpu().numpy()
    assert (np.diff(ids_np) >= 0).all()
    f = flat2.cpu().numpy()
    assert f.min() >= 0 and f.max() < sc.n
    assert int(off2.max()) <= cap


def test_async_empty_view(cuda):
    from xsimgs_b200 import _C
    n = 1000
    m2 = torch.full((n, 2), -1e4, device=cuda)
    radii = torch.zeros(n, 2, device=cuda)
    dep = torch.ones(n, device=cuda)
    tpg, ids, flat, off, counts = _C.isect_regular_tiles_async(m2, radii, dep, 640, 480, 16, 16, capacity=64)
    assert counts.tolist() == [0, 0]
    assert int(tpg.abs().sum()) == 0
    assert off.shape == (30, 40) and int(off.abs().sum()) == 0


def _render(cuda, sc, cam, W, H, monkeypatch, sync):
    from xsimgs_b200 import scenes, ut_gs_render
    if sync:
        monkeypatch.setenv("XSIMGS_B200_SYNC_TILING", "1")
    else:
        monkeypatch.delenv("XSIMGS_B200_SYNC_TILING", raising=False)
    p = {k: v.detach().clone().requires_grad_(True) for k, v in
         dict(means=sc.means, scales=sc.scales, quats=sc.quats, opacities=sc.opacities).items()}
    colors = torch.rand(sc.n, 3, generator=torch.Generator().manual_seed(5)).to(cuda).requires_grad_(True)
    color, depth, alpha, _ = ut_gs_render(cam, p["means"], p["scales"], p["quats"], p["opacities"], W, H,
                                          colors=colors)
    ups = [t.to(cuda) for t in scenes.upstream_grads(H, W, 3)]
    torch.autograd.backward([color, depth, alpha], ups)
    return [color.detach(), depth.detach(), alpha.detach()], [p[k].grad for k in p] + [colors.grad]


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _same(imgs, grads, imgs_ref, grads_ref, spread):
    for a, b in zip(imgs, imgs_ref):
        assert torch.equal(a, b)
    names = ("means", "scales", "quats", "opacities", "colors")
    for name, a, b, s in zip(names, grads, grads_ref, spread):
        err = _rel(a, b)
        assert err <= max(8.0 * s, 1e-6), f"{name}: relative L2 {err} vs run-to-run {s}"


def test_render_async_equals_exact_and_recovers_from_overflow(cuda, monkeypatch):
    from xsimgs_b200.rendering import render as R
    sc, cam, W, H = _view(cuda)
    R._capacity.clear()
    imgs_ref, grads_ref = _render(cuda, sc, cam, W, H, monkeypatch, sync=True)
    # the backward's float atomics make gradients differ run to run: measure that spread
    _, grads_again = _render(cuda, sc, cam, W, H, monkeypatch, sync=True)
    spread = [_rel(a, b) for a, b in zip(grads_again, grads_ref)]
    print("run-to-run gradient spread", spread)
    assert not R._capacity
    # first render learns the capacity on the exact path, the second uses it
    for _ in range(2):
        imgs, grads = _render(cuda, sc, cam, W, H, monkeypatch, sync=False)
        assert len(R._capacity) == 1
        _same(imgs, grads, imgs_ref, grads_ref, spread)
    key, cap = next(iter(R._capacity.items()))
    # too small a capacity: the view is rendered again on exact lists
    R._capacity[key] = cap // 4
    imgs, grads = _render(cuda, sc, cam, W, H, monkeypatch, sync=False)
    _same(imgs, grads, imgs_ref, grads_ref, spread)
    assert R._capacity[key] >= cap
    R._capacity.clear()
