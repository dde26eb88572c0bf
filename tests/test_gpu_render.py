"""End-to-end `ut_gs_render` (public API, autograd) vs the oracle pipeline on
C1, and size-independent properties of the full C2 workload on the GPU."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_grads_close, assert_images_close, camera_inputs, to_np

pytestmark = pytest.mark.gpu


def test_ut_gs_render_e2e_c1(cuda):
    from xsimgs_b200 import scenes, ut_gs_render, spherical_harmonics_fused
    sc = scenes.c1_scene()
    spec = scenes.c1_camera()
    cam, pack, _ = camera_inputs(spec, cuda)
    W, H = spec.width, spec.height
    p = {k: v.to(cuda).requires_grad_(True) for k, v in sc.params().items()}
    origin = torch.zeros(3, device=cuda)
    colors = spherical_harmonics_fused(p["sh"], p["means"], origin, 0)
    color, depth, alpha, meta = ut_gs_render(cam, p["means"], p["scales"], p["quats"], p["opacities"], W, H,
                                             colors=colors)
    vr, vd, va = (t.to(cuda) for t in scenes.upstream_grads(H, W, 3))
    loss = (color * vr).sum() + (depth * vd).sum() + (alpha * va).sum()
    loss.backward()

    # oracle pipeline on the same inputs
    flags, radii, m2, dep = O.projection_utgs("pinhole", pack, sc.means.numpy(), None, sc.scales.numpy(),
                                              sc.quats.numpy(), sc.opacities.numpy(), W, H)
    tpg, ids, flat = O.isect_regular(m2, radii, dep, W, H)
    off = O.isect_offset_encode(ids, 16, 16)
    ro, rd, _ = O.camera_rays("pinhole", pack, W, H)
    rcol = O.sh_fwd(0, np.zeros(3, np.float32), sc.means.numpy(), sc.sh.numpy())
    rrgb, rdep, ralpha, rlast, near = O.rasterize_fwd(sc.means.numpy(), sc.quats.numpy(), sc.scales.numpy(), rcol,
                                                      sc.opacities.numpy(), W, H, 16, 16, ro, rd, off, flat)
    assert_images_close(color, rrgb, near, what="rgb")
    assert_images_close(depth, rdep, near, atol=1e-4, what="depth")
    assert_images_close(alpha, ralpha, near, what="alpha")
    assert torch.isfinite(p["means"].grad).all()
    assert meta["radii"].shape == (sc.n, 2)


def test_c2_full_size_properties(cuda):
    """1M Gaussians at 1920x1080: tiling invariants hold at full size."""
    from xsimgs_b200 import _C, scenes
    sc = scenes.street_scene(1_000_000).to(cuda)
    spec = scenes.c2_camera()
    cam = spec.make(cuda)
    W, H = spec.width, spec.height
    flags, radii, m2, dep = cam.ut_gs_projection(sc.means, sc.scales, sc.quats, W, H, opacity=sc.opacities)
    tpg, ids, flat = _C.isect_regular_tiles(m2, radii, dep, W, H, 16, 16)
    n_isects = ids.numel()
    assert n_isects == int(tpg.sum())
    # sorted by (tile, depth bits) ascending
    ids_np = to_np(ids)
    assert (np.diff(ids_np) >= 0).all()
    # each Gaussian appears exactly tiles_per_gauss times
    counts = np.bincount(to_np(flat), minlength=sc.n)
    np.testing.assert_array_equal(counts, to_np(tpg))
    tw, th = (W + 15) // 16, (H + 15) // 16
    off = to_np(_C.isect_offset_encode(ids, tw, th)).reshape(-1)
    tiles = ids_np >> 32
    # offsets[t] = number of intersections with tile < t
    expect = np.searchsorted(tiles, np.arange(tw * th), side="left")
    np.testing.assert_array_equal(off, expect)
    # the unsorted emission is a permutation of the sorted one
    tpg2, ids2, flat2 = _C.isect_regular_tiles(m2, radii, dep, W, H, 16, 16, sort=False)
    order = np.lexsort((to_np(flat2), to_np(ids2)))
    np.testing.assert_array_equal(to_np(ids2)[order], ids_np)
