"""Generates tests/golden/c1_small.npz: the CPU oracle's outputs on a small
seeded C1-style scene (2000 Gaussians, 64x64 pinhole), stage by stage.

The reference cannot be built or run here, so these are regression fixtures
of the oracle itself (they pin the oracle against unintended change), not
reference outputs.  Regenerate with `python -m tests.golden.make_golden`.
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "c1_small.npz")


def compute():
    from oracle import oracle as O
    from xsimgs_b200 import scenes

    sc = scenes.c1_scene(n=2000, seed=3)
    W = H = 64
    pack = np.zeros(22, np.float32)
    pack[0] = 1.0
    pack[18:22] = [1.0, 1.0, 0.5, 0.5]
    m, q, s, o = (t.numpy() for t in (sc.means, sc.quats, sc.scales, sc.opacities))
    cols = (sc.sh[:, 0, :].numpy() * 0.28209479177387814 + 0.5).astype(np.float32)
    flags, radii, m2, dep = O.projection_utgs("pinhole", pack, m, None, s, q, o, W, H)
    tpg, ids, flat = O.isect_regular(m2, radii, dep, W, H, 16, 16)
    off = O.isect_offset_encode(ids, 4, 4)
    ro, rd, _ = O.camera_rays("pinhole", pack, W, H)
    rgb, depth, alpha, last, near = O.rasterize_fwd(m, q, s, cols, o, W, H, 16, 16, ro, rd, off, flat)
    rng = np.random.default_rng(7)
    vr = rng.normal(size=(H, W, 3)).astype(np.float32)
    vd = rng.normal(size=(H, W)).astype(np.float32)
    va = rng.normal(size=(H, W)).astype(np.float32)
    g = O.rasterize_bwd(m, q, s, cols, o, W, H, 16, 16, ro, rd, off, flat, alpha, last, vr, vd, va)
    return dict(flags=flags, radii=radii, means2d=m2, depths=dep, tiles_per_gauss=tpg, isect_ids=ids,
                flatten_ids=flat, offsets=off, ray_d=rd, rgb=rgb, depth=depth, alpha=alpha, last_ids=last,
                v_means=g["v_means"], v_quats=g["v_quats"], v_scales=g["v_scales"],
                v_opacities=g["v_opacities"], v_colors=g["v_colors"])


if __name__ == "__main__":
    np.savez_compressed(OUT, **compute())
    print(OUT, os.path.getsize(OUT), "bytes")
