"""The multi-view SH backward split (used by the multi-GPU step) on the GPU:
the position gradient of a rank's own views and the coefficient gradient
summed over views, each against the oracle's per-view SH backward summed,
and the MultiViewSH autograd Function against per-view autograd."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_grads_close, to_np

pytestmark = pytest.mark.gpu


def _case(seed, n, degree, views, extra_bands=1):
    rng = np.random.default_rng(seed)
    k = (degree + 1) ** 2 + extra_bands
    return (rng.normal(size=(n, 3)).astype(np.float32) * 8, rng.normal(size=(n, k, 3)).astype(np.float32),
            rng.normal(size=(views, 3)).astype(np.float32), rng.normal(size=(views, n, 3)).astype(np.float32))


@pytest.mark.parametrize("degree", [0, 1, 3, 4])
def test_split_backward_matches_oracle_sum(cuda, degree):
    from xsimgs_b200 import _C
    pos, coeffs, origins, d_out = _case(degree, 5000, degree, views=3)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    ref_c = np.zeros_like(coeffs)
    ref_p = np.zeros_like(pos)
    for v in range(origins.shape[0]):
        dc, _, dp, _ = O.sh_bwd(degree, origins[v], pos, coeffs, d_out[v])
        ref_c += dc
        ref_p += dp
    d_pos = _C.spherical_harmonics_positions_bwd(degree, t(origins), t(pos), t(coeffs), t(d_out))
    d_coeffs = _C.spherical_harmonics_coeffs_bwd_multi(degree, t(origins), t(pos), t(d_out), coeffs.shape[1])
    np.testing.assert_allclose(to_np(d_coeffs), ref_c, atol=2e-5, rtol=1e-5)
    assert (to_np(d_coeffs)[:, (degree + 1) ** 2:] == 0).all()
    assert_grads_close(d_pos, ref_p, "d_positions", rtol=2e-4)


def test_multiview_sh_function_matches_per_view_autograd(cuda):
    import xsimgs_b200 as X
    from xsimgs_b200.multiview import multiview_colors
    pos, coeffs, origins, d_out = _case(11, 4000, 3, views=2, extra_bands=0)
    t = lambda a, g=False: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).requires_grad_(g)
    sh1, m1 = t(coeffs, True), t(pos, True)
    cols = multiview_colors(sh1, m1, t(origins), 3, 2)
    (cols * t(d_out)).sum().backward()
    sh2, m2 = t(coeffs, True), t(pos, True)
    loss = sum((X.spherical_harmonics_fused(sh2, m2, t(origins[v]), 3) * t(d_out[v])).sum() for v in range(2))
    loss.backward()
    np.testing.assert_allclose(to_np(cols[0]), to_np(X.spherical_harmonics_fused(sh2, m2, t(origins[0]), 3)),
                               atol=1e-6)
    np.testing.assert_allclose(to_np(sh1.grad), to_np(sh2.grad), atol=2e-5, rtol=1e-5)
    assert_grads_close(m1.grad, m2.grad, "means", rtol=2e-4)
