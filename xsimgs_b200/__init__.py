"""xsimgs_b200 — B200-native (sm_100a) Gaussian sensor rendering behind the
xsimgs operator surface.

Drop-in for the reference's render path: `xsimgs_b200._C` carries the same op
names as `xsimgs._C`, and `ut_gs_render` / `ut_gs_tiling` /
`spherical_harmonics_fused` / the camera classes keep the reference's Python
API.  Importing the package loads the in-tree CUDA extension and fails loudly
if it has not been built.
"""
from ._native import _C  # noqa: F401
from .rendering import (  # noqa: F401
    ut_gs_render, ut_gs_tiling, ut_gs_rasterize, ut_gs_dynamic_rasterize,
    spherical_harmonics_fused, rgb_to_sh0, sh0_to_rgb, sh_degree_to_bands,
)
from . import cameras  # noqa: F401

__version__ = "0.1.0"
