from .render import ut_gs_render, ut_gs_tiling  # noqa: F401
from .rasterize import ut_gs_rasterize, UTGSRasterize  # noqa: F401
from .rasterize_dynamic import ut_gs_dynamic_rasterize, UTGSDynamicRasterize  # noqa: F401
from .sh import (  # noqa: F401
    SphericalHarmonicsFused, spherical_harmonics_fused, sh_degree_to_bands,
    sh_degree_to_specular_dim, rgb_to_sh0, sh0_to_rgb,
)
