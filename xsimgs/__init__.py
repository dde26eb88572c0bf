"""The reference's import path, served by xsimgs_b200.

Code written against the reference imports `xsimgs` (`from xsimgs._C import
rasterize_eval3d_fwd`, `from xsimgs.rendering import ut_gs_render`,
`xsimgs.cameras.ext.PerspectiveCamera`, `xsimgs.nodes.smpl_lbs_skinning`,
...; src/xsimgs/rendering/rasterize.py:4, src/xsimgs/rendering/sh.py:3-6,
src/xsimgs/rendering/render.py:3).  This package registers those module
names as aliases of the B200 implementation, so such code runs unchanged:
`xsimgs._C` IS `xsimgs_b200._C` (the same extension object), and the
Python modules are the same module objects under both names.

The reference's camera modules live in one file here
(xsimgs_b200/cameras/ext_camera.py), so `xsimgs.cameras.ext.perspective`,
`.fisheye`, `.lidar`, ... all name that module.  Out-of-scope parts of the
reference (MCMC noise, box / voxel structures) have no alias.
"""
import importlib
import sys

import xsimgs_b200 as _impl

_ALIASES = {
    "xsimgs._C": "xsimgs_b200._C",
    "xsimgs.rendering": "xsimgs_b200.rendering",
    "xsimgs.rendering.render": "xsimgs_b200.rendering.render",
    "xsimgs.rendering.rasterize": "xsimgs_b200.rendering.rasterize",
    "xsimgs.rendering.rasterize_dynamic": "xsimgs_b200.rendering.rasterize_dynamic",
    "xsimgs.rendering.sh": "xsimgs_b200.rendering.sh",
    "xsimgs.cameras": "xsimgs_b200.cameras",
    "xsimgs.cameras.ext": "xsimgs_b200.cameras",
    "xsimgs.cameras.ext.ext_camera": "xsimgs_b200.cameras.ext_camera",
    "xsimgs.cameras.ext.perspective": "xsimgs_b200.cameras.ext_camera",
    "xsimgs.cameras.ext.distorted_perspective": "xsimgs_b200.cameras.ext_camera",
    "xsimgs.cameras.ext.fisheye": "xsimgs_b200.cameras.ext_camera",
    "xsimgs.cameras.ext.spherical": "xsimgs_b200.cameras.ext_camera",
    "xsimgs.cameras.ext.lidar": "xsimgs_b200.cameras.ext_camera",
    "xsimgs.nodes": "xsimgs_b200.nodes",
    "xsimgs.nodes.container": "xsimgs_b200.nodes.container",
    "xsimgs.nodes.img_layout": "xsimgs_b200.nodes.img_layout",
    "xsimgs.nodes.smpl": "xsimgs_b200.nodes.smpl",
}

for _name, _target in _ALIASES.items():
    sys.modules[_name] = importlib.import_module(_target)

_C = sys.modules["xsimgs._C"]
rendering = sys.modules["xsimgs.rendering"]
cameras = sys.modules["xsimgs.cameras"]
nodes = sys.modules["xsimgs.nodes"]
__version__ = _impl.__version__
