"""Scene-assembly nodes around the render path (the reference's
src/xsimgs/nodes): SMPL skinning of articulated bodies into the scene's
Gaussian container."""
from .smpl import (  # noqa: F401
    SMPLLocalToGlobalPose, LBSSkinningSMPL, smpl_local_to_global_pose, smpl_lbs_skinning,
    valid_instances_indices,
)
