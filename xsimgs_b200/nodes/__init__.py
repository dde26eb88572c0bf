"""Scene-assembly nodes around the render path (the reference's
src/xsimgs/nodes): SMPL skinning of articulated bodies into the scene's
Gaussian container, rigid per-instance transforms, instance masks and
keyframe-pose interpolation."""
from .smpl import (  # noqa: F401
    InterpolateSMPLPoses, SMPLLocalToGlobalPose, LBSSkinningSMPL, interpolate_smpl_poses,
    smpl_local_to_global_pose, smpl_lbs_skinning, valid_instances_indices,
)
from .container import RigidTransformAndPut, rigid_transform_and_put  # noqa: F401
