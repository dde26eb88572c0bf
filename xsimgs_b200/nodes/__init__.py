"""Scene-assembly nodes around the render path (the reference's
src/xsimgs/nodes): SMPL skinning of articulated bodies into the scene's
Gaussian container, rigid per-instance transforms, instance masks,
keyframe-pose interpolation and image byte layouts."""
from .smpl import (  # noqa: F401
    InterpolateSMPLPoses, SMPLLocalToGlobalPose, LBSSkinningSMPL, interpolate_smpl_poses,
    smpl_local_to_global_pose, smpl_lbs_skinning, valid_instances_indices,
)
from .container import RigidTransformAndPut, rigid_transform_and_put, packed_mask_from_instances  # noqa: F401
from .img_layout import image_to_chw_rgb_byte, image_to_hwc_rgb_byte, image_to_hwc_rgba_byte  # noqa: F401
