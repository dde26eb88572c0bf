from .ext_camera import (  # noqa: F401
    FusedRSCamera, PerspectiveCamera, FisheyeCamera, SphericalCamera, LidarCamera, DistortedPerspectiveCamera,
    max_valid_radius,
    look_at_quat, rotmat_to_quat, data_addr_tensor, cornering_values_from_pixel_values,
)
