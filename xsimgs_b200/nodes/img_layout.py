"""Float RGB images to 8-bit layouts for display / encoding: the reference's
src/xsimgs/nodes/img_layout.py:1-47.  CUDA images go through the
`_C.image_to_*_byte` kernels (each channel (uint8)(saturate(x) * 255));
images in host memory are converted with torch on the host, as the
reference does for them."""
import torch

from .._native import _C


def _check_image(image: torch.Tensor):
    assert image.ndim == 3, "Image must be [H, W, 3] tensor"
    assert image.shape[-1] == 3, "Image must be [H, W, 3] tensor"
    assert image.dtype == torch.float32, "Image must be float32 tensor"


def image_to_chw_rgb_byte(image: torch.Tensor) -> torch.Tensor:
    """[H, W, 3] float32 -> [3, H, W] uint8."""
    _check_image(image)
    if image.is_cpu:
        return image.permute(2, 0, 1).clamp(0, 1).mul(255.0).byte()
    return _C.image_to_chw_rgb_byte(image.contiguous())


def image_to_hwc_rgb_byte(image: torch.Tensor) -> torch.Tensor:
    """[H, W, 3] float32 -> [H, W, 3] uint8."""
    _check_image(image)
    if image.is_cpu:
        return image.clamp(0, 1).mul(255.0).byte()
    return _C.image_to_hwc_rgb_byte(image.contiguous())


def image_to_hwc_rgba_byte(image: torch.Tensor) -> torch.Tensor:
    """[H, W, 3] float32 -> [H, W, 4] uint8, alpha 255."""
    _check_image(image)
    if image.is_cpu:
        rgb = image.clamp(0, 1).mul(255.0).byte()
        return torch.cat([rgb, torch.full((*rgb.shape[:2], 1), 255, dtype=torch.uint8)], dim=-1)
    return _C.image_to_hwc_rgba_byte(image.contiguous())
