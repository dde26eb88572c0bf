"""Spherical-harmonics colour with autograd; mirrors the reference's
SphericalHarmonicsFused and helpers (src/xsimgs/rendering/sh.py:11-71)."""
import torch

from .._native import _C
from ..utils import apply_grad_mask


class SphericalHarmonicsFused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, coeffs, positions, origin, degree_to_use: int, mask=None,
                layout_3kn: bool = False, coeffs_dc=None):
        ctx.layout_3kn = layout_3kn
        ctx.degree_to_use = degree_to_use
        ctx.save_for_backward(origin, positions, coeffs, mask, coeffs_dc)
        return _C.spherical_harmonics_fused_fwd(
            degree_to_use, origin, positions, coeffs, mask, layout_3kn, coeffs_dc)

    @staticmethod
    def backward(ctx, grad_out):
        origin, positions, coeffs, mask, coeffs_dc = ctx.saved_tensors
        d_coeffs, d_coeffs_dc, d_positions, d_origin = _C.spherical_harmonics_fused_bwd(
            ctx.degree_to_use, origin, positions, coeffs, mask, ctx.layout_3kn,
            grad_out.contiguous(), coeffs_dc)
        # order of the forward inputs:
        # coeffs, positions, origin, degree_to_use, mask, layout_3kn, coeffs_dc
        grads = (d_coeffs, d_positions, d_origin, None, None, None, d_coeffs_dc)
        return apply_grad_mask(ctx, grads)


def spherical_harmonics_fused(coeffs, positions, origin, degree_to_use: int, mask=None,
                              layout_3kn: bool = False, coeffs_dc=None):
    return SphericalHarmonicsFused.apply(coeffs, positions, origin, degree_to_use, mask,
                                         layout_3kn, coeffs_dc)


def sh_degree_to_bands(degree: int):
    return (degree + 1) ** 2


def sh_degree_to_specular_dim(degree: int):
    """Number of dimensions used by SH of deg [1...degree], inclusive"""
    return 3 * (sh_degree_to_bands(degree) - 1)


SH_C0 = 0.28209479177387814


def rgb_to_sh0(rgb: torch.Tensor) -> torch.Tensor:
    return (rgb - 0.5) / SH_C0


def sh0_to_rgb(sh: torch.Tensor) -> torch.Tensor:
    return sh * SH_C0 + 0.5
