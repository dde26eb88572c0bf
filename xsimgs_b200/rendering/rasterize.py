"""Autograd wrapper of the static compositing ops.

Mirrors the reference's UTGSRasterize (src/xsimgs/rendering/rasterize.py:6-100):
same forward inputs, saved tensors and gradient order.
"""
import torch

from .._native import _C
from ..utils import apply_grad_mask


class UTGSRasterize(torch.autograd.Function):
    @staticmethod
    def forward(ctx, positions, rotation, scale, density, colors, ray_o, ray_d,
                isect_offsets, flatten_ids, tile_size_x: int, tile_size_y: int, n_isects=None):
        height, width = ray_o.shape[:2]
        channels = colors.shape[-1] if colors is not None else 0
        ws = torch.empty(_C.rasterize_workspace_size(positions.shape[0], channels, n_isects=flatten_ids.numel(),
                                                     n_tiles=isect_offsets.numel(),
                                                     tile_pixels=tile_size_x * tile_size_y), dtype=torch.uint8,
                         device=positions.device)
        out_rgb, out_depth, out_alpha, last_ids = _C.rasterize_eval3d_fwd(
            means=positions,
            quats=rotation,
            scales=scale,
            opacities=density.view(1, -1),
            colors=colors.unsqueeze(0) if colors is not None else None,
            ray_origs=ray_o,
            ray_dirs=ray_d,
            image_width=width,
            image_height=height,
            tile_size_width=tile_size_x,
            tile_size_height=tile_size_y,
            tile_offsets=isect_offsets,
            flatten_ids=flatten_ids,
            workspace=ws,
            n_isects=n_isects,
        )
        # the backward reuses the forward's packed records and tile order
        ctx.workspace = ws
        ctx.n_isects = n_isects
        ctx.tile_size_x = tile_size_x
        ctx.tile_size_y = tile_size_y
        ctx.save_for_backward(positions, rotation, scale, density, colors, ray_o, ray_d,
                              isect_offsets, flatten_ids, out_alpha, last_ids)
        return out_rgb, out_depth, out_alpha

    @staticmethod
    def backward(ctx, grad_rgb, grad_depth, grad_alpha):
        (positions, rotation, scale, density, colors, ray_o, ray_d,
         isect_offsets, flatten_ids, out_alpha, last_ids) = ctx.saved_tensors
        # v_points, v_quat, v_scale, v_opacity, v_colors, v_ray_o, v_ray_d; the
        # per-pixel ray gradients are computed only when a ray needs them
        grads = _C.rasterize_eval3d_bwd(
            positions, scale, rotation, density, colors, ray_o, ray_d,
            ctx.tile_size_x, ctx.tile_size_y, isect_offsets, flatten_ids,
            out_alpha, last_ids,
            grad_rgb.contiguous() if grad_rgb is not None else None,
            grad_depth.contiguous(),
            grad_alpha.contiguous(),
            forward_workspace=ctx.workspace,
            n_isects=ctx.n_isects,
            ray_grads=bool(ctx.needs_input_grad[5] or ctx.needs_input_grad[6]),
        )
        return apply_grad_mask(ctx, list(grads) + [None, None, None, None, None])


def ut_gs_rasterize(positions, rotation, scale, density, colors, ray_o, ray_d,
                    isect_offsets, flatten_ids, tile_size_x: int, tile_size_y: int, n_isects=None):
    """`n_isects` (not in the reference): an int64 device tensor holding the
    length of a capacity-sized `flatten_ids` (isect_regular_tiles_async)."""
    return UTGSRasterize.apply(positions, rotation, scale, density, colors, ray_o, ray_d,
                               isect_offsets, flatten_ids, tile_size_x, tile_size_y, n_isects)
