"""Rigid per-instance transforms of Gaussians into the scene container, with
autograd: the reference's Python contract (src/xsimgs/nodes/container.py:13-137).

Each Gaussian p of an enabled instance k = instance_id[p] is written at row
buffer_offset + p (or buffer_offset + per_instance_offsets[k] +
gs_inst_offsets[p]) as position R(q_k) x_p + t_k, rotation q_k (x) r_p and
velocity v_k + w_k x R(q_k) x_p (quaternions w, x, y, z).
"""
from __future__ import annotations

import torch

from .._native import _C
from ..utils import apply_grad_mask

packed_mask_from_instances = _C.packed_mask_from_instances


class RigidTransformAndPut(torch.autograd.Function):
    @staticmethod
    def forward(ctx, positions, rotations, instance_id, inst_q, inst_t, inst_v, inst_w, inst_mask,
                out_positions, out_rotation, out_velocity, out_mask, buffer_offset: int, per_instance_offsets,
                gs_inst_offsets):
        _C.copy_gs_rigid_transform_fwd(positions, rotations, instance_id, inst_q, inst_t, inst_v, inst_w, inst_mask,
                                       out_positions, out_rotation, out_velocity, out_mask, buffer_offset,
                                       per_instance_offsets, gs_inst_offsets)
        ctx.buffer_offset = buffer_offset
        ctx.save_for_backward(positions, rotations, instance_id, inst_q, inst_w, inst_mask, per_instance_offsets,
                              gs_inst_offsets)
        # out_mask is written in place too but, as in the reference, not returned
        ctx.mark_dirty(*[t for t in (out_positions, out_rotation, out_velocity) if t is not None])
        return out_positions, out_rotation, out_velocity

    @staticmethod
    def backward(ctx, v_positions, v_rotation, v_velocity):
        (positions, rotations, instance_id, inst_q, inst_w, inst_mask, per_instance_offsets,
         gs_inst_offsets) = ctx.saved_tensors
        v_positions = v_positions.contiguous()
        v_rotation = v_rotation.contiguous()
        v_velocity = v_velocity.contiguous() if v_velocity is not None else None
        gp, gr, gq, gt, gv, gw = _C.copy_gs_rigid_transform_bwd(
            positions, rotations, instance_id, inst_q, inst_w, inst_mask, ctx.buffer_offset, per_instance_offsets,
            gs_inst_offsets, v_positions, v_rotation, v_velocity)
        return apply_grad_mask(ctx, (gp, gr, None, gq, gt, gv, gw, None, v_positions, v_rotation, v_velocity, None,
                                     None, None, None))


def rigid_transform_and_put(positions, rotations, instance_id, inst_q, inst_t, inst_v, inst_w, inst_mask,
                            out_positions=None, out_rotation=None, out_velocity=None, out_mask=None,
                            buffer_offset: int = 0, per_instance_offsets=None, gs_inst_offsets=None):
    """Returns (out_positions, out_rotation, out_velocity, out_mask); missing
    outputs are allocated as zeros of the input's size (container.py:84-137)."""
    if out_positions is None:
        out_positions = torch.zeros_like(positions.detach())
    if out_rotation is None:
        out_rotation = torch.zeros_like(rotations.detach())
    if out_velocity is None:
        out_velocity = torch.zeros_like(positions.detach())
    if out_mask is None:
        out_mask = torch.zeros_like(positions.detach()[..., 0], dtype=torch.bool)
    out_positions, out_rotation, out_velocity = RigidTransformAndPut.apply(
        positions, rotations, instance_id, inst_q, inst_t, inst_v, inst_w, inst_mask, out_positions, out_rotation,
        out_velocity, out_mask, buffer_offset, per_instance_offsets, gs_inst_offsets)
    return out_positions, out_rotation, out_velocity, out_mask
