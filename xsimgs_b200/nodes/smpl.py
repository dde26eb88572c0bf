"""SMPL skinning with autograd, the reference's Python contract
(src/xsimgs/nodes/smpl.py:46-233): `smpl_local_to_global_pose` turns
per-joint local rotations into global joint transforms, and
`smpl_lbs_skinning` blends them into each body's Gaussians and writes the
result into the scene container at `global_offset`.

Shapes: N bodies ("objects") with V Gaussians each, B of them selected by
`local_q_ids` / `valid_ids`, K instances; quaternions are (w, x, y, z); id
tensors are 32-bit integers.
"""
from __future__ import annotations

import torch

from .._native import _C
from ..utils import apply_grad_mask


class InterpolateSMPLPoses(torch.autograd.Function):
    """Joint rotations of each body at `query_time`, slerped between its two
    bracketing keyframes (joint 0 taken from root_q[instance_ids]); gradients
    flow to the keyframe rotations, root_q and the query time
    (smpl.py:18-43)."""

    @staticmethod
    def forward(ctx, smpl_poses, smpl_poses_time, root_q, instance_ids, query_time):
        ctx.save_for_backward(smpl_poses, smpl_poses_time, root_q, instance_ids, query_time)
        return _C.interpolate_smpl_poses_fwd(smpl_poses, smpl_poses_time, root_q, instance_ids, query_time)

    @staticmethod
    def backward(ctx, grad_quat_out):
        smpl_poses, smpl_poses_time, root_q, instance_ids, query_time = ctx.saved_tensors
        d_poses, d_root, d_query = _C.interpolate_smpl_poses_bwd(smpl_poses, smpl_poses_time, root_q, instance_ids,
                                                                 query_time, grad_quat_out.contiguous())
        return apply_grad_mask(ctx, [d_poses, None, d_root, None, d_query])


class SMPLLocalToGlobalPose(torch.autograd.Function):
    """(local_q_ids [B], local_q [N,24,4], joints [N,24,3], a0_inv_q [N,24,4],
    a0_inv_t [N,24,3]) -> (global_q [B,24,4], global_t [B,24,3]); gradients
    flow to local_q and a0_inv_* (smpl.py:46-80)."""

    @staticmethod
    def forward(ctx, local_q_ids, local_q, joints, a0_inv_q, a0_inv_t):
        out_q, out_t = _C.smpl_local_to_global_fwd(local_q_ids, local_q, joints, a0_inv_q, a0_inv_t)
        ctx.save_for_backward(local_q_ids, local_q, joints, a0_inv_q, a0_inv_t, out_q, out_t)
        return out_q, out_t

    @staticmethod
    def backward(ctx, grad_q, grad_t):
        local_q_ids, local_q, joints, a0_inv_q, a0_inv_t, out_q, out_t = ctx.saved_tensors
        grad_q = torch.zeros_like(out_q) if grad_q is None else grad_q.contiguous()
        grad_t = torch.zeros_like(out_t) if grad_t is None else grad_t.contiguous()
        d_local_q, d_a0_q, d_a0_t = _C.smpl_local_to_global_bwd(local_q_ids, local_q, joints, a0_inv_q, a0_inv_t,
                                                                 out_q, out_t, grad_q, grad_t)
        return apply_grad_mask(ctx, [None, d_local_q, None, d_a0_q, d_a0_t])


class LBSSkinningSMPL(torch.autograd.Function):
    """Linear-blend skinning into the container (smpl.py:83-163).  The
    container tensors are written in place and returned; their incoming
    gradients pass through to them, as in the reference."""

    @staticmethod
    def forward(ctx, valid_ids, global_q, global_t, vertices, quats, weights, instance_ids, instance_t, instance_v,
                global_offset, out_positions, out_rotations, out_velocities, out_mask):
        _C.smpl_lbs_skinning(valid_ids, global_q, global_t, vertices, quats, weights, instance_ids, instance_t,
                             instance_v, global_offset, out_positions, out_rotations, out_velocities, out_mask)
        ctx.global_offset = global_offset
        ctx.num_instances = instance_t.shape[0]
        ctx.save_for_backward(valid_ids, instance_ids, global_q, global_t, vertices, quats, weights)
        ctx.mark_dirty(*[t for t in (out_positions, out_rotations, out_velocities, out_mask) if t is not None])
        return out_positions, out_rotations, out_velocities, out_mask

    @staticmethod
    def backward(ctx, v_positions, v_rotations, v_velocities, v_mask):
        valid_ids, instance_ids, global_q, global_t, vertices, quats, weights = ctx.saved_tensors
        v_positions = v_positions.contiguous()
        v_rotations = v_rotations.contiguous()
        v_velocities = v_velocities.contiguous() if v_velocities is not None else None
        (d_global_q, d_global_t, d_vertices, d_quats, d_weights, d_instance_v,
         d_instance_t) = _C.smpl_lbs_skinning_bwd(valid_ids, instance_ids, global_q, global_t, vertices, quats,
                                                  weights, ctx.global_offset, ctx.num_instances, v_positions,
                                                  v_rotations, v_velocities)
        return apply_grad_mask(ctx, (None, d_global_q, d_global_t, d_vertices, d_quats, d_weights, None,
                                     d_instance_t, d_instance_v, None, v_positions, v_rotations, v_velocities,
                                     None))


def smpl_lbs_skinning(valid_ids, global_q, global_t, vertices, quats, weights, instance_ids, instance_t, instance_v,
                      global_offset: int, out_positions, out_rotations, out_velocities=None, out_mask=None):
    """Skins B bodies into rows [global_offset + obj * V, ... + V) of the
    container; returns (out_positions, out_rotations, out_velocities,
    out_mask) (smpl.py:166-189)."""
    return LBSSkinningSMPL.apply(valid_ids.contiguous(), global_q.contiguous(), global_t.contiguous(),
                                 vertices.contiguous(), quats.contiguous(), weights.contiguous(),
                                 instance_ids.contiguous(), instance_t.contiguous(), instance_v.contiguous(),
                                 global_offset, out_positions, out_rotations, out_velocities, out_mask)


def smpl_local_to_global_pose(local_q_ids, local_q, joints, a0_inv_q, a0_inv_t):
    """(global_q [B,24,4], global_t [B,24,3]) of the bodies `local_q_ids`
    (smpl.py:192-203)."""
    return SMPLLocalToGlobalPose.apply(local_q_ids.contiguous(), local_q.contiguous(), joints.contiguous(),
                                       a0_inv_q.contiguous(), a0_inv_t.contiguous())


def valid_instances_indices(instance_ids: torch.Tensor, instance_mask: torch.Tensor) -> torch.Tensor:
    """Indices of the bodies whose instance is enabled in `instance_mask`
    (smpl.py:219-233): the compaction kernel for small contiguous inputs,
    else a torch gather."""
    if len(instance_ids) < 1024 and instance_ids.is_contiguous() and instance_mask.is_contiguous():
        return _C.smpl_ids_compaction(instance_ids, instance_mask)
    idxs = torch.arange(len(instance_ids), device=instance_ids.device)
    return idxs[instance_mask[instance_ids.long()]]


def interpolate_smpl_poses(smpl_poses, smpl_poses_time, root_q, instance_ids, query_time):
    """[N, 24, 4] joint rotations at query_time (smpl.py:206-216)."""
    return InterpolateSMPLPoses.apply(smpl_poses.contiguous(), smpl_poses_time.contiguous(), root_q.contiguous(),
                                      instance_ids.contiguous(), query_time)
