"""Shared helpers of the parity tests: run one view through the GPU ops and
through the CPU oracle on the same inputs, stage by stage."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O

SH_C0 = 0.28209479177387814

# Tolerances (the targets of this port):
#   images (colour, depth, alpha): max-abs 1e-4, except "ambiguous" pixels:
#     those where one of the compositing's threshold tests (alpha >= 1/255,
#     T (1 - alpha) <= 1e-4, the backward's opacity * vis <= 0.99 gate) came
#     within the float32 error band of that pair's alpha (computed by the
#     oracle from the pair's conditioning) — two float32 implementations,
#     including the reference's own CUDA, may decide those tests either way;
#     they must stay below 1 % of the pixels;
#   parameter gradients: computed from upstream gradients that are zero at
#     the ambiguous pixels (on both sides), then |gpu - ref| <= 1e-3 * |ref|
#     + 1e-3 * max|ref| per element and a relative L2 error below 1e-3 per
#     tensor;
#   integers (tile counts, ids, offsets): bit-exact on identical inputs.
IMG_ATOL = 1e-4
GRAD_RTOL = 1e-3
AMBIGUOUS_MAX_FRAC = 1e-2


def to_np(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t


def assert_images_close(gpu, ref, near, atol=IMG_ATOL, what="image"):
    gpu, ref = to_np(gpu), to_np(ref)
    near = to_np(near).astype(bool)
    assert near.mean() < AMBIGUOUS_MAX_FRAC, f"{what}: too many threshold-ambiguous pixels {near.mean()}"
    diff = np.abs(gpu - ref)
    if diff.ndim == 3:
        diff = diff.max(axis=-1)
    diff = np.where(near, 0.0, diff)
    worst = float(diff.max()) if diff.size else 0.0
    assert worst <= atol, f"{what}: max-abs {worst} > {atol} at {np.unravel_index(diff.argmax(), diff.shape)}"


def assert_grads_close(gpu, ref, what="grad", rtol=GRAD_RTOL, pixel_mask=None):
    """Per-element and relative-L2 check; `pixel_mask` [H, W] (True = compare)
    drops the threshold-ambiguous pixels from per-pixel gradient images."""
    gpu, ref = to_np(gpu).astype(np.float64), to_np(ref).astype(np.float64)
    if pixel_mask is not None:
        keep = to_np(pixel_mask).astype(bool)
        gpu, ref = gpu[keep], ref[keep]
    assert gpu.shape == ref.shape, f"{what}: shape {gpu.shape} vs {ref.shape}"
    scale = np.abs(ref).max() if ref.size else 0.0
    err = np.abs(gpu - ref)
    bound = rtol * np.abs(ref) + rtol * scale
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements off, worst err {err.max()} "
                           f"(scale {scale}) at {np.unravel_index(err.argmax(), err.shape)}")
    rel = np.linalg.norm(gpu - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel < rtol, f"{what}: relative L2 error {rel}"


def camera_inputs(spec, device):
    cam = spec.make(device)
    pack = to_np(cam.pack).reshape(-1)
    elev = to_np(cam.beam_v) if hasattr(cam, "beam_v") else None
    return cam, pack, elev


def sh_colors(sh, degree):
    """Band-0 colour (view independent) for degree-0 scenes."""
    assert degree == 0
    return sh[:, 0, :] * SH_C0 + 0.5


def zero_at(near, *images):
    """Copies of the upstream-gradient images with the ambiguous pixels
    (`near`, [H, W]) set to zero, so a threshold test decided differently
    there changes no gradient on either side."""
    keep = torch.from_numpy(~to_np(near).astype(bool))
    out = []
    for im in images:
        m = keep.to(im.device)
        out.append(im * (m[..., None] if im.dim() == 3 else m).to(im.dtype))
    return out
