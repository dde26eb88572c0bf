"""Small helpers the reference takes from its `pytoast` dependency."""
from __future__ import annotations

import torch


def apply_grad_mask(ctx, grads):
    """Return `grads` with None where the matching forward input does not need
    a gradient (the role of toast.ops.ext.apply_grad_mask, used by the
    reference's autograd Functions, e.g. rendering/rasterize.py:72)."""
    needs = ctx.needs_input_grad
    out = []
    for i, g in enumerate(grads):
        out.append(g if (i < len(needs) and needs[i]) else None)
    return tuple(out)


def pack_bits(mask: torch.Tensor) -> torch.Tensor:
    """bool[N] -> packed uint32[ceil(N/32)] with bit i%32 of word i//32 = mask[i]
    (the packed-mask format of mask_radii_packed and the SH mask)."""
    n = mask.numel()
    words = (n + 31) // 32
    m = torch.zeros(words * 32, dtype=torch.int64, device=mask.device)
    m[:n] = mask.reshape(-1).to(torch.int64)
    w = (m.view(words, 32) << torch.arange(32, device=mask.device)).sum(dim=1)
    return w.to(torch.int32).view(torch.uint32) if hasattr(torch, "uint32") else w.to(torch.int32)
