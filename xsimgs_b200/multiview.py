"""Multi-GPU host logic of the render path: one process per GPU, each
rendering its share of the sensor views against a full replica of the
Gaussians, then one exchange — the sum of the per-Gaussian gradients over
ranks (NCCL all-reduce on NVLink / NVSwitch; gloo on CPU for tests).

No kernel reads another GPU's memory: the only remote data is what the
collective delivers into local buffers.
"""
from __future__ import annotations

from typing import Iterable, Sequence

import torch
import torch.distributed as dist


def assign_views(costs: Sequence[float], world: int) -> list[list[int]]:
    """Views -> ranks, balancing the summed cost (greedy longest first, ties
    to the lowest rank; deterministic, so every rank computes the same
    assignment).  A rank may get no view when there are fewer views than
    ranks."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    load = [0.0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += float(costs[i])
    for v in out:
        v.sort()
    return out


class GradientAllReduce:
    """Sums the gradients of `leaves` over the ranks of `group`, one
    asynchronous all-reduce per leaf, always issued in the order of `leaves`
    (so every rank issues the same collectives in the same order).

    A leaf's collective is issued as soon as autograd has accumulated its
    gradient for the current backward pass and all leaves before it are
    issued: list the leaves in the order backward finishes them (for the
    render step: rotations, scales, opacities — done by the compositing
    backward — then means and SH, done after the SH backward) and the
    exchange of the first ones overlaps the rest of the backward.

    Run one backward() per pass (sum the losses of all of a rank's views
    first): a second backward in the same pass would add to gradients whose
    collectives were already issued.

    `wait()` issues whatever is left — with a zero gradient for a leaf this
    rank never touched in the pass (a rank without views) — and blocks the
    current stream on all collectives of the pass; call it once per pass,
    after backward()."""

    def __init__(self, leaves: Iterable[torch.Tensor], group=None):
        self.leaves = list(leaves)
        self.group = group
        self.enabled = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
        self.handles = []
        self._reset()
        if self.enabled:
            for i, t in enumerate(self.leaves):
                self.handles.append(t.register_post_accumulate_grad_hook(self._make_hook(i)))

    def _reset(self):
        self.ready = [False] * len(self.leaves)
        self.next = 0
        self.works = []

    def _make_hook(self, i):
        def hook(_t):
            self.ready[i] = True
            self._flush()
        return hook

    def _issue(self, i):
        t = self.leaves[i]
        if t.grad is None:
            t.grad = torch.zeros_like(t)
        self.works.append(dist.all_reduce(t.grad, group=self.group, async_op=True))

    def _flush(self):
        while self.next < len(self.leaves) and self.ready[self.next]:
            self._issue(self.next)
            self.next += 1

    def wait(self) -> int:
        """Issues the remaining collectives, waits for all of the pass;
        returns how many were issued."""
        if not self.enabled:
            return 0
        while self.next < len(self.leaves):
            self._issue(self.next)
            self.next += 1
        n = len(self.works)
        for w in self.works:
            w.wait()
        self._reset()
        return n

    def remove(self):
        for h in self.handles:
            h.remove()
        self.handles = []
