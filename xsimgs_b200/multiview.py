"""Multi-GPU host logic of the render path: one process per GPU, each
rendering its share of the sensor views against a full replica of the
Gaussians, then one exchange — the sum of the per-Gaussian gradients over
ranks (NCCL all-reduce on NVLink / NVSwitch; gloo on CPU for tests).

With NCCL no kernel of this package touches another GPU's memory; the
alternative exchange in exchange.py does it with its own NVSwitch kernels.
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


def exchanged_leaves(names: Iterable[str], multiview_sh: bool) -> list[str]:
    """The leaves whose gradients a step sums over ranks, in the order the
    backward finishes them: the compositing's (quats, scales, opacities),
    then means, then the SH coefficients and any other leaf (skinning
    parameters ...).  With the multi-view SH exchange (MultiViewSH) the SH
    gradient comes out of the backward already summed over ranks and is not
    exchanged again."""
    names = list(names)
    order = [k for k in ("quats", "scales", "opacities", "means") if k in names]
    order += [k for k in names if k not in order and not (multiview_sh and k == "sh")]
    return order


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
    after backward().  It returns the number of collectives issued (one per
    bucket).

    `gated=True` holds every all-reduce of a pass until `open_gate()` is
    called (MultiViewSH.backward calls it right after issuing its
    all-gathers on the same group), so that every rank issues its
    collectives in the same order whatever order autograd runs the ready
    nodes in: the view exchange first, then the all-reduces in leaf order.
    A rank whose graphs differ from its peers' (other view counts) could
    otherwise interleave the two kinds differently and mismatch the
    collectives."""

    def __init__(self, leaves: Iterable[torch.Tensor], group=None, gated: bool = False,
                 buckets: Sequence[int] | None = None):
        self.leaves = list(leaves)
        self.group = group
        self.gated = gated
        # consecutive leaves that get ready together can share one
        # collective: `buckets` gives the group sizes in leaf order
        sizes = list(buckets) if buckets is not None else [1] * len(self.leaves)
        if sum(sizes) != len(self.leaves) or min(sizes, default=1) < 1:
            raise ValueError("buckets must split the leaves into consecutive non-empty groups")
        self.bucket_of, self.bucket_leaves = [], []
        k = 0
        for b, n in enumerate(sizes):
            self.bucket_leaves.append(list(range(k, k + n)))
            self.bucket_of += [b] * n
            k += n
        self.enabled = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
        self.handles = []
        self._reset()
        if self.enabled:
            for i, t in enumerate(self.leaves):
                self.handles.append(t.register_post_accumulate_grad_hook(self._make_hook(i)))

    def _reset(self):
        self.ready = [False] * len(self.leaves)
        self.next = 0  # next bucket to issue
        self.works = []
        self.unpack = []
        self.gate_open = not self.gated

    def open_gate(self):
        """Lets the pass's all-reduces go (issuing those already ready)."""
        self.gate_open = True
        self._flush()

    def _make_hook(self, i):
        def hook(_t):
            self.ready[i] = True
            self._flush()
        return hook

    def _issue(self, b):
        idx = self.bucket_leaves[b]
        for i in idx:
            t = self.leaves[i]
            if t.grad is None:
                t.grad = torch.zeros_like(t)
        if len(idx) == 1:
            self.works.append(dist.all_reduce(self.leaves[idx[0]].grad, group=self.group, async_op=True))
            return
        # one flat buffer per bucket; after the collective each leaf's
        # gradient becomes a view of it
        flat = torch.cat([self.leaves[i].grad.reshape(-1) for i in idx])
        self.works.append(dist.all_reduce(flat, group=self.group, async_op=True))
        self.unpack.append((flat, idx))

    def _bucket_ready(self, b):
        return all(self.ready[i] for i in self.bucket_leaves[b])

    def _flush(self):
        if not self.gate_open:
            return
        while self.next < len(self.bucket_leaves) and self._bucket_ready(self.next):
            self._issue(self.next)
            self.next += 1

    def wait(self) -> int:
        """Issues the remaining collectives, waits for all of the pass;
        returns how many were issued."""
        if not self.enabled:
            return 0
        self.gate_open = True
        while self.next < len(self.bucket_leaves):
            self._issue(self.next)
            self.next += 1
        n = len(self.works)
        for w in self.works:
            w.wait()
        for flat, idx in self.unpack:
            off = 0
            for i in idx:
                t = self.leaves[i]
                t.grad = flat[off:off + t.numel()].view_as(t)
                off += t.numel()
        timeline.mark("exchange_end")
        self._reset()
        return n

    def remove(self):
        for h in self.handles:
            h.remove()
        self.handles = []


class MultiViewSH(torch.autograd.Function):
    """Colours of one Gaussian set seen from each of this rank's views, with a
    backward that exchanges colour gradients instead of SH-coefficient
    gradients.

    forward(sh [N, K, 3], means [N, 3], origins [k, 3]) -> colours [k, N, 3]
    (one spherical_harmonics_fused per view).  The coefficient gradient summed
    over every view of every rank is sum_j Y(dir_j) (x) dcolour_j, so the
    backward all-gathers the k colour gradients [N, 3] and origins of every
    rank (3 floats per Gaussian and view, instead of an all-reduce of
    3 x (deg+1)^2 floats per Gaussian) and rebuilds that sum locally; the
    returned `sh` gradient is therefore already the sum over ranks and must
    not be all-reduced again.  The `means` gradient covers this rank's views
    only (sum it over ranks with the other geometry gradients).

    Every rank of `group` must call it with the same k_max >= its own k
    (ranks pad to k_max), and with at least one view, in the same order
    relative to its other collectives on `group`.  Either give it a group of
    its own (its all-gathers then run beside the gradient all-reduces, each
    group in one order on every rank), or share the all-reduces' group and
    pass the step's GradientAllReduce (built with gated=True) as `reducer`:
    its all-reduces are then released only after the all-gathers are issued.
    Coefficients [N, K, 3] with band 0 included; no mask."""

    @staticmethod
    def forward(ctx, sh, means, origins, degree: int, k_max: int, group=None, reducer=None, exchange=None):
        from ._native import _C
        cols = torch.stack([_C.spherical_harmonics_fused_fwd(degree, origins[v].contiguous(), means, sh, None, False)
                            for v in range(origins.shape[0])])
        ctx.degree, ctx.k_max, ctx.group, ctx.reducer, ctx.exchange = degree, k_max, group, reducer, exchange
        ctx.save_for_backward(sh, means, origins)
        return cols

    @staticmethod
    def backward(ctx, d_cols):
        from ._native import _C
        sh, means, origins = ctx.saved_tensors
        d_cols = d_cols.contiguous()
        k, n = origins.shape[0], means.shape[0]
        if ctx.exchange is not None:
            return MultiViewSH._backward_nvls(ctx, sh, means, origins, d_cols)
        distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size(ctx.group) > 1
        if distributed:
            world = dist.get_world_size(ctx.group)
            kmax = ctx.k_max
            pad_d = torch.zeros(kmax, n, 3, device=d_cols.device, dtype=d_cols.dtype)
            pad_d[:k] = d_cols
            # padded views carry zero gradient from a real origin (finite basis)
            pad_o = origins[:1].expand(kmax, 3).clone()
            pad_o[:k] = origins
            all_d = torch.empty(world * kmax, n, 3, device=d_cols.device, dtype=d_cols.dtype)
            all_o = torch.empty(world * kmax, 3, device=d_cols.device, dtype=d_cols.dtype)
            w_d = dist.all_gather_into_tensor(all_d, pad_d, group=ctx.group, async_op=True)
            w_o = dist.all_gather_into_tensor(all_o, pad_o, group=ctx.group, async_op=True)
        else:
            all_d, all_o = d_cols, origins
        if ctx.reducer is not None:
            ctx.reducer.open_gate()
        timeline.mark("sh_bwd_start")
        d_means = _C.spherical_harmonics_positions_bwd(ctx.degree, origins, means, sh, d_cols)
        if distributed:
            w_d.wait()
            w_o.wait()
        timeline.mark("sh_gathered")
        d_sh = _C.spherical_harmonics_coeffs_bwd_multi(ctx.degree, all_o, means, all_d, sh.shape[1])
        timeline.mark("sh_bwd_end")
        return d_sh, d_means, None, None, None, None, None, None

    @staticmethod
    def _backward_nvls(ctx, sh, means, origins, d_cols):
        """The same with the view exchange on this package's NVSwitch kernels
        (exchange.NvlsExchange.all_gather) on the compute stream."""
        from ._native import _C
        ex = ctx.exchange
        k, n, kmax = origins.shape[0], means.shape[0], ctx.k_max
        timeline.mark("sh_bwd_start")
        d_means = _C.spherical_harmonics_positions_bwd(ctx.degree, origins, means, sh, d_cols)
        if k < kmax:
            pad_d = torch.zeros(kmax, n, 3, device=d_cols.device, dtype=d_cols.dtype)
            pad_d[:k] = d_cols
            pad_o = origins[:1].expand(kmax, 3).clone()
            pad_o[:k] = origins
        else:
            pad_d, pad_o = d_cols, origins
        if ex.defer_views:
            # the step's NvlsGradientSum gathers these with its all-reduce and
            # adds the rebuilt SH gradient to the SH leaf after backward
            ex.pending_views = {"d": pad_d, "o": pad_o, "means": means, "degree": ctx.degree, "k_max": kmax,
                                "K": sh.shape[1]}
            return None, d_means, None, None, None, None, None, None
        all_d, all_o = ex.all_gather(pad_d, pad_o)
        all_d = all_d.reshape(ex.world * kmax, n, 3)
        all_o = all_o.reshape(ex.world * kmax, 3)
        timeline.mark("sh_gathered")
        d_sh = _C.spherical_harmonics_coeffs_bwd_multi(ctx.degree, all_o.contiguous(), means, all_d.contiguous(),
                                                       sh.shape[1])
        timeline.mark("sh_bwd_end")
        return d_sh, d_means, None, None, None, None, None, None


def multiview_colors(sh, means, origins, degree: int, k_max: int, group=None, reducer=None, exchange=None):
    """[k, N, 3] colours of this rank's k views (see MultiViewSH); with
    `exchange` (an exchange.NvlsExchange made for k_max * N * 3 and
    k_max * 3 gathered floats) the backward gathers the views over NVSwitch
    with this package's kernels instead of NCCL."""
    return MultiViewSH.apply(sh.contiguous(), means.contiguous(), origins.contiguous(), degree, k_max, group,
                             reducer, exchange)


class Timeline:
    """Optional named CUDA events on the current stream, for per-phase step
    timing (off unless enabled; marks cost one event record each)."""

    def __init__(self):
        self.enabled = False
        self.events: list[tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.events.append((name, e))

    def take(self) -> list[tuple[str, torch.cuda.Event]]:
        ev, self.events = self.events, []
        return ev


timeline = Timeline()
