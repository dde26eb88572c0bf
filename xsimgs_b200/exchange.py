"""Gradient exchange of the sensor-sharded render step with this package's
own NVLink / NVSwitch kernels (csrc/exchange.cu) instead of NCCL.

The exchange buffers are symmetric (torch's symmetric memory allocates the
same buffer on every rank of the group and maps all copies behind one
NVSwitch multicast address).  The kernels run on the compute stream:

  * `all_reduce_(tensors)`: the tensors are packed into the reduce buffer,
    every rank sums its 1/world slice over all copies with one in-switch
    read-reduce (`multimem.ld_reduce`) and writes the sum to every copy
    (`multimem.st`), and the sums are unpacked back into the tensors — each
    rank's link carries its slice once each way, and no SM time goes to
    adding;
  * `all_gather(d, o)`: every rank writes its own slice into every copy of the
    gather buffers (`multimem.st`);

each between two barriers over per-rank flag words (bounded waits: a rank
that never arrives sets an error flag that `check()` raises on).

`NvlsExchange.supported()` says whether this can run (CUDA, an initialised
NCCL process group, torch symmetric memory, and NVLink multicast, which is
only known once the buffers exist: the constructor raises without it).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ._native import _C


def _pad4(n: int) -> int:
    return (int(n) + 3) // 4 * 4


def _multicast_address(t: torch.Tensor, handle) -> int:
    mc = int(handle.multicast_ptr)
    if mc == 0:
        raise RuntimeError("no NVLink multicast for this group (NVSwitch with multicast support is required)")
    addr = mc + (t.data_ptr() - int(handle.buffer_ptrs[handle.rank]))
    if addr % 16:
        raise RuntimeError("multicast address of the exchange buffer is not 16-byte aligned")
    return addr


class NvlsExchange:
    """Symmetric exchange buffers of one process group on this device:
    `n_reduce` floats to all-reduce and, per rank, `n_gather` floats (plus
    `n_gather_small`) to all-gather."""

    TIMEOUT_S = 10.0
    # set by NvlsGradientSum(sh_leaf=...): MultiViewSH leaves its view
    # gradients here for the step's single exchange window
    defer_views = False
    pending_views = None

    @staticmethod
    def supported(group=None) -> tuple[bool, str]:
        if not torch.cuda.is_available():
            return False, "no CUDA device"
        if not (dist.is_available() and dist.is_initialized()):
            return False, "no process group"
        if dist.get_backend(group) != "nccl":
            return False, "process group backend is not NCCL"
        try:
            import torch.distributed._symmetric_memory  # noqa: F401
        except ImportError:
            return False, "torch symmetric memory unavailable"
        return True, ""

    def __init__(self, group, n_reduce: int, n_gather: int = 0, n_gather_small: int = 0, device=None):
        import torch.distributed._symmetric_memory as symm
        self.group = group if group is not None else dist.group.WORLD
        name = self.group.group_name
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self._handles = []

        def sym(n, dtype):
            t = symm.empty(max(int(n), 4), dtype=dtype, device=dev)
            h = symm.rendezvous(t, name)
            self._handles.append(h)
            return t, h

        self.flags, hf = sym(_pad4(self.world), torch.int32)
        self.flags.zero_()
        self.peer_flags = int(hf.buffer_ptrs_dev)
        self.n_reduce = _pad4(n_reduce)
        self.red, hr = sym(self.n_reduce, torch.float32)
        self.red_mc = _multicast_address(self.red, hr)
        self.n_gather, self.n_small = int(n_gather), int(n_gather_small)
        self.slice, self.slice_small = _pad4(self.n_gather), _pad4(self.n_small)
        if self.n_gather:
            self.gat, hg = sym(self.world * self.slice, torch.float32)
            self.gat_mc = _multicast_address(self.gat, hg)
        if self.n_small:
            self.gat_small, hs = sym(self.world * self.slice_small, torch.float32)
            self.small_mc = _multicast_address(self.gat_small, hs)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        self._side = None
        # every rank's flags are zero before any rank's first barrier
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def barrier(self):
        self.epoch += 1
        _C.exchange_barrier(self.peer_flags, self.rank, self.world, self.epoch & 0xFFFFFFFF, self.TIMEOUT_S,
                            self.err)

    def all_reduce_(self, tensors) -> None:
        """Sums the float32 `tensors` over the group's ranks, in place (every
        rank passes tensors of the same sizes in the same order)."""
        tensors = list(tensors)
        total = sum(t.numel() for t in tensors)
        if total > self.n_reduce:
            raise ValueError(f"all_reduce_: {total} floats exceed the buffer ({self.n_reduce})")
        torch.cat([t.reshape(-1) for t in tensors], out=self.red[:total])
        self.barrier()
        _C.nvls_allreduce_sum(self.red_mc, self.n_reduce, self.rank, self.world, self.red)
        self.barrier()
        off = 0
        for t in tensors:
            t.copy_(self.red[off:off + t.numel()].view_as(t))
            off += t.numel()

    def exchange(self, tensors, d: torch.Tensor | None = None, small: torch.Tensor | None = None):
        """all_reduce_(tensors) and, when `d` is given, all_gather(d, small)
        inside ONE pair of barriers (the two kinds of traffic share the
        window instead of each waiting out its own pair); returns the
        gathered views as all_gather does (None, None without `d`)."""
        tensors = list(tensors)
        total = sum(t.numel() for t in tensors)
        if total > self.n_reduce:
            raise ValueError(f"exchange: {total} floats exceed the reduce buffer ({self.n_reduce})")
        if d is not None and (d.numel() != self.n_gather or (small is not None and small.numel() != self.n_small)):
            raise ValueError("exchange: gather sizes differ from the ones the buffers were made for")
        if total:
            torch.cat([t.reshape(-1) for t in tensors], out=self.red[:total])
        if d is not None:
            d, small = d.contiguous(), (small.contiguous() if small is not None else None)
        self.barrier()  # inputs written everywhere, previous contents read everywhere
        main = torch.cuda.current_stream(self.device)
        if d is not None:
            # the gather's stores on a side stream, beside the all-reduce
            if self._side is None:
                self._side = torch.cuda.Stream(device=self.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                _C.nvls_broadcast(d.reshape(-1), self.gat_mc + 4 * self.rank * self.slice)
                if small is not None:
                    _C.nvls_broadcast(small.reshape(-1), self.small_mc + 4 * self.rank * self.slice_small)
            d.record_stream(self._side)
            if small is not None:
                small.record_stream(self._side)
        if total:
            _C.nvls_allreduce_sum(self.red_mc, self.n_reduce, self.rank, self.world, self.red)
        if d is not None:
            main.wait_stream(self._side)
        self.barrier()  # every store has landed
        off = 0
        for t in tensors:
            t.copy_(self.red[off:off + t.numel()].view_as(t))
            off += t.numel()
        if d is None:
            return None, None
        out_d = self.gat.view(self.world, self.slice)[:, :self.n_gather]
        out_s = self.gat_small.view(self.world, self.slice_small)[:, :self.n_small] if small is not None else None
        return out_d, out_s

    def leave_no_views(self, means: torch.Tensor, degree: int, n_coeffs: int, k_max: int) -> None:
        """For a rank that renders no view in this pass while the others run
        MultiViewSH: its share of the view gather is k_max views of zero
        colour gradient (from an origin outside the Gaussians' bounding box,
        so every SH basis value stays finite), which add nothing to the
        rebuilt SH gradient.  Call it where MultiViewSH would have run."""
        n = means.shape[0]
        o = (means.detach().amax(0) + 1.0).reshape(1, 3).expand(k_max, 3).contiguous()
        self.pending_views = {"d": torch.zeros(k_max, n, 3, device=means.device, dtype=means.dtype), "o": o,
                              "means": means.detach(), "degree": degree, "k_max": k_max, "K": n_coeffs}

    def all_gather(self, d: torch.Tensor, small: torch.Tensor | None = None):
        """Every rank's `d` (n_gather floats) and `small` (n_gather_small
        floats): ([world, n_gather], [world, n_gather_small]) views of the
        gather buffers, valid until the next all_gather."""
        if d.numel() != self.n_gather or (small is not None and small.numel() != self.n_small):
            raise ValueError("all_gather: sizes differ from the ones the buffers were made for")
        self.barrier()  # every rank is done reading the previous contents
        _C.nvls_broadcast(d.contiguous().reshape(-1), self.gat_mc + 4 * self.rank * self.slice)
        if small is not None:
            _C.nvls_broadcast(small.contiguous().reshape(-1), self.small_mc + 4 * self.rank * self.slice_small)
        self.barrier()  # every rank's slices have landed
        out_d = self.gat.view(self.world, self.slice)[:, :self.n_gather]
        out_s = self.gat_small.view(self.world, self.slice_small)[:, :self.n_small] if small is not None else None
        return out_d, out_s

    def check(self) -> None:
        """Raises if a barrier timed out (reads the device flag: synchronises)."""
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"exchange barrier timed out: rank {e - 1} did not arrive within {self.TIMEOUT_S} s")


class NvlsGradientSum:
    """After a rank's backward pass, sums the gradients of `leaves` over the
    ranks (a zero gradient for a leaf this rank did not reach) with one
    NvlsExchange window.  Same `wait()` contract as
    multiview.GradientAllReduce.

    With `sh_leaf`, the multi-view SH exchange joins the same window:
    MultiViewSH (given this exchange) then leaves its view gradients with the
    exchange instead of gathering them inside backward, and wait() gathers
    them together with the all-reduce and adds the rebuilt SH-coefficient
    gradient (summed over every view of every rank) to `sh_leaf.grad`.  So
    `sh_leaf.grad` is complete only after wait(), like every other exchanged
    gradient."""

    def __init__(self, leaves, exchange: NvlsExchange, sh_leaf: torch.Tensor | None = None):
        self.leaves = list(leaves)
        self.exchange = exchange
        self.sh_leaf = sh_leaf
        exchange.defer_views = sh_leaf is not None
        exchange.pending_views = None

    def wait(self) -> int:
        from .multiview import timeline
        from ._native import _C
        ex = self.exchange
        for t in self.leaves:
            if t.grad is None:
                t.grad = torch.zeros_like(t)
        pend, ex.pending_views = ex.pending_views, None
        if self.sh_leaf is not None and pend is None:
            raise RuntimeError("NvlsGradientSum.wait: no view gradients were left by MultiViewSH in this pass")
        all_d, all_o = ex.exchange([t.grad for t in self.leaves], *((pend["d"], pend["o"]) if pend else ()))
        timeline.mark("exchange_end")
        if pend is not None:
            kmax, n = pend["k_max"], pend["means"].shape[0]
            d_sh = _C.spherical_harmonics_coeffs_bwd_multi(
                pend["degree"], all_o.reshape(ex.world * kmax, 3).contiguous(), pend["means"],
                all_d.reshape(ex.world * kmax, n, 3).contiguous(), pend["K"])
            g = self.sh_leaf
            g.grad = d_sh.view_as(g) if g.grad is None else g.grad + d_sh.view_as(g)
            timeline.mark("sh_bwd_end")
        return 1

    def remove(self):
        pass
