"""The NVSwitch gradient exchange (csrc/exchange.cu, xsimgs_b200/exchange.py).

  * The barrier's bounded wait, on one GPU: a peer whose flag nothing sets
    makes the barrier give up after its timeout and report that peer in the
    error word (the context stays usable); a peer that did arrive does not.
  * With two or more GPUs, two NCCL ranks: the all-gather returns every
    rank's slice bit for bit, the in-switch all-reduce returns the exact sum
    of two ranks' values, and a render-shaped step exchanged in one NVSwitch
    window (NvlsGradientSum with the SH leaf, MultiViewSH leaving its view
    gradients to it) ends with the same gradients as the NCCL exchange, also
    when one rank renders no view (it gathers zero view gradients).
"""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_times_out_when_a_peer_never_arrives(cuda):
    from xsimgs_b200 import _C
    mine = torch.zeros(4, dtype=torch.int32, device=cuda)
    other = torch.zeros(4, dtype=torch.int32, device=cuda)  # stands in for rank 1's flags
    ptrs = torch.tensor([mine.data_ptr(), other.data_ptr()], dtype=torch.int64, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _C.exchange_barrier(ptrs.data_ptr(), 0, 2, 1, 0.2, err)
    torch.cuda.synchronize()
    assert int(err) == 2  # 1 + the rank that never arrived
    assert int(other[0]) == 1  # rank 0 announced epoch 1 to rank 1
    # the peer arrives (its flag word in rank 0's flags reaches epoch 2): no error
    err.zero_()
    mine[1] = 2
    _C.exchange_barrier(ptrs.data_ptr(), 0, 2, 2, 0.2, err)
    torch.cuda.synchronize()
    assert int(err) == 0 and int(other[0]) == 2
    # the device is still usable
    assert float(torch.ones(8, device=cuda).sum()) == 8.0


def _multiview_step_both_ways(rank, world, dev):
    """A render-shaped step (a colour per view from the SH coefficients, the
    means feeding the colours and the 'compositing', quaternions only the
    latter) backpropagated and exchanged twice: NCCL (GradientAllReduce +
    MultiViewSH gathering inside backward) and this package's NVSwitch window
    (NvlsGradientSum with the SH leaf).  Gradients must agree."""
    import torch.distributed as dist
    from xsimgs_b200.exchange import NvlsExchange, NvlsGradientSum
    from xsimgs_b200.multiview import GradientAllReduce, exchanged_leaves, multiview_colors
    n, K = 2000, 16
    g = torch.Generator().manual_seed(100 + rank)
    means = (torch.randn(n, 3, generator=g) * 3).to(dev).requires_grad_(True)
    sh = (torch.randn(n, K, 3, generator=g) * 0.3).to(dev).requires_grad_(True)
    quats = torch.randn(n, 4, generator=g).to(dev).requires_grad_(True)
    origins = torch.randn(1, 3, generator=g).to(dev)
    d_cols = torch.randn(1, n, 3, generator=g).to(dev)
    w_q, w_m = torch.randn(n, 4, generator=g).to(dev), torch.randn(n, 3, generator=g).to(dev)
    leaves = {"means": means, "sh": sh, "quats": quats}
    order = exchanged_leaves(leaves, multiview_sh=True)

    def step(red, **kw):
        for t in leaves.values():
            t.grad = None
        cols = multiview_colors(sh, means, origins, 3, k_max=1, **kw)
        loss = (cols * d_cols).sum() + (quats * w_q).sum() + (means * w_m).sum()
        loss.backward()
        red.wait()
        return {k: t.grad.detach().clone() for k, t in leaves.items()}

    grp = dist.new_group([0, 1])
    red_nccl = GradientAllReduce([leaves[k] for k in order])
    nccl = step(red_nccl, group=grp)
    red_nccl.remove()  # its hooks would otherwise all-reduce the next pass too
    ex = NvlsExchange(None, sum(leaves[k].numel() for k in order), n * 3, 3, device=dev)
    red = NvlsGradientSum([leaves[k] for k in order], ex, sh_leaf=sh)
    out = {}
    for it in range(2):
        mine = step(red, exchange=ex)
        for k in leaves:
            out[f"mv_{k}_{it}"] = bool(torch.allclose(mine[k], nccl[k], rtol=1e-5, atol=1e-5))
    # rank 1 renders no view: in the NVSwitch window it gathers k_max views of
    # zero colour gradient (leave_no_views); the NCCL reference for that is
    # rank 1 rendering its view with a zero upstream colour gradient
    def step_viewless(red, nvls):
        for t in leaves.values():
            t.grad = None
        loss = (quats * w_q).sum() + (means * w_m).sum()
        if rank == 0 or not nvls:
            cols = multiview_colors(sh, means, origins, 3, k_max=1,
                                    **({"exchange": ex} if nvls else {"group": grp}))
            loss = loss + (cols * (d_cols if rank == 0 else torch.zeros_like(d_cols))).sum()
        else:
            ex.leave_no_views(means, 3, K, 1)
        loss.backward()
        red.wait()
        return {k: t.grad.detach().clone() for k, t in leaves.items()}

    red_nccl = GradientAllReduce([leaves[k] for k in order])
    want = step_viewless(red_nccl, nvls=False)
    red_nccl.remove()
    got = step_viewless(red, nvls=True)
    for k in leaves:
        out[f"mv_viewless_{k}_0"] = bool(torch.allclose(got[k], want[k], rtol=1e-5, atol=1e-5))
    torch.cuda.synchronize()
    ex.check()
    return out


def _two_rank_worker(rank, world, port, out_q):
    import torch.distributed as dist
    from xsimgs_b200.exchange import NvlsExchange
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    res = {}
    try:
        n = 10_003  # not a multiple of 4: padded buffers
        ex = NvlsExchange(None, n_reduce=2 * n, n_gather=3 * n, n_gather_small=3, device=dev)
        g = torch.Generator().manual_seed(7)
        vals = [torch.randn(2 * n, generator=g) for _ in range(world)]
        gath = [torch.randn(3 * n, generator=g) for _ in range(world)]
        small = [torch.randn(3, generator=g) for _ in range(world)]
        for it in range(3):  # repeated use of the same buffers
            t = vals[rank].to(dev).clone() * (it + 1)
            ex.all_reduce_([t[:n], t[n:]])
            want = sum(v * (it + 1) for v in vals)
            res[f"sum_exact_{it}"] = bool(torch.equal(t.cpu(), want))
            d, s = ex.all_gather(gath[rank].to(dev) + it, small[rank].to(dev))
            res[f"gather_exact_{it}"] = bool(torch.equal(d.cpu(), torch.stack(gath) + it) and
                                             torch.equal(s.cpu(), torch.stack(small)))
        torch.cuda.synchronize()
        ex.check()
        res.update(_multiview_step_both_ways(rank, world, dev))
        res["ok"] = True
    except Exception as e:  # noqa: BLE001
        res["error"] = repr(e)[:300]
    finally:
        dist.barrier()
        dist.destroy_process_group()
    out_q.put((rank, res))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nvls_exchange_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, res in got.items():
        if "error" in res and "multicast" in res["error"]:
            pytest.skip(f"no NVLink multicast here: {res['error']}")
        assert res.get("ok"), (r, res)
        bad = [k for k, v in res.items() if k.endswith(tuple("012")) and not v]
        assert not bad, (r, bad)
        assert sum(k.startswith("mv_") for k in res) == 9, res
