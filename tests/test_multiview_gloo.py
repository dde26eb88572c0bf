"""Host logic of the multi-GPU path on CPU: view assignment, and the
gradient all-reduce over two gloo ranks (the same code runs over NCCL on
GPUs).  Each rank builds a small autograd graph shaped like the render step
(a leaf feeding two consumers, like the Gaussian means feeding both the SH
colour and the compositing) and checks that after backward + wait() every
rank holds the sum of all ranks' gradients."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from xsimgs_b200.multiview import GradientAllReduce, assign_views, exchanged_leaves


def test_assign_views_balanced_and_deterministic():
    costs = [2.07, 1.23, 2.07, 1.23, 2.07, 1.23]  # C3: 3 x 1080p pinholes, 3 x 1280x960 fisheyes (Mpix)
    for world in (1, 2, 3, 4, 6, 8):
        a = assign_views(costs, world)
        assert a == assign_views(costs, world)
        assert sorted(i for v in a for i in v) == list(range(len(costs)))
        loads = [sum(costs[i] for i in v) for v in a]
        assert max(loads) - min(loads) <= max(costs) + 1e-9
    assert assign_views([1.0], 4) == [[0], [], [], []]
    with pytest.raises(ValueError):
        assign_views(costs, 0)


def test_exchanged_leaves_order_and_multiview_sh():
    names = ["means", "quats", "scales", "opacities", "sh", "local_q", "vertices"]
    assert exchanged_leaves(names, multiview_sh=False) == ["quats", "scales", "opacities", "means", "sh",
                                                           "local_q", "vertices"]
    # the multi-view SH backward already returns the SH gradient summed over ranks
    assert exchanged_leaves(names[:5], multiview_sh=True) == ["quats", "scales", "opacities", "means"]
    assert exchanged_leaves(["sh", "means"], multiview_sh=False) == ["means", "sh"]


def _plain(t):
    # a numpy copy pickles by value: a tensor would travel as a file
    # descriptor its worker must still hold when the parent reads the queue
    return t.detach().cpu().numpy().copy()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    """Two backward passes with the hooks registered once: each pass issues
    one collective per leaf, and afterwards every rank holds the same
    gradient."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        g = torch.Generator().manual_seed(100 + rank)
        means = torch.randn(50, 3, generator=g).requires_grad_(True)
        quats = torch.randn(50, 4, generator=g).requires_grad_(True)
        sh = torch.randn(50, 16, 3, generator=g).requires_grad_(True)
        red = GradientAllReduce([means, quats, sh])
        for _ in range(2):
            for t in (means, quats, sh):
                t.grad = None
            w = torch.randn(50, 3, generator=g)
            ((sh[:, 0, :] * means.sin()).sum() + (means * w).sum() + (quats ** 2).sum() * (rank + 1)).backward()
            n = red.wait()
            assert n == 3, f"{n} collectives in one pass"
            for t in (means, quats, sh):
                lst = [torch.empty_like(t.grad) for _ in range(world)]
                dist.all_gather(lst, t.grad)
                assert all(torch.equal(o, t.grad) for o in lst)
        red.remove()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def _reference_sum(world, idle=()):
    """The summed gradients recomputed without any collective."""
    tot = None
    for rank in range(world):
        if rank in idle:
            continue
        g = torch.Generator().manual_seed(100 + rank)
        means = torch.randn(50, 3, generator=g).requires_grad_(True)
        quats = torch.randn(50, 4, generator=g).requires_grad_(True)
        sh = torch.randn(50, 16, 3, generator=g).requires_grad_(True)
        w = torch.randn(50, 3, generator=g)
        ((sh[:, 0, :] * means.sin()).sum() + (means * w).sum() + (quats ** 2).sum() * (rank + 1)).backward()
        grads = [means.grad, quats.grad, sh.grad]
        tot = grads if tot is None else [a + b for a, b in zip(tot, grads)]
    return tot


def _worker_values(rank, world, port, q, idle=(), buckets=None):
    """`idle` ranks run no backward (a rank without views): they contribute
    zeros and still take part in every collective.  With `buckets`, leaves
    share collectives (their gradients become views of one flat buffer)."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        g = torch.Generator().manual_seed(100 + rank)
        means = torch.randn(50, 3, generator=g).requires_grad_(True)
        quats = torch.randn(50, 4, generator=g).requires_grad_(True)
        sh = torch.randn(50, 16, 3, generator=g).requires_grad_(True)
        red = GradientAllReduce([means, quats, sh], buckets=buckets)
        w = torch.randn(50, 3, generator=g)
        if rank not in idle:
            ((sh[:, 0, :] * means.sin()).sum() + (means * w).sum() + (quats ** 2).sum() * (rank + 1)).backward()
        assert red.wait() == (3 if buckets is None else len(buckets))
        q.put((rank, [_plain(t.grad) for t in (means, quats, sh)]))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.parametrize("target", ["consistency", "values", "idle_rank", "buckets", "buckets_idle_rank"])
def test_gradient_allreduce_two_gloo_ranks(target):
    world = 2
    idle = (1,) if target.endswith("idle_rank") else ()
    buckets = [2, 1] if target.startswith("buckets") else None
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    if target == "consistency":
        procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    else:
        procs = [ctx.Process(target=_worker_values, args=(r, world, port, q, idle, buckets)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, v = q.get(timeout=120)
        results[r] = v if isinstance(v, str) else [torch.from_numpy(x) for x in v]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if target == "consistency":
        assert all(v == "ok" for v in results.values()), results
    else:
        assert all(not isinstance(v, str) for v in results.values()), results
        ref = _reference_sum(world, idle)
        for r in range(world):
            for got, want in zip(results[r], ref):
                torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)


def _torch_ops():
    """CPU stand-ins for the three _C ops MultiViewSH calls (the CUDA ones are
    checked against the oracle in tests/test_gpu_multiview_sh.py)."""
    from tests.test_oracle import _torch_sh

    def cols(deg, origin, means, sh):
        d = means - origin
        return _torch_sh(deg, d / d.norm(dim=-1, keepdim=True), sh).float()

    def fwd(deg, origin, means, sh, mask, layout):
        return cols(deg, origin, means, sh)

    def pos_bwd(deg, origins, means, sh, d_out):
        with torch.enable_grad():
            m = means.detach().double().requires_grad_(True)
            sum((cols(deg, origins[v].double(), m, sh.detach().double()) * d_out[v]).sum()
                for v in range(origins.shape[0])).backward()
        return m.grad.float()

    def coeff_bwd(deg, origins, means, d_out, dim):
        with torch.enable_grad():
            s = torch.zeros(means.shape[0], dim, 3, dtype=torch.float64, requires_grad=True)
            sum((cols(deg, origins[v].double(), means.detach().double(), s) * d_out[v]).sum()
                for v in range(origins.shape[0])).backward()
        return s.grad.float()

    return fwd, pos_bwd, coeff_bwd


def _mvsh_setup(rank):
    g = torch.Generator().manual_seed(5)           # replicated scene
    means = torch.randn(40, 3, generator=g) * 4
    sh = torch.randn(40, 16, 3, generator=g)
    views = [2, 1][rank]                            # uneven views per rank
    gr = torch.Generator().manual_seed(50 + rank)
    origins = torch.randn(views, 3, generator=gr)
    d_cols = torch.randn(views, 40, 3, generator=gr)
    return means, sh, origins, d_cols


def _worker_mvsh(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from xsimgs_b200._native import _C
        from xsimgs_b200.multiview import multiview_colors
        _C.spherical_harmonics_fused_fwd, _C.spherical_harmonics_positions_bwd, \
            _C.spherical_harmonics_coeffs_bwd_multi = _torch_ops()
        means, sh, origins, d_cols = _mvsh_setup(rank)
        means.requires_grad_(True)
        sh.requires_grad_(True)
        cols = multiview_colors(sh, means, origins, 3, k_max=2)
        (cols * d_cols).sum().backward()
        q.put((rank, (_plain(means.grad), _plain(sh.grad))))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


def test_multiview_sh_exchange_two_gloo_ranks():
    """The SH gradient each rank gets is the sum over every view of every
    rank (uneven view counts, padded), the means gradient its own views'."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_mvsh, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: (v if isinstance(v, str) else [torch.from_numpy(x) for x in v])
           for r, v in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(not isinstance(v, str) for v in res.values()), res
    fwd, pos_bwd, coeff_bwd = _torch_ops()
    all_o, all_d = [], []
    for r in range(world):
        means, sh, origins, d_cols = _mvsh_setup(r)
        all_o.append(origins)
        all_d.append(d_cols)
        torch.testing.assert_close(res[r][0], pos_bwd(3, origins, means, sh, d_cols), rtol=1e-5, atol=1e-5)
    want_sh = coeff_bwd(3, torch.cat(all_o), means, torch.cat(all_d), 16)
    for r in range(world):
        torch.testing.assert_close(res[r][1], want_sh, rtol=1e-5, atol=1e-5)


def _worker_mvsh_gated(rank, world, port, q, own_group=False):
    """The render step's two exchanges together: the geometry all-reduces
    (GradientAllReduce) and MultiViewSH's all-gathers, with different view
    counts (so different autograd graphs) per rank — either on one group
    with the all-reduces gated behind the all-gathers, or with the view
    exchange on a group of its own (each group keeps one order)."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from xsimgs_b200._native import _C
        from xsimgs_b200.multiview import multiview_colors
        _C.spherical_harmonics_fused_fwd, _C.spherical_harmonics_positions_bwd, \
            _C.spherical_harmonics_coeffs_bwd_multi = _torch_ops()
        means, sh, origins, d_cols = _mvsh_setup(rank)
        g = torch.Generator().manual_seed(7)
        quats = torch.randn(40, 4, generator=g)
        w_q, w_m = _gated_weights(rank)
        for t in (means, sh, quats):
            t.requires_grad_(True)
        sh_group = dist.new_group([0, 1]) if own_group else None
        # the leaves a step exchanges, chosen as the bench chooses them: the
        # SH gradient (already summed by the view exchange) is left out
        leaves = {"means": means, "sh": sh, "quats": quats}
        red = GradientAllReduce([leaves[k] for k in exchanged_leaves(leaves, multiview_sh=True)],
                                gated=not own_group)
        for _ in range(2):  # hooks registered once, two passes
            for t in (means, sh, quats):
                t.grad = None
            cols = (multiview_colors(sh, means, origins, 3, k_max=2, group=sh_group) if own_group else
                    multiview_colors(sh, means, origins, 3, k_max=2, reducer=red))
            # "compositing": quats and means feed it as well as the colours
            loss = (cols * d_cols).sum() + (quats * w_q).sum() + (means * w_m).sum()
            loss.backward()
            assert red.wait() == 2
        q.put((rank, (_plain(means.grad), _plain(sh.grad), _plain(quats.grad))))
        red.remove()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


def _gated_weights(rank):
    g = torch.Generator().manual_seed(70 + rank)
    return torch.randn(40, 4, generator=g), torch.randn(40, 3, generator=g)


@pytest.mark.parametrize("own_group", [False, True], ids=["gated", "own_group"])
def test_allreduce_with_multiview_exchange_two_gloo_ranks(own_group):
    """Every rank ends with the sum over ranks of the geometry gradients and
    the SH gradient of every view of every rank, uneven view counts."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_mvsh_gated, args=(r, world, port, q, own_group)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: (v if isinstance(v, str) else [torch.from_numpy(x) for x in v])
           for r, v in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(not isinstance(v, str) for v in res.values()), res
    fwd, pos_bwd, coeff_bwd = _torch_ops()
    all_o, all_d = [], []
    want_m = 0
    want_q = 0
    for r in range(world):
        means, sh, origins, d_cols = _mvsh_setup(r)
        all_o.append(origins)
        all_d.append(d_cols)
        w_q, w_m = _gated_weights(r)
        want_m = want_m + pos_bwd(3, origins, means, sh, d_cols) + w_m
        want_q = want_q + w_q
    want_sh = coeff_bwd(3, torch.cat(all_o), means, torch.cat(all_d), 16)
    for r in range(world):
        torch.testing.assert_close(res[r][0], want_m, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(res[r][1], want_sh, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(res[r][2], want_q, rtol=1e-5, atol=1e-5)
