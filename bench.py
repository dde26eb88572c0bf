#!/usr/bin/env python
"""Benchmark of the Gaussian render path: fwd+bwd Mpix/s on the C2 workload
(1M Gaussians, SH degree 3, one 1920x1080 pinhole per GPU).

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]

One step = SH colour forward -> ut_gs_render (UT projection, tile
intersection + sort + offsets, rays, forward compositing) -> backward
(compositing backward, SH backward) through the public API and autograd, and
with N > 1 ranks the NCCL all-reduce (sum) of all Gaussian gradients
(views are sharded one per rank; weak scaling).  Rank r renders the C2 view;
every rank holds the full scene.

value  : whole-job Mpix/s with inputs resident in HBM, device-timed with CUDA
         events (max over ranks).
e2e    : the same step through the same public API with the upstream
         gradient images copied in from pinned host memory and the loss read
         back to the host every step (copies buffered on a copy stream,
         each loss read while the next steps run).
--impl reference : the CPU oracle restatement of the reference (the
         reference itself cannot be built here), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

W_C2, H_C2, N_C2, DEG_C2 = 1920, 1080, 1_000_000, 3
METRIC = "Gaussian-render fwd+bwd Mpix/s (1M Gaussians, 1080p)"
L2_BYTES = 126 * 2**20


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-lidar", action="store_true", help="skip the C4 lidar rays/s measurement")
    p.add_argument("--gaussians", type=int, default=0, help="override the workload's Gaussian count")
    p.add_argument("--workload", default="c2", choices=["c2", "c3", "c3-8"],
                   help="c2: one C2 view per rank (weak scaling, the default); c3 / c3-8: the rig's views "
                        "sharded over the ranks (strong scaling)")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_count():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ------------------------------------------------------------ CPU oracle --
def oracle_view(sc, spec, rows=None):
    """One fwd+bwd view (pinhole or fisheye) on the CPU oracle; `rows` limits
    compositing to a band of tile rows (projection and tiling always cover
    the whole view).  Returns (seconds, pixels composited)."""
    import numpy as np
    from oracle import oracle as O
    from xsimgs_b200 import scenes
    cam = spec.make("cpu")
    pack = cam.pack.numpy().reshape(-1)
    W, H = spec.width, spec.height
    m, q, s, o, sh = (t.numpy() for t in (sc.means, sc.quats, sc.scales, sc.opacities, sc.sh))
    vr, vd, va = (t.numpy() for t in scenes.upstream_grads(H, W, 3))
    t0 = time.perf_counter()
    flags, radii, m2, dep = O.projection_utgs(spec.kind, pack, m, None, s, q, o, W, H)
    tpg, ids, flat = O.isect_regular(m2, radii, dep, W, H, 16, 16)
    tw, th = (W + 15) // 16, (H + 15) // 16
    off = O.isect_offset_encode(ids, tw, th)
    ro, rd, _ = O.camera_rays(spec.kind, pack, W, H)
    cols = O.sh_fwd(DEG_C2, pack[4:7], m, sh)
    y0, y1 = (0, th) if rows is None else rows
    band = slice(y0 * 16, min(H, y1 * 16))
    start = int(off[y0, 0])
    end = int(off[y1, 0]) if y1 < th else len(flat)
    offb = off[y0:y1] - start
    flb = flat[start:end]
    Hb = band.stop - band.start
    rgb, d, a, last, _ = O.rasterize_fwd(m, q, s, cols, o, W, Hb, 16, 16, ro[band], rd[band], offb, flb)
    g = O.rasterize_bwd(m, q, s, cols, o, W, Hb, 16, 16, ro[band], rd[band], offb, flb, a, last,
                        vr[band], vd[band], va[band])
    O.sh_bwd(DEG_C2, pack[4:7], m, sh, g["v_colors"])
    return time.perf_counter() - t0, W * Hb


def reference_arm(args, world, rank):
    """--impl reference: the CPU oracle on the box's host cores, on the same
    workload (every view of one step), rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as O
    from xsimgs_b200 import scenes
    specs, n_default, scaling = workload_views(args.workload)
    n_gauss = args.gaussians or n_default
    # torchrun sets OMP_NUM_THREADS=1 per process: use every host core
    O.set_threads(cpu_count())
    sc = scenes.street_scene(n_gauss)
    if scaling == "weak":
        specs = specs * world   # every rank's view
    cores = O.num_threads()
    # calibrate on full views; bound the whole run to about three minutes by
    # compositing a centred band of tile rows of each view
    t_full = sum(oracle_view(sc, sp)[0] for sp in specs[:1]) * len(specs)
    steps = args.steps + args.warmup
    budget = 170.0 / max(1, steps)
    frac = min(1.0, budget / t_full)
    bands = []
    for sp in specs:
        th = (sp.height + 15) // 16
        if frac >= 1.0:
            bands.append(None)
        else:
            nrows = max(1, int(th * frac))
            y0 = max(0, th // 2 - nrows // 2)
            bands.append((y0, y0 + nrows))
    for _ in range(args.warmup):
        for sp, rows in zip(specs, bands):
            oracle_view(sc, sp, rows)
    tot_t, tot_px = 0.0, 0
    for _ in range(args.steps):
        for sp, rows in zip(specs, bands):
            t, px = oracle_view(sc, sp, rows)
            tot_t += t
            tot_px += px
    value = tot_px / tot_t / 1e6
    if all(b is None for b in bands):
        sample = f"every view of the step in full ({len(specs)} view(s))"
    else:
        sample = (f"projection + tiling of all {n_gauss} Gaussians and fwd+bwd compositing of a centred band of "
                  f"{bands[0][1] - bands[0][0]} tile rows per view, {len(specs)} view(s) per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "Mpix/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * tot_t / args.steps, 2), "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32", "data": f"synthetic (seeded {args.workload.upper()} scene)",
        "config": {"workload": WORKLOAD_DESC[args.workload],
                   "implementation": "CPU oracle restatement (reference not buildable here)"},
        "cpu_baseline": {"value": round(value, 4), "unit": "Mpix/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU arm ----
class ClockSampler:
    """nvidia-smi clock / throttle sampling while a timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ln in open(self.path):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        mx = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def workload_views(name: str):
    """(camera specs, Gaussians, scaling) of a bench workload."""
    from xsimgs_b200 import scenes
    if name == "c2":
        return [scenes.c2_camera()], N_C2, "weak"
    if name in ("c3", "c3-8"):
        return scenes.c3_rig(eight=name == "c3-8"), 2 * N_C2, "strong"
    raise ValueError(name)


WORKLOAD_DESC = {
    "c2": "C2: 1M Gaussians, SH deg 3, pinhole 1920x1080, fwd+bwd per view (every rank renders the C2 view)",
    "c3": "C3: 2M Gaussians, SH deg 3, 6-camera rig (3 pinholes 1920x1080, 3 KB fisheyes 1280x960), "
          "fwd+bwd of all views per step, views sharded over ranks",
    "c3-8": "C3-8: C3 plus 2 pinholes at yaw 30/210 deg (8 views), views sharded over ranks",
}


def gpu_arm(args, world, rank, local):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import xsimgs_b200 as X
    from xsimgs_b200 import capi, scenes, roofline
    from xsimgs_b200.multiview import GradientAllReduce, assign_views, multiview_colors

    specs, n_default, scaling = workload_views(args.workload)
    n_gauss = args.gaussians if args.gaussians else n_default
    sc = scenes.street_scene(n_gauss).to(dev)
    if scaling == "weak":
        assignment = [[0]] * world   # every rank renders the workload's one view
        px_per_step = world * specs[0].width * specs[0].height
    else:
        assignment = assign_views([s.width * s.height for s in specs], world)
        px_per_step = sum(s.width * s.height for s in specs)
    mine = assignment[rank]
    # with a view on every rank, ranks exchange per-view colour gradients and
    # rebuild the SH-coefficient gradient locally (MultiViewSH) instead of
    # all-reducing it
    mvsh = world > 1 and min(len(v) for v in assignment) >= 1
    k_max = max(len(v) for v in assignment)
    views = [(specs[i], specs[i].make(dev)) for i in mine]
    leaves = {k: v.clone().requires_grad_(True) for k, v in sc.params().items()}
    # backward finishes the compositing's leaves first, then the SH backward's
    red = GradientAllReduce([leaves[k] for k in ("quats", "scales", "opacities", "means")] +
                            ([] if mvsh else [leaves["sh"]]))
    upstream = [tuple(t.to(dev) for t in scenes.upstream_grads(sp.height, sp.width, 3, seed=1 + rank * 16 + k))
                for k, (sp, _) in enumerate(views)]

    def step(grads):
        for v in leaves.values():
            v.grad = None
        loss = torch.zeros((), device=dev)
        if mvsh:
            cols = multiview_colors(leaves["sh"], leaves["means"], torch.stack([cam.t0 for _, cam in views]),
                                    DEG_C2, k_max)
        for v, ((sp, cam), (gr, gd, ga)) in enumerate(zip(views, grads)):
            colors = cols[v] if mvsh else X.spherical_harmonics_fused(leaves["sh"], leaves["means"], cam.t0, DEG_C2)
            color, depth, alpha, _ = X.ut_gs_render(cam, leaves["means"], leaves["scales"], leaves["quats"],
                                                    leaves["opacities"], sp.width, sp.height, colors=colors)
            loss = loss + (torch.dot(color.reshape(-1), gr.reshape(-1)) + torch.dot(depth.reshape(-1), gd.reshape(-1))
                           + torch.dot(alpha.reshape(-1), ga.reshape(-1)))
        if views:
            loss.backward()
        red.wait()
        return loss

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(upstream)
    barrier()

    # -------------------------------------------------- timed: value ----
    clocks = ClockSampler(local)
    clocks.start()
    capi.timing_reset()
    capi.timing_enable(True)
    launches0 = capi.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record()
    for _ in range(args.steps):
        step(upstream)
    ev1.record()
    barrier()
    launches = capi.launch_count() - launches0
    capi.timing_enable(False)
    t_ms = ev0.elapsed_time(ev1)
    bwd_ms, bwd_n = capi.timing_query("rasterize_bwd")
    fwd_ms, fwd_n = capi.timing_query("rasterize_fwd")
    capi.timing_reset()

    # ---------------------------------------------------- timed: e2e ----
    # Each step's upstream gradients come from pinned host memory and each
    # step's loss goes back to pinned host memory and is read on the host.
    # The copies are buffered on a copy stream (later steps' inputs arrive
    # while step k computes) and the loss of step k is read while the next
    # steps run, as a training loop with asynchronous loss logging does.
    host = [[t.cpu().pin_memory() for t in g] for g in upstream]
    h2d = sum(t.numel() * t.element_size() for g in host for t in g)
    comp = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(device=dev)
    NB = 3  # buffers: the host reads step k's loss while steps k+1 and k+2 are queued
    dbufs = [[[torch.empty_like(t) for t in g] for g in upstream] for _ in range(NB)]
    loss_host = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(NB)]
    ev_in = [torch.cuda.Event() for _ in range(NB)]
    ev_free = [torch.cuda.Event() for _ in range(NB)]  # compute is done with dbufs[b]
    ev_out = [torch.cuda.Event() for _ in range(NB)]
    for ev in ev_free:
        ev.record(comp)
    losses = []

    def e2e_steps(n, start_event=None):
        pending = []
        for k in range(n):
            b = k % NB
            if len(pending) == NB - 1:  # buffer b's previous loss must be read before it is reused
                p = pending.pop(0)
                ev_out[p].synchronize()
                losses.append(float(loss_host[p]))
            with torch.cuda.stream(copy_stream):
                if start_event is not None and k == 0:
                    copy_stream.wait_event(start_event)
                copy_stream.wait_event(ev_free[b])
                for dg, hg in zip(dbufs[b], host):
                    for d, h in zip(dg, hg):
                        d.copy_(h, non_blocking=True)
                ev_in[b].record(copy_stream)
            comp.wait_event(ev_in[b])
            loss = step(dbufs[b])
            ev_free[b].record(comp)
            loss_host[b].copy_(loss.detach(), non_blocking=True)
            ev_out[b].record(comp)
            pending.append(b)
        for p in pending:
            ev_out[p].synchronize()
            losses.append(float(loss_host[p]))

    e2e_steps(max(1, args.warmup // 2))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_steps(args.steps, start_event=e0)
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    assert all(math.isfinite(v) for v in losses)

    # ------------------------------ timed: C4 lidar rays/s (c2 scene) ----
    lidar_ms = {}
    if args.workload == "c2" and not args.no_lidar:
        lspec = scenes.c4_lidar()
        lcam = lspec.make(dev)
        LW, LH = lspec.width, lspec.height
        gen = torch.Generator().manual_seed(3)
        inten = torch.rand(n_gauss, 1, generator=gen).to(dev).requires_grad_(True)
        lg = [t.to(dev) for t in scenes.upstream_grads(LH, LW, 1, seed=40 + rank)]

        def lstep(phm):
            for v in list(leaves.values()) + [inten]:
                v.grad = None
            color, depth, alpha, _ = X.ut_gs_render(lcam, leaves["means"], leaves["scales"], leaves["quats"],
                                                    leaves["opacities"], LW, LH, colors=inten, use_phm=phm)
            (torch.dot(color.reshape(-1), lg[0].reshape(-1)) + torch.dot(depth.reshape(-1), lg[1].reshape(-1))
             + torch.dot(alpha.reshape(-1), lg[2].reshape(-1))).backward()
            red.wait()

        for phm in (False, True):
            for _ in range(args.warmup):
                lstep(phm)
            barrier()
            l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0.record()
            for _ in range(args.steps):
                lstep(phm)
            l1.record()
            barrier()
            lidar_ms["phm" if phm else "central"] = l0.elapsed_time(l1)

    clk = clocks.stop()

    # max over ranks
    tt = torch.tensor([t_ms, e2e_ms, lidar_ms.get("central", 0.0), lidar_ms.get("phm", 0.0)], device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, l_c, l_p = tt.tolist()
    lidar = None
    if lidar_ms:
        rays = world * 128 * 2048 * args.steps
        lidar = {"metric": "lidar rays/s (C4: 128 beams x 2048 azimuth bins, the C2 scene, depth + intensity + "
                           "ray-drop alpha, fwd+bwd)", "unit": "rays/s", "scaling": "weak",
                 "value": round(rays / (l_c * 1e-3)), "ms_per_step": round(l_c / args.steps, 3),
                 "phm": {"value": round(rays / (l_p * 1e-3)), "ms_per_step": round(l_p / args.steps, 3)}}

    # ------------------------------------------------ roofline inputs ----
    roof = None
    if rank == 0 and views:
        fl_b = fl_f = 0.0
        pairs = {"evaluated_fwd": 0, "evaluated_bwd": 0, "contributing": 0}
        for sp, cam in views:
            W, H = sp.width, sp.height
            cnt = torch.zeros(8, dtype=torch.int64, device=dev)
            capi.set_pair_counters(cnt.data_ptr())
            with torch.no_grad():
                colors = X.spherical_harmonics_fused(sc.sh, sc.means, cam.t0, DEG_C2)
                td = X.ut_gs_tiling(cam, sc.means, sc.scales, sc.quats, W, H, opacity=sc.opacities)
                ro, rd = cam.camera_rays(W, H)
                _, _, alpha, last = X._C.rasterize_eval3d_fwd(
                    means=sc.means, quats=sc.quats, scales=sc.scales, colors=colors.unsqueeze(0),
                    opacities=sc.opacities.view(1, -1), image_width=W, image_height=H, tile_size_width=16,
                    tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=td["isect_offsets"],
                    flatten_ids=td["flatten_ids"])
            torch.cuda.synchronize()
            capi.set_pair_counters(None)
            n_eval_f, n_contrib = (int(x) for x in cnt.tolist()[:2])
            # backward replays every pair up to each pixel's last contributor
            tw = (W + 15) // 16
            ty = torch.arange(H, device=dev) // 16
            tx = torch.arange(W, device=dev) // 16
            start = td["isect_offsets"].view(-1)[(ty[:, None] * tw + tx[None, :])]
            n_eval_b = int(torch.where(alpha > 0, last - start + 1, torch.zeros_like(last)).sum())
            # the render step's rays come from the camera: no ray gradients
            fl_b += roofline.bwd_flops(n_eval_b, n_contrib, 3, ray_grads=False)
            fl_f += roofline.fwd_flops(n_eval_f, n_contrib, 3)
            pairs["evaluated_fwd"] += n_eval_f
            pairs["evaluated_bwd"] += n_eval_b
            pairs["contributing"] += n_contrib
        peak_flops = fp32_peak(dev)
        # kernel time per step over the timed region (all of this rank's views)
        bwd_step = bwd_ms / args.steps
        fwd_step = fwd_ms / args.steps
        ach_b = fl_b / (bwd_step * 1e-3) / 1e12
        ach_f = fl_f / (fwd_step * 1e-3) / 1e12
        c2_full = args.workload == "c2" and n_gauss == N_C2
        roof = {"kernel": "rasterize_bwd (raster_bwd_px2_kernel<3>: static scene, no ray gradients, two pixels a lane)", "bound": "fp32",
                "achieved": round(ach_b, 2), "peak": round(peak_flops / 1e12, 2), "unit": "TFLOP/s",
                "frac": round(ach_b / (peak_flops / 1e12), 3),
                "traffic": roofline.BWD_DRAM_BYTES_C2 if c2_full else None,
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum, one capture of this kernel "
                                   "on this workload (bytes per launch)") if c2_full else None,
                "peak_source": "measured: FP32 FMA probe in this run (MEASURED_PEAKS.json has only HBM and bf16)",
                "avg_launch_ms": round(bwd_ms / max(1, bwd_n), 4),
                "flops_per_launch": fl_b / len(views), "pairs": pairs,
                "fwd": {"achieved": round(ach_f, 2), "avg_launch_ms": round(fwd_ms / max(1, fwd_n), 4),
                        "frac": round(ach_f / (peak_flops / 1e12), 3)},
                "step_share": round((bwd_step + fwd_step) / (t_ms / args.steps), 3)}

    red.remove()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    cpu = None
    if world == 1 and not args.no_cpu_baseline and args.workload == "c2":
        from oracle import oracle as O
        O.set_threads(cpu_count())
        t, px = oracle_view(scenes.street_scene(n_gauss), specs[0])
        cpu = {"value": round(px / t / 1e6, 4), "unit": "Mpix/s", "cores": O.num_threads(), "kind": "port",
               "sample": "one full C2 view (projection, tiling, SH, fwd+bwd compositing) on the CPU oracle"}

    px_total = px_per_step * args.steps
    value = px_total / (t_ms * 1e-3) / 1e6
    e2e = px_total / (e2e_ms * 1e-3) / 1e6
    gbytes = sum(v.numel() * 4 for v in leaves.values())
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "Mpix/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 3), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded {args.workload.upper()} scene)",
        "config": {"workload": WORKLOAD_DESC[args.workload],
                   "views_per_gpu": len(views) if scaling == "weak" else
                   [len(v) for v in assign_views([s.width * s.height for s in specs], world)],
                   "parallelism": f"view-sharded dp{world} + NCCL all-reduce of grads",
                   "gradient_exchange": ("all-reduce of the geometry gradients + all-gather of the per-view colour "
                                         "gradients, SH-coefficient gradient rebuilt on every rank") if mvsh else
                                        ("all-reduce of every Gaussian gradient" if world > 1 else "none"),
                   "gaussians": n_gauss, "pixels_per_step": px_per_step, "tile": 16,
                   "l2": f"inputs larger than L2: Gaussian params {gbytes / 1e6:.0f} MB > 126 MB L2"},
        "e2e": {"value": round(e2e, 2), "unit": "Mpix/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches), "gpu_launches_per_step": round(launches / args.steps, 1),
        "clocks": clk, "roofline": roof, "cpu_baseline": cpu, "lidar": lidar,
    }
    print(json.dumps(line), flush=True)


def fp32_peak(dev) -> float:
    """FLOP/s of the FMA probe kernel (8 x 148 SM-filling blocks), best of 3."""
    import torch
    from xsimgs_b200 import capi
    scratch = torch.empty(512, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    stream = torch.cuda.current_stream(dev).cuda_stream
    best = 0.0
    for _ in range(4):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fl = capi.fp32_probe(scratch.data_ptr(), 4096, sms * 4, stream)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, fl / (e0.elapsed_time(e1) * 1e-3))
    return best


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    gpu_arm(args, world, rank, local)


if __name__ == "__main__":
    main()
