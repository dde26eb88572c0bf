#!/usr/bin/env python
"""Benchmark of the Gaussian render path: fwd+bwd Mpix/s on the C2 workload
(1M Gaussians, SH degree 3, one 1920x1080 pinhole per GPU).

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]
                    [--workload c2|c3|c3-8|c5]

One step = SH colour forward -> ut_gs_render (UT projection, tile
intersection + sort + offsets, rays, forward compositing) -> backward from
N(0, 1) upstream gradients of the colour, depth and alpha images
(compositing backward, SH backward) through the public API and autograd, and
with N > 1 ranks the exchange of the Gaussian gradients over NVLink (views
are sharded over the ranks; this package's NVSwitch multicast kernels, or
NCCL with --exchange bucketed / per-leaf).  Every rank holds the full scene.

value  : whole-job Mpix/s with inputs resident in HBM, device-timed with CUDA
         events (max over ranks).
e2e    : the same step through the same public API with the upstream
         gradient images copied in from pinned host memory and the step's
         scalar result (mean alpha) read back to the host every step (copies
         buffered on a copy stream, each result read while the next steps
         run).
Extra keys of the default (c2) line, each timed the same way at the same N:
  lidar  C4: 128 x 2048 lidar rays/s over the C2 scene, with and without PHM
  rig    C3-8: the 8-camera rig (5 pinholes 1920x1080, 3 KB fisheyes
         1280x960) over the 2M-Gaussian scene, views sharded over the ranks
         (strong scaling); also C3 (the 6-camera rig) as rig.c3
  c5     C5: 8 SMPL bodies x 20k Gaussians skinned into the 1M static scene,
         rendered into the 6 rig cameras, skinning + render fwd + bwd
         (strong scaling)
  phases per-phase device times of a step (forward, backward, view exchange,
         all-reduce tail)
  stages per-stage launch times and HBM fractions (projection, tiling, SH,
         skinning) from the library's timed scopes
--impl reference : the CPU oracle restatement of the reference on the box's
         host cores (the reference has no CPU implementation of this path and
         its GPU kernels are a test oracle here), rank 0 only.
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

W_C2, H_C2, N_C2, DEG = 1920, 1080, 1_000_000, 3
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
    p.add_argument("--no-rig", action="store_true", help="skip the C3 / C3-8 rig measurement")
    p.add_argument("--no-c5", action="store_true", help="skip the C5 skinned-actor measurement")
    p.add_argument("--gaussians", type=int, default=0, help="override the workload's Gaussian count")
    p.add_argument("--exchange", default="nvls", choices=["nvls", "bucketed", "per-leaf"],
                   help="gradient exchange at N > 1: this package's NVSwitch multicast kernels (nvls, the "
                        "default; NCCL bucketed where NVLink multicast is unavailable), or NCCL with the "
                        "geometry gradients ready together in one all-reduce (bucketed) or one per leaf")
    p.add_argument("--workload", default="c2", choices=["c2", "c3", "c3-8", "c5"],
                   help="c2: one C2 view per rank (weak scaling, the default); c3 / c3-8 / c5: the rig's views "
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


WORKLOAD_DESC = {
    "c2": "C2: 1M Gaussians, SH deg 3, pinhole 1920x1080, fwd+bwd per view (every rank renders the C2 view)",
    "c3": "C3: 2M Gaussians, SH deg 3, 6-camera rig (3 pinholes 1920x1080, 3 KB fisheyes 1280x960), "
          "fwd+bwd of all views per step, views sharded over ranks",
    "c3-8": "C3-8: C3 plus 2 pinholes at yaw 30/210 deg (8 views), views sharded over ranks",
    "c5": "C5: 8 SMPL bodies x 20k Gaussians skinned into the 1M-Gaussian C2 scene, 6-camera rig, skinning + "
          "fwd+bwd of all views per step, views sharded over ranks",
}


def workload_views(name: str):
    """(camera specs, Gaussians, scaling) of a bench workload."""
    from xsimgs_b200 import scenes
    if name == "c2":
        return [scenes.c2_camera()], N_C2, "weak"
    if name in ("c3", "c3-8"):
        return scenes.c3_rig(eight=name == "c3-8"), 2 * N_C2, "strong"
    if name == "c5":
        return scenes.c3_rig(), N_C2, "strong"
    raise ValueError(name)


def mvsh_enabled(name: str, world: int, views_everywhere: bool, exchange: str) -> bool:
    """Whether a step exchanges per-view colour gradients (MultiViewSH)
    instead of all-reducing the SH gradient."""
    return world > 1 and name != "c5" and (views_everywhere or exchange == "nvls")


def workload_config(name: str, world: int, n_gauss: int, exchange: str = "nvls") -> dict:
    """The `config` dict of a workload at `world` ranks; both arms print it."""
    from xsimgs_b200.multiview import assign_views
    specs, _, scaling = workload_views(name)
    if scaling == "weak":
        px = world * specs[0].width * specs[0].height
        views = 1
    else:
        px = sum(s.width * s.height for s in specs)
        views = [len(v) for v in assign_views([s.width * s.height for s in specs], world)]
    mvsh = mvsh_enabled(name, world, scaling == "weak" or min(views) >= 1, exchange)
    cfg = {"workload": WORKLOAD_DESC[name], "views_per_gpu": views,
           "parallelism": f"view-sharded dp{world} + gradient exchange over NVLink",
           "gradient_exchange": ("all-reduce of the geometry gradients + all-gather of the per-view colour "
                                 "gradients, SH-coefficient gradient rebuilt on every rank") if mvsh else
                                ("all-reduce of every Gaussian gradient" if world > 1 else "none"),
           "gaussians": n_gauss + (8 * 20_000 if name == "c5" else 0), "pixels_per_step": px, "tile": 16,
           "l2": "inputs larger than L2 (Gaussian parameters > 126 MB L2)"}
    return cfg


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
    cols = O.sh_fwd(DEG, pack[4:7], m, sh)
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
    O.sh_bwd(DEG, pack[4:7], m, sh, g["v_colors"])
    return time.perf_counter() - t0, W * Hb


def reference_arm(args, world, rank):
    """--impl reference: the CPU oracle on the box's host cores, on the same
    workload (every view of one step), rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as O
    from xsimgs_b200 import scenes
    name = "c3" if args.workload == "c5" else args.workload
    specs, n_default, scaling = workload_views(name)
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
                  f"{bands[0][1] - bands[0][0]} of {(specs[0].height + 15) // 16} tile rows per view (the image "
                  f"centre, a denser pixel mix than the whole view), {len(specs)} view(s) per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "Mpix/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * tot_t / args.steps, 2), "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32", "data": f"synthetic (seeded {args.workload.upper()} scene)",
        "config": workload_config(args.workload, world, n_gauss, args.exchange),
        "cpu_baseline": {"value": round(value, 4), "unit": "Mpix/s", "cores": cores, "kind": "port",
                         "sample": sample,
                         "implementation": "CPU oracle restatement of the reference (oracle/xsg_oracle.cpp)"},
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


class Workload:
    """One rank's share of a bench workload: its views, the scene leaves,
    the gradient exchange and a `step(upstream)` that runs one fwd+bwd pass
    of every view of this rank and the exchange."""

    def __init__(self, name, world, rank, dev, n_gauss=0, exchange="bucketed"):
        import torch
        import xsimgs_b200 as X
        from xsimgs_b200 import scenes
        from xsimgs_b200.multiview import GradientAllReduce, assign_views, exchanged_leaves, multiview_colors
        self.X, self.torch, self.mvc = X, torch, multiview_colors
        self.name, self.world, self.rank, self.dev = name, world, rank, dev
        specs, n_default, self.scaling = workload_views(name)
        self.n_gauss = n_gauss or n_default
        self.specs = specs
        if self.scaling == "weak":
            self.assignment = [[0]] * world
            self.px_per_step = world * specs[0].width * specs[0].height
        else:
            self.assignment = assign_views([s.width * s.height for s in specs], world)
            self.px_per_step = sum(s.width * s.height for s in specs)
        mine = self.assignment[rank]
        self.views = [(specs[i], specs[i].make(dev)) for i in mine]
        self.k_max = max(len(v) for v in self.assignment)
        sc = scenes.street_scene(self.n_gauss).to(dev)
        self.leaves = {k: v.clone().requires_grad_(True) for k, v in sc.params().items()}
        self.smpl = None
        if name == "c5":
            self._setup_c5(dev)
        # with a view on every rank, ranks exchange per-view colour gradients
        # and rebuild the SH-coefficient gradient locally (MultiViewSH), on a
        # communicator of their own: its all-gathers and the all-reduces
        # below each keep one order on every rank and run side by side
        import torch.distributed as dist
        views_everywhere = min(len(v) for v in self.assignment) >= 1
        # the NVSwitch window lets a rank without views join the view gather
        # with zero gradients; NCCL's gather inside backward needs a view on
        # every rank
        self.mvsh = mvsh_enabled(name, world, views_everywhere, exchange)
        order = exchanged_leaves(self.leaves, self.mvsh)
        self.ex = None
        self.sh_group = None
        if exchange == "nvls" and world > 1:
            # this package's NVSwitch kernels on the compute stream: the view
            # exchange inside the SH backward, one all-reduce after backward
            from xsimgs_b200.exchange import NvlsExchange, NvlsGradientSum
            n_red = sum(self.leaves[k].numel() for k in order)
            n_gat = self.k_max * self.n_gauss * 3 if self.mvsh else 0
            try:
                self.ex = NvlsExchange(None, n_red, n_gat, 3 * self.k_max if self.mvsh else 0, device=dev)
            except RuntimeError as e:  # no NVLink multicast here: every rank finds the same
                print(f"[bench] NVSwitch exchange unavailable ({e}); using NCCL", flush=True)
                exchange = "bucketed"
                self.mvsh = mvsh_enabled(name, world, views_everywhere, exchange)
                order = exchanged_leaves(self.leaves, self.mvsh)
        self.exchange = exchange if world > 1 else "none"
        if self.ex is not None:
            # the view gather joins the all-reduce's window (one barrier pair)
            self.red = NvlsGradientSum([self.leaves[k] for k in order], self.ex,
                                       sh_leaf=self.leaves["sh"] if self.mvsh else None)
        else:
            # NCCL: the view exchange on a communicator of its own (its
            # all-gathers and the all-reduces each keep one order on every
            # rank and run side by side); backward finishes the compositing's
            # leaves first (quats, scales and opacities together: one
            # bucket), then the SH backward's
            self.sh_group = dist.new_group(list(range(world))) if self.mvsh else None
            buckets = ([3] + [1] * (len(order) - 3)) if exchange == "bucketed" else None
            self.red = GradientAllReduce([self.leaves[k] for k in order], buckets=buckets)
        self.upstream = [tuple(t.to(dev) for t in scenes.upstream_grads(sp.height, sp.width, 3,
                                                                         seed=1 + rank * 16 + k))
                         for k, (sp, _) in enumerate(self.views)]

    def _setup_c5(self, dev):
        import torch
        from xsimgs_b200 import scenes
        s = scenes.c5_smpl()
        g = lambda t: t.to(dev).contiguous()
        self.smpl = {k: g(v) for k, v in s.items()}
        nb = s["vertices"].shape[0] * s["vertices"].shape[1]
        self.n_bodies = s["vertices"].shape[0]
        self.n_body_gauss = nb
        gen = torch.Generator().manual_seed(21)
        self.leaves["local_q"] = self.smpl.pop("local_q").clone().requires_grad_(True)
        self.leaves["vertices"] = self.smpl.pop("vertices").clone().requires_grad_(True)
        self.body_scales = g(torch.exp(torch.randn(nb, 3, generator=gen) * 0.3 - 3.5))
        self.body_opac = g(torch.sigmoid(torch.randn(nb, generator=gen) + 1.0))
        self.body_sh = g(scenes._sh(gen, nb, DEG))

    def _scene(self):
        """(means, quats, scales, opacities, sh, velocity) of the step's scene."""
        L = self.leaves
        if self.smpl is None:
            return L["means"], L["quats"], L["scales"], L["opacities"], L["sh"], None
        from xsimgs_b200.nodes import smpl_lbs_skinning, smpl_local_to_global_pose
        torch, s, dev = self.torch, self.smpl, self.dev
        gq, gt = smpl_local_to_global_pose(s["valid_ids"], L["local_q"], s["joints"], s["a0_inv_q"], s["a0_inv_t"])
        n_s, nb = self.n_gauss, self.n_body_gauss
        pos = torch.cat([L["means"], torch.zeros(nb, 3, device=dev)])
        rot = torch.cat([L["quats"], torch.zeros(nb, 4, device=dev)])
        vel = torch.zeros(n_s + nb, 3, device=dev)
        pos, rot, vel, _ = smpl_lbs_skinning(s["valid_ids"], gq, gt, L["vertices"], s["quats"], s["weights"],
                                             s["instance_ids"], s["instance_t"], s["instance_v"], n_s, pos, rot,
                                             vel)
        scales = torch.cat([L["scales"], self.body_scales])
        opac = torch.cat([L["opacities"], self.body_opac])
        sh = torch.cat([L["sh"], self.body_sh])
        return pos, rot, scales, opac, sh, vel

    def step(self, grads, marks=None):
        X, torch = self.X, self.torch
        for v in self.leaves.values():
            v.grad = None
        means, quats, scales, opac, sh, vel = self._scene()
        if self.mvsh and self.views:
            cols = self.mvc(sh, means, torch.stack([cam.t0 for _, cam in self.views]), DEG, self.k_max,
                            group=self.sh_group, exchange=self.ex)
        elif self.mvsh:
            self.ex.leave_no_views(means, DEG, sh.shape[1], self.k_max)
        outs, ups = [], []
        for v, ((sp, cam), g) in enumerate(zip(self.views, grads)):
            colors = cols[v] if self.mvsh else X.spherical_harmonics_fused(sh, means, cam.t0, DEG)
            color, depth, alpha, _ = X.ut_gs_render(cam, means, scales, quats, opac, sp.width, sp.height,
                                                    colors=colors, points_velocity=vel)
            outs += [color, depth, alpha]
            ups += list(g)
        # the step's reported result: mean alpha of this rank's views (one
        # reduction; the upstream gradients enter the backward directly)
        result = (torch.stack([o.mean() for o in outs[2::3]]).mean() if outs
                  else torch.zeros((), device=self.dev))
        if marks is not None:
            marks.append(("fwd_end", _event()))
        if outs:
            # backward from the upstream gradient images (~N(0,1)) of the
            # colour, depth and alpha images of every view
            torch.autograd.backward(outs, ups)
        if marks is not None:
            marks.append(("bwd_end", _event()))
        self.red.wait()
        return result


def _event():
    import torch
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    return e


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(values, world, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def time_steps(wl, steps, warmup, world):
    """Device time (ms) of `steps` steps after `warmup` untimed ones, this
    rank; barrier + synchronize on both sides."""
    import torch
    for _ in range(warmup):
        wl.step(wl.upstream)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        wl.step(wl.upstream)
    e1.record()
    barrier(world)
    return e0.elapsed_time(e1)


PHASE_NAMES = {"fwd_end": "forward", "sh_bwd_start": "backward_compute", "sh_gathered": "sh_bwd_exchange_wait",
               "sh_bwd_end": "sh_coeff_rebuild", "bwd_end": "backward_rest", "exchange_end": "exchange"}


def phase_times(wl, steps, world):
    """Mean per-phase device times (ms) of a step, each from the previous
    mark: forward (everything queued before backward), backward compute up
    to the SH backward, the view all-gather wait (NCCL path), the
    SH-coefficient rebuild, the rest of backward, and the gradient exchange
    (all-reduce; with the NVSwitch kernels also the view gather)."""
    from xsimgs_b200.multiview import timeline
    acc = {}
    barrier(world)
    timeline.enabled = True
    timeline.take()
    for _ in range(steps):
        marks = [("start", _event())]
        wl.step(wl.upstream, marks)
        marks += timeline.take()
        barrier(world)
        ev = dict(marks)
        # each phase ends at a mark and starts at the one before it in time
        # (the NVSwitch exchange rebuilds the SH gradient after the exchange
        # window, the NCCL path inside backward)
        t_of = sorted((ev["start"].elapsed_time(e), k) for k, e in ev.items() if k != "start")
        prev = 0.0
        for t, k in t_of:
            acc[PHASE_NAMES[k]] = acc.get(PHASE_NAMES[k], 0.0) + (t - prev)
            prev = t
    timeline.enabled = False
    mine = {k: v / steps for k, v in acc.items()}
    if world == 1:
        return {k: round(v, 4) for k, v in mine.items()}
    # every rank's phases: the max and min over ranks show the load skew the
    # collectives wait out
    import torch
    import torch.distributed as dist
    keys = list(PHASE_NAMES.values())
    t = torch.tensor([mine.get(k, 0.0) for k in keys], dtype=torch.float64, device=torch.device("cuda"))
    all_t = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(all_t, t)
    m = torch.stack(all_t)
    return {k: {"rank0": round(float(m[0, i]), 4), "max": round(float(m[:, i].max()), 4),
                "min": round(float(m[:, i].min()), 4)} for i, k in enumerate(keys) if k in mine}


def exchange_probe(wl, world, dev, reps=10):
    """The step's gradient exchange alone (no compute running): the
    all-gather of one colour gradient per rank and the all-reduces of the
    geometry gradients, as the step issues them; mean ms over `reps`."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return None
    n = wl.n_gauss
    geo = [torch.zeros(n, k, device=dev) for k in (4, 3, 1, 3)]
    d = torch.zeros(n, 3, device=dev)
    out = torch.empty(world * n, 3, device=dev)
    flat = torch.zeros(n * 11, device=dev)

    def run(split):
        w = [dist.all_gather_into_tensor(out, d, async_op=True)] if wl.mvsh else []
        if split:
            w += [dist.all_reduce(t, async_op=True) for t in geo]
        else:
            w += [dist.all_reduce(flat, async_op=True)]
        for x in w:
            x.wait()

    res = {}
    if wl.ex is not None:
        # this package's NVSwitch kernels: the view all-gather and the
        # all-reduce of every exchanged gradient in one window, as the step
        # runs them
        ex = wl.ex
        dv = torch.zeros(ex.n_gather, device=dev)
        ov = torch.zeros(ex.n_small, device=dev)
        red = torch.zeros(ex.n_reduce, device=dev)

        def run_nvls():
            ex.exchange([red], *((dv, ov) if ex.n_gather else ()))

        for _ in range(3):
            run_nvls()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run_nvls()
        e1.record()
        barrier(world)
        res["nvls"] = round(e0.elapsed_time(e1) / reps, 4)
        ex.check()
    for split in (True, False):
        for _ in range(3):
            run(split)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run(split)
        e1.record()
        barrier(world)
        res["per_leaf" if split else "one_bucket"] = round(e0.elapsed_time(e1) / reps, 4)
    res["bytes_all_reduced"] = 4 * 11 * n
    res["bytes_all_gathered_per_rank"] = 12 * n if wl.mvsh else 0
    return res


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

    wl = Workload(args.workload, world, rank, dev, args.gaussians, args.exchange)
    views, leaves = wl.views, wl.leaves

    for _ in range(args.warmup):
        wl.step(wl.upstream)
    barrier(world)

    # -------------------------------------------------- timed: value ----
    clocks = ClockSampler(local)
    clocks.start()
    capi.timing_reset()
    capi.timing_enable(True)
    launches0 = capi.launch_count()
    t_ms = time_steps(wl, args.steps, 0, world)
    launches = capi.launch_count() - launches0
    capi.timing_enable(False)
    timed = {}
    for name in ("rasterize_fwd", "rasterize_bwd", "projection_utgs", "isect_count", "isect_emit_sort", "sh_fwd",
                 "sh_bwd", "sh_positions_bwd", "sh_coeffs_bwd_multi", "lbs_fwd", "lbs_bwd"):
        ms, n = capi.timing_query(name)
        if n:
            timed[name] = (ms, n)
    capi.timing_reset()

    # ---------------------------------------------------- timed: e2e ----
    # Each step's upstream gradients come from pinned host memory and each
    # step's loss goes back to pinned host memory and is read on the host.
    # The copies are buffered on a copy stream (later steps' inputs arrive
    # while step k computes) and the loss of step k is read while the next
    # steps run, as a training loop with asynchronous loss logging does.
    host = [[t.cpu().pin_memory() for t in g] for g in wl.upstream]
    h2d = sum(t.numel() * t.element_size() for g in host for t in g)
    comp = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(device=dev)
    NB = 3  # buffers: the host reads step k's loss while steps k+1 and k+2 are queued
    dbufs = [[[torch.empty_like(t) for t in g] for g in wl.upstream] for _ in range(NB)]
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
            loss = wl.step(dbufs[b])
            ev_free[b].record(comp)
            loss_host[b].copy_(loss.detach(), non_blocking=True)
            ev_out[b].record(comp)
            pending.append(b)
        for p in pending:
            ev_out[p].synchronize()
            losses.append(float(loss_host[p]))

    e2e_steps(max(1, args.warmup // 2))
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_steps(args.steps, start_event=e0)
    e1.record()
    barrier(world)
    e2e_ms = e0.elapsed_time(e1)
    assert all(math.isfinite(v) for v in losses)

    # ----------------------------------------------------- phases ----
    phases = phase_times(wl, min(10, args.steps), world)
    xprobe = exchange_probe(wl, world, dev)

    extra = {}
    main_default = args.workload == "c2"
    # ------------------------------ timed: C4 lidar rays/s (c2 scene) ----
    if main_default and not args.no_lidar:
        extra["lidar"] = lidar_leg(args, wl, world, rank, dev)
    # --------------------------------------- strong scaling: rig, C5 ----
    if main_default and not args.no_rig:
        extra["rig"] = strong_leg(args, "c3-8", world, rank, dev)
        extra["rig"]["c3"] = strong_leg(args, "c3", world, rank, dev, phases=False)
    if main_default and not args.no_c5:
        extra["c5"] = strong_leg(args, "c5", world, rank, dev, roofline=False)

    clk = clocks.stop()

    t_ms, e2e_ms = max_over_ranks([t_ms, e2e_ms], world, dev)

    # ------------------------------------------------ roofline inputs ----
    roof, stages = None, None
    if rank == 0 and views:
        roof, n_isects = roofline_fields(wl, timed, args.steps, dev)
        stages = stage_fields(wl, timed, n_isects)

    wl.red.remove()
    if wl.ex is not None:
        wl.ex.check()  # raises if a barrier of the exchange timed out
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    cpu = None
    if world == 1 and not args.no_cpu_baseline and args.workload == "c2":
        from oracle import oracle as O
        O.set_threads(cpu_count())
        t, px = oracle_view(scenes.street_scene(wl.n_gauss), wl.specs[0])
        cpu = {"value": round(px / t / 1e6, 4), "unit": "Mpix/s", "cores": O.num_threads(), "kind": "port",
               "sample": "one full C2 view (projection, tiling, SH, fwd+bwd compositing) on the CPU oracle"}

    px_total = wl.px_per_step * args.steps
    value = px_total / (t_ms * 1e-3) / 1e6
    e2e = px_total / (e2e_ms * 1e-3) / 1e6
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "Mpix/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 3), "higher_is_better": True,
        "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded {args.workload.upper()} scene)",
        "config": workload_config(args.workload, world, wl.n_gauss, wl.exchange),
        "e2e": {"value": round(e2e, 2), "unit": "Mpix/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "note": "per step: the upstream gradient images in (pinned host -> device), the step's scalar "
                        "result (mean alpha) out; rendered images and parameter gradients stay on the device, "
                        "as in a training loop"},
        "gpu_launches": int(launches), "gpu_launches_per_step": round(launches / args.steps, 1),
        "clocks": clk, "roofline": roof, "cpu_baseline": cpu, "phases": phases, "stages": stages,
        "exchange_alone_ms": xprobe,
        "exchange": wl.exchange,
    }
    line.update(extra)
    print(json.dumps(line), flush=True)


def lidar_leg(args, wl, world, rank, dev):
    """C4: the 128 x 2048 lidar over the C2 scene (intensity channel),
    fwd+bwd, weak scaling (every rank renders the sweep)."""
    import torch
    import xsimgs_b200 as X
    from xsimgs_b200 import scenes
    lspec = scenes.c4_lidar()
    lcam = lspec.make(dev)
    LW, LH = lspec.width, lspec.height
    gen = torch.Generator().manual_seed(3)
    inten = torch.rand(wl.n_gauss, 1, generator=gen).to(dev).requires_grad_(True)
    lg = [t.to(dev) for t in scenes.upstream_grads(LH, LW, 1, seed=40 + rank)]
    L = wl.leaves

    class Lidar:
        def __init__(self, phm):
            self.phm = phm
            self.upstream = None

        def step(self, _grads, marks=None):
            for v in list(L.values()) + [inten]:
                v.grad = None
            color, depth, alpha, _ = X.ut_gs_render(lcam, L["means"], L["scales"], L["quats"], L["opacities"], LW,
                                                    LH, colors=inten, use_phm=self.phm)
            torch.autograd.backward([color, depth, alpha], lg)
            wl.red.wait()

    out = {}
    for phm in (False, True):
        ms = time_steps(Lidar(phm), args.steps, args.warmup, world)
        out["phm" if phm else "central"] = ms
    c, p = max_over_ranks([out["central"], out["phm"]], world, dev)
    rays = world * LW * LH * args.steps
    return {"metric": "lidar rays/s (C4: 128 beams x 2048 azimuth bins, the C2 scene, depth + intensity + "
                      "ray-drop alpha, fwd+bwd)", "unit": "rays/s", "scaling": "weak",
            "value": round(rays / (c * 1e-3)), "ms_per_step": round(c / args.steps, 3),
            "phm": {"value": round(rays / (p * 1e-3)), "ms_per_step": round(p / args.steps, 3)}}


def strong_leg(args, name, world, rank, dev, phases=True, roofline=True):
    """A strong-scaling workload (all views of the rig per step, sharded over
    the ranks) timed like the main line; Mpix/s of the whole job, and the
    compositing kernels' FP32 fractions on rank 0's views."""
    import torch
    from xsimgs_b200 import capi
    wl = Workload(name, world, rank, dev, exchange=args.exchange)
    steps = max(3, min(args.steps, 20))
    ms = time_steps(wl, steps, max(3, args.warmup), world)
    ph = phase_times(wl, min(5, steps), world) if phases else None
    ms, = max_over_ranks([ms], world, dev)
    roof = None
    if roofline:
        # a few more steps with the library's timed scopes on (every rank
        # steps: the exchange is collective); the pair counts on rank 0
        capi.timing_reset()
        capi.timing_enable(True)
        time_steps(wl, 3, 0, world)
        capi.timing_enable(False)
        timed = {}
        for kname in ("rasterize_fwd", "rasterize_bwd"):
            t, n = capi.timing_query(kname)
            if n:
                timed[kname] = (t, n)
        capi.timing_reset()
        if rank == 0 and wl.views and timed:
            r, _ = roofline_fields(wl, timed, 3, dev)
            roof = {"bwd": {k: r[k] for k in ("achieved", "frac", "avg_launch_ms")},
                    "bwd_executed_frac": r["executed"]["frac"], "fwd": r["fwd"], "peak": r["peak"],
                    "unit": r["unit"], "views": len(wl.views), "pairs": r["pairs"],
                    "fwd_warp_entries": r["fwd_warp_entries"]}
    if wl.ex is not None:
        wl.ex.check()
    wl.red.remove()
    out = {"metric": f"Gaussian-render fwd+bwd Mpix/s ({name.upper()})", "unit": "Mpix/s", "scaling": "strong",
           "value": round(wl.px_per_step * steps / (ms * 1e-3) / 1e6, 2), "ms_per_step": round(ms / steps, 3),
           "steps": steps, "config": workload_config(name, world, wl.n_gauss, wl.exchange)}
    if ph is not None:
        out["phases_rank0"] = ph
    if roof is not None:
        out["roofline_rank0"] = roof
    del wl
    torch.cuda.empty_cache()
    return out


def roofline_fields(wl, timed, steps, dev):
    """Roofline of the dominant kernel (compositing backward, FP32-issue
    bound) with pair counts measured live on this rank's views."""
    import torch
    import xsimgs_b200 as X
    from xsimgs_b200 import capi, roofline
    fl_b = fl_bx = fl_f = 0.0
    pairs = {"evaluated_fwd": 0, "evaluated_bwd": 0, "contributing": 0}
    # the forward's (warp, list entry) work: staged, passing the warp's cone
    # test, passing the per-lane quadric test, evaluated (pair counters 2-5)
    warp_work = {"staged": 0, "cone_passed": 0, "quadric_passed": 0, "evaluated": 0}
    n_isects = 0
    L = wl.leaves
    for sp, cam in wl.views:
        W, H = sp.width, sp.height
        cnt = torch.zeros(12, dtype=torch.int64, device=dev)
        capi.set_pair_counters(cnt.data_ptr())
        with torch.no_grad():
            colors = X.spherical_harmonics_fused(L["sh"], L["means"], cam.t0, DEG)
            td = X.ut_gs_tiling(cam, L["means"], L["scales"], L["quats"], W, H, opacity=L["opacities"])
            ro, rd = cam.camera_rays(W, H)
            _, _, alpha, last = X._C.rasterize_eval3d_fwd(
                means=L["means"], quats=L["quats"], scales=L["scales"], colors=colors.unsqueeze(0),
                opacities=L["opacities"].view(1, -1), image_width=W, image_height=H, tile_size_width=16,
                tile_size_height=16, ray_origs=ro, ray_dirs=rd, tile_offsets=td["isect_offsets"],
                flatten_ids=td["flatten_ids"])
        torch.cuda.synchronize()
        capi.set_pair_counters(None)
        cl = cnt.tolist()
        n_eval_f, n_contrib = int(cl[0]), int(cl[1])
        for key, i in (("staged", 2), ("cone_passed", 3), ("quadric_passed", 4), ("evaluated", 5)):
            warp_work[key] += int(cl[i])
        n_isects += int(td["flatten_ids"].numel())
        touched = int((td["radii"] > 0).all(-1).sum())
        # backward replays every pair up to each pixel's last contributor
        tw = (W + 15) // 16
        ty = torch.arange(H, device=dev) // 16
        tx = torch.arange(W, device=dev) // 16
        start = td["isect_offsets"].view(-1)[(ty[:, None] * tw + tx[None, :])]
        n_eval_b = int(torch.where(alpha > 0, last - start + 1, torch.zeros_like(last)).sum())
        # the render step's rays come from the camera: no ray gradients
        fl_b += roofline.bwd_flops(n_eval_b, n_contrib, 3, ray_grads=False)
        fl_bx += roofline.bwd_flops_executed(n_eval_b, n_contrib, touched, 3, ray_grads=False)
        fl_f += roofline.fwd_flops(n_eval_f, n_contrib, 3)
        pairs["evaluated_fwd"] += n_eval_f
        pairs["evaluated_bwd"] += n_eval_b
        pairs["contributing"] += n_contrib
    peak = fp32_peak(dev)
    bwd_ms, bwd_n = timed.get("rasterize_bwd", (0.0, 0))
    fwd_ms, fwd_n = timed.get("rasterize_fwd", (0.0, 0))
    bwd_step, fwd_step = bwd_ms / steps, fwd_ms / steps
    ach_b = fl_b / (bwd_step * 1e-3) / 1e12
    ach_bx = fl_bx / (bwd_step * 1e-3) / 1e12
    ach_f = fl_f / (fwd_step * 1e-3) / 1e12
    c2_full = wl.name == "c2" and wl.n_gauss == N_C2
    pk = peak / 1e12
    roof = {"kernel": "rasterize_bwd (raster_bwd_px2_kernel<3>: static scene, no ray gradients, two pixels a lane)",
            "bound": "fp32", "achieved": round(ach_b, 2), "peak": round(pk, 2), "unit": "TFLOP/s",
            "frac": round(ach_b / pk, 3),
            "executed": {"achieved": round(ach_bx, 2), "frac": round(ach_bx / pk, 3),
                         "note": "FLOPs the kernel executes: the quat/scale VJP runs once per Gaussian in the "
                                 "finalize pass, not per contributing pair"},
            "traffic": roofline.BWD_DRAM_BYTES_C2 if c2_full else None,
            "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum, one capture of this kernel "
                               "on this workload (bytes per launch)") if c2_full else None,
            "peak_source": "measured: FP32 FMA probe in this run (MEASURED_PEAKS.json has only HBM and bf16)",
            "avg_launch_ms": round(bwd_ms / max(1, bwd_n), 4),
            "flops_per_launch": fl_b / len(wl.views), "pairs": pairs, "fwd_warp_entries": warp_work,
            "fwd": {"achieved": round(ach_f, 2), "avg_launch_ms": round(fwd_ms / max(1, fwd_n), 4),
                    "frac": round(ach_f / pk, 3)}}
    return roof, n_isects


def stage_fields(wl, timed, n_isects):
    """Per-stage launch time and HBM fraction (algorithmic bytes per launch
    over the launch's mean device time, against the measured copy peak)."""
    from xsimgs_b200 import roofline
    peak = hbm_peak()
    out = {}
    n = wl.n_gauss
    views = len(wl.views)
    for name, (ms, cnt) in timed.items():
        if name.startswith("rasterize"):
            continue
        avg = ms / cnt
        by = roofline.stage_bytes(name, n, sh_bands=(DEG + 1) ** 2,
                                  views=(wl.world * wl.k_max if name == "sh_coeffs_bwd_multi" else views))
        d = {"launches": cnt, "avg_launch_ms": round(avg, 4)}
        if by is not None:
            gbs = by / (avg * 1e-3) / 1e9
            d.update({"bytes_per_launch": by, "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 3)})
        if name == "isect_emit_sort":
            d["isects_per_launch"] = n_isects // max(1, views)
        out[name] = d
    out["hbm_peak_gbs"] = peak
    out["hbm_peak_source"] = "MEASURED_PEAKS.json hbm_gbs (copy, read + write bytes)"
    return out


def hbm_peak() -> float:
    try:
        return float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except Exception:
        return 6650.0  # fallback figure of this pool


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
