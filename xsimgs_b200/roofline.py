"""Frozen algorithmic work model of the compositing kernels (FLOP counts per
pair), used by bench.py for `roofline.achieved`.

Counts are of the reference's expressions (csrc/rasterization/eval3d_fwd.cu
and eval3d_bwd.cu), one FLOP per add/mul/compare/min, two per FMA, and one
per MUFU operation (rsqrt, ex2, rcp), independent of how a kernel schedules
them:

forward, every evaluated (pixel, Gaussian) pair (eval3d_fwd.cu:116-131)
    o - mu 3, M (o - mu) 15, M d 15, |Md|^2 5, normalise 3 + rsqrt 1,
    cross 9, |cross|^2 5, power 1, exp 1 + ex2 1, opacity * 1, min 1,
    alpha test 1                                                      = 62
forward, every contributing pair (eval3d_fwd.cu:133-153)
    hit distance 5 + 5 + 1 + div 1, T (1 - alpha) 2, test 1, vis 1,
    depth 2, colour 2 C                                            = 18 + 2C
backward, every pair up to the pixel's last contributor (eval3d_bwd.cu:172-206)
    the forward's 62
backward, every contributing pair (eval3d_bwd.cu:219-271): 1/(1-alpha),
    T, fac 4; colour grad C; v_alpha 4 C + 7; hit-distance terms 30;
    power-term branch 135 (cross products, normalise backward, outer
    products, M^T products); quat/scale VJP 136; opacity 1; buffers 2 C + 2
                                                                  = 315 + 7 C
"""

FWD_EVAL = 62
BWD_EVAL = 62


def fwd_contrib(cdim: int) -> int:
    return 18 + 2 * cdim


# per contributing pair, only for the per-pixel ray gradients (v_ray_d =
# M^T v_grd: 9 mul + 6 add; accumulating v_ray_o / v_ray_d: 6 add); a
# backward that is not asked for ray gradients does not owe them
RAY_GRAD_FLOPS = 21


def bwd_contrib(cdim: int, ray_grads: bool = True) -> int:
    return 315 + 7 * cdim - (0 if ray_grads else RAY_GRAD_FLOPS)


def fwd_flops(n_eval: int, n_contrib: int, cdim: int) -> float:
    return float(FWD_EVAL * n_eval + fwd_contrib(cdim) * n_contrib)


def bwd_flops(n_eval_bwd: int, n_contrib: int, cdim: int, ray_grads: bool = True) -> float:
    return float(BWD_EVAL * n_eval_bwd + bwd_contrib(cdim, ray_grads) * n_contrib)


# DRAM bytes per launch of the compositing backward (static scene, no ray
# gradients, two pixels a lane, the forward's contributor masks) on the C2
# view (1M Gaussians, 1920x1080, 16x16 tiles), dram__bytes_read.sum +
# dram__bytes_write.sum from one capture:
#   ncu --set full --clock-control none -k "regex:raster_(fwd|bwd_px2)" -s 2 -c 2 \
#       python bench.py --steps 2 --warmup 1 --no-cpu-baseline --no-lidar --no-rig --no-c5
BWD_DRAM_BYTES_C2 = 270.41e6 + 35.77e6


# The quaternion / scale part of the backward (quat_scale_to_preci_half_vjp,
# rasterization/utils.h:232-263) is linear in dL/dM for a fixed Gaussian:
# this package's backward sums dL/dM over the pairs and applies the VJP once
# per Gaussian in its finalize pass, so of the algorithmic count above it
# executes 136 FLOP per contributing pair fewer (and 136 per Gaussian more).
QUAT_SCALE_VJP = 136


def bwd_flops_executed(n_eval_bwd: int, n_contrib: int, n_gauss_touched: int, cdim: int,
                       ray_grads: bool = True) -> float:
    return bwd_flops(n_eval_bwd, n_contrib, cdim, ray_grads) - QUAT_SCALE_VJP * (n_contrib - n_gauss_touched)


# Algorithmic HBM bytes per launch of the memory-bound stages (inputs read
# once, outputs written once), by the timing names of the C ABI:
#   projection_utgs   means, scales 12 + 12, quats 16, opacity 4 read;
#                     flag 1, radii 8, means2d 8, depth 4 written    65 B / Gaussian
#   isect_count       means2d, radii read, count written             20 B / Gaussian
#   sh_fwd            position 12 + coefficients 12 K read, colour 12 written
#   sh_bwd            position, coefficients, colour gradient read; coefficient
#                     and position gradients written
#   sh_positions_bwd  position, coefficients, J colour gradients read; position
#                     gradient written
#   sh_coeffs_bwd_multi  position, J colour gradients read; coefficient
#                     gradient written
#   lbs_fwd           vertex 12, quat 16, 24 weights 96 read; position 12,
#                     rotation 16, velocity 12, mask 1 written     165 B / element
#   lbs_bwd           vertex, quat, weights and the position / rotation /
#                     velocity gradients read; vertex, quat, weight gradients
#                     written                                      288 B / element
def stage_bytes(name: str, n: int, sh_bands: int = 16, views: int = 1) -> float | None:
    k = 12 * sh_bands
    table = {
        "projection_utgs": 65, "projection_utgs_phm": 65,
        "isect_count": 20,
        "sh_fwd": 12 + k + 12,
        "sh_bwd": 12 + k + 12 + k + 12,
        "sh_positions_bwd": 12 + k + 12 * views + 12,
        "sh_coeffs_bwd_multi": 12 + 12 * views + k,
        "lbs_fwd": 165,
        "lbs_bwd": 288,
    }
    per = table.get(name)
    return None if per is None else float(per) * n
