"""The camera-parameter gradients of the CPU oracle (oracle/xsg_oracle_camgrad.cpp)
against float64 autograd of an independent torch restatement of the ray and
pixel-time forward (ray_kernels.h:8-59, camera.h:89-131, the impls'
pixel_to_camera_ray): rotation through the quaternion's matrix instead of the
quaternion polynomial, the fisheye angle through one differentiable Newton
step at the converged root (which has the implicit-function derivative), and
the spherical angle limits held constant (the reference gives them no ray
gradient).  Covers every camera model, world / camera space, normalised or
raw rays, no / small / large angular velocity (both branches of the
axis-angle series), and a non-unit q0 with a negative real part."""
import numpy as np
import pytest
import torch

from oracle import oracle as O


DIST8 = (-0.25, 0.07, 3e-4, -2e-4, -0.008, 0.03, 0.002, 0.0005)  # k1 k2 p1 p2 k3 k4 k5 k6


def distort_t(x, y, k):
    """OpenCV rational + tangential distortion of (x, y) (torch, any dtype)."""
    k1, k2, p1, p2, k3, k4, k5, k6 = (k[i] for i in range(8))
    r2 = x * x + y * y
    sc = (1 + r2 * (k1 + r2 * (k2 + r2 * k3))) / (1 + r2 * (k4 + r2 * (k5 + r2 * k6)))
    return (x * sc + 2 * p1 * x * y + p2 * (r2 + 2 * x * x), y * sc + p1 * (r2 + 2 * y * y) + 2 * p2 * x * y)


def undistort_t(xd, yd, k):
    """D(x) = xd solved by Newton with a differentiable last step: the step
    at the converged root has the implicit-function derivative in k and xd."""
    with torch.no_grad():
        x, y = xd.clone(), yd.clone()
        kd = k.detach()
        for _ in range(20):
            x.requires_grad_(True)
            y.requires_grad_(True)
            with torch.enable_grad():
                fx, fy = distort_t(x, y, kd)
                jxx, jxy = torch.autograd.grad(fx.sum(), (x, y), retain_graph=True)
                jyx, jyy = torch.autograd.grad(fy.sum(), (x, y))
            det = jxx * jyy - jxy * jyx
            rx, ry = fx.detach() - xd, fy.detach() - yd
            x = (x - (jyy * rx - jxy * ry) / det).detach()
            y = (y - (jxx * ry - jyx * rx) / det).detach()
    x.requires_grad_(True)
    y.requires_grad_(True)
    with torch.enable_grad():
        fx, fy = distort_t(x, y, kd)
        jxx, jxy = torch.autograd.grad(fx.sum(), (x, y), retain_graph=True)
        jyx, jyy = torch.autograd.grad(fy.sum(), (x, y))
    x, y = x.detach(), y.detach()
    det = jxx * jyy - jxy * jyx
    rx, ry = distort_t(x, y, k)
    rx, ry = rx - xd, ry - yd
    return x - (jyy * rx - jxy * ry) / det, y - (jxx * ry - jyx * rx) / det


def _base(words, w=(0.01, -0.02, 0.3), q0=(0.9, 0.1, -0.3, 0.2)):
    p = np.zeros(words, np.float32)
    p[0:4] = q0
    p[4:7] = (0.5, -1.0, 1.6)
    p[7:10] = (3.0, 0.5, -0.2)
    p[10:13] = w
    p[14:16] = (0.02, 0.03)
    p[16] = 0.01
    p[17] = 0.02
    return p


def camera_pack(kind, w=(0.01, -0.02, 0.3), q0=(0.9, 0.1, -0.3, 0.2)):
    p = _base(O.WORDS[kind], w, q0)
    i = O.INTR[kind]
    if kind in ("pinhole", "fisheye", "distorted"):
        p[i:i + 4] = (0.45, 0.6, 0.52, 0.47)
        if kind == "fisheye":
            p[i + 4:i + 8] = (0.03, -0.02, 0.01, -0.004)
        if kind == "distorted":
            p[i:i + 2] = (0.9, 1.2)  # the image stays inside the model's monotone range
            p[i + 4:i + 12] = DIST8
            p[i + 12] = 4.0
    else:
        p[i:i + 4] = (0.1, 6.0, -0.4, 0.9)  # phi_min, phi_range, theta_min, theta_range
    return p


def _grid_uv(kind, W, H, elev):
    u = ((np.arange(W, dtype=np.float32) + np.float32(0.5)) / np.float32(W)).astype(np.float32)
    if kind == "lidar":
        v = elev.astype(np.float32)
    else:
        v = ((np.arange(H, dtype=np.float32) + np.float32(0.5)) / np.float32(H)).astype(np.float32)
    U, V = np.meshgrid(u, v)
    return U, V


def _fe_solve_f32(delta, k):
    """The forward's float32 fisheye solve (vectorised), for the validity decision."""
    f = np.float32
    k1, k2, k3, k4 = (f(x) for x in k)
    th = delta.astype(np.float32).copy()
    res = np.zeros_like(th)
    done = np.zeros(th.shape, bool)
    for _ in range(20):
        t2 = th * th
        d = t2 * k4 + k3
        d = t2 * d + k2
        d = t2 * d + k1
        d = t2 * d + f(1)
        r = th * d - delta
        dd = t2 * f(9) * k4 + f(7) * k3
        dd = t2 * dd + f(5) * k2
        dd = t2 * dd + f(3) * k1
        dd = t2 * dd + f(1)
        nt = np.clip(th - r / np.maximum(dd, f(0.1)), f(0), f(np.pi)).astype(np.float32)
        th = np.where(done, th, nt)
        res = np.where(done, res, r)
        done |= np.abs(r) < f(1e-6)
    t2 = th * th
    dd = t2 * f(9) * k4 + f(7) * k3
    dd = t2 * dd + f(5) * k2
    dd = t2 * dd + f(3) * k1
    dd = t2 * dd + f(1)
    return th, res, dd


def _rotmat(q):
    w, x, y, z = q.unbind(-1)
    return torch.stack([
        torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)], -2)


def _qmul(a, b):
    aw, av = a[..., :1], a[..., 1:]
    bw, bv = b[..., :1], b[..., 1:]
    return torch.cat([aw * bw - (av * bv).sum(-1, keepdim=True), aw * bv + bw * av + torch.cross(av, bv, dim=-1)], -1)


def torch_rays(kind, pk, W, H, world, normalized, elev=None):
    U, V = _grid_uv(kind, W, H, elev)
    Ut, Vt = torch.tensor(U, dtype=torch.float64), torch.tensor(V, dtype=torch.float64)
    i = O.INTR[kind]
    if kind in ("pinhole", "fisheye", "distorted"):
        ux, uy = (Ut - pk[i + 2]) / pk[i], (Vt - pk[i + 3]) / pk[i + 1]
        if kind == "pinhole":
            ray = torch.stack([ux, uy, torch.ones_like(ux)], -1)
        elif kind == "distorted":
            x, y = undistort_t(ux, uy, pk[i + 4:i + 12])
            ray = torch.stack([x, y, torch.ones_like(x)], -1)
        else:
            k = pk[i + 4:i + 8]
            p32 = pk.detach().numpy().astype(np.float32)
            uxf = (U - p32[i + 2]) / p32[i]
            uyf = (V - p32[i + 3]) / p32[i + 1]
            dlf = np.sqrt(uxf * uxf + uyf * uyf)
            thf, resf, derf = _fe_solve_f32(dlf, p32[i + 4:i + 8])
            valid = (thf > 0) & (dlf > 1e-8) & (np.abs(resf) < 1e-5) & (derf > 1e-3)
            assert valid.all(), "test camera must converge everywhere"
            delta = torch.sqrt(ux * ux + uy * uy)
            with torch.no_grad():
                th = torch.tensor(thf, dtype=torch.float64)
                for _ in range(6):
                    t2 = th * th
                    th = th - (th * (1 + t2 * (k[0] + t2 * (k[1] + t2 * (k[2] + t2 * k[3])))) - delta) / (
                        1 + t2 * (3 * k[0] + t2 * (5 * k[1] + t2 * (7 * k[2] + t2 * 9 * k[3]))))
            t2 = th * th
            res = th * (1 + t2 * (k[0] + t2 * (k[1] + t2 * (k[2] + t2 * k[3])))) - delta
            der = 1 + t2 * (3 * k[0] + t2 * (5 * k[1] + t2 * (7 * k[2] + t2 * 9 * k[3])))
            th = th - res / der.detach()
            s = torch.sin(th) / delta
            ray = torch.stack([s * ux, s * uy, torch.cos(th)], -1)
    else:
        lim = pk[i:i + 4].detach()
        az, el = lim[0] + Ut * lim[1], lim[2] + Vt * lim[3]
        ray = torch.stack([torch.cos(el) * torch.sin(az), torch.cos(el) * torch.cos(az), torch.sin(el)], -1)
    nray = ray / ray.norm(dim=-1, keepdim=True) if normalized else ray
    if not world:
        return torch.zeros_like(nray), nray
    dt = pk[16] + Ut * pk[14] + Vt * pk[15] - pk[17]
    q0 = pk[0:4]
    q0s = q0 / q0.norm() * (1.0 if float(q0[0].detach()) >= 0 else -1.0)
    a = pk[10:13] * dt[..., None]
    th2 = (a * a).sum(-1)
    small = th2 < 1e-4
    ths = torch.sqrt(torch.where(small, torch.ones_like(th2), th2))
    sc = torch.where(small, 0.5 - th2 / 48, torch.sin(0.5 * ths) / ths)
    ch = torch.where(small, 1 - th2 / 8 + th2 * th2 / 384, torch.cos(0.5 * ths))
    qa = torch.cat([ch[..., None], sc[..., None] * a], -1)
    q = _qmul(qa, q0s.expand_as(qa))
    ray_d = (_rotmat(q) @ nray[..., None])[..., 0]
    ray_o = pk[4:7] + pk[7:10] * dt[..., None]
    return ray_o, ray_d


def _elev(H):
    return np.sort(np.random.default_rng(5).uniform(0.02, 0.98, H)).astype(np.float32)


def _check(got, want, what):
    """Per camera tensor: |got - want| <= 1e-6 * (|want| + max|want| of the tensor)."""
    groups = [(0, 4), (4, 7), (7, 10), (10, 13), (13, 14), (14, 16), (16, 17), (17, 18), (18, 20), (20, 22),
              (22, 24), (24, 28), (28, 32), (32, 33), (33, 36)]
    for a, b in groups:
        if a >= len(want):
            break
        g, w = got[a:b], want[a:b]
        bound = 1e-6 * (np.abs(w) + np.abs(w).max()) + 1e-12
        assert (np.abs(g - w) <= bound).all(), f"{what} words {a}:{b}: {g} vs {w}"


@pytest.mark.parametrize("kind", ["pinhole", "fisheye", "spherical", "lidar", "distorted"])
@pytest.mark.parametrize("world,normalized", [(True, True), (False, True), (True, False), (False, False)])
def test_oracle_ray_backward_is_autograd(kind, world, normalized):
    W, H = 24, 16
    elev = _elev(H) if kind == "lidar" else None
    pack = camera_pack(kind)
    rng = np.random.default_rng(3)
    go = (rng.normal(size=(H, W, 3)) + 0.3).astype(np.float32)
    gd = (rng.normal(size=(H, W, 3)) + 0.3).astype(np.float32)
    got = O.camera_rays_bwd(kind, pack, W, H, go, gd, world, normalized, elev=elev)
    pk = torch.tensor(pack.astype(np.float64), requires_grad=True)
    ro, rd = torch_rays(kind, pk, W, H, world, normalized, elev)
    loss = (ro * torch.tensor(go, dtype=torch.float64)).sum() + (rd * torch.tensor(gd, dtype=torch.float64)).sum()
    if loss.requires_grad:  # camera-space range-image rays depend on no differentiable word
        loss.backward()
    want = pk.grad.numpy() if pk.grad is not None else np.zeros(len(pack))
    if kind == "lidar":
        want[22:24] = 0.0
    _check(got, want, f"{kind} world={world} normalized={normalized}")
    assert got[13] == 0.0
    if kind in ("spherical", "lidar"):
        assert not got[18:].any()
    if kind in ("fisheye", "distorted"):
        assert not got[18:20].any()  # padding before the 16-byte aligned impl


@pytest.mark.parametrize("w", [(0.0, 0.0, 0.0), (0.01, -0.02, 0.05), (2.0, -1.0, 9.0)])
@pytest.mark.parametrize("q0", [(0.9, 0.1, -0.3, 0.2), (-1.2, 0.4, 0.7, -0.1)])
def test_oracle_ray_backward_motion_branches(w, q0):
    """Angular velocity zero, inside the series branch of the axis angle
    (|w dt| < 1e-2) and far outside it (up to ~0.5 rad), for a unit q0 and a
    non-unit one with a negative real part (std() flips it)."""
    W, H = 20, 12
    pack = camera_pack("pinhole", w=w, q0=q0)
    pack[14:16] = (0.02, 0.05)
    rng = np.random.default_rng(4)
    go = (rng.normal(size=(H, W, 3)) + 0.3).astype(np.float32)
    gd = (rng.normal(size=(H, W, 3)) + 0.3).astype(np.float32)
    got = O.camera_rays_bwd("pinhole", pack, W, H, go, gd)
    pk = torch.tensor(pack.astype(np.float64), requires_grad=True)
    ro, rd = torch_rays("pinhole", pk, W, H, True, True)
    ((ro * torch.tensor(go, dtype=torch.float64)).sum() + (rd * torch.tensor(gd, dtype=torch.float64)).sum()).backward()
    _check(got, pk.grad.numpy(), f"w={w} q0={q0}")


@pytest.mark.parametrize("kind", ["pinhole", "lidar"])
@pytest.mark.parametrize("delta", [False, True])
def test_oracle_pixel_time_backward_is_autograd(kind, delta):
    W, H = 24, 16
    elev = _elev(H) if kind == "lidar" else None
    pack = camera_pack(kind)
    rng = np.random.default_rng(6)
    g = rng.normal(size=(H, W)).astype(np.float32)
    got, _ = O.pixel_time_bwd(kind, pack, g, delta, W=W, H=H, elev=elev)
    pk = torch.tensor(pack.astype(np.float64), requires_grad=True)
    U, V = _grid_uv(kind, W, H, elev)
    t = pk[16] + torch.tensor(U, dtype=torch.float64) * pk[14] + torch.tensor(V, dtype=torch.float64) * pk[15]
    if delta:
        t = t - pk[17]
    (t * torch.tensor(g, dtype=torch.float64)).sum().backward()
    _check(got, pk.grad.numpy()[:len(got)] * (np.arange(len(got)) < 22), f"{kind} delta={delta}")
    uv = rng.uniform(0, 1, size=(50, 2)).astype(np.float32)
    gu = rng.normal(size=50).astype(np.float32)
    got, d_uv = O.pixel_time_bwd(kind, pack, gu, delta, uv=uv)
    pk.grad = None
    tuv = torch.tensor(uv, dtype=torch.float64, requires_grad=True)
    t = pk[16] + tuv[:, 0] * pk[14] + tuv[:, 1] * pk[15] - (pk[17] if delta else 0.0)
    (t * torch.tensor(gu, dtype=torch.float64)).sum().backward()
    _check(got, pk.grad.numpy(), f"{kind} uv delta={delta}")
    np.testing.assert_allclose(d_uv, tuv.grad.numpy(), rtol=1e-6)
