// xsimgs-b200 CPU ORACLE — test infrastructure only, never a product path.
//
// Camera-parameter gradients of the per-pixel rays and pixel times: a scalar
// restatement of the reference's camera_ray_backward_kernel_cuda
// (include/cameras/ray_kernels.h:61-123), the impl backward passes
// (csrc/cameras/perspective.cu:18-34, csrc/cameras/fisheye_opencv.cu:77-141;
// the spherical and lidar impls keep BaseCameraImpl's empty backward,
// include/cameras/base_camera_impl.h:20-23) and the pixel-time backward
// kernels (include/cameras/time_kernels.h:115-297).
//
// PARITY STATUS: unpinned (the reference cannot be built here and ships no
// golden vectors).  The quaternion steps the reference takes from pytoast
// (apply_backward, apply_angular_velocity_backward, std_backward) are
// restated from their mathematics: the oracle is checked against float64
// autograd of an independent torch restatement in tests/.
//
// Arithmetic: every per-pixel gradient and the sums are in double; the
// pixel's uv and the fisheye convergence test (which decides whether a pixel
// gets an intrinsics gradient) are evaluated in float32 as the forward does.

#include <cmath>
#include <cstdint>
#include <vector>

namespace {

struct D3 { double x, y, z; };
inline D3 operator+(D3 a, D3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline D3 operator-(D3 a, D3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline D3 operator*(double s, D3 a) { return {s * a.x, s * a.y, s * a.z}; }
inline double dot(D3 a, D3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline D3 cross(D3 a, D3 b) { return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }

struct DQ { double w; D3 v; };
inline DQ qmul(DQ a, DQ b) { return {a.w * b.w - dot(a.v, b.v), a.w * b.v + b.w * a.v + cross(a.v, b.v)}; }
// R(q) p for unit q
inline D3 qrot(DQ q, D3 p) {
    const D3 t = 2.0 * cross(q.v, p);
    return p + q.w * t + cross(q.v, t);
}

enum { CAM_PINHOLE = 0, CAM_FISHEYE = 1, CAM_SPHERICAL = 2, CAM_LIDAR = 3, CAM_DISTORTED = 4 };

// OpenCV 8-coefficient distortion D(x) = x scale(r2) + delta(x) in double,
// with its symmetric Jacobian (distorted_perspective.cu:43-78); k = the
// eight coefficients k1 k2 p1 p2 k3 k4 k5 k6 (pack words 24..31).
struct DistD {
    double scale, denom, dx, dy, juu, juv, jvv;
    double det() const { return juu * jvv - juv * juv; }
};
inline DistD dist_state(const float* k, double u, double v) {
    const double k1 = k[0], k2 = k[1], p1 = k[2], p2 = k[3], k3 = k[4], k4 = k[5], k5 = k[6], k6 = k[7];
    const double r2 = u * u + v * v;
    const double num = 1 + r2 * (k1 + r2 * (k2 + r2 * k3));
    const double den = 1 + r2 * (k4 + r2 * (k5 + r2 * k6));
    const double sc = num / den;
    const double dsc = ((k1 + r2 * (2 * k2 + 3 * k3 * r2)) * den - num * (k4 + r2 * (2 * k5 + 3 * k6 * r2))) /
                       (den * den);
    return {sc, den, 2 * p1 * u * v + p2 * (r2 + 2 * u * u), p1 * (r2 + 2 * v * v) + 2 * p2 * u * v,
            sc + 2 * u * u * dsc + 2 * p1 * v + 6 * p2 * u, 2 * u * v * dsc + 2 * p1 * u + 2 * p2 * v,
            sc + 2 * v * v * dsc + 6 * p1 * v + 2 * p2 * u};
}
// Newton on D(x) = xd (a fixed-point step where |det J| <= 1e-3), run to
// double precision.
inline void undistort_d(const float* k, double xdu, double xdv, double& u, double& v) {
    u = xdu;
    v = xdv;
    for (int j = 0; j < 12; ++j) {
        const DistD s = dist_state(k, u, v);
        const double rx = u * s.scale + s.dx - xdu, ry = v * s.scale + s.dy - xdv;
        const double det = s.det();
        if (std::fabs(det) > 1e-3) {
            u -= (s.jvv * rx - s.juv * ry) / det;
            v -= (s.juu * ry - s.juv * rx) / det;
        } else {
            u = (xdu - s.dx) / s.scale;
            v = (xdv - s.dy) / s.scale;
        }
    }
}

// The float32 fisheye re-solve of the forward (fisheye_opencv.cu:14-47),
// used only for the convergence / validity decision.
struct FisheyeF {
    float k1, k2, k3, k4;
    float dist(float t) const {
        const float t2 = t * t;
        float d = t2 * k4 + k3;
        d = t2 * d + k2;
        d = t2 * d + k1;
        d = t2 * d + 1.0f;
        return t * d;
    }
    float deriv(float t) const {
        const float t2 = t * t;
        float d = t2 * 9.0f * k4 + 7.0f * k3;
        d = t2 * d + 5.0f * k2;
        d = t2 * d + 3.0f * k1;
        d = t2 * d + 1.0f;
        return d;
    }
    float solve(float delta, float& res) const {
        float t = delta;
        res = 0.0f;
        for (int i = 0; i < 20; ++i) {
            res = dist(t) - delta;
            t -= res / std::fmax(deriv(t), 0.1f);
            t = std::fmin(std::fmax(t, 0.0f), float(M_PI));
            if (std::fabs(res) < 1e-6f) break;
        }
        return t;
    }
};

struct Pixel { float u, v; };

// base_camera_impl.h:9-14; lidar rows take v from the beam table.
inline Pixel pixel_uv(int type, int px, int py, int W, int H, const float* elev) {
    const float u = (float(px) + 0.5f) / float(W);
    if (type == CAM_LIDAR) return {u, elev[py]};
    return {u, (float(py) + 0.5f) / float(H)};
}

struct RayGrad {
    const float* p;
    int type;
    FisheyeF fe;

    // Camera-frame ray in double; theta_out = the fisheye angle (the forward
    // returns (0, 0, 1) when its float32 solve ends at theta <= 0).
    D3 ray(Pixel uv, double& theta_out) const {
        const double u = uv.u, v = uv.v;
        if (type == CAM_PINHOLE) return {(u - p[20]) / p[18], (v - p[21]) / p[19], 1.0};
        if (type == CAM_DISTORTED) {
            double x, y;
            undistort_d(p + 22, (u - p[20]) / p[18], (v - p[21]) / p[19], x, y);
            return {x, y, 1.0};
        }
        if (type == CAM_FISHEYE) {
            const float uxf = (uv.u - p[20]) / p[18], uyf = (uv.v - p[21]) / p[19];
            float res;
            const float thf = fe.solve(std::sqrt(uxf * uxf + uyf * uyf), res);
            if (thf <= 0.0f) { theta_out = 0.0; return {0.0, 0.0, 1.0}; }
            const double ux = (u - p[20]) / p[18], uy = (v - p[21]) / p[19];
            const double delta = std::sqrt(ux * ux + uy * uy);
            double th = thf;  // refined in double where the float32 solve converged
            const bool conv = std::fabs(res) < 1e-5f && fe.deriv(thf) > 1e-3f;
            for (int i = 0; i < (conv ? 4 : 0); ++i) {
                const double t2 = th * th;
                const double f = th * (1 + t2 * (p[22] + t2 * (p[23] + t2 * (p[24] + t2 * p[25])))) - delta;
                const double d = 1 + t2 * (3 * p[22] + t2 * (5 * p[23] + t2 * (7 * p[24] + t2 * 9 * p[25])));
                th -= f / d;
            }
            theta_out = th;
            const double s = std::sin(th) / delta;
            return {s * ux, s * uy, std::cos(th)};
        }
        const double az = p[18] + u * p[19], el = p[20] + v * p[21];
        return {std::cos(el) * std::sin(az), std::cos(el) * std::cos(az), std::sin(el)};
    }

    void impl_bwd(Pixel uv, double theta, D3 d, double* acc) const {
        if (type == CAM_PINHOLE) {
            const double fx = p[18], fy = p[19];
            acc[18] += -d.x * (uv.u - p[20]) / (fx * fx);
            acc[19] += -d.y * (uv.v - p[21]) / (fy * fy);
            acc[20] += -d.x / fx;
            acc[21] += -d.y / fy;
            return;
        }
        if (type == CAM_DISTORTED) {  // distorted_perspective.cu:115-190
            const double fx = p[18], fy = p[19];
            const double xdu = (uv.u - p[20]) / fx, xdv = (uv.v - p[21]) / fy;
            double x, y;
            undistort_d(p + 22, xdu, xdv, x, y);
            const DistD s = dist_state(p + 22, x, y);
            const double det = s.det();
            double gx, gy;  // J^-T d.xy
            if (std::fabs(det) <= 1e-3) {
                gx = d.x / s.scale;
                gy = d.y / s.scale;
            } else {
                gx = (s.jvv * d.x - s.juv * d.y) / det;
                gy = (s.juu * d.y - s.juv * d.x) / det;
            }
            acc[18] += -gx * xdu / fx;
            acc[19] += -gy * xdv / fy;
            acc[20] += -gx / fx;
            acc[21] += -gy / fy;
            const double r2 = x * x + y * y, r4 = r2 * r2, r6 = r4 * r2;
            const double rad = -(gx * x + gy * y) / s.denom, rad_den = -rad * s.scale;
            acc[22] += rad * r2;
            acc[23] += rad * r4;
            acc[24] += -(gx * 2 * x * y + gy * (r2 + 2 * y * y));
            acc[25] += -(gx * (r2 + 2 * x * x) + gy * 2 * x * y);
            acc[26] += rad * r6;
            acc[27] += rad_den * r2;
            acc[28] += rad_den * r4;
            acc[29] += rad_den * r6;
            return;
        }
        if (type != CAM_FISHEYE) return;
        const float uxf = (uv.u - p[20]) / p[18], uyf = (uv.v - p[21]) / p[19];
        const float deltaf = std::sqrt(uxf * uxf + uyf * uyf);
        float res;
        const float thf = fe.solve(deltaf, res);
        if (!((thf > 0.0f) && (deltaf > 1e-8f) && (std::fabs(res) < 1e-5f) && (fe.deriv(thf) > 1e-3f))) return;
        const double fx = p[18], fy = p[19];
        const double ux = (uv.u - p[20]) / fx, uy = (uv.v - p[21]) / fy;
        const double delta = std::sqrt(ux * ux + uy * uy);
        const double th = theta, t2 = th * th;
        const double der = 1 + t2 * (3 * p[22] + t2 * (5 * p[23] + t2 * (7 * p[24] + t2 * 9 * p[25])));
        const double sn = std::sin(th), cs = std::cos(th);
        // ray = (sin(th)/delta * uc, cos(th)), th = th(delta, k)
        const double d_s = d.x * ux + d.y * uy;
        const double d_th = d_s * cs / delta - d.z * sn;
        const double g = d_th / der;
        double tp = th * t2;
        for (int i = 0; i < 4; ++i) {
            acc[22 + i] += -g * tp;
            tp *= t2;
        }
        const double d_delta = -d_s * sn / (delta * delta) + g;
        const double s = sn / delta;
        const double dux = s * d.x + d_delta * ux / delta;
        const double duy = s * d.y + d_delta * uy / delta;
        acc[18] += -dux * ux / fx;
        acc[19] += -duy * uy / fy;
        acc[20] += -dux / fx;
        acc[21] += -duy / fy;
    }
};

inline D3 normalize_bwd(D3 r, D3 g) {
    const double l = std::sqrt(dot(r, r));
    const D3 n = (1.0 / l) * r;
    return (1.0 / l) * (g - dot(n, g) * n);
}

}  // namespace

extern "C" {

// d_pack[words] (double) = gradient of sum(d_ray_o . ray_o + d_ray_d . ray_d)
// with respect to the pack; ray_kernels.h:61-123.
void xsgo_camera_rays_bwd(int type, const float* pack, const float* elev, int W, int H, int world_space,
                          int normalized, const float* d_ray_o, const float* d_ray_d, int words, double* d_pack) {
    // RayGrad indexes the intrinsics from word 18; impls holding a float4
    // start at word 20 in the pack (the reference's struct alignment), so
    // those read and accumulate two words further on
    const int shift = (type == CAM_FISHEYE || type == CAM_DISTORTED) ? 2 : 0;
    RayGrad k{pack + shift, type, {0.0f, 0.0f, 0.0f, 0.0f}};
    if (type == CAM_FISHEYE) k.fe = {k.p[22], k.p[23], k.p[24], k.p[25]};
    const double qn = std::sqrt(double(pack[0]) * pack[0] + double(pack[1]) * pack[1] + double(pack[2]) * pack[2] +
                                double(pack[3]) * pack[3]);
    const double sg = pack[0] < 0.0f ? -1.0 : 1.0;
    const DQ q0s{sg * pack[0] / qn, {sg * pack[1] / qn, sg * pack[2] / qn, sg * pack[3] / qn}};
    const D3 vel{pack[7], pack[8], pack[9]}, wv{pack[10], pack[11], pack[12]};
    std::vector<double> rows(size_t(H) * words, 0.0);
#pragma omp parallel for schedule(static)
    for (int py = 0; py < H; ++py) {
        double* acc = rows.data() + size_t(py) * words;
        for (int px = 0; px < W; ++px) {
            const int64_t idx = int64_t(py) * W + px;
            const Pixel uv = pixel_uv(type, px, py, W, H, elev);
            double theta = 0.0;
            const D3 ray = k.ray(uv, theta);
            const D3 gd{d_ray_d[3 * idx], d_ray_d[3 * idx + 1], d_ray_d[3 * idx + 2]};
            D3 dray = gd;
            if (world_space) {
                const D3 go = d_ray_o ? D3{d_ray_o[3 * idx], d_ray_o[3 * idx + 1], d_ray_o[3 * idx + 2]}
                                      : D3{0, 0, 0};
                const double dt = double(pack[16]) + double(uv.u) * pack[14] + double(uv.v) * pack[15] - pack[17];
                acc[4] += go.x; acc[5] += go.y; acc[6] += go.z;
                acc[7] += dt * go.x; acc[8] += dt * go.y; acc[9] += dt * go.z;
                double d_dt = dot(go, vel);
                const D3 n = normalized ? (1.0 / std::sqrt(dot(ray, ray))) * ray : ray;
                // q = q_aa(w dt) (x) std(q0), q_aa = (cos(th/2), sin(th/2)/th a)
                const D3 a = dt * wv;
                const double th = std::sqrt(dot(a, a));
                const double sc = th > 1e-12 ? std::sin(0.5 * th) / th : 0.5;
                const double ch = std::cos(0.5 * th);
                const DQ qa{ch, sc * a};
                const DQ q = qmul(qa, q0s);
                // y = R(q) n: dL/dq (tangent part is all that matters, std_backward
                // removes the rest) and dL/dn = R(q)^T g
                const D3 u = q.v;
                const DQ gq{2.0 * dot(gd, cross(u, n)),
                            2.0 * q.w * cross(n, gd) + 2.0 * dot(u, n) * gd + 2.0 * dot(u, gd) * n -
                                4.0 * dot(n, gd) * u};
                const D3 dn = qrot(DQ{q.w, -1.0 * q.v}, gd);
                // Hamilton product backward
                const double d_aw = gq.w * q0s.w + dot(gq.v, q0s.v);
                const D3 d_av = q0s.w * gq.v - gq.w * q0s.v + cross(q0s.v, gq.v);
                const double d_bw = gq.w * qa.w + dot(gq.v, qa.v);
                const D3 d_bv = qa.w * gq.v - gq.w * qa.v + cross(gq.v, qa.v);
                // q_aa(a) backward: d cos(th/2)/da = -sc/2 a, d(sc a)/da = sc I + (sc'/th) a a^T
                const double dsc = th > 1e-3 ? (0.5 * ch - sc) / (th * th) : -1.0 / 24.0 + th * th / 960.0;
                const D3 ga = (-0.5 * sc * d_aw) * a + sc * d_av + (dot(a, d_av) * dsc) * a;
                acc[10] += dt * ga.x; acc[11] += dt * ga.y; acc[12] += dt * ga.z;
                d_dt += dot(wv, ga);
                // std(q0) = sign(w) q0/|q0| backward
                const DQ qh{pack[0] / qn, {pack[1] / qn, pack[2] / qn, pack[3] / qn}};
                const double proj = qh.w * d_bw + dot(qh.v, d_bv);
                acc[0] += sg / qn * (d_bw - proj * qh.w);
                acc[1] += sg / qn * (d_bv.x - proj * qh.v.x);
                acc[2] += sg / qn * (d_bv.y - proj * qh.v.y);
                acc[3] += sg / qn * (d_bv.z - proj * qh.v.z);
                acc[14] += d_dt * uv.u;
                acc[15] += d_dt * uv.v;
                acc[16] += d_dt;
                acc[17] -= d_dt;
                dray = dn;
            }
            if (normalized) dray = normalize_bwd(ray, dray);
            k.impl_bwd(uv, theta, dray, acc + shift);
        }
    }
    for (int j = 0; j < words; ++j) d_pack[j] = 0.0;
    for (int py = 0; py < H; ++py)
        for (int j = 0; j < words; ++j) d_pack[j] += rows[size_t(py) * words + j];
}

// time_kernels.h:115-297: t = trigger + uv . rolling (- pose when delta);
// uv from the pixel grid (uv == NULL, n = W * H) or given [n, 2], in which
// case d_uv (may be NULL) = grad * rolling.
void xsgo_pixel_time_bwd(int type, const float* pack, const float* elev, int W, int H, const float* uv,
                         int64_t n, int delta, const float* grad, int words, double* d_pack, float* d_uv) {
    for (int j = 0; j < words; ++j) d_pack[j] = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        Pixel p;
        if (uv) p = {uv[2 * i], uv[2 * i + 1]};
        else p = pixel_uv(type, int(i % W), int(i / W), W, H, elev);
        const double g = grad[i];
        d_pack[14] += g * p.u;
        d_pack[15] += g * p.v;
        d_pack[16] += g;
        if (delta) d_pack[17] -= g;
        if (d_uv) {
            d_uv[2 * i] = float(g * pack[14]);
            d_uv[2 * i + 1] = float(g * pack[15]);
        }
    }
}

}  // extern "C"
