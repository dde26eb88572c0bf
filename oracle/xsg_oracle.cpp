// xsimgs-b200 CPU ORACLE — test infrastructure only, never a product path.
//
// A scalar C++17 restatement of the xsimgs Gaussian render path
// (whesense/xsimgs, the "reference"), written from the reference's CUDA
// sources and used as the checker for the B200 kernels in this repository.
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
// it.  Every function names the reference file:line it follows (paths are
// relative to the reference project root).
//
// PARITY STATUS: unpinned.  The reference cannot be built (its `pytoast`
// dependency is absent and unpinned, third_party/glm is empty) and it ships no
// tests, fixtures or golden vectors.  The parts of the path that the reference
// delegates to pytoast (quaternion std()/to_matrix()/from_matrix(), vector
// normalize(), apply_velocity) are restated from the conventions the
// reference's own sources spell out (wxyz quaternions, utils.h:61-83; the
// motion model, projection_kernels.h:74-113) and are marked "toast:" below.
//
// Floating point: built with -ffp-contract=off and without -march flags, so
// every float operation rounds exactly as written.  Transcendentals come from
// the host libm; the B200 kernels use CUDA's, so results agree to a few ulp,
// not bit for bit (see the tolerances in tests/).
//
// Built by oracle/build.py into oracle/_build/libxsg_oracle.so.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------- vectors --
struct f2 { float x, y; };
struct f3 { float x, y, z; };
struct f4 { float x, y, z, w; };
struct quat { float w, x, y, z; };

inline f2 operator+(f2 a, f2 b) { return {a.x + b.x, a.y + b.y}; }
inline f2 operator-(f2 a, f2 b) { return {a.x - b.x, a.y - b.y}; }
inline f2 operator*(f2 a, f2 b) { return {a.x * b.x, a.y * b.y}; }
inline f2 operator/(f2 a, f2 b) { return {a.x / b.x, a.y / b.y}; }
inline f2 operator*(float s, f2 a) { return {s * a.x, s * a.y}; }
inline f2 operator*(f2 a, float s) { return {a.x * s, a.y * s}; }
inline f2 operator/(f2 a, float s) { return {a.x / s, a.y / s}; }
inline f3 operator+(f3 a, f3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline f3 operator-(f3 a, f3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline f3 operator-(f3 a) { return {-a.x, -a.y, -a.z}; }
inline f3 operator*(float s, f3 a) { return {s * a.x, s * a.y, s * a.z}; }
inline f3 operator*(f3 a, float s) { return {a.x * s, a.y * s, a.z * s}; }
inline f3 operator/(f3 a, float s) { return {a.x / s, a.y / s, a.z / s}; }
inline f3& operator+=(f3& a, f3 b) { a = a + b; return a; }
inline float dot(f2 a, f2 b) { return a.x * b.x + a.y * b.y; }
inline float dot(f3 a, f3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline f3 cross(f3 a, f3 b) {
    return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
inline float length(f2 a) { return std::sqrt(dot(a, a)); }
inline float length(f3 a) { return std::sqrt(dot(a, a)); }
// toast: normalize(v) = v * rsqrt(dot(v, v)) (helper_math convention).
inline f3 normalize(f3 v) { return v * (1.0f / std::sqrt(dot(v, v))); }

// float -> int32 with the GPU's cvt.rzi.s32.f32 semantics (saturating, NaN->0),
// which the reference's `static_cast<int>(floorf(..))` compiles to on device.
inline int32_t f2i(float v) {
    if (std::isnan(v)) return 0;
    if (v >= 2147483648.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return static_cast<int32_t>(v);
}

// ------------------------------------------------------------- quaternions --
// toast: quaternion std() — unit length with a non-negative real part.
inline quat q_std(quat q) {
    float n = 1.0f / std::sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    if (q.w < 0.0f) n = -n;
    return {q.w * n, q.x * n, q.y * n, q.z * n};
}
inline f3 q_img(quat q) { return {q.x, q.y, q.z}; }

// Rotate p by unit quaternion (w, xyz); reference projection_kernels.h:67-71.
inline f3 quat_apply(float w, f3 xyz, f3 p) {
    const f3 uv = cross(xyz, p);
    const f3 uuv = cross(xyz, uv);
    return p + 2.0f * (w * uv + uuv);
}

// Rotation vector w*t -> quaternion; projection_kernels.h:12-36 (values only).
inline void quat_from_axis_angle(f3 w, float t, float& qw, f3& qxyz) {
    const float w_norm2 = dot(w, w);
    const float w_norm = std::sqrt(w_norm2);
    const float theta = w_norm * std::fabs(t);
    const float sin_half = std::sin(0.5f * theta);
    const float cos_half = std::cos(0.5f * theta);
    const float scale = (theta < 1e-2f) ? 0.5f - theta * theta * (1.0f / 48.0f)
                                        : sin_half / theta;
    qw = cos_half;
    qxyz = scale * w * t;
}

// q1 (x) q2 Hamilton product; projection_kernels.h:38-51 (values only).
inline void quat_mul(float w1, f3 x1, float w2, f3 x2, float& w, f3& x) {
    w = w1 * w2 - dot(x1, x2);
    x = w1 * x2 + w2 * x1 + cross(x1, x2);
}

// toast: apply_angular_velocity(q0, w, t) = q_aa(w t) (x) q0, the composition
// the reference spells out in jac_world_to_camera (projection_kernels.h:88-101).
inline quat apply_angular_velocity(quat q0, f3 w, float t) {
    float w1; f3 x1;
    quat_from_axis_angle(w, t, w1, x1);
    quat r; f3 rx;
    quat_mul(w1, x1, q0.w, q_img(q0), r.w, rx);
    r.x = rx.x; r.y = rx.y; r.z = rx.z;
    return r;
}

// toast: rotation matrix rows of a quaternion (normalised first, as the
// rasteriser's quat_to_rotmat does, rasterization/utils.h:61-83).
inline void quat_to_rows(quat q, f3 rows[3]) {
    const float inv = 1.0f / std::sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    const float w = q.w * inv, x = q.x * inv, y = q.y * inv, z = q.z * inv;
    const float x2 = x * x, y2 = y * y, z2 = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    rows[0] = {1.f - 2.f * (y2 + z2), 2.f * (xy - wz), 2.f * (xz + wy)};
    rows[1] = {2.f * (xy + wz), 1.f - 2.f * (x2 + z2), 2.f * (yz - wx)};
    rows[2] = {2.f * (xz - wy), 2.f * (yz + wx), 1.f - 2.f * (x2 + y2)};
}

// ----------------------------------------------------------------- cameras --
// Camera pack layout of this project (floats):
//   [0:4) q0 wxyz  [4:7) t0  [7:10) v  [10:13) w  [13] pad
//   [14:16) rolling_time  [16] trigger_time  [17] pose_time  [18:) intrinsics
// The reference's field order is camera.h:71-79.
enum CamType { CAM_PINHOLE = 0, CAM_FISHEYE = 1, CAM_SPHERICAL = 2, CAM_LIDAR = 3, CAM_DISTORTED = 4 };
enum ProjMode { MODE_CENTRAL = 0, MODE_NEG = 1, MODE_POS = 2 };

struct Cam {
    int type;
    quat q0; f3 t0, v, w; f2 rolling; float trigger, pose;
    f2 f, c; f4 dist;                                       // pinhole / fisheye
    f4 d0, d1; float max_r2;                                 // distorted pinhole
    float phi_min, phi_range, theta_min, theta_range;        // spherical / lidar
    const float* elev;                                       // lidar beam v table

    static Cam load(int type, const float* p, const float* elev_values) {
        Cam k{};
        k.type = type;
        k.q0 = {p[0], p[1], p[2], p[3]};
        k.t0 = {p[4], p[5], p[6]};
        k.v = {p[7], p[8], p[9]};
        k.w = {p[10], p[11], p[12]};
        k.rolling = {p[14], p[15]};
        k.trigger = p[16];
        k.pose = p[17];
        if (type == CAM_PINHOLE || type == CAM_FISHEYE || type == CAM_DISTORTED) {
            // impls holding a float4 start at word 20 (16-byte aligned, as in
            // the reference's Camera<Impl> struct), the others at word 18
            const float* in = p + ((type == CAM_PINHOLE) ? 18 : 20);
            k.f = {in[0], in[1]};
            k.c = {in[2], in[3]};
            if (type == CAM_FISHEYE) k.dist = {in[4], in[5], in[6], in[7]};
            if (type == CAM_DISTORTED) {
                k.d0 = {in[4], in[5], in[6], in[7]};
                k.d1 = {in[8], in[9], in[10], in[11]};
                k.max_r2 = in[12];
            }
        } else {
            k.phi_min = p[18]; k.phi_range = p[19];
            k.theta_min = p[20]; k.theta_range = p[21];
        }
        k.elev = elev_values;
        return k;
    }

    bool has_jacobian() const { return type != CAM_FISHEYE && type != CAM_DISTORTED; }

    // DistortedPerspectiveCameraImpl::DistortionState at (u, v)
    // (distorted_perspective.cu:11-78): D(x) = x scale + delta and its
    // symmetric Jacobian.
    struct DState { float scale, denom, dx, dy, juu, juv, jvv; };
    DState dstate(float u, float v) const {
        const float r2 = u * u + v * v;
        const float num = 1.0f + r2 * (d0.x + r2 * (d0.y + r2 * d1.x));
        const float den = 1.0f + r2 * (d1.y + r2 * (d1.z + r2 * d1.w));
        const float sc = num / den;
        const float dn = d0.x + r2 * (2.0f * d0.y + 3.0f * d1.x * r2);
        const float dd = d1.y + r2 * (2.0f * d1.z + 3.0f * d1.w * r2);
        const float dsc = (dn * den - num * dd) / (den * den);
        return {sc, den,
                2.0f * d0.z * u * v + d0.w * (r2 + 2.0f * u * u),
                d0.z * (r2 + 2.0f * v * v) + 2.0f * d0.w * u * v,
                sc + 2.0f * u * u * dsc + 2.0f * d0.z * v + 6.0f * d0.w * u,
                2.0f * u * v * dsc + 2.0f * d0.z * u + 2.0f * d0.w * v,
                sc + 2.0f * v * v * dsc + 6.0f * d0.z * v + 2.0f * d0.w * u};
    }
    // undistort_uv, distorted_perspective.cu:80-99 (st = the state at the
    // start of the last step)
    f2 undistort(f2 xd, DState& st) const {
        f2 x = xd;
        for (int j = 0; j < 5; ++j) {
            st = dstate(x.x, x.y);
            const float rx = x.x * st.scale + st.dx - xd.x;
            const float ry = x.y * st.scale + st.dy - xd.y;
            const float det = st.juu * st.jvv - st.juv * st.juv;
            if (std::fabs(det) > 1e-3f) {
                x.x -= (st.jvv * rx - st.juv * ry) / det;
                x.y -= (st.juu * ry - st.juv * rx) / det;
            } else {
                x = {(xd.x - st.dx) / st.scale, (xd.y - st.dy) / st.scale};
            }
        }
        return x;
    }
    // uv_distortion, distortion.h:8-30, applied to x
    f2 distort(f2 x) const {
        const float uu = x.x * x.x, vv = x.y * x.y;
        const float r2 = uu + vv;
        const float num = 1.0f + r2 * (d0.x + r2 * (d0.y + r2 * d1.x));
        const float den = 1.0f + r2 * (d1.y + r2 * (d1.z + r2 * d1.w));
        const float sc = num / den;
        const float uv2 = 2.0f * x.x * x.y;
        return {x.x * sc + (d0.z * uv2 + d0.w * (r2 + 2.0f * uu)),
                x.y * sc + (d0.z * (r2 + 2.0f * vv) + d0.w * uv2)};
    }

    // base_camera_impl.h:9-14; lidar rows from the beam table, spherical.h:77-82
    f2 pixel_to_uv(int px, int py, int W, int H) const {
        const float u = (static_cast<float>(px) + 0.5f) / static_cast<float>(W);
        if (type == CAM_LIDAR) return {u, elev[py]};
        return {u, (static_cast<float>(py) + 0.5f) / static_cast<float>(H)};
    }
    // camera.h:89-99
    float pixel_time(f2 uv) const { return trigger + dot(uv, rolling); }
    float pixel_time_delta(f2 uv) const { return pixel_time(uv) - pose; }

    // fisheye_opencv.cu:14-47
    float fe_dist(float theta) const {
        const float t2 = theta * theta;
        float d = t2 * dist.w + dist.z;
        d = t2 * d + dist.y;
        d = t2 * d + dist.x;
        d = t2 * d + 1.0f;
        return theta * d;
    }
    float fe_deriv(float theta) const {
        const float t2 = theta * theta;
        float d = t2 * 9.0f * dist.w + 7.0f * dist.z;
        d = t2 * d + 5.0f * dist.y;
        d = t2 * d + 3.0f * dist.x;
        d = t2 * d + 1.0f;
        return d;
    }
    float fe_solve(float delta, float& residual) const {
        float theta = delta;
        residual = 0.0f;
        for (int i = 0; i < 20; ++i) {
            residual = fe_dist(theta) - delta;
            theta -= residual / std::fmax(fe_deriv(theta), 0.1f);
            theta = std::fmin(std::fmax(theta, 0.0f), float(M_PI));
            if (std::fabs(residual) < 1e-6f) break;
        }
        return theta;
    }

    // spherical.h:21-32
    static f3 sph_to_cart(float az, float el, float d) {
        const float es = std::sin(el), ec = std::cos(el);
        const float as = std::sin(az), ac = std::cos(az);
        const float xy = d * ec;
        return {xy * as, xy * ac, d * es};
    }

    // perspective.cu:13-16, fisheye_opencv.cu:49-64, spherical.h:40-46
    f3 pixel_to_camera_ray(f2 uv) const {
        if (type == CAM_DISTORTED) {  // distorted_perspective.cu:101-106
            DState st;
            const f2 x = undistort((uv - c) / f, st);
            return {x.x, x.y, 1.0f};
        }
        if (type == CAM_PINHOLE) {
            const f2 uc = (uv - c) / f;
            return {uc.x, uc.y, 1.0f};
        }
        if (type == CAM_FISHEYE) {
            const f2 uc = (uv - c) / f;
            const float delta = length(uc);
            float residual;
            const float theta = fe_solve(delta, residual);
            if (theta <= 0.0f) return {0.0f, 0.0f, 1.0f};
            const float s = std::sin(theta) / delta;
            return {s * uc.x, s * uc.y, std::cos(theta)};
        }
        return sph_to_cart(phi_min + uv.x * phi_range, theta_min + uv.y * theta_range, 1.0f);
    }

    // camera.h:117-123, fisheye_opencv.cu:66-74
    bool ray_valid(f2 uv) const {
        if (type == CAM_DISTORTED) {  // distorted_perspective.cu:108-118
            DState st;
            const f2 xd = (uv - c) / f;
            const f2 x = undistort(xd, st);
            const float rx = x.x * st.scale + st.dx - xd.x;
            const float ry = x.y * st.scale + st.dy - xd.y;
            const float r2 = x.x * x.x + x.y * x.y;
            return (r2 <= max_r2) && (std::fabs(rx) < 1e-5f) && (std::fabs(ry) < 1e-5f);
        }
        if (type != CAM_FISHEYE) return true;
        const float delta = length((uv - c) / f);
        if (delta <= 1e-8f) return true;
        float residual;
        const float theta = fe_solve(delta, residual);
        return (std::fabs(residual) < 1e-5f) && (fe_deriv(theta) > 0.0f);
    }

    // spherical.h:109-125
    f2 angles_to_uv(int mode, float phi, float theta) const {
        float u = (phi - phi_min) / phi_range;
        const float u_pose = (std::fabs(rolling.x) > 0.0f) ? (pose - trigger) / rolling.x : 0.5f;
        const float u_off = (2.0f * float(M_PI) / std::fabs(phi_range));
        if (rolling.x > 0) {
            if (mode == MODE_NEG && u > u_pose) u = u - u_off;
            if (mode == MODE_POS && u < u_pose) u = u + u_off;
        } else {
            if (mode == MODE_NEG && u < u_pose) u = u + u_off;
            if (mode == MODE_POS && u > u_pose) u = u - u_off;
        }
        const float v = (theta - theta_min) / theta_range;
        return {u, v};
    }

    // perspective.cu:54-60, fisheye_opencv.cu:143-153, spherical.h:127-131
    f3 point_to_uvd(int mode, f3 p) const {
        if (type == CAM_DISTORTED) {  // distorted_perspective.cu:192-199
            const f2 x{p.x / p.z, p.y / p.z};
            const f2 xd = distort(x);
            const float r2 = x.x * x.x + x.y * x.y;
            return {xd.x * f.x + c.x, xd.y * f.y + c.y, (r2 <= max_r2) ? p.z : 0.0f};
        }
        if (type == CAM_PINHOLE)
            return {p.x * f.x / p.z + c.x, p.y * f.y / p.z + c.y, p.z};
        if (type == CAM_FISHEYE) {
            const float norm = std::fmax(1e-6f, std::hypot(p.x, p.y));
            const float theta = std::atan2(norm, p.z);
            const bool valid = fe_deriv(theta) > 0.0f;
            const float delta = fe_dist(theta) / norm;
            const f2 uv = f * delta * f2{p.x, p.y} + c;
            const float depth = (valid && delta > 0.0f) ? length(p) : 0.0f;
            return {uv.x, uv.y, depth};
        }
        const float dist_ = length(p);
        const float phi = std::atan2(-p.x, -p.y) + float(M_PI);
        const float theta = std::asin(p.z / dist_);
        const f2 uv = angles_to_uv(mode, phi, theta);
        return {uv.x, uv.y, dist_};
    }

    // perspective.cu:62-70, spherical.h:133-153
    void point_to_uvd_jacob(int mode, f3 p, f3 dp, f3& uvd, f2& duv) const {
        if (type == CAM_PINHOLE) {
            uvd = point_to_uvd(mode, p);
            const float du = f.x * (dp.x - uvd.x * dp.z) / uvd.z;
            const float dv = f.y * (dp.y - uvd.y * dp.z) / uvd.z;
            duv = {du, dv};
            return;
        }
        const float x2y2 = p.x * p.x + p.y * p.y;
        const float r = std::sqrt(x2y2 + p.z * p.z);
        // double M_PI, as spherical.h:140 adds it (one rounding from double)
        const float phi = float(double(std::atan2(-p.x, -p.y)) + M_PI);
        const float theta = std::asin(p.z / r);
        const f2 uv = angles_to_uv(mode, phi, theta);
        uvd = {uv.x, uv.y, r};
        const float x2y2_sqrt = std::sqrt(x2y2);
        const float r2 = r * r;
        const float mul = p.z / (r2 * x2y2_sqrt);
        duv = {((-p.x * dp.y + p.y * dp.x) / x2y2) / phi_range,
               ((x2y2_sqrt * dp.z) / r2 - mul * (p.x * dp.x + p.y * dp.y)) / theta_range};
    }
};

// World point -> camera point at time t and d/dt; projection_kernels.h:74-113
void world_to_camera_jac(const Cam& k, f3 P, f3 Pv, float t, f3& res, f3& dres) {
    // quaternion of the rotation vector w t and its derivative (:12-36)
    const float w_norm = std::sqrt(dot(k.w, k.w));
    const float theta = w_norm * std::fabs(t);
    const float sh = std::sin(0.5f * theta), ch = std::cos(0.5f * theta);
    const float scale = (theta < 1e-2f) ? 0.5f - theta * theta * (1.0f / 48.0f) : sh / theta;
    const float w1 = ch;
    const f3 x1 = scale * k.w * t;
    const float dw1 = -0.5f * std::copysign(1.0f, t) * sh * w_norm;
    const f3 dx1 = (0.5f * ch) * k.w;
    // product with q0 (:38-51)
    const f3 x2 = q_img(k.q0);
    const float w2 = k.q0.w;
    float w = w1 * w2 - dot(x1, x2);
    f3 xyz = w1 * x2 + w2 * x1 + cross(x1, x2);
    float dw = dw1 * w2 - dot(dx1, x2);
    f3 dxyz = dw1 * x2 + w2 * dx1 + cross(dx1, x2);
    xyz = -1.0f * xyz;   // inverse rotation
    dxyz = -1.0f * dxyz;
    const f3 vd = Pv - k.v;
    const f3 p = P - k.t0 + vd * t;
    // rotation and its derivative (:53-65)
    const f3 uv = cross(xyz, p);
    const f3 uuv = cross(xyz, uv);
    res = p + 2.0f * (w * uv + uuv);
    const f3 duv = cross(dxyz, p);
    const f3 dp = 2.0f * (dw * uv + w * duv + cross(dxyz, uv) + cross(xyz, duv));
    dres = dp + quat_apply(w, xyz, vd);
}

// Rolling-shutter Newton projection; projection_kernels.h:116-256.
void camera_projection(const Cam& k, f3 P, f3 Pv, float thr, float max_res, float margin,
                       int mode, bool force_nojac, f4& uvdt, bool& valid) {
    f3 uvd{0, 0, 0};
    float pt = 0.0f;
    if (mode == MODE_NEG) pt = -std::fabs(k.rolling.x) * 0.5f;
    else if (mode == MODE_POS) pt = std::fabs(k.rolling.x) * 0.5f;
    float residual = 0.0f;
    for (int i = 0; i < 5; ++i) {
        if (k.has_jacobian() && !force_nojac) {
            f3 pc, jpc; f2 duv;
            world_to_camera_jac(k, P, Pv, pt, pc, jpc);
            k.point_to_uvd_jacob(mode, pc, jpc, uvd, duv);
            const float assumed = k.pose + pt;
            const float real = k.pixel_time(f2{uvd.x, uvd.y});
            residual = assumed - real;
            const float dres = 1.0f - dot(duv, k.rolling);
            pt -= residual / dres;
        } else {
            const quat q = apply_angular_velocity(k.q0, k.w, pt);
            const f3 p = P - k.t0 + (Pv - k.v) * pt;
            const f3 pc = quat_apply(q.w, -q_img(q), p);
            uvd = k.point_to_uvd(mode, pc);
            const float assumed = k.pose + pt;
            const float real = k.pixel_time(f2{uvd.x, uvd.y});
            residual = assumed - real;
            pt -= residual;
        }
        if ((uvd.z <= 0.0f) || (uvd.x < -margin) || (uvd.x > 1.0f + margin) ||
            (uvd.y < -margin) || (uvd.y > 1.0f + margin)) {
            valid = false;
            uvdt = {0, 0, 0, 0};
            return;
        }
        if (std::fabs(residual) < thr) break;
    }
    uvdt = {uvd.x, uvd.y, uvd.z, pt};
    valid = valid && (std::fabs(residual) < max_res) && (uvd.z > 0.0f);
}

// ---------------------------------------------------------------------- UT --
struct UTW { float m0, c0, w, sq; };
// ut_kernels.h:17-36 (float arithmetic on the host)
UTW ut_weights(float a, float b, float kappa) {
    const float lam = a * a * (3 + kappa) - 3;
    UTW r;
    r.m0 = lam / (3 + lam);
    r.c0 = lam / (3 + lam) + (1 - a * a + b);
    r.w = 1 / (2 * (3 + lam));
    r.sq = std::sqrt(lam + 3);
    return r;
}

// ut_kernels.h:38-49: columns of R(q) scaled by s_i * sqrt(3 + lambda)
void ut_deltas(float sq, quat q, f3 s, f3 d[3]) {
    quat_to_rows({q.w, -q.x, -q.y, -q.z}, d);
    d[0] = d[0] * (s.x * sq);
    d[1] = d[1] * (s.y * sq);
    d[2] = d[2] * (s.z * sq);
}

struct UTArgs { float thr, max_res, margin; f2 img; UTW w; };

// ut_kernels.h:52-137
bool unscented_transform(const Cam& k, const UTArgs& a, int mode, f3 P, f3 Pv, const f3 d[3],
                         f2& mean2d, float& depth, float& u_dist, f3& cov) {
    f4 uvdt; bool valid = true;
    f2 pts[7];
    camera_projection(k, P, Pv, a.thr, a.max_res, a.margin, mode, false, uvdt, valid);
    if (!valid) return false;
    pts[0] = f2{uvdt.x, uvdt.y} * a.img;
    mean2d = a.w.m0 * pts[0];
    depth = uvdt.z;
    float umin = pts[0].x, umax = pts[0].x;
    float sign = 1.0f;
    for (int i = 0; i < 6; ++i) {
        camera_projection(k, P + sign * d[i / 2], Pv, a.thr, a.max_res, a.margin, mode, false,
                          uvdt, valid);
        pts[i + 1] = f2{uvdt.x, uvdt.y} * a.img;
        mean2d = mean2d + a.w.w * pts[i + 1];
        umin = std::fmin(umin, pts[i + 1].x);
        umax = std::fmax(umax, pts[i + 1].x);
        sign *= -1.0f;
    }
    if (!valid) return false;
    u_dist = umax - umin;
    f2 vec = pts[0] - mean2d;
    cov = a.w.c0 * f3{vec.x * vec.x, vec.x * vec.y, vec.y * vec.y};
    for (int i = 1; i < 7; ++i) {
        vec = pts[i] - mean2d;
        cov = cov + a.w.w * f3{vec.x * vec.x, vec.x * vec.y, vec.y * vec.y};
    }
    const float det = cov.x * cov.z - cov.y * cov.y;
    if (det <= 0.0f || cov.x < 0 || cov.z < 0) return false;
    return true;
}

// ut_kernels.h:145-184
bool ut_projection(const Cam& k, const UTArgs& a, int mode, f3 P, f3 Pv, float opac,
                   const f3 d[3], f2& mean2d, f2& radii, float& depth, float& u_dist) {
    f3 cov{0, 0, 0};
    mean2d = {0, 0}; depth = 0; u_dist = 0;
    const bool res = unscented_transform(k, a, mode, P, Pv, d, mean2d, depth, u_dist, cov);
    const float extend = std::fmin(3.33f, std::sqrt(2.0f * std::log(opac / (1.0f / 255.0f))));
    radii = {extend * std::sqrt(std::fmax(0.0f, cov.x)), extend * std::sqrt(std::fmax(0.0f, cov.z))};
    const bool ix = !(((mean2d.x + radii.x) < 0) || (a.img.x < (mean2d.x - radii.x)));
    const bool iy = !(((mean2d.y + radii.y) < 0) || (a.img.y < (mean2d.y - radii.y)));
    return res && ix && iy;
}

// --------------------------------------------------------------- tiling ----
// tiling_common.cuh:25-73: key = (tile << 32) | sign-extended depth bits
inline int64_t make_key(int64_t tile, float depth) {
    int32_t bits;
    std::memcpy(&bits, &depth, 4);
    return (tile << 32) | static_cast<int64_t>(bits);
}

// Stable ascending sort of pairs on key bits [0, 32 + tile_n_bits) — the
// effect of cub::DeviceRadixSort::SortPairs in tiling_common.cu:102-162.
void sort_pairs(std::vector<int64_t>& keys, std::vector<int32_t>& vals, int tile_n_bits) {
    const int nb = 32 + tile_n_bits;
    const uint64_t mask = nb >= 64 ? ~0ull : ((1ull << nb) - 1ull);
    std::vector<size_t> idx(keys.size());
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
        return (static_cast<uint64_t>(keys[a]) & mask) < (static_cast<uint64_t>(keys[b]) & mask);
    });
    std::vector<int64_t> k2(keys.size());
    std::vector<int32_t> v2(vals.size());
    for (size_t i = 0; i < idx.size(); ++i) { k2[i] = keys[idx[i]]; v2[i] = vals[idx[i]]; }
    keys.swap(k2);
    vals.swap(v2);
}

int tile_bits(int n_tiles) {
    return static_cast<int>(std::floor(std::log2(static_cast<float>(n_tiles)))) + 1;
}

// phm_lidar_tiling.cu:16-49
void bounds_increasing(float vmin, float vmax, int N, const float* v, int& lo, int& hi) {
    int i = 0;
    while (i < N && v[i] < vmin) ++i;
    lo = std::min(std::max(i - 1, 0), N - 1);
    while (i < N && v[i] < vmax) ++i;
    hi = std::min(std::max(i - 1, 0), N - 1);
}

}  // namespace

// ===================================================================== API ==
extern "C" {

int xsgo_num_threads() {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void xsgo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

void xsgo_ut_weights(float a, float b, float k, float* out4) {
    const UTW w = ut_weights(a, b, k);
    out4[0] = w.m0; out4[1] = w.c0; out4[2] = w.w; out4[3] = w.sq;
}

// Per-pixel rays; ray_kernels.h:8-59 and camera.h:125-131.
void xsgo_camera_rays(int type, const float* pack, const float* elev, int W, int H,
                      int world_space, int normalized, float* ray_o, float* ray_d,
                      uint8_t* valid) {
    const Cam k = Cam::load(type, pack, elev);
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < int64_t(W) * H; ++idx) {
        const int px = int(idx % W), py = int(idx / W);
        const f2 uv = k.pixel_to_uv(px, py, W, H);
        f3 ray = k.pixel_to_camera_ray(uv);
        if (normalized) ray = normalize(ray);
        f3 o{0, 0, 0}, d = ray;
        if (world_space) {
            const float dt = k.pixel_time_delta(uv);
            const quat q = apply_angular_velocity(q_std(k.q0), k.w, dt);
            o = k.t0 + k.v * dt;
            d = quat_apply(q.w, q_img(q), ray);
        }
        if (ray_o) { ray_o[3 * idx] = o.x; ray_o[3 * idx + 1] = o.y; ray_o[3 * idx + 2] = o.z; }
        ray_d[3 * idx] = d.x; ray_d[3 * idx + 1] = d.y; ray_d[3 * idx + 2] = d.z;
        if (valid) valid[idx] = k.ray_valid(uv) ? 1 : 0;
    }
}

// time_kernels.h:5-112
void xsgo_pixel_time(int type, const float* pack, const float* elev, int W, int H, int delta,
                     float* out) {
    const Cam k = Cam::load(type, pack, elev);
    for (int64_t idx = 0; idx < int64_t(W) * H; ++idx) {
        const f2 uv = k.pixel_to_uv(int(idx % W), int(idx / W), W, H);
        out[idx] = delta ? k.pixel_time_delta(uv) : k.pixel_time(uv);
    }
}

void xsgo_pixel_time_from_uv(int type, const float* pack, const float* uv, int64_t n, int delta,
                             float* out) {
    const Cam k = Cam::load(type, pack, nullptr);
    for (int64_t i = 0; i < n; ++i) {
        const f2 u{uv[2 * i], uv[2 * i + 1]};
        out[i] = delta ? k.pixel_time_delta(u) : k.pixel_time(u);
    }
}

// undistort_map, distortion.h:33-56: distorted uv of every pixel centre,
// mapped to [-1, 1] unless normalized_range.
void xsgo_undistort_map(const float* pack, int W, int H, int normalized_range, float* out) {
    const Cam k = Cam::load(CAM_DISTORTED, pack, nullptr);
    for (int64_t idx = 0; idx < int64_t(W) * H; ++idx) {
        const f2 uv = k.pixel_to_uv(int(idx % W), int(idx / W), W, H);
        const f2 xd = k.distort((uv - k.c) / k.f);
        f2 r{xd.x * k.f.x + k.c.x, xd.y * k.f.y + k.c.y};
        if (!normalized_range) r = {r.x * 2.0f - 1.0f, r.y * 2.0f - 1.0f};
        out[2 * idx] = r.x;
        out[2 * idx + 1] = r.y;
    }
}

// camera_projection_fwd, projection_kernels.h:259-309
void xsgo_projection(int type, const float* pack, const float* elev, const float* pts,
                     const float* vel, int64_t n, float thr, float max_res, float margin,
                     int mode, int force_nojac, float* uvdt_out, uint8_t* mask_out) {
    const Cam k = Cam::load(type, pack, elev);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const f3 P{pts[3 * i], pts[3 * i + 1], pts[3 * i + 2]};
        const f3 V = vel ? f3{vel[3 * i], vel[3 * i + 1], vel[3 * i + 2]} : f3{0, 0, 0};
        bool m = true; f4 u;
        camera_projection(k, P, V, thr, max_res, margin, mode, force_nojac != 0, u, m);
        u.w += k.pose;
        uvdt_out[4 * i] = u.x; uvdt_out[4 * i + 1] = u.y; uvdt_out[4 * i + 2] = u.z;
        uvdt_out[4 * i + 3] = u.w;
        m = m && (u.x >= 0.0f && u.y >= 0.0f) && (u.x <= 1.0f && u.y <= 1.0f);
        mask_out[i] = m ? 1 : 0;
    }
}

// unscented_transform_kernel (ut_kernels.h:192-246) and the phase-modelling
// variant unscented_transform_phm_kernel (ut_phm_kernels.h:13-114).
// Outputs must be zero-initialised by the caller (the reference zero-fills).
void xsgo_projection_utgs(int type, const float* pack, const float* elev, const float* pts,
                          const float* vel, const float* scales, const float* quats,
                          const float* opac, int64_t n, float W, float H, float ua, float ub,
                          float uk, float thr, float max_res, float margin, int phm,
                          uint8_t* flags, float* radii, float* means2d, float* depths) {
    const Cam k = Cam::load(type, pack, elev);
    UTArgs a{thr, max_res, margin, {W, H}, ut_weights(ua, ub, uk)};
#pragma omp parallel for schedule(dynamic, 1024)
    for (int64_t i = 0; i < n; ++i) {
        const f3 P{pts[3 * i], pts[3 * i + 1], pts[3 * i + 2]};
        const f3 V = vel ? f3{vel[3 * i], vel[3 * i + 1], vel[3 * i + 2]} : f3{0, 0, 0};
        const f3 S{scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
        const quat Q{quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
        const float o = opac ? opac[i] : 1.0f;
        if (o < 1.0f / 255.0f) continue;
        f3 d[3];
        ut_deltas(a.w.sq, Q, S, d);
        if (!phm) {
            f2 m, r; float dep, ud;
            if (!ut_projection(k, a, MODE_CENTRAL, P, V, o, d, m, r, dep, ud)) continue;
            radii[2 * i] = r.x; radii[2 * i + 1] = r.y;
            flags[i] = 1;
            means2d[2 * i] = m.x; means2d[2 * i + 1] = m.y;
            depths[i] = dep;
            continue;
        }
        f2 mc{0, 0}, ml{0, 0}, mr{0, 0}, rc{0, 0}, rl{0, 0}, rr{0, 0};
        float dc = 0, dl = 0, dr = 0, ud = 0;
        bool res = ut_projection(k, a, MODE_CENTRAL, P, V, o, d, mc, rc, dc, ud);
        if (!res) continue;
        const float u_pi = float(M_PI) * a.img.x / std::fabs(k.phi_range);
        const int r_c = int(res) * (int(ud > u_pi) + 1);
        res = ut_projection(k, a, MODE_NEG, P, V, o, d, ml, rl, dl, ud);
        const int r_l = int(res) * (int(ud > u_pi) + 1);
        res = ut_projection(k, a, MODE_POS, P, V, o, d, mr, rr, dr, ud);
        const int r_r = int(res) * (int(ud > u_pi) + 1);
        f2 m, r; float dep; uint8_t fl;
        if (r_l == 1 && r_r == 1) { fl = 2; r = rl; m = ml; dep = dl; }
        else if (r_c == 1) { fl = 1; r = rc; m = mc; dep = dc; }
        else if (r_l != 1 && r_r != 1) continue;
        else {
            const bool use_left = r_l != 1;
            fl = 1; r = use_left ? rl : rr; m = use_left ? ml : mr; dep = use_left ? dl : dr;
        }
        flags[i] = fl;
        radii[2 * i] = r.x; radii[2 * i + 1] = r.y;
        means2d[2 * i] = m.x; means2d[2 * i + 1] = m.y;
        depths[i] = dep;
    }
}

// mask_radii.cu:10-58
void xsgo_mask_radii(const uint8_t* mask, const uint32_t* packed, int64_t n, float* radii) {
    for (int64_t i = 0; i < n; ++i) {
        const bool keep = mask ? (mask[i] != 0) : ((packed[i / 32] >> (i % 32)) & 1u);
        if (!keep) { radii[2 * i] = 0.0f; radii[2 * i + 1] = 0.0f; }
    }
}

// Regular tiling, regular_tiling.cu:13-135 (+ sort, tiling_common.cu:102-162).
// Call once with isect_ids == nullptr to get the count (returned); then again
// with buffers of that size.  Returns the number of intersections.
int64_t xsgo_isect_regular(const float* means2d, const float* radii, const float* depths,
                           int64_t n, int W, int H, int tsx, int tsy, int sort,
                           int32_t* tiles_per_gauss, int64_t* isect_ids, int32_t* flatten_ids) {
    const int ntx = (W + tsx - 1) / tsx, nty = (H + tsy - 1) / tsy;
    const f2 ts{float(tsx), float(tsy)};
    std::vector<int64_t> cum(n);
    int64_t total = 0;
    std::vector<int> tmin(2 * n), tmax(2 * n);
    for (int64_t i = 0; i < n; ++i) {
        f2 r{radii[2 * i], radii[2 * i + 1]};
        int cnt = 0;
        if (!(r.x <= 0 || r.y <= 0)) {
            const f2 m = f2{means2d[2 * i], means2d[2 * i + 1]} / ts;
            r = r / ts;
            const int x0 = std::min(ntx, std::max(0, f2i(std::floor(m.x - r.x))));
            const int y0 = std::min(nty, std::max(0, f2i(std::floor(m.y - r.y))));
            const int x1 = std::min(ntx, std::max(0, f2i(std::ceil(m.x + r.x))));
            const int y1 = std::min(nty, std::max(0, f2i(std::ceil(m.y + r.y))));
            tmin[2 * i] = x0; tmin[2 * i + 1] = y0; tmax[2 * i] = x1; tmax[2 * i + 1] = y1;
            cnt = (y1 - y0) * (x1 - x0);
        }
        tiles_per_gauss[i] = cnt;
        total += cnt;
        cum[i] = total;
    }
    if (!isect_ids) return total;
    std::vector<int64_t> keys(total);
    std::vector<int32_t> vals(total);
    for (int64_t i = 0; i < n; ++i) {
        if (tiles_per_gauss[i] <= 0) continue;
        int64_t off = i > 0 ? cum[i - 1] : 0;
        for (int y = tmin[2 * i + 1]; y < tmax[2 * i + 1]; ++y)
            for (int x = tmin[2 * i]; x < tmax[2 * i]; ++x) {
                keys[off] = make_key(int64_t(y) * ntx + x, depths[i]);
                vals[off] = int32_t(i);
                ++off;
            }
    }
    if (sort && total) sort_pairs(keys, vals, tile_bits(ntx * nty));
    std::memcpy(isect_ids, keys.data(), total * 8);
    std::memcpy(flatten_ids, vals.data(), total * 4);
    return total;
}

// Lidar (irregular elevation) and spherical (regular) azimuth/elevation
// tiling with the wrap re-projection for flag 2:
// phm_lidar_tiling.cu:52-351 and phm_spherical_tiling.cu:15-291.
int64_t xsgo_isect_spherical(int lidar, const float* pack, const float* elev_values,
                             const float* pts, const float* vel, const float* scales,
                             const float* quats, const float* opac, const uint8_t* flags,
                             const float* means2d, const float* radii, const float* depths,
                             const float* elev_bounds, int n_elev_bounds, int64_t n, int tsx,
                             int tsy, float W, float H, float ua, float ub, float uk, int sort,
                             int32_t* tiles_per_gauss, int64_t* isect_ids, int32_t* flatten_ids) {
    const Cam k = Cam::load(lidar ? CAM_LIDAR : CAM_SPHERICAL, pack, elev_values);
    const int n_az = lidar ? (static_cast<int>(W) + tsx - 1) / tsx
                           : static_cast<int>(std::ceil(W / static_cast<float>(tsx)));
    const int n_el = lidar ? n_elev_bounds
                           : static_cast<int>(std::ceil(H / static_cast<float>(tsy)));
    const float u_per_tile = static_cast<float>(tsx) / W;
    const float v_per_tile = lidar ? std::ceil(H / static_cast<float>(n_el)) / H
                                   : static_cast<float>(tsy) / H;
    const f2 img{W, H};
    UTArgs a{1e-4f, 0.002f, 1.0f, img, ut_weights(ua, ub, uk)};

    // one tile rectangle [x0, x1) x [y0, y1) in the regular/exclusive form
    struct Rect { int x0, y0, x1, y1; };
    auto limits = [&](f2 m, f2 r, float umin, float umax, Rect& rc) -> int {
        const float lo = std::fmax(m.x - r.x, umin);
        const float hi = std::fmin(m.x + r.x, umax);
        if (lidar) {
            rc = {0, 0, 0, 0};
            if (hi <= lo) return 0;
            int tx0 = f2i(std::floor(lo / u_per_tile));
            int tx1 = f2i(std::ceil(hi / u_per_tile)) - 1;
            int ty0, ty1;
            bounds_increasing(m.y - r.y, m.y + r.y, n_el, elev_bounds, ty0, ty1);
            rc = {tx0, ty0, tx1 + 1, ty1 + 1};
            return (ty1 - ty0 + 1) * (tx1 - tx0 + 1);
        }
        rc = {0, 0, 0, 0};
        if (hi <= lo) return 0;
        const int tx0 = f2i(std::floor(lo / u_per_tile));
        const int ty0 = std::min(n_el, std::max(0, f2i(std::floor((m.y - r.y) / v_per_tile))));
        const int tx1 = f2i(std::ceil(hi / u_per_tile));
        const int ty1 = std::min(n_el, std::max(0, f2i(std::ceil((m.y + r.y) / v_per_tile))));
        rc = {tx0, ty0, tx1, ty1};
        return (ty1 - ty0) * (tx1 - tx0);
    };

    std::vector<Rect> r1(n), r2(n);
    std::vector<float> dep2(n);
    std::vector<uint8_t> has2(n, 0);
    int64_t total = 0;
    std::vector<int64_t> cum(n);
    const float u_pose = std::fabs(k.rolling.x) > 0.0f ? (k.pose - k.trigger) / k.rolling.x : 0.5f;
    for (int64_t i = 0; i < n; ++i) {
        f2 rr{radii[2 * i], radii[2 * i + 1]};
        const uint8_t fl = flags[i];
        int cnt = 0;
        r1[i] = {0, 0, 0, 0};
        if (!(rr.x <= 0 || rr.y <= 0 || fl == 0)) {
            float umin = 0.0f, umax = 1.0f;
            if (fl == 2) {
                if (k.rolling.x > 0) umax = u_pose; else umin = u_pose;
            }
            const f2 m = f2{means2d[2 * i], means2d[2 * i + 1]} / img;
            rr = rr / img;
            cnt += limits(m, rr, umin, umax, r1[i]);
            if (fl == 2) {
                const f3 P{pts[3 * i], pts[3 * i + 1], pts[3 * i + 2]};
                const f3 V = vel ? f3{vel[3 * i], vel[3 * i + 1], vel[3 * i + 2]} : f3{0, 0, 0};
                const f3 S{scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
                const quat Q{quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
                const float o = opac ? opac[i] : 1.0f;
                f3 d[3];
                ut_deltas(a.w.sq, Q, S, d);
                f2 m2, rad2; float dp2, tmp;
                if (ut_projection(k, a, MODE_POS, P, V, o, d, m2, rad2, dp2, tmp)) {
                    if (k.rolling.x > 0) {
                        umin = std::ceil(u_pose / u_per_tile) * u_per_tile + 1e-6f;
                        umax = 1.0f;
                    } else {
                        umin = 0.0f;
                        umax = std::floor(u_pose / u_per_tile) * u_per_tile - 1e-6f;
                    }
                    cnt += limits(m2 / img, rad2 / img, umin, umax, r2[i]);
                    dep2[i] = dp2;
                    has2[i] = 1;
                }
            }
        }
        tiles_per_gauss[i] = cnt;
        total += cnt;
        cum[i] = total;
    }
    if (!isect_ids) return total;
    std::vector<int64_t> keys(total);
    std::vector<int32_t> vals(total);
    for (int64_t i = 0; i < n; ++i) {
        if (tiles_per_gauss[i] <= 0) continue;
        int64_t off = i > 0 ? cum[i - 1] : 0;
        auto fill = [&](const Rect& rc, float depth) {
            for (int y = rc.y0; y < rc.y1; ++y)
                for (int x = rc.x0; x < rc.x1; ++x) {
                    keys[off] = make_key(int64_t(y) * n_az + x, depth);
                    vals[off] = int32_t(i);
                    ++off;
                }
        };
        fill(r1[i], depths[i]);
        if (has2[i]) fill(r2[i], dep2[i]);
    }
    if (sort && total) sort_pairs(keys, vals, tile_bits(n_az * n_el));
    std::memcpy(isect_ids, keys.data(), total * 8);
    std::memcpy(flatten_ids, vals.data(), total * 4);
    return total;
}

// isect_offset_encode, tiling_common.cu:25-99
void xsgo_isect_offset_encode(const int64_t* isect_ids, int64_t n_isects, int tw, int th,
                              int32_t* offsets) {
    const int64_t n_tiles = int64_t(tw) * th;
    if (n_isects == 0) {
        std::fill(offsets, offsets + n_tiles, 0);
        return;
    }
    const int tb = tile_bits(int(n_tiles));
    auto tile_of = [&](int64_t key) {
        const int64_t hi = key >> 32;
        return (hi >> tb) * n_tiles + (hi & ((1 << tb) - 1));
    };
    for (int64_t idx = 0; idx < n_isects; ++idx) {
        const int64_t cur = tile_of(isect_ids[idx]);
        if (idx == 0)
            for (int64_t t = 0; t < cur + 1; ++t) offsets[t] = 0;
        if (idx == n_isects - 1)
            for (int64_t t = cur + 1; t < n_tiles; ++t) offsets[t] = int32_t(n_isects);
        if (idx > 0) {
            const int64_t hp = isect_ids[idx - 1] >> 32, hc = isect_ids[idx] >> 32;
            if (hp == hc) continue;
            const int64_t prev = tile_of(isect_ids[idx - 1]);
            for (int64_t t = prev + 1; t < cur + 1; ++t) offsets[t] = int32_t(idx);
        }
    }
}

// ------------------------------------------------------------ rasteriser --
// One Gaussian's world-to-"unit sphere" transform M = S^-1 R^T
// (eval3d_fwd.cu:90-106, rasterization/utils.h:61-83); M[i] is row i.
static void gauss_M(const float* q4, const float* s3, f3 M[3], f3 R[3]) {
    float w = q4[0], x = q4[1], y = q4[2], z = q4[3];
    const float inv = 1.0f / std::sqrt(x * x + y * y + z * z + w * w);
    x *= inv; y *= inv; z *= inv; w *= inv;
    const float x2 = x * x, y2 = y * y, z2 = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    // R rows (R = [c0 c1 c2] with the columns of utils.h:70-80)
    R[0] = {1.f - 2.f * (y2 + z2), 2.f * (xy - wz), 2.f * (xz + wy)};
    R[1] = {2.f * (xy + wz), 1.f - 2.f * (x2 + z2), 2.f * (yz - wx)};
    R[2] = {2.f * (xz - wy), 2.f * (yz + wx), 1.f - 2.f * (x2 + y2)};
    const float is[3] = {1.0f / s3[0], 1.0f / s3[1], 1.0f / s3[2]};
    // row i of S^-1 R^T = (1/s_i) * column i of R
    for (int i = 0; i < 3; ++i) {
        const f3 col{(&R[0].x)[i], (&R[1].x)[i], (&R[2].x)[i]};
        M[i] = is[i] * col;
    }
}
static inline f3 mat_vec(const f3 M[3], f3 v) { return {dot(M[0], v), dot(M[1], v), dot(M[2], v)}; }
static inline f3 safe_normalize(f3 v) {
    const float l = dot(v, v);
    return l > 0.0f ? v * (1.0f / std::sqrt(l)) : v;
}

// How far apart two float32 evaluations of one pair's alpha may land,
// relative (different summation order or fused multiply-adds, 2-ulp exp /
// rsqrt).  gro = M (o - mu) sums terms of size |M_ij| |(o - mu)_j| and
// cancels down to |gro|; gc = normalize(grd) x gro cancels again down to
// |gc|; so gc moves by a few ulps of (terms + |gro|) and power = -|gc|^2 / 2
// by |gc| |d gc|.  The factor 3 is about five times the largest difference
// seen between this oracle and the CUDA kernels on the parity scenes.
static inline float alpha_rel_error(const f3 M[3], f3 mu, f3 om, f3 gro, f3 gc, float power, bool moving) {
    const float eps = 5.97e-8f;  // 2^-24
    float terms = 0.f, mmax = 0.f;
    for (int i = 0; i < 3; ++i) {
        terms = std::fmax(terms, std::fabs(M[i].x * om.x) + std::fabs(M[i].y * om.y) + std::fabs(M[i].z * om.z));
        mmax = std::fmax(mmax, std::fabs(M[i].x) + std::fabs(M[i].y) + std::fabs(M[i].z));
    }
    // a moving centre mu + t v may round differently (fused or not)
    const float d_mu = moving ? mmax * std::fmax(std::fmax(std::fabs(mu.x), std::fabs(mu.y)), std::fabs(mu.z)) : 0.f;
    const float d_gc = 3.f * eps * (terms + d_mu + std::sqrt(dot(gro, gro)));
    return std::sqrt(dot(gc, gc)) * d_gc + 8.f * eps * (1.f + std::fabs(power)) + 1e-6f;
}

// Front-to-back 3D-evaluation compositing, eval3d_fwd.cu:34-166 (static) and
// eval3d_dynamic_fwd.cu:38-173 (velocity, per-pixel time).  `near` (may be
// null) returns, per pixel, 1 when a test whose outcome two float32
// evaluations may decide differently was within the pair's alpha error
// band of its threshold: the alpha >= 1/255 test, the termination test
// T (1 - alpha) <= 1e-4 (with the accumulated error of T), or the backward's
// opacity * vis <= 0.99 gate (eval3d_bwd.cu:190-205), which switches the
// power-term gradient on or off.
void xsgo_rasterize_fwd(const float* means, const float* vel, const float* quats,
                        const float* scales, const float* colors, int cdim, const float* opac,
                        int W, int H, int tsx, int tsy, const float* ray_o, const float* ray_d,
                        const float* ray_t, const int32_t* offsets, int ntx, int nty,
                        const int32_t* flatten, int64_t n_isects, float* out_rgb,
                        float* out_depth, float* out_alpha, int32_t* last_ids, uint8_t* near) {
    const int64_t npx = int64_t(W) * H;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t pix = 0; pix < npx; ++pix) {
        const int i = int(pix / W), j = int(pix % W);
        const int tile = (i / tsy) * ntx + (j / tsx);
        const int64_t start = offsets[tile];
        const int64_t end = (tile == ntx * nty - 1) ? n_isects : offsets[tile + 1];
        const f3 o{ray_o[3 * pix], ray_o[3 * pix + 1], ray_o[3 * pix + 2]};
        const f3 d{ray_d[3 * pix], ray_d[3 * pix + 1], ray_d[3 * pix + 2]};
        const float t_ray = ray_t ? ray_t[pix] : 0.0f;
        float T = 1.0f, depth = 0.0f;
        float acc[600] = {0};
        int64_t cur = 0;
        bool amb = false;
        float t_err = 1e-5f;  // relative error bound of T
        for (int64_t k = start; k < end; ++k) {
            const int32_t g = flatten[k];
            f3 M[3], R[3];
            gauss_M(quats + 4 * g, scales + 3 * g, M, R);
            f3 mu{means[3 * g], means[3 * g + 1], means[3 * g + 2]};
            if (vel) mu = mu + t_ray * f3{vel[3 * g], vel[3 * g + 1], vel[3 * g + 2]};
            const f3 om = o - mu;
            const f3 gro = mat_vec(M, om);
            const f3 grd = mat_vec(M, d);
            const f3 gc = cross(safe_normalize(grd), gro);
            const float power = -0.5f * dot(gc, gc);
            const float a_raw = opac[g] * std::exp(power);
            const float alpha = std::fmin(0.999f, a_raw);
            if (near) {
                const float band = alpha_rel_error(M, mu, om, gro, gc, power, vel != nullptr);
                if (std::fabs(a_raw * 255.0f - 1.0f) < band) amb = true;
                if (a_raw >= 1.f / 255.f && std::fabs(a_raw / 0.99f - 1.0f) < band) amb = true;
                if (alpha >= 1.f / 255.f) t_err += band * alpha / std::fmax(1.0f - alpha, 1e-3f);
            }
            if (alpha < 1.f / 255.f) continue;
            const float hit_t = -dot(gro, grd) / dot(grd, grd);
            const float nT = T * (1.0f - alpha);
            if (std::fabs(nT * 1e4f - 1.0f) < t_err) amb = true;
            if (nT <= 1e-4f) break;
            const float vis = alpha * T;
            depth += vis * hit_t;
            for (int c = 0; c < cdim; ++c) acc[c] += colors[int64_t(g) * cdim + c] * vis;
            cur = k;
            T = nT;
        }
        out_alpha[pix] = 1.0f - T;
        out_depth[pix] = depth;
        for (int c = 0; c < cdim; ++c) out_rgb[pix * cdim + c] = acc[c];
        last_ids[pix] = int32_t(cur);
        if (near) near[pix] = amb ? 1 : 0;
    }
}

// Back-to-front gradient replay, eval3d_bwd.cu:38-294 (static) and
// eval3d_dynamic_bwd.cu:68-310 (dynamic: vel and ray_t non-null).  Gradient
// outputs must be zero-filled by the caller; per-Gaussian gradients are
// accumulated here with a per-thread buffer and reduced at the end.
void xsgo_rasterize_bwd(const float* means, const float* vel, const float* quats,
                        const float* scales, const float* colors, int cdim, const float* opac,
                        int W, int H, int tsx, int tsy, const float* ray_o, const float* ray_d,
                        const float* ray_t, const int32_t* offsets, int ntx, int nty,
                        const int32_t* flatten, int64_t n_isects, int64_t n_gauss,
                        const float* render_alpha, const int32_t* last_ids, const float* v_rgb,
                        const float* v_depth, const float* v_alpha, float* v_means,
                        float* v_vel, float* v_quats, float* v_scales, float* v_colors,
                        float* v_opac, float* v_ray_o, float* v_ray_d, float* v_ray_t) {
    const int64_t npx = int64_t(W) * H;
    const int stride = 3 + 3 + 4 + 3 + 1 + cdim;   // mean, vel, quat, scale, opac, colour
    int nthreads = 1;
#ifdef _OPENMP
    nthreads = omp_get_max_threads();
#endif
    std::vector<std::vector<double>> part(nthreads);
#pragma omp parallel
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        std::vector<double>& buf = part[tid];
        buf.assign(size_t(n_gauss) * stride, 0.0);
#pragma omp for schedule(dynamic, 64)
        for (int64_t pix = 0; pix < npx; ++pix) {
            const int i = int(pix / W), j = int(pix % W);
            const int tile = (i / tsy) * ntx + (j / tsx);
            const int64_t start = offsets[tile];
            const int64_t end = (tile == ntx * nty - 1) ? n_isects : offsets[tile + 1];
            const f3 o{ray_o[3 * pix], ray_o[3 * pix + 1], ray_o[3 * pix + 2]};
            const f3 d{ray_d[3 * pix], ray_d[3 * pix + 1], ray_d[3 * pix + 2]};
            const float t_ray = ray_t ? ray_t[pix] : 0.0f;
            const float T_final = 1.0f - render_alpha[pix];
            float T = T_final;
            float buffer[600] = {0};
            const int64_t bin_final = last_ids[pix];
            float vc[600];
            for (int c = 0; c < cdim; ++c) vc[c] = v_rgb ? v_rgb[pix * cdim + c] : 0.0f;
            const float vd = v_depth[pix], va = v_alpha[pix];
            f3 vro{0, 0, 0}, vrd{0, 0, 0};
            float vtime = 0.0f, dbuf = 0.0f;
            for (int64_t k = end - 1; k >= start; --k) {
                if (k > bin_final) continue;
                const int32_t g = flatten[k];
                f3 M[3], R[3];
                gauss_M(quats + 4 * g, scales + 3 * g, M, R);
                f3 v_g{0, 0, 0};
                if (vel) v_g = {vel[3 * g], vel[3 * g + 1], vel[3 * g + 2]};
                const f3 mu = f3{means[3 * g], means[3 * g + 1], means[3 * g + 2]} + t_ray * v_g;
                const f3 omm = o - mu;
                const f3 gro = mat_vec(M, omm);
                const f3 grd = mat_vec(M, d);
                const f3 grd_n = safe_normalize(grd);
                const f3 gc = cross(grd_n, gro);
                const float power = -0.5f * dot(gc, gc);
                const float vis = std::exp(power);
                const float op = opac[g];
                const float alpha = std::fmin(0.99f, op * vis);
                if (alpha < 1.f / 255.f) continue;
                const float hit_t = -dot(grd, gro) / dot(grd, grd);
                const float ra = 1.0f / std::fmax(1e-6f, 1.0f - alpha);
                T *= ra;
                const float fac = alpha * T;
                double* G = &buf[size_t(g) * stride];
                for (int c = 0; c < cdim; ++c) G[14 + c] += double(vc[c] * fac);
                float v_alpha_ = 0.0f;
                const float* rgb = colors ? colors + int64_t(g) * cdim : nullptr;
                for (int c = 0; c < cdim; ++c) v_alpha_ += (rgb[c] * T - buffer[c] * ra) * vc[c];
                v_alpha_ += (hit_t * T - dbuf * ra) * vd;
                v_alpha_ += T_final * ra * va;
                const float dd = dot(grd, grd);
                const float od = dot(gro, grd);
                const float dLdt = vd * fac;
                f3 v_gro = (-1.0f * grd) * dLdt / dd;
                f3 v_grd = (2.0f * od * grd - dd * gro) * dLdt / (dd * dd);
                if (op * vis <= 0.99f) {
                    const float v_vis = op * v_alpha_;
                    const float v_dist = -0.5f * vis * v_vis;
                    const f3 v_gc = 2.0f * v_dist * gc;
                    const f3 v_grd_n = -cross(v_gc, gro);
                    v_gro += cross(v_gc, grd_n);
                    // safe_normalize_bwd, rasterization/utils.h:197-205
                    const float l = dot(grd, grd);
                    if (l > 0.0f) {
                        const float il = 1.0f / std::sqrt(l);
                        v_grd += il * v_grd_n - (il * il * il) * dot(v_grd_n, grd) * grd;
                    } else {
                        v_grd += v_grd_n;
                    }
                    // v_M = outer(v_grd, d) + outer(v_gro, o - mu), row-major rows
                    f3 vM[3];
                    for (int r = 0; r < 3; ++r)
                        vM[r] = (&v_grd.x)[r] * d + (&v_gro.x)[r] * omm;
                    // v_(o - mu) = M^T v_gro ; v_d = M^T v_grd
                    const f3 v_omm = (&v_gro.x)[0] * M[0] + (&v_gro.x)[1] * M[1] + (&v_gro.x)[2] * M[2];
                    const f3 v_dd = (&v_grd.x)[0] * M[0] + (&v_grd.x)[1] * M[1] + (&v_grd.x)[2] * M[2];
                    G[0] += -double(v_omm.x); G[1] += -double(v_omm.y); G[2] += -double(v_omm.z);
                    vro += v_omm;
                    vrd += v_dd;
                    if (vel) {
                        G[3] += -double(v_omm.x * t_ray); G[4] += -double(v_omm.y * t_ray);
                        G[5] += -double(v_omm.z * t_ray);
                        vtime += -dot(v_omm, v_g);
                    }
                    // M = S^-1 R^T: v_scale_i = -(1/s_i)^2 (R col_i . vM row_i)
                    //               v_R[a][i] = vM[i][a] / s_i
                    const float* s3 = scales + 3 * g;
                    float vR[3][3];
                    for (int r = 0; r < 3; ++r) {
                        const float is = 1.0f / s3[r];
                        const f3 col{(&R[0].x)[r], (&R[1].x)[r], (&R[2].x)[r]};
                        G[10 + r] += double(-is * is * dot(col, vM[r]));
                        for (int a2 = 0; a2 < 3; ++a2) vR[a2][r] = (&vM[r].x)[a2] * is;
                    }
                    // d R / d quat through the normalisation (utils.h:208-230)
                    const float* q4 = quats + 4 * g;
                    float w = q4[0], x = q4[1], y = q4[2], z = q4[3];
                    const float inv = 1.0f / std::sqrt(x * x + y * y + z * z + w * w);
                    x *= inv; y *= inv; z *= inv; w *= inv;
                    // vR[row][col]; reference's v_R[c][r] is column-major
                    auto VR = [&](int cidx, int ridx) { return vR[ridx][cidx]; };
                    const float gw = 2.f * (x * (VR(1, 2) - VR(2, 1)) + y * (VR(2, 0) - VR(0, 2)) +
                                            z * (VR(0, 1) - VR(1, 0)));
                    const float gx = 2.f * (-2.f * x * (VR(1, 1) + VR(2, 2)) + y * (VR(0, 1) + VR(1, 0)) +
                                            z * (VR(0, 2) + VR(2, 0)) + w * (VR(1, 2) - VR(2, 1)));
                    const float gy = 2.f * (x * (VR(0, 1) + VR(1, 0)) - 2.f * y * (VR(0, 0) + VR(2, 2)) +
                                            z * (VR(1, 2) + VR(2, 1)) + w * (VR(2, 0) - VR(0, 2)));
                    const float gz = 2.f * (x * (VR(0, 2) + VR(2, 0)) + y * (VR(1, 2) + VR(2, 1)) -
                                            2.f * z * (VR(0, 0) + VR(1, 1)) + w * (VR(0, 1) - VR(1, 0)));
                    const float dq = gw * w + gx * x + gy * y + gz * z;
                    G[6] += double((gw - dq * w) * inv);
                    G[7] += double((gx - dq * x) * inv);
                    G[8] += double((gy - dq * y) * inv);
                    G[9] += double((gz - dq * z) * inv);
                    G[13] += double(vis * v_alpha_);
                }
                for (int c = 0; c < cdim; ++c) buffer[c] += rgb[c] * fac;
                dbuf += fac * hit_t;
            }
            v_ray_o[3 * pix] = vro.x; v_ray_o[3 * pix + 1] = vro.y; v_ray_o[3 * pix + 2] = vro.z;
            v_ray_d[3 * pix] = vrd.x; v_ray_d[3 * pix + 1] = vrd.y; v_ray_d[3 * pix + 2] = vrd.z;
            if (v_ray_t) v_ray_t[pix] = vtime;
        }
    }
    for (int64_t g = 0; g < n_gauss; ++g) {
        double acc[14 + 600] = {0};
        for (int t = 0; t < nthreads; ++t) {
            if (part[t].empty()) continue;
            const double* G = &part[t][size_t(g) * stride];
            for (int s = 0; s < stride; ++s) acc[s] += G[s];
        }
        for (int a = 0; a < 3; ++a) v_means[3 * g + a] = float(acc[a]);
        if (v_vel) for (int a = 0; a < 3; ++a) v_vel[3 * g + a] = float(acc[3 + a]);
        for (int a = 0; a < 4; ++a) v_quats[4 * g + a] = float(acc[6 + a]);
        for (int a = 0; a < 3; ++a) v_scales[3 * g + a] = float(acc[10 + a]);
        v_opac[g] = float(acc[13]);
        if (v_colors) for (int c = 0; c < cdim; ++c) v_colors[g * cdim + c] = float(acc[14 + c]);
    }
}

// -------------------------------------------------- spherical harmonics --
// Real SH basis up to degree 4 evaluated at a unit direction, the polynomial
// forms of sh_fwd.cu:16-115; basis[i] for band i.
static void sh_basis(int deg, float x, float y, float z, float* b) {
    b[0] = 0.2820947917738781f;
    if (deg < 1) return;
    b[1] = -0.48860251190292f * y;
    b[2] = 0.48860251190292f * z;
    b[3] = -0.48860251190292f * x;
    if (deg < 2) return;
    const float z2 = z * z;
    const float t0B = -1.092548430592079f * z;
    const float c1 = x * x - y * y, s1 = 2.f * x * y;
    b[4] = 0.5462742152960395f * s1;
    b[5] = t0B * y;
    b[6] = 0.9461746957575601f * z2 - 0.3153915652525201f;
    b[7] = t0B * x;
    b[8] = 0.5462742152960395f * c1;
    if (deg < 3) return;
    const float t0C = -2.285228997322329f * z2 + 0.4570457994644658f;
    const float t1B = 1.445305721320277f * z;
    const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
    b[9] = -0.5900435899266435f * s2;
    b[10] = t1B * s1;
    b[11] = t0C * y;
    b[12] = z * (1.865881662950577f * z2 - 1.119528997770346f);
    b[13] = t0C * x;
    b[14] = t1B * c1;
    b[15] = -0.5900435899266435f * c2;
    if (deg < 4) return;
    const float t0D = z * (-4.683325804901025f * z2 + 2.007139630671868f);
    const float t1C = 3.31161143515146f * z2 - 0.47308734787878f;
    const float t2B = -1.770130769779931f * z;
    const float c3 = x * c2 - y * s2, s3 = x * s2 + y * c2;
    b[16] = 0.6258357354491763f * s3;
    b[17] = t2B * s2;
    b[18] = t1C * s1;
    b[19] = t0D * y;
    b[20] = 1.984313483298443f * z * b[12] - 1.006230589874905f * b[6];
    b[21] = t0D * x;
    b[22] = t1C * c1;
    b[23] = t2B * c2;
    b[24] = 0.6258357354491763f * c3;
}

// Partial derivatives of the basis polynomials with respect to x, y, z
// (treated as independent, as sh_bwd.cu:20-247 does), computed in double by
// central differences of the polynomial in double precision would be
// inexact, so they are differentiated analytically here.
static void sh_basis_grad(int deg, double x, double y, double z, double* bx, double* by,
                          double* bz) {
    for (int i = 0; i < 25; ++i) bx[i] = by[i] = bz[i] = 0.0;
    if (deg < 1) return;
    const double K1 = 0.48860251190292;
    by[1] = -K1; bz[2] = K1; bx[3] = -K1;
    if (deg < 2) return;
    const double K4 = 0.5462742152960395, K5 = -1.092548430592079, K6 = 0.9461746957575601;
    bx[4] = K4 * 2 * y; by[4] = K4 * 2 * x;
    by[5] = K5 * z; bz[5] = K5 * y;
    bz[6] = 2 * K6 * z;
    bx[7] = K5 * z; bz[7] = K5 * x;
    bx[8] = K4 * 2 * x; by[8] = -K4 * 2 * y;
    if (deg < 3) return;
    const double K9 = -0.5900435899266435, KT = 1.445305721320277;
    const double A = -2.285228997322329, B = 0.4570457994644658;
    const double C = 1.865881662950577, D = -1.119528997770346;
    // s2 = 3x^2 y - y^3 ; c2 = x^3 - 3 x y^2
    bx[9] = K9 * 6 * x * y; by[9] = K9 * (3 * x * x - 3 * y * y);
    bx[10] = KT * z * 2 * y; by[10] = KT * z * 2 * x; bz[10] = KT * 2 * x * y;
    by[11] = A * z * z + B; bz[11] = 2 * A * z * y;
    bz[12] = 3 * C * z * z + D;
    bx[13] = A * z * z + B; bz[13] = 2 * A * z * x;
    bx[14] = KT * z * 2 * x; by[14] = -KT * z * 2 * y; bz[14] = KT * (x * x - y * y);
    bx[15] = K9 * (3 * x * x - 3 * y * y); by[15] = K9 * (-6 * x * y);
    if (deg < 4) return;
    const double K16 = 0.6258357354491763, E = -4.683325804901025, F = 2.007139630671868;
    const double G = 3.31161143515146, Hh = -0.47308734787878, I = -1.770130769779931;
    // s3 = 4x^3 y - 4 x y^3 ; c3 = x^4 - 6 x^2 y^2 + y^4
    bx[16] = K16 * (12 * x * x * y - 4 * y * y * y); by[16] = K16 * (4 * x * x * x - 12 * x * y * y);
    bx[17] = I * z * 6 * x * y; by[17] = I * z * (3 * x * x - 3 * y * y); bz[17] = I * (3 * x * x * y - y * y * y);
    bx[18] = (G * z * z + Hh) * 2 * y; by[18] = (G * z * z + Hh) * 2 * x; bz[18] = 2 * G * z * 2 * x * y;
    by[19] = E * z * z * z + F * z; bz[19] = (3 * E * z * z + F) * y;
    // b20 = 1.98 z b12 - 1.006 b6, b12 = z (C z^2 + D), b6 = K6 z^2 - c
    bz[20] = 1.984313483298443 * (z * (C * z * z + D) + z * (3 * C * z * z + D)) -
             1.006230589874905 * (2 * K6 * z);
    bx[21] = E * z * z * z + F * z; bz[21] = (3 * E * z * z + F) * x;
    bx[22] = (G * z * z + Hh) * 2 * x; by[22] = -(G * z * z + Hh) * 2 * y; bz[22] = 2 * G * z * (x * x - y * y);
    bx[23] = I * z * (3 * x * x - 3 * y * y); by[23] = I * z * (-6 * x * y); bz[23] = I * (x * x * x - 3 * x * y * y);
    bx[24] = K16 * (4 * x * x * x - 12 * x * y * y); by[24] = K16 * (-12 * x * x * y + 4 * y * y * y);
}

// spherical_harmonics_fused_fwd, sh_fwd.cu:119-245.  layout_3kn selects
// [3, K, N] coefficients (else [N, K, 3]); dc (optional) holds band 0 apart.
void xsgo_sh_fwd(int deg, const float* origin, const float* pos, const float* coeffs,
                 const float* dc, const uint32_t* mask, int layout_3kn, int64_t n, int dim,
                 float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        if (mask && !((mask[i / 32] >> (i % 32)) & 1u)) continue;
        const f3 dir = normalize(f3{pos[3 * i] - origin[0], pos[3 * i + 1] - origin[1],
                                    pos[3 * i + 2] - origin[2]});
        float b[25];
        sh_basis(deg, dir.x, dir.y, dir.z, b);
        const int bands = (deg + 1) * (deg + 1);
        for (int ch = 0; ch < 3; ++ch) {
            double acc = 0.0;
            for (int k = 0; k < bands; ++k) {
                float cf;
                if (dc && k == 0)
                    cf = layout_3kn ? dc[int64_t(ch) * n + i] : dc[i * 3 + ch];
                else {
                    const int kk = dc ? k - 1 : k;
                    cf = layout_3kn ? coeffs[(int64_t(ch) * dim + kk) * n + i]
                                    : coeffs[(i * dim + kk) * 3 + ch];
                }
                acc += double(b[k]) * double(cf);
            }
            out[3 * i + ch] = float(acc) + 0.5f;
        }
    }
}

// spherical_harmonics_fused_bwd, sh_bwd.cu:250-376.  d_coeffs/d_dc/d_pos
// must be zero-filled by the caller; d_origin gets the total.
void xsgo_sh_bwd(int deg, const float* origin, const float* pos, const float* coeffs,
                 const float* dc, const uint32_t* mask, int layout_3kn, int64_t n, int dim,
                 const float* d_out, float* d_coeffs, float* d_dc, float* d_pos,
                 float* d_origin) {
    double o_acc[3] = {0, 0, 0};
    for (int64_t i = 0; i < n; ++i) {
        if (mask && !((mask[i / 32] >> (i % 32)) & 1u)) continue;
        const f3 diff{pos[3 * i] - origin[0], pos[3 * i + 1] - origin[1], pos[3 * i + 2] - origin[2]};
        const f3 dir = normalize(diff);
        float b[25];
        sh_basis(deg, dir.x, dir.y, dir.z, b);
        double bx[25], by[25], bz[25];
        sh_basis_grad(deg, dir.x, dir.y, dir.z, bx, by, bz);
        const int bands = (deg + 1) * (deg + 1);
        double gd[3] = {0, 0, 0};
        for (int ch = 0; ch < 3; ++ch) {
            const float g = d_out[3 * i + ch];
            for (int k = 0; k < bands; ++k) {
                float cf;
                float* dst;
                if (dc && k == 0) {
                    const int64_t o = layout_3kn ? int64_t(ch) * n + i : i * 3 + ch;
                    cf = dc[o]; dst = d_dc + o;
                } else {
                    const int kk = dc ? k - 1 : k;
                    const int64_t o = layout_3kn ? (int64_t(ch) * dim + kk) * n + i
                                                 : (i * dim + kk) * 3 + ch;
                    cf = coeffs[o]; dst = d_coeffs + o;
                }
                *dst = b[k] * g;
                gd[0] += bx[k] * cf * g; gd[1] += by[k] * cf * g; gd[2] += bz[k] * cf * g;
            }
        }
        // normalize backward: (g - n (n.g)) / |v|
        const double l = std::sqrt(double(diff.x) * diff.x + double(diff.y) * diff.y +
                                   double(diff.z) * diff.z);
        const double nx = diff.x / l, ny = diff.y / l, nz = diff.z / l;
        const double ng = nx * gd[0] + ny * gd[1] + nz * gd[2];
        const double dx = (gd[0] - nx * ng) / l, dy = (gd[1] - ny * ng) / l, dz = (gd[2] - nz * ng) / l;
        d_pos[3 * i] += float(dx); d_pos[3 * i + 1] += float(dy); d_pos[3 * i + 2] += float(dz);
        o_acc[0] -= dx; o_acc[1] -= dy; o_acc[2] -= dz;
    }
    d_origin[0] = float(o_acc[0]); d_origin[1] = float(o_acc[1]); d_origin[2] = float(o_acc[2]);
}

}  // extern "C"
