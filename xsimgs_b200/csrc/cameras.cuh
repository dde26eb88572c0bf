// Rolling-shutter camera models on the device (pinhole, OpenCV fisheye,
// spherical, lidar) and the Newton-iteration point projection.
//
// Semantics follow the reference's Camera<Impl> (include/cameras/camera.h:67-183),
// PerspectiveCameraImpl (csrc/cameras/perspective.cu:7-71),
// OpenCVFisheyeCameraImpl (csrc/cameras/fisheye_opencv.cu:5-188),
// SphericalCamera / LidarCameraImpl (csrc/cameras/spherical.h:9-163) and
// camera_projection (include/cameras/projection_kernels.h:12-256).  The pack
// layout is documented in include/xsimgs_b200.h.
#pragma once

#include "common.cuh"

namespace xsg {

enum { MODE_CENTRAL = 0, MODE_NEG = 1, MODE_POS = 2 };

struct CamBase {
    float qw, qx, qy, qz;  // camera->world rotation at pose_time (wxyz)
    v3 t0, v, w;
    float2 rolling;
    float trigger, pose;

    __device__ __forceinline__ void load_base(const float* p) {
        qw = p[0]; qx = p[1]; qy = p[2]; qz = p[3];
        t0 = mk3(p[4], p[5], p[6]);
        v = mk3(p[7], p[8], p[9]);
        w = mk3(p[10], p[11], p[12]);
        rolling = make_float2(p[14], p[15]);
        trigger = p[16];
        pose = p[17];
    }
    __device__ __forceinline__ float pixel_time(float u, float vv) const {
        return trigger + (u * rolling.x + vv * rolling.y);
    }
};

// ---------------------------------------------------------------- models --
struct Pinhole : CamBase {
    static constexpr int kType = XSG_CAM_PINHOLE;
    static constexpr bool kJacobian = true;
    static constexpr int kWords = 22;
    float2 f, c;
    __device__ __forceinline__ void load(const float* p) {
        load_base(p);
        f = make_float2(p[18], p[19]);
        c = make_float2(p[20], p[21]);
    }
    __device__ __forceinline__ float2 pixel_to_uv(int px, int py, int W, int H) const {
        return make_float2((float(px) + 0.5f) / float(W), (float(py) + 0.5f) / float(H));
    }
    __device__ __forceinline__ v3 ray_cs(float2 uv) const {
        return mk3((uv.x - c.x) / f.x, (uv.y - c.y) / f.y, 1.0f);
    }
    __device__ __forceinline__ bool ray_valid(float2) const { return true; }
    // d(ray_cs)/d(f, c) applied to d_ray, added to pack words 18..21
    // (perspective.cu:18-34).
    template <int P>
    __device__ __forceinline__ void ray_cs_bwd(float2 uv, v3 d, float (&acc)[P]) const {
        const float ifx = 1.0f / f.x, ify = 1.0f / f.y;
        acc[18] -= d.x * (uv.x - c.x) * ifx * ifx;
        acc[19] -= d.y * (uv.y - c.y) * ify * ify;
        acc[20] -= d.x * ifx;
        acc[21] -= d.y * ify;
    }
    __device__ __forceinline__ v3 to_uvd(int, v3 p) const {
        return mk3(p.x * f.x / p.z + c.x, p.y * f.y / p.z + c.y, p.z);
    }
    __device__ __forceinline__ void to_uvd_jac(int mode, v3 p, v3 dp, v3& uvd, float2& duv) const {
        uvd = to_uvd(mode, p);
        duv = make_float2(f.x * (dp.x - uvd.x * dp.z) / uvd.z, f.y * (dp.y - uvd.y * dp.z) / uvd.z);
    }
};

struct Fisheye : CamBase {
    static constexpr int kType = XSG_CAM_FISHEYE;
    static constexpr bool kJacobian = false;
    static constexpr int kWords = 28;
    float2 f, c;
    float4 k;
    __device__ __forceinline__ void load(const float* p) {
        load_base(p);
        f = make_float2(p[20], p[21]);
        c = make_float2(p[22], p[23]);
        k = make_float4(p[24], p[25], p[26], p[27]);
    }
    __device__ __forceinline__ float2 pixel_to_uv(int px, int py, int W, int H) const {
        return make_float2((float(px) + 0.5f) / float(W), (float(py) + 0.5f) / float(H));
    }
    __device__ __forceinline__ float distort(float th) const {
        const float t2 = th * th;
        float d = t2 * k.w + k.z;
        d = t2 * d + k.y;
        d = t2 * d + k.x;
        d = t2 * d + 1.0f;
        return th * d;
    }
    __device__ __forceinline__ float distort_deriv(float th) const {
        const float t2 = th * th;
        float d = t2 * 9.0f * k.w + 7.0f * k.z;
        d = t2 * d + 5.0f * k.y;
        d = t2 * d + 3.0f * k.x;
        d = t2 * d + 1.0f;
        return d;
    }
    // theta_d(theta) = delta by clamped Newton steps (fisheye_opencv.cu:34-47)
    __device__ __forceinline__ float solve(float delta, float& residual) const {
        float th = delta;
        residual = 0.0f;
#pragma unroll 1
        for (int i = 0; i < 20; ++i) {
            residual = distort(th) - delta;
            th -= residual / fmaxf(distort_deriv(th), 0.1f);
            th = fminf(fmaxf(th, 0.0f), float(M_PI));
            if (fabsf(residual) < 1e-6f) break;
        }
        return th;
    }
    __device__ __forceinline__ v3 ray_cs(float2 uv) const {
        const float ux = (uv.x - c.x) / f.x, uy = (uv.y - c.y) / f.y;
        const float delta = sqrtf(ux * ux + uy * uy);
        float res;
        const float th = solve(delta, res);
        if (th <= 0.0f) return mk3(0.0f, 0.0f, 1.0f);
        float s, co;
        sincosf(th, &s, &co);
        const float sf = s / delta;
        return mk3(sf * ux, sf * uy, co);
    }
    __device__ __forceinline__ bool ray_valid(float2 uv) const {
        const float ux = (uv.x - c.x) / f.x, uy = (uv.y - c.y) / f.y;
        const float delta = sqrtf(ux * ux + uy * uy);
        if (delta <= 1e-8f) return true;
        float res;
        const float th = solve(delta, res);
        return (fabsf(res) < 1e-5f) && (distort_deriv(th) > 0.0f);
    }
    // Backward of ray_cs into f, c (words 20..23) and k1..k4 (24..27),
    // fisheye_opencv.cu:77-141.  theta(delta, k) is implicit in
    // distort(theta) = delta, so dtheta/ddelta = 1/distort' and
    // dtheta/dk_i = -theta^(2i+3)/distort'; rays whose re-solve did not
    // converge, or sit on the axis, get no gradient.
    template <int P>
    __device__ __forceinline__ void ray_cs_bwd(float2 uv, v3 d, float (&acc)[P]) const {
        const float ux = (uv.x - c.x) / f.x, uy = (uv.y - c.y) / f.y;
        const float delta = sqrtf(ux * ux + uy * uy);
        float res;
        const float th = solve(delta, res);
        const float der = distort_deriv(th);
        if (!((th > 0.0f) && (delta > 1e-8f) && (fabsf(res) < 1e-5f) && (der > 1e-3f))) return;
        float sn, cs;
        sincosf(th, &sn, &cs);
        const float idl = 1.0f / delta;
        const float s = sn * idl;
        const float d_s = d.x * ux + d.y * uy;
        const float d_th = d_s * cs * idl - d.z * sn;
        const float d_ths = d_th / der;
        const float t2 = th * th, t3 = t2 * th;
        acc[24] -= d_ths * t3;
        acc[25] -= d_ths * t3 * t2;
        acc[26] -= d_ths * t3 * t2 * t2;
        acc[27] -= d_ths * t3 * t2 * t2 * t2;
        const float d_dl = -d_s * sn * idl * idl + d_ths;
        const float dux = s * d.x + d_dl * ux * idl;
        const float duy = s * d.y + d_dl * uy * idl;
        acc[20] -= dux * ux / f.x;
        acc[21] -= duy * uy / f.y;
        acc[22] -= dux / f.x;
        acc[23] -= duy / f.y;
    }
    __device__ __forceinline__ v3 to_uvd(int, v3 p) const {
        const float norm = fmaxf(1e-6f, hypotf(p.x, p.y));
        const float th = atan2f(norm, p.z);
        const bool valid = distort_deriv(th) > 0.0f;
        const float delta = distort(th) / norm;
        const float u = f.x * delta * p.x + c.x;
        const float vv = f.y * delta * p.y + c.y;
        const float depth = (valid && (delta > 0.0f)) ? sqrtf(dot3(p, p)) : 0.0f;
        return mk3(u, vv, depth);
    }
    __device__ __forceinline__ void to_uvd_jac(int, v3, v3, v3&, float2&) const {}
};

// OpenCV 8-coefficient pinhole (k1 k2 p1 p2 | k3 k4 k5 k6, rational radial
// model + tangential), DistortedPerspectiveCameraImpl,
// csrc/cameras/distorted_perspective.cu:6-230 and include/cameras/distortion.h:8-30.
// Pack words 18..30: f.x f.y c.x c.y, k1 k2 p1 p2, k3 k4 k5 k6, max_radius^2.
struct Distorted : CamBase {
    static constexpr int kType = XSG_CAM_DISTORTED;
    static constexpr bool kJacobian = false;
    static constexpr int kWords = 36;
    static constexpr float kMinDet = 1e-3f;
    float2 f, c;
    float4 d0, d1;  // (k1, k2, p1, p2), (k3, k4, k5, k6)
    float max_r2;
    __device__ __forceinline__ void load(const float* p) {
        load_base(p);
        f = make_float2(p[20], p[21]);
        c = make_float2(p[22], p[23]);
        d0 = make_float4(p[24], p[25], p[26], p[27]);
        d1 = make_float4(p[28], p[29], p[30], p[31]);
        max_r2 = p[32];
    }
    __device__ __forceinline__ float2 pixel_to_uv(int px, int py, int W, int H) const {
        return make_float2((float(px) + 0.5f) / float(W), (float(py) + 0.5f) / float(H));
    }
    // Distortion D(x) = x * scale(r2) + delta(x) at x, with its (symmetric)
    // Jacobian; DistortionState, distorted_perspective.cu:11-78.
    struct State {
        float scale, denom, dx, dy, juu, juv, jvv;
        __device__ __forceinline__ float det() const { return juu * jvv - juv * juv; }
    };
    __device__ __forceinline__ State state_at(float u, float v) const {
        const float r2 = u * u + v * v;
        const float num = 1.0f + r2 * (d0.x + r2 * (d0.y + r2 * d1.x));
        const float den = 1.0f + r2 * (d1.y + r2 * (d1.z + r2 * d1.w));
        const float sc = num / den;
        const float dn = d0.x + r2 * (2.0f * d0.y + 3.0f * d1.x * r2);
        const float dd = d1.y + r2 * (2.0f * d1.z + 3.0f * d1.w * r2);
        const float dsc = (dn * den - num * dd) / (den * den);
        State st;
        st.scale = sc;
        st.denom = den;
        st.dx = 2.0f * d0.z * u * v + d0.w * (r2 + 2.0f * u * u);
        st.dy = d0.z * (r2 + 2.0f * v * v) + 2.0f * d0.w * u * v;
        st.juu = sc + 2.0f * u * u * dsc + 2.0f * d0.z * v + 6.0f * d0.w * u;
        st.juv = 2.0f * u * v * dsc + 2.0f * d0.z * u + 2.0f * d0.w * v;
        st.jvv = sc + 2.0f * v * v * dsc + 6.0f * d0.z * v + 2.0f * d0.w * u;
        return st;
    }
    // Five Newton steps on D(x) = xd (a fixed-point step where the Jacobian
    // is near singular); `st` is left at the last step's starting point.
    __device__ __forceinline__ float2 undistort(float2 xd, State& st) const {
        float2 x = xd;
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            st = state_at(x.x, x.y);
            const float rx = x.x * st.scale + st.dx - xd.x;
            const float ry = x.y * st.scale + st.dy - xd.y;
            const float det = st.det();
            if (fabsf(det) > kMinDet) {
                x.x -= (st.jvv * rx - st.juv * ry) / det;
                x.y -= (st.juu * ry - st.juv * rx) / det;
            } else {
                x = make_float2((xd.x - st.dx) / st.scale, (xd.y - st.dy) / st.scale);
            }
        }
        return x;
    }
    __device__ __forceinline__ v3 ray_cs(float2 uv) const {
        State st;
        const float2 x = undistort(make_float2((uv.x - c.x) / f.x, (uv.y - c.y) / f.y), st);
        return mk3(x.x, x.y, 1.0f);
    }
    __device__ __forceinline__ bool ray_valid(float2 uv) const {
        State st;
        const float2 xd = make_float2((uv.x - c.x) / f.x, (uv.y - c.y) / f.y);
        const float2 x = undistort(xd, st);
        const float rx = x.x * st.scale + st.dx - xd.x;
        const float ry = x.y * st.scale + st.dy - xd.y;
        const float r2 = x.x * x.x + x.y * x.y;
        return (r2 <= max_r2) && (fabsf(rx) < 1e-5f) && (fabsf(ry) < 1e-5f);
    }
    // Backward into f, c (18..21) and the eight coefficients (22..29) at the
    // re-solved point, implicit in D(x; k) = (uv - c) / f:
    // g_d = J^-T d_ray.xy, dL/dk = -g_d . dD/dk (distorted_perspective.cu:115-190).
    template <int P>
    __device__ __forceinline__ void ray_cs_bwd(float2 uv, v3 d, float (&acc)[P]) const {
        const float ifx = 1.0f / f.x, ify = 1.0f / f.y;
        const float2 xd = make_float2((uv.x - c.x) * ifx, (uv.y - c.y) * ify);
        State st;
        const float2 x = undistort(xd, st);
        st = state_at(x.x, x.y);
        const float det = st.det();
        float gx, gy;
        if (fabsf(det) <= kMinDet) {
            gx = d.x / st.scale;
            gy = d.y / st.scale;
        } else {
            gx = (st.jvv * d.x - st.juv * d.y) / det;
            gy = (st.juu * d.y - st.juv * d.x) / det;
        }
        acc[20] -= gx * xd.x * ifx;
        acc[21] -= gy * xd.y * ify;
        acc[22] -= gx * ifx;
        acc[23] -= gy * ify;
        const float r2 = x.x * x.x + x.y * x.y, r4 = r2 * r2, r6 = r4 * r2;
        const float rad = -(gx * x.x + gy * x.y) / st.denom;
        const float rad_den = -rad * st.scale;
        acc[24] += rad * r2;
        acc[25] += rad * r4;
        acc[26] -= gx * 2.0f * x.x * x.y + gy * (r2 + 2.0f * x.y * x.y);
        acc[27] -= gx * (r2 + 2.0f * x.x * x.x) + gy * 2.0f * x.x * x.y;
        acc[28] += rad * r6;
        acc[29] += rad_den * r2;
        acc[30] += rad_den * r4;
        acc[31] += rad_den * r6;
    }
    // uv_distortion (distortion.h:8-30) applied to x.
    __device__ __forceinline__ float2 distort(float2 x) const {
        const float uu = x.x * x.x, vv = x.y * x.y;
        const float r2 = uu + vv;
        const float num = 1.0f + r2 * (d0.x + r2 * (d0.y + r2 * d1.x));
        const float den = 1.0f + r2 * (d1.y + r2 * (d1.z + r2 * d1.w));
        const float sc = num / den;
        const float uv2 = 2.0f * x.x * x.y;
        return make_float2(x.x * sc + (d0.z * uv2 + d0.w * (r2 + 2.0f * uu)),
                           x.y * sc + (d0.z * (r2 + 2.0f * vv) + d0.w * uv2));
    }
    // camera_point_to_uvd, distorted_perspective.cu:192-199: depth 0 beyond
    // the trusted radius.
    __device__ __forceinline__ v3 to_uvd(int, v3 p) const {
        const float2 x = make_float2(p.x / p.z, p.y / p.z);
        const float2 xd = distort(x);
        const float r2 = x.x * x.x + x.y * x.y;
        return mk3(xd.x * f.x + c.x, xd.y * f.y + c.y, (r2 <= max_r2) ? p.z : 0.0f);
    }
    __device__ __forceinline__ void to_uvd_jac(int, v3, v3, v3&, float2&) const {}
    // distort_uv, distorted_perspective.cu:201-205
    __device__ __forceinline__ float2 distort_uv(float2 uv) const {
        const float2 xd = distort(make_float2((uv.x - c.x) / f.x, (uv.y - c.y) / f.y));
        return make_float2(xd.x * f.x + c.x, xd.y * f.y + c.y);
    }
};

template <bool kLidar>
struct Spherical : CamBase {
    static constexpr int kType = kLidar ? XSG_CAM_LIDAR : XSG_CAM_SPHERICAL;
    static constexpr bool kJacobian = true;
    static constexpr int kWords = kLidar ? 24 : 22;
    float phi_min, phi_range, theta_min, theta_range;
    const float* elev;
    __device__ __forceinline__ void load(const float* p) {
        load_base(p);
        phi_min = p[18]; phi_range = p[19]; theta_min = p[20]; theta_range = p[21];
        elev = nullptr;
        if (kLidar) {
            uint32_t lo = __float_as_uint(p[22]), hi = __float_as_uint(p[23]);
            elev = reinterpret_cast<const float*>((uint64_t(hi) << 32) | uint64_t(lo));
        }
    }
    __device__ __forceinline__ float2 pixel_to_uv(int px, int py, int W, int H) const {
        const float u = (float(px) + 0.5f) / float(W);
        if (kLidar) return make_float2(u, elev[py]);
        return make_float2(u, (float(py) + 0.5f) / float(H));
    }
    __device__ __forceinline__ v3 ray_cs(float2 uv) const {
        const float az = phi_min + uv.x * phi_range;
        const float el = theta_min + uv.y * theta_range;
        float es, ec, as, ac;
        sincosf(el, &es, &ec);
        sincosf(az, &as, &ac);
        const float xy = 1.0f * ec;
        return mk3(xy * as, xy * ac, 1.0f * es);
    }
    // The reference gives the angle limits no ray gradient (spherical.h:34-100
    // keeps BaseCameraImpl's empty pixel_to_camera_ray_backward).
    template <int P>
    __device__ __forceinline__ void ray_cs_bwd(float2, v3, float (&)[P]) const {}
    __device__ __forceinline__ bool ray_valid(float2) const { return true; }
    __device__ __forceinline__ float2 angles_to_uv(int mode, float phi, float theta) const {
        float u = (phi - phi_min) / phi_range;
        const float u_pose = (fabsf(rolling.x) > 0.0f) ? (pose - trigger) / rolling.x : 0.5f;
        const float u_off = (2.0f * float(M_PI) / fabsf(phi_range));
        if (rolling.x > 0) {
            if (mode == MODE_NEG && u > u_pose) u = u - u_off;
            if (mode == MODE_POS && u < u_pose) u = u + u_off;
        } else {
            if (mode == MODE_NEG && u < u_pose) u = u + u_off;
            if (mode == MODE_POS && u > u_pose) u = u - u_off;
        }
        return make_float2(u, (theta - theta_min) / theta_range);
    }
    __device__ __forceinline__ v3 to_uvd(int mode, v3 p) const {
        const float d = sqrtf(dot3(p, p));
        const float phi = atan2f(-p.x, -p.y) + float(M_PI);
        const float th = asinf(p.z / d);
        const float2 uv = angles_to_uv(mode, phi, th);
        return mk3(uv.x, uv.y, d);
    }
    __device__ __forceinline__ void to_uvd_jac(int mode, v3 p, v3 dp, v3& uvd, float2& duv) const {
        const float x2y2 = p.x * p.x + p.y * p.y;
        const float r = sqrtf(x2y2 + p.z * p.z);
        // the reference adds the double constant M_PI here (spherical.h:140),
        // so the sum is rounded once from double (cartesian_to_spherical,
        // used by to_uvd above, adds float(M_PI))
        const float phi = float(double(atan2f(-p.x, -p.y)) + M_PI);
        const float th = asinf(p.z / r);
        const float2 uv = angles_to_uv(mode, phi, th);
        uvd = mk3(uv.x, uv.y, r);
        const float sq = sqrtf(x2y2);
        const float r2 = r * r;
        const float mul = p.z / (r2 * sq);
        duv = make_float2(((-p.x * dp.y + p.y * dp.x) / x2y2) / phi_range,
                          ((sq * dp.z) / r2 - mul * (p.x * dp.x + p.y * dp.y)) / theta_range);
    }
};

// ------------------------------------------------------------- motion ----
// Quaternion of the rotation vector w*t: projection_kernels.h:12-36.
__device__ __forceinline__ void axis_angle_quat(v3 w, float t, float& qw, v3& qv, float& dqw, v3& dqv) {
    const float wn = sqrtf(dot3(w, w));
    const float th = wn * fabsf(t);
    float sh, ch;
    sincosf(0.5f * th, &sh, &ch);
    const float sc = (th < 1e-2f) ? 0.5f - th * th * (1.0f / 48.0f) : sh / th;
    qw = ch;
    qv = sc * w * t;
    dqw = -0.5f * copysignf(1.0f, t) * sh * wn;
    dqv = (0.5f * ch) * w;
}

__device__ __forceinline__ v3 quat_rotate(float w, v3 q, v3 p) {
    const v3 uv = cross3(q, p);
    const v3 uuv = cross3(q, uv);
    return p + 2.0f * (w * uv + uuv);
}

// Camera->world rotation at time offset t: q_aa(w t) (x) q0 (toast
// apply_angular_velocity, as spelled out in projection_kernels.h:88-101).
template <typename Cam>
__device__ __forceinline__ void pose_rotation(const Cam& k, float q0w, v3 q0v, float t, float& rw, v3& rv) {
    float w1, dw1;
    v3 x1, dx1;
    axis_angle_quat(k.w, t, w1, x1, dw1, dx1);
    rw = w1 * q0w - dot3(x1, q0v);
    rv = w1 * q0v + q0w * x1 + cross3(x1, q0v);
}

// World point -> camera point at time t, and its time derivative
// (projection_kernels.h:74-113).
template <typename Cam>
__device__ __forceinline__ void world_to_camera_jac(const Cam& k, v3 P, v3 Pv, float t, v3& res, v3& dres) {
    float w1, dw1;
    v3 x1, dx1;
    axis_angle_quat(k.w, t, w1, x1, dw1, dx1);
    const v3 x2 = mk3(k.qx, k.qy, k.qz);
    const float w2 = k.qw;
    const float w = w1 * w2 - dot3(x1, x2);
    v3 xyz = w1 * x2 + w2 * x1 + cross3(x1, x2);
    const float dw = dw1 * w2 - dot3(dx1, x2);
    v3 dxyz = dw1 * x2 + w2 * dx1 + cross3(dx1, x2);
    xyz = -1.0f * xyz;
    dxyz = -1.0f * dxyz;
    const v3 vd = Pv - k.v;
    const v3 p = P - k.t0 + vd * t;
    const v3 uv = cross3(xyz, p);
    const v3 uuv = cross3(xyz, uv);
    res = p + 2.0f * (w * uv + uuv);
    const v3 duv = cross3(dxyz, p);
    const v3 dp = 2.0f * (dw * uv + w * duv + cross3(dxyz, uv) + cross3(xyz, duv));
    dres = dp + quat_rotate(w, xyz, vd);
}

// Solve for the capture time of a world point and project it
// (camera_projection, projection_kernels.h:201-256).  Returns uvdt and
// clears `valid` on failure (valid is never set here).
template <typename Cam, bool kUseJac>
__device__ __forceinline__ void project_point(const Cam& k, v3 P, v3 Pv, float thr, float max_res,
                                              float margin, int mode, float4& uvdt, bool& valid) {
    v3 uvd = mk3(0.f, 0.f, 0.f);
    float pt = 0.0f;
    if (mode == MODE_NEG) pt = -fabsf(k.rolling.x) * 0.5f;
    else if (mode == MODE_POS) pt = fabsf(k.rolling.x) * 0.5f;
    float residual = 0.0f;
    if (k.w.x == 0.0f && k.w.y == 0.0f && k.w.z == 0.0f && Pv.x == k.v.x && Pv.y == k.v.y && Pv.z == k.v.z) {
        // No angular velocity and no relative motion: the camera-frame point
        // does not depend on the capture time, so every Newton step below
        // projects the same point and has d residual / d t = 1.  Project
        // once and iterate only the time update (same checks, same result).
        // the camera's Jacobian projection where the reference iterates
        // with it (its uvd can differ in the last bit from to_uvd's)
        if constexpr (kUseJac && Cam::kJacobian) {
            float2 duv;
            k.to_uvd_jac(mode, quat_rotate(k.qw, mk3(-k.qx, -k.qy, -k.qz), P - k.t0), mk3(0.f, 0.f, 0.f), uvd, duv);
        } else {
            uvd = k.to_uvd(mode, quat_rotate(k.qw, mk3(-k.qx, -k.qy, -k.qz), P - k.t0));
        }
        if ((uvd.z <= 0.0f) || (uvd.x < -margin) || (uvd.x > 1.0f + margin) || (uvd.y < -margin) ||
            (uvd.y > 1.0f + margin)) {
            valid = false;
            uvdt = make_float4(0.f, 0.f, 0.f, 0.f);
            return;
        }
        const float real = k.pixel_time(uvd.x, uvd.y);
#pragma unroll 1
        for (int it = 0; it < 5; ++it) {
            residual = (k.pose + pt) - real;
            pt -= residual;
            if (fabsf(residual) < thr) break;
        }
        uvdt = make_float4(uvd.x, uvd.y, uvd.z, pt);
        valid = valid && (fabsf(residual) < max_res) && (uvd.z > 0.0f);
        return;
    }
#pragma unroll 1
    for (int it = 0; it < 5; ++it) {
        if constexpr (kUseJac && Cam::kJacobian) {
            v3 pc, jpc;
            float2 duv;
            world_to_camera_jac(k, P, Pv, pt, pc, jpc);
            k.to_uvd_jac(mode, pc, jpc, uvd, duv);
            const float assumed = k.pose + pt;
            const float real = k.pixel_time(uvd.x, uvd.y);
            residual = assumed - real;
            const float dres = 1.0f - (duv.x * k.rolling.x + duv.y * k.rolling.y);
            pt -= residual / dres;
        } else {
            float rw;
            v3 rv;
            pose_rotation(k, k.qw, mk3(k.qx, k.qy, k.qz), pt, rw, rv);
            const v3 p = P - k.t0 + (Pv - k.v) * pt;
            const v3 pc = quat_rotate(rw, -1.0f * rv, p);
            uvd = k.to_uvd(mode, pc);
            const float assumed = k.pose + pt;
            const float real = k.pixel_time(uvd.x, uvd.y);
            residual = assumed - real;
            pt -= residual;
        }
        if ((uvd.z <= 0.0f) || (uvd.x < -margin) || (uvd.x > 1.0f + margin) || (uvd.y < -margin) ||
            (uvd.y > 1.0f + margin)) {
            valid = false;
            uvdt = make_float4(0.f, 0.f, 0.f, 0.f);
            return;
        }
        if (fabsf(residual) < thr) break;
    }
    uvdt = make_float4(uvd.x, uvd.y, uvd.z, pt);
    valid = valid && (fabsf(residual) < max_res) && (uvd.z > 0.0f);
}

// Dispatch a templated functor over the camera type.
template <typename F>
int dispatch_camera(int type, F&& f) {
    switch (type) {
        case XSG_CAM_PINHOLE: f(Pinhole{}); return XSG_OK;
        case XSG_CAM_FISHEYE: f(Fisheye{}); return XSG_OK;
        case XSG_CAM_SPHERICAL: f(Spherical<false>{}); return XSG_OK;
        case XSG_CAM_LIDAR: f(Spherical<true>{}); return XSG_OK;
        case XSG_CAM_DISTORTED: f(Distorted{}); return XSG_OK;
        default: return set_error(XSG_ERR_INVALID_ARGUMENT, "unknown camera type");
    }
}

}  // namespace xsg
