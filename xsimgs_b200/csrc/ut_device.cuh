// Unscented-transform projection of one Gaussian (device), shared by the
// projection kernels and the range-image tiling (which re-projects
// wrap-around Gaussians).
#pragma once

#include <cmath>

#include "cameras.cuh"

namespace xsg {

// ------------------------------------------------------------------- UT --
struct UTParams {
    float m0, c0, w, sq;  // mean-0 weight, cov-0 weight, other weight, sqrt(3+lambda)
    float thr, max_res, margin;
    float img_w, img_h;
};

// ut_kernels.h:17-36, evaluated on the host in float
inline UTParams ut_params(float a, float b, float kappa, float thr, float max_res, float margin,
                          float W, float H) {
    const float lam = a * a * (3 + kappa) - 3;
    UTParams p;
    p.m0 = lam / (3 + lam);
    p.c0 = lam / (3 + lam) + (1 - a * a + b);
    p.w = 1 / (2 * (3 + lam));
    p.sq = std::sqrt(lam + 3);
    p.thr = thr; p.max_res = max_res; p.margin = margin;
    p.img_w = W; p.img_h = H;
    return p;
}

// Sigma-point offsets: columns of R(q) scaled by s_i*sqrt(3+lambda)
// (ut_kernels.h:38-49; toast to_matrix of the conjugate, normalised).
__device__ __forceinline__ void ut_deltas(float sq, float4 q, v3 s, v3 d[3]) {
    const float inv = 1.0f / sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
    const float w = q.x * inv, x = -q.y * inv, y = -q.z * inv, z = -q.w * inv;
    const float x2 = x * x, y2 = y * y, z2 = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    d[0] = mk3(1.f - 2.f * (y2 + z2), 2.f * (xy - wz), 2.f * (xz + wy));
    d[1] = mk3(2.f * (xy + wz), 1.f - 2.f * (x2 + z2), 2.f * (yz - wx));
    d[2] = mk3(2.f * (xz - wy), 2.f * (yz + wx), 1.f - 2.f * (x2 + y2));
    d[0] = d[0] * (s.x * sq);
    d[1] = d[1] * (s.y * sq);
    d[2] = d[2] * (s.z * sq);
}

// unscented_transform + unscented_transform_projection, ut_kernels.h:52-184
template <typename Cam>
__device__ __forceinline__ bool ut_project(const Cam& k, const UTParams& p, int mode, v3 P, v3 Pv,
                                           float opac, const v3 d[3], float2& mean2d, float2& radii,
                                           float& depth, float& u_dist) {
    float4 uvdt;
    bool valid = true;
    float3 cov = make_float3(0.f, 0.f, 0.f);
    bool ok = false;
    mean2d = make_float2(0.f, 0.f);
    depth = 0.f;
    u_dist = 0.f;
    project_point<Cam, true>(k, P, Pv, p.thr, p.max_res, p.margin, mode, uvdt, valid);
    if (valid) {
        float2 pts[7];
        pts[0] = make_float2(uvdt.x * p.img_w, uvdt.y * p.img_h);
        mean2d = make_float2(p.m0 * pts[0].x, p.m0 * pts[0].y);
        depth = uvdt.z;
        float umin = pts[0].x, umax = pts[0].x;
        float sign = 1.0f;
#pragma unroll
        for (int i = 0; i < 6; ++i) {
            project_point<Cam, true>(k, P + sign * d[i / 2], Pv, p.thr, p.max_res, p.margin, mode, uvdt,
                                     valid);
            pts[i + 1] = make_float2(uvdt.x * p.img_w, uvdt.y * p.img_h);
            mean2d.x += p.w * pts[i + 1].x;
            mean2d.y += p.w * pts[i + 1].y;
            umin = fminf(umin, pts[i + 1].x);
            umax = fmaxf(umax, pts[i + 1].x);
            sign *= -1.0f;
        }
        if (valid) {
            u_dist = umax - umin;
            float vx = pts[0].x - mean2d.x, vy = pts[0].y - mean2d.y;
            cov = make_float3(p.c0 * (vx * vx), p.c0 * (vx * vy), p.c0 * (vy * vy));
#pragma unroll
            for (int i = 1; i < 7; ++i) {
                vx = pts[i].x - mean2d.x;
                vy = pts[i].y - mean2d.y;
                cov.x += p.w * (vx * vx);
                cov.y += p.w * (vx * vy);
                cov.z += p.w * (vy * vy);
            }
            const float det = cov.x * cov.z - cov.y * cov.y;
            ok = !(det <= 0.0f || cov.x < 0 || cov.z < 0);
        }
    }
    const float extend = fminf(3.33f, sqrtf(2.0f * logf(opac / (1.0f / 255.0f))));
    radii = make_float2(extend * sqrtf(fmaxf(0.0f, cov.x)), extend * sqrtf(fmaxf(0.0f, cov.z)));
    const bool ix = !(((mean2d.x + radii.x) < 0) || (p.img_w < (mean2d.x - radii.x)));
    const bool iy = !(((mean2d.y + radii.y) < 0) || (p.img_h < (mean2d.y - radii.y)));
    return ok && ix && iy;
}

}  // namespace xsg
