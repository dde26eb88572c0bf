// Test infrastructure: a minimal stand-in for pytoast's <toast/math/motion.h>
// (see quat.h in this folder for why and for the quaternion conventions).
// The motion model is the one the reference spells out in
// projection_kernels.h:12-113: q(t) = q_aa(w t) (x) q0 with
// q_aa(a) = (cos(|a|/2), sin(|a|/2)/|a| a) (its small-angle series below
// |a| = 1e-2), t(t) = t0 + v t.
#pragma once

#include <tuple>
#include "../utils/vector_math.h"
#include "quat.h"
#include "../utils/bwd_math_utils.h"

HOSTDEVICE float lerp(float a, float b, float t) { return a + t * (b - a); }
HOSTDEVICE float2 lerp(float2 a, float2 b, float t) { return make_float2(lerp(a.x, b.x, t), lerp(a.y, b.y, t)); }
HOSTDEVICE float3 lerp(float3 a, float3 b, float t) {
    return make_float3(lerp(a.x, b.x, t), lerp(a.y, b.y, t), lerp(a.z, b.z, t));
}
HOSTDEVICE float4 lerp(float4 a, float4 b, float t) {
    return make_float4(lerp(a.x, b.x, t), lerp(a.y, b.y, t), lerp(a.z, b.z, t), lerp(a.w, b.w, t));
}

// rotation-vector quaternion of w * t
HOSTDEVICE quatf quat_from_angular_velocity(const float3& w, float t) {
    const float w_norm = sqrtf(dot(w, w));
    const float theta = w_norm * fabsf(t);
    float sin_half, cos_half;
    sincosf(0.5f * theta, &sin_half, &cos_half);
    const float scale = (theta < 1e-2f) ? 0.5f - theta * theta * (1.0f / 48.0f) : sin_half / theta;
    return quatf{cos_half, scale * w * t};
}

HOSTDEVICE quatf apply_angular_velocity(const quatf& q0, const float3& w, float t) {
    return quat_from_angular_velocity(w, t) * q0;
}

HOSTDEVICE std::tuple<quatf, float3> apply_velocity(const quatf& q0, const float3& t0, const float3& v,
                                                    const float3& w, float t) {
    return {apply_angular_velocity(q0, w, t), t0 + v * t};
}

// dL/dq0, dL/dw, dL/dt of q = q_aa(w t) (x) q0 given dL/dq
HOSTDEVICE std::tuple<quatf, float3, float> apply_angular_velocity_backward(const quatf& q0, const float3& w,
                                                                            float t, const quatf& dq) {
    const quatf a = quat_from_angular_velocity(w, t);
    // q = a (x) q0 is linear in each factor: dL/dq0 = conj(a) (x) dq, dL/da = dq (x) conj(q0)
    const quatf dq0 = a.conjugate() * dq;
    const quatf da = dq * q0.conjugate();
    // a = (cos(th/2), s(th) w t), th = |w| |t|
    const float wn = sqrtf(dot(w, w));
    const float theta = wn * fabsf(t);
    float sin_half, cos_half;
    sincosf(0.5f * theta, &sin_half, &cos_half);
    float s, ds_dth;
    if (theta < 1e-2f) {
        s = 0.5f - theta * theta * (1.0f / 48.0f);
        ds_dth = -theta * (1.0f / 24.0f);
    } else {
        s = sin_half / theta;
        ds_dth = (0.5f * cos_half * theta - sin_half) / (theta * theta);
    }
    const float3 dav = da.img();
    // dL/dtheta through cos(th/2) and s(th)
    const float g_th = -0.5f * sin_half * da.w + ds_dth * dot(dav, w * t);
    // theta = |w| |t|: dtheta/dw = |t| w/|w|, dtheta/dt = |w| sign(t)
    const float3 dw_dir = wn > 0.0f ? (fabsf(t) / wn) * w : make_float3(0.f, 0.f, 0.f);
    const float3 dw = g_th * dw_dir + s * t * dav;
    const float dt = g_th * wn * copysignf(1.0f, t) + s * dot(dav, w);
    return {dq0, dw, dt};
}
