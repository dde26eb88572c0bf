// Quaternion helpers shared by the SMPL and scene-assembly kernels:
// (w, x, y, z) in memory, Hamilton products, R(q) p as the quaternion
// polynomial p + 2 (w (u x p) + u x (u x p)), std() = unit length with
// w >= 0, and the matching backward formulas.
#pragma once

#include "common.cuh"

namespace xsg {

struct Q {
    float w, x, y, z;
};
__device__ __forceinline__ Q ldq(const float* p) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    return {v.x, v.y, v.z, v.w};
}
__device__ __forceinline__ void stq(float* p, Q q) { *reinterpret_cast<float4*>(p) = make_float4(q.w, q.x, q.y, q.z); }
__device__ __forceinline__ Q qadd(Q a, Q b) { return {a.w + b.w, a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ Q conj(Q q) { return {q.w, -q.x, -q.y, -q.z}; }
__device__ __forceinline__ v3 vec(Q q) { return {q.x, q.y, q.z}; }
__device__ __forceinline__ Q qmul(Q a, Q b) {
    const v3 av = vec(a), bv = vec(b);
    const v3 v = a.w * bv + b.w * av + cross3(av, bv);
    return {a.w * b.w - dot3(av, bv), v.x, v.y, v.z};
}
// R(q) p = p + 2 (w (u x p) + u x (u x p))
__device__ __forceinline__ v3 rot(Q q, v3 p) {
    const v3 u = vec(q);
    const v3 uv = cross3(u, p);
    return p + 2.0f * (q.w * uv + cross3(u, uv));
}
// d/dq of g . R(q) p
__device__ __forceinline__ Q rot_bwd_q(Q q, v3 p, v3 g) {
    const v3 u = vec(q);
    const float up = dot3(u, p), ug = dot3(u, g), pg = dot3(p, g);
    const v3 du = (2.0f * q.w) * cross3(p, g) + (2.0f * up) * g + (2.0f * ug) * p - (4.0f * pg) * u;
    return {2.0f * dot3(g, cross3(u, p)), du.x, du.y, du.z};
}
__device__ __forceinline__ Q qstd(Q q) {
    float n = rsqrtf(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    if (q.w < 0.f) n = -n;
    return {q.w * n, q.x * n, q.y * n, q.z * n};
}
__device__ __forceinline__ Q qstd_bwd(Q raw, Q g) {
    const float il = rsqrtf(raw.w * raw.w + raw.x * raw.x + raw.y * raw.y + raw.z * raw.z);
    const Q n{raw.w * il, raw.x * il, raw.y * il, raw.z * il};
    const float ng = n.w * g.w + n.x * g.x + n.y * g.y + n.z * g.z;
    const float k = raw.w < 0.f ? -il : il;
    return {k * (g.w - n.w * ng), k * (g.x - n.x * ng), k * (g.y - n.y * ng), k * (g.z - n.z * ng)};
}
}  // namespace xsg
