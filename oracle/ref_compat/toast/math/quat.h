// Test infrastructure: a minimal stand-in for pytoast's <toast/math/quat.h>,
// written for this project so that the reference's own camera, UT-projection
// and range-image tiling sources compile into the GPU test oracle under
// oracle/_ref.  Nothing in the shipped library includes it.
//
// pytoast is not available and nothing in the reference pins these
// semantics; the conventions below are the ones the CPU oracle and the
// shipped kernels assume, so a disagreement with the reference's kernels can
// only come from the reference's own code, not from this header:
//   * quatf holds w, x, y, z in that memory order (wxyz, as the reference's
//     rasteriser reads quaternions, rasterization/utils.h:61-62), plain
//     floats (4-byte alignment);
//   * std(): unit length (scaled by rsqrt(|q|^2)) with a non-negative real
//     part;
//   * to_matrix(rows): the three rows of the rotation matrix of the
//     quaternion scaled by 1 / sqrt(|q|^2) (the polynomial of
//     rasterization/utils.h:61-83);
//   * apply(p) = p + 2 (w (v x p) + v x (v x p)), v = (x, y, z), the form the
//     reference spells out in projection_kernels.h:67-71 (no normalisation);
//     apply_inv(p) = the same with v negated;
//   * products are Hamilton products;
//   * slerp: shortest arc, normalised linear interpolation when the
//     quaternions are within acos(0.9995) of each other;
//   * apply_backward / std_backward: the vector-Jacobian products of apply
//     and std from their mathematics.
#pragma once

#include <tuple>
#include "../utils/vector_math.h"

struct quatf {
    float w, x, y, z;

    quatf() = default;
    HOSTDEVICE constexpr quatf(float w_, float x_, float y_, float z_) : w(w_), x(x_), y(y_), z(z_) {}
    HOSTDEVICE constexpr quatf(float w_, float3 v) : w(w_), x(v.x), y(v.y), z(v.z) {}
    // a float4 read from a wxyz tensor: .x is the real part
    HOSTDEVICE explicit constexpr quatf(float4 v) : w(v.x), x(v.y), y(v.z), z(v.w) {}
    HOSTDEVICE operator float4() const { return make_float4(w, x, y, z); }

    [[nodiscard]] HOSTDEVICE float real() const { return w; }
    [[nodiscard]] HOSTDEVICE float3 img() const { return make_float3(x, y, z); }

    [[nodiscard]] HOSTDEVICE float norm2() const { return w * w + x * x + y * y + z * z; }

    [[nodiscard]] HOSTDEVICE quatf conjugate() const { return {w, -x, -y, -z}; }

    [[nodiscard]] HOSTDEVICE quatf std() const {
#ifdef __CUDA_ARCH__
        float n = rsqrtf(norm2());
#else
        float n = 1.0f / std::sqrt(norm2());
#endif
        if (w < 0.0f) n = -n;
        return {w * n, x * n, y * n, z * n};
    }

    HOSTDEVICE void to_matrix(float3* rows) const {
        const float inv = 1.0f / sqrtf(norm2());
        const float qw = w * inv, qx = x * inv, qy = y * inv, qz = z * inv;
        const float x2 = qx * qx, y2 = qy * qy, z2 = qz * qz;
        const float xy = qx * qy, xz = qx * qz, yz = qy * qz;
        const float wx = qw * qx, wy = qw * qy, wz = qw * qz;
        rows[0] = make_float3(1.f - 2.f * (y2 + z2), 2.f * (xy - wz), 2.f * (xz + wy));
        rows[1] = make_float3(2.f * (xy + wz), 1.f - 2.f * (x2 + z2), 2.f * (yz - wx));
        rows[2] = make_float3(2.f * (xz - wy), 2.f * (yz + wx), 1.f - 2.f * (x2 + y2));
    }

    [[nodiscard]] HOSTDEVICE float3 apply(const float3& p) const {
        const float3 v = img();
        const float3 uv = cross(v, p);
        const float3 uuv = cross(v, uv);
        return p + 2.0f * (w * uv + uuv);
    }

    [[nodiscard]] HOSTDEVICE float3 apply_inv(const float3& p) const { return conjugate().apply(p); }

    [[nodiscard]] HOSTDEVICE quatf slerp(const quatf& other, float t) const {
        float d = w * other.w + x * other.x + y * other.y + z * other.z;
        quatf b = other;
        if (d < 0.0f) {
            d = -d;
            b = {-b.w, -b.x, -b.y, -b.z};
        }
        float s0, s1;
        if (d > 0.9995f) {
            s0 = 1.0f - t;
            s1 = t;
        } else {
            const float th = acosf(d);
            const float sn = sinf(th);
            s0 = sinf((1.0f - t) * th) / sn;
            s1 = sinf(t * th) / sn;
        }
        quatf r{s0 * w + s1 * b.w, s0 * x + s1 * b.x, s0 * y + s1 * b.y, s0 * z + s1 * b.z};
        const float n = 1.0f / sqrtf(r.norm2());
        return {r.w * n, r.x * n, r.y * n, r.z * n};
    }

    // dL/dq and dL/dp of y = apply(p) (q taken as is, not normalised)
    HOSTDEVICE static std::tuple<quatf, float3> apply_backward(const quatf& q, const float3& p, const float3& g) {
        const float3 v = q.img();
        const float3 uv = cross(v, p);
        // y = p + 2 w (v x p) + 2 v x (v x p)
        // dy/dw^T g = 2 (v x p) . g
        const float dw = 2.0f * dot(uv, g);
        // d/dv of 2 w (v x p): g . (2 w (dv x p)) = dv . (2 w (p x g))
        // d/dv of 2 v x (v x p) = 2 [ dv x (v x p) + v x (dv x p) ]
        //   g . (dv x uv) = dv . (uv x g);  g . (v x (dv x p)) = (g x v) . (dv x p) = dv . (p x (g x v))
        const float3 dv = 2.0f * q.w * cross(p, g) + 2.0f * (cross(uv, g) + cross(p, cross(g, v)));
        // dy/dp^T g = R^T g for the rotation part: p + 2 w (v x p) + 2 v x (v x p)
        //   g . (v x dp) = dp . (g x v);  g . (v x (v x dp)) = (g x v) . (v x dp) = dp . ((g x v) x v)
        const float3 gv = cross(g, v);
        const float3 dp = g + 2.0f * (q.w * gv + cross(gv, v));
        return {quatf{dw, dv}, dp};
    }

    // dL/dq of s = std(q) given dL/ds (the sign flip is locally constant)
    HOSTDEVICE static float4 std_backward(const quatf& q, const quatf& ds) {
        const float n2 = q.norm2();
        const float inv = 1.0f / sqrtf(n2);
        const float sg = q.w < 0.0f ? -1.0f : 1.0f;
        const float dot_qd = q.w * ds.w + q.x * ds.x + q.y * ds.y + q.z * ds.z;
        const float k = dot_qd / n2;
        return make_float4(sg * inv * (ds.w - k * q.w), sg * inv * (ds.x - k * q.x), sg * inv * (ds.y - k * q.y),
                           sg * inv * (ds.z - k * q.z));
    }
};

HOSTDEVICE quatf operator*(const quatf& a, const quatf& b) {
    const float3 av = a.img(), bv = b.img();
    return quatf{a.w * b.w - dot(av, bv), a.w * bv + b.w * av + cross(av, bv)};
}
