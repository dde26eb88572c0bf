// Test infrastructure: a minimal stand-in for pytoast's
// <toast/utils/bwd_math_utils.h> (see vector_math.h in this folder for why).
// normalize_bwd<Tag>(v, g) is the vector-Jacobian product of
// normalize(v) = v / |v|:  (g - n (n . g)) / |v| with n = v / |v|, written as
// g * il - v * (il^3 (v . g)), il = rsqrt(v . v) — the same expression the
// reference spells out for its own safe_normalize_bwd
// (rasterization/utils.h:197-205).
#pragma once

#include "vector_math.h"
#include "../math/scalar.h"

template <typename Tag>
HOSTDEVICE float3 normalize_bwd(const float3& v, const float3& d_out) {
    const float l = dot(v, v);
#ifdef __CUDA_ARCH__
    const float il = rsqrtf(l);
#else
    const float il = 1.0f / std::sqrt(l);
#endif
    const float il3 = il * il * il;
    return il * d_out - il3 * dot(d_out, v) * v;
}
