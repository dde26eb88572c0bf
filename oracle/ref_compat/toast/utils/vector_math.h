// Test infrastructure: a minimal stand-in for pytoast's
// <toast/utils/vector_math.h>, written for this project so that the
// reference's own CUDA sources compile into the GPU test oracle under
// oracle/_ref (pytoast is not available and has no pinned version).  Nothing
// in the shipped library includes it.
//
// What it provides is what those sources use: the DEVICE / HOSTDEVICE
// function qualifiers (inline, so headers that define functions can be
// included by several translation units) and component-wise arithmetic on
// CUDA's float2/float3/float4/int2 vector types, dot, cross,
// length(v) = sqrtf(dot(v, v)) and
// normalize(v) = v * rsqrt(dot(v, v)) (the helper_math convention; the same
// assumption the CPU oracle makes).
#pragma once

#include <cstdint>
#include <cmath>
#include <cuda_runtime.h>
#include <sys/types.h>

#ifndef DEVICE
#define DEVICE __device__ __forceinline__
#endif
#ifndef HOSTDEVICE
#define HOSTDEVICE __host__ __device__ __forceinline__
#endif

// ------------------------------------------------------------------ float2 --
HOSTDEVICE float2 operator+(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
HOSTDEVICE float2 operator-(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
HOSTDEVICE float2 operator-(float2 a) { return make_float2(-a.x, -a.y); }
HOSTDEVICE float2 operator*(float2 a, float2 b) { return make_float2(a.x * b.x, a.y * b.y); }
HOSTDEVICE float2 operator/(float2 a, float2 b) { return make_float2(a.x / b.x, a.y / b.y); }
HOSTDEVICE float2 operator*(float2 a, float s) { return make_float2(a.x * s, a.y * s); }
HOSTDEVICE float2 operator*(float s, float2 a) { return make_float2(s * a.x, s * a.y); }
HOSTDEVICE float2 operator/(float2 a, float s) { return make_float2(a.x / s, a.y / s); }
HOSTDEVICE float2 operator/(float s, float2 a) { return make_float2(s / a.x, s / a.y); }
HOSTDEVICE float2 operator+(float2 a, float s) { return make_float2(a.x + s, a.y + s); }
HOSTDEVICE float2 operator-(float2 a, float s) { return make_float2(a.x - s, a.y - s); }
HOSTDEVICE float2& operator+=(float2& a, float2 b) { a.x += b.x; a.y += b.y; return a; }
HOSTDEVICE float2& operator-=(float2& a, float2 b) { a.x -= b.x; a.y -= b.y; return a; }
HOSTDEVICE float2& operator*=(float2& a, float2 b) { a.x *= b.x; a.y *= b.y; return a; }
HOSTDEVICE float2& operator/=(float2& a, float2 b) { a.x /= b.x; a.y /= b.y; return a; }
HOSTDEVICE float2& operator*=(float2& a, float s) { a.x *= s; a.y *= s; return a; }
HOSTDEVICE float2& operator/=(float2& a, float s) { a.x /= s; a.y /= s; return a; }
HOSTDEVICE float dot(float2 a, float2 b) { return a.x * b.x + a.y * b.y; }
HOSTDEVICE float length(float2 v) { return sqrtf(dot(v, v)); }

// ------------------------------------------------------------------ float3 --
HOSTDEVICE float3 operator+(float3 a, float3 b) { return make_float3(a.x + b.x, a.y + b.y, a.z + b.z); }
HOSTDEVICE float3 operator-(float3 a, float3 b) { return make_float3(a.x - b.x, a.y - b.y, a.z - b.z); }
HOSTDEVICE float3 operator-(float3 a) { return make_float3(-a.x, -a.y, -a.z); }
HOSTDEVICE float3 operator*(float3 a, float3 b) { return make_float3(a.x * b.x, a.y * b.y, a.z * b.z); }
HOSTDEVICE float3 operator/(float3 a, float3 b) { return make_float3(a.x / b.x, a.y / b.y, a.z / b.z); }
HOSTDEVICE float3 operator*(float3 a, float s) { return make_float3(a.x * s, a.y * s, a.z * s); }
HOSTDEVICE float3 operator*(float s, float3 a) { return make_float3(s * a.x, s * a.y, s * a.z); }
HOSTDEVICE float3 operator/(float3 a, float s) { return make_float3(a.x / s, a.y / s, a.z / s); }
HOSTDEVICE float3 operator/(float s, float3 a) { return make_float3(s / a.x, s / a.y, s / a.z); }
HOSTDEVICE float3 operator+(float3 a, float s) { return make_float3(a.x + s, a.y + s, a.z + s); }
HOSTDEVICE float3 operator-(float3 a, float s) { return make_float3(a.x - s, a.y - s, a.z - s); }
HOSTDEVICE float3& operator+=(float3& a, float3 b) { a.x += b.x; a.y += b.y; a.z += b.z; return a; }
HOSTDEVICE float3& operator-=(float3& a, float3 b) { a.x -= b.x; a.y -= b.y; a.z -= b.z; return a; }
HOSTDEVICE float3& operator*=(float3& a, float3 b) { a.x *= b.x; a.y *= b.y; a.z *= b.z; return a; }
HOSTDEVICE float3& operator*=(float3& a, float s) { a.x *= s; a.y *= s; a.z *= s; return a; }
HOSTDEVICE float3& operator/=(float3& a, float s) { a.x /= s; a.y /= s; a.z /= s; return a; }
HOSTDEVICE float dot(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
HOSTDEVICE float3 cross(float3 a, float3 b) {
    return make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
HOSTDEVICE float length(float3 v) { return sqrtf(dot(v, v)); }
HOSTDEVICE float3 normalize(float3 v) {
#ifdef __CUDA_ARCH__
    return v * rsqrtf(dot(v, v));
#else
    return v * (1.0f / std::sqrt(dot(v, v)));
#endif
}

// ------------------------------------------------------------------ float4 --
HOSTDEVICE float4 operator+(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
HOSTDEVICE float4 operator-(float4 a, float4 b) { return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
HOSTDEVICE float4 operator-(float4 a) { return make_float4(-a.x, -a.y, -a.z, -a.w); }
HOSTDEVICE float4 operator*(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
HOSTDEVICE float4 operator/(float4 a, float s) { return make_float4(a.x / s, a.y / s, a.z / s, a.w / s); }
HOSTDEVICE float4& operator*=(float4& a, float s) { a.x *= s; a.y *= s; a.z *= s; a.w *= s; return a; }
HOSTDEVICE float4 operator*(float4 a, float s) { return make_float4(a.x * s, a.y * s, a.z * s, a.w * s); }
HOSTDEVICE float4 operator*(float s, float4 a) { return make_float4(s * a.x, s * a.y, s * a.z, s * a.w); }
HOSTDEVICE float4& operator+=(float4& a, float4 b) { a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w; return a; }
HOSTDEVICE float dot(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

// -------------------------------------------------------------------- int2 --
HOSTDEVICE int2 operator+(int2 a, int2 b) { return make_int2(a.x + b.x, a.y + b.y); }
HOSTDEVICE int2 operator-(int2 a, int2 b) { return make_int2(a.x - b.x, a.y - b.y); }
