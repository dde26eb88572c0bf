// Test infrastructure: a minimal stand-in for the GLM headers, written for
// this project so that the reference's own rasteriser sources
// (csrc/rasterization/*.cu, whose `third_party/glm` submodule is empty in
// the reference checkout) compile into the GPU test oracle under oracle/_ref.
// Nothing in the shipped library includes it.
//
// Semantics follow the GLSL/GLM conventions the reference relies on:
//   * fvecN: N packed floats, no over-alignment (fvec3 is 12 bytes, fvec4 is
//     16 bytes with 4-byte alignment), so device arrays of float triples can
//     be reinterpreted as fvec3 arrays as the reference does;
//   * fmatC: column-major, m[c] is column c, m[c][r] is the element in row r;
//     the 9-scalar constructor takes column 0 first;
//   * m * v = sum_c m[c] * v[c]; (a * b)[c][r] = sum_k a[k][r] * b[c][k];
//     outerProduct(c, r)[i][j] = c[j] * r[i] (c r^T);
//   * dot/cross/transpose as in linear algebra; sums are taken in index
//     order, except the 4-component dot, summed as (x + y) + (z + w).
#pragma once

#include <cuda_runtime.h>

#ifndef GLMC_FN
#define GLMC_FN __host__ __device__ __forceinline__
#endif

namespace glm {

struct fvec2 {
    float x, y;
    fvec2() = default;
    GLMC_FN constexpr fvec2(float a, float b) : x(a), y(b) {}
    template <typename U>
    GLMC_FN explicit constexpr fvec2(U s) : x(static_cast<float>(s)), y(static_cast<float>(s)) {}
    GLMC_FN float& operator[](int i) { return i == 0 ? x : y; }
    GLMC_FN const float& operator[](int i) const { return i == 0 ? x : y; }
};

struct fvec3 {
    float x, y, z;
    fvec3() = default;
    GLMC_FN constexpr fvec3(float a, float b, float c) : x(a), y(b), z(c) {}
    template <typename U>
    GLMC_FN explicit constexpr fvec3(U s)
        : x(static_cast<float>(s)), y(static_cast<float>(s)), z(static_cast<float>(s)) {}
    GLMC_FN float& operator[](int i) { return i == 0 ? x : (i == 1 ? y : z); }
    GLMC_FN const float& operator[](int i) const { return i == 0 ? x : (i == 1 ? y : z); }
    GLMC_FN fvec3& operator+=(const fvec3& o) { x += o.x; y += o.y; z += o.z; return *this; }
    GLMC_FN fvec3& operator-=(const fvec3& o) { x -= o.x; y -= o.y; z -= o.z; return *this; }
    GLMC_FN fvec3& operator*=(float s) { x *= s; y *= s; z *= s; return *this; }
    GLMC_FN fvec3& operator/=(float s) { x /= s; y /= s; z /= s; return *this; }
};

struct fvec4 {
    float x, y, z, w;
    fvec4() = default;
    GLMC_FN constexpr fvec4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
    template <typename U>
    GLMC_FN explicit constexpr fvec4(U s)
        : x(static_cast<float>(s)), y(static_cast<float>(s)), z(static_cast<float>(s)), w(static_cast<float>(s)) {}
    GLMC_FN float& operator[](int i) { return i == 0 ? x : (i == 1 ? y : (i == 2 ? z : w)); }
    GLMC_FN const float& operator[](int i) const { return i == 0 ? x : (i == 1 ? y : (i == 2 ? z : w)); }
    GLMC_FN fvec4& operator+=(const fvec4& o) { x += o.x; y += o.y; z += o.z; w += o.w; return *this; }
    GLMC_FN fvec4& operator-=(const fvec4& o) { x -= o.x; y -= o.y; z -= o.z; w -= o.w; return *this; }
    GLMC_FN fvec4& operator*=(float s) { x *= s; y *= s; z *= s; w *= s; return *this; }
};

using vec2 = fvec2;
using vec3 = fvec3;
using vec4 = fvec4;

// ---------------------------------------------------------------- vec ops --
GLMC_FN fvec2 operator+(fvec2 a, fvec2 b) { return {a.x + b.x, a.y + b.y}; }
GLMC_FN fvec2 operator-(fvec2 a, fvec2 b) { return {a.x - b.x, a.y - b.y}; }
GLMC_FN fvec2 operator*(fvec2 a, float s) { return {a.x * s, a.y * s}; }
GLMC_FN fvec2 operator*(float s, fvec2 a) { return {s * a.x, s * a.y}; }

GLMC_FN fvec3 operator-(fvec3 a) { return {-a.x, -a.y, -a.z}; }
GLMC_FN fvec3 operator+(fvec3 a, fvec3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
GLMC_FN fvec3 operator-(fvec3 a, fvec3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
GLMC_FN fvec3 operator*(fvec3 a, fvec3 b) { return {a.x * b.x, a.y * b.y, a.z * b.z}; }
GLMC_FN fvec3 operator*(fvec3 a, float s) { return {a.x * s, a.y * s, a.z * s}; }
GLMC_FN fvec3 operator*(float s, fvec3 a) { return {s * a.x, s * a.y, s * a.z}; }
GLMC_FN fvec3 operator/(fvec3 a, float s) { return {a.x / s, a.y / s, a.z / s}; }
GLMC_FN fvec3 operator/(float s, fvec3 a) { return {s / a.x, s / a.y, s / a.z}; }
GLMC_FN fvec3 operator/(fvec3 a, fvec3 b) { return {a.x / b.x, a.y / b.y, a.z / b.z}; }

GLMC_FN fvec4 operator-(fvec4 a) { return {-a.x, -a.y, -a.z, -a.w}; }
GLMC_FN fvec4 operator+(fvec4 a, fvec4 b) { return {a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w}; }
GLMC_FN fvec4 operator-(fvec4 a, fvec4 b) { return {a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w}; }
GLMC_FN fvec4 operator*(fvec4 a, fvec4 b) { return {a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w}; }
GLMC_FN fvec4 operator*(fvec4 a, float s) { return {a.x * s, a.y * s, a.z * s, a.w * s}; }
GLMC_FN fvec4 operator*(float s, fvec4 a) { return {s * a.x, s * a.y, s * a.z, s * a.w}; }
GLMC_FN fvec4 operator/(fvec4 a, float s) { return {a.x / s, a.y / s, a.z / s, a.w / s}; }

GLMC_FN float dot(fvec2 a, fvec2 b) { return a.x * b.x + a.y * b.y; }
GLMC_FN float dot(fvec3 a, fvec3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
GLMC_FN float dot(fvec4 a, fvec4 b) { return (a.x * b.x + a.y * b.y) + (a.z * b.z + a.w * b.w); }
GLMC_FN fvec3 cross(fvec3 a, fvec3 b) {
    return {a.y * b.z - b.y * a.z, a.z * b.x - b.z * a.x, a.x * b.y - b.x * a.y};
}

// ---------------------------------------------------------------- matrices --
struct fmat2 {
    fvec2 value[2];
    fmat2() = default;
    GLMC_FN fvec2& operator[](int c) { return value[c]; }
    GLMC_FN const fvec2& operator[](int c) const { return value[c]; }
};

struct fmat3 {
    fvec3 value[3];
    fmat3() = default;
    GLMC_FN constexpr fmat3(float a0, float a1, float a2, float b0, float b1, float b2, float c0, float c1, float c2)
        : value{fvec3(a0, a1, a2), fvec3(b0, b1, b2), fvec3(c0, c1, c2)} {}
    GLMC_FN constexpr fmat3(fvec3 c0, fvec3 c1, fvec3 c2) : value{c0, c1, c2} {}
    GLMC_FN explicit constexpr fmat3(float d)
        : value{fvec3(d, 0.f, 0.f), fvec3(0.f, d, 0.f), fvec3(0.f, 0.f, d)} {}
    GLMC_FN fvec3& operator[](int c) { return value[c]; }
    GLMC_FN const fvec3& operator[](int c) const { return value[c]; }
    GLMC_FN fmat3& operator+=(const fmat3& o) {
        value[0] += o.value[0]; value[1] += o.value[1]; value[2] += o.value[2];
        return *this;
    }
};

struct fmat4 {
    fvec4 value[4];
    fmat4() = default;
    GLMC_FN fvec4& operator[](int c) { return value[c]; }
    GLMC_FN const fvec4& operator[](int c) const { return value[c]; }
};

using mat2 = fmat2;
using mat3 = fmat3;
using mat4 = fmat4;

GLMC_FN fmat3 operator+(const fmat3& a, const fmat3& b) { return {a[0] + b[0], a[1] + b[1], a[2] + b[2]}; }
GLMC_FN fmat3 operator-(const fmat3& a, const fmat3& b) { return {a[0] - b[0], a[1] - b[1], a[2] - b[2]}; }
GLMC_FN fmat3 operator*(const fmat3& a, float s) { return {a[0] * s, a[1] * s, a[2] * s}; }
GLMC_FN fmat3 operator*(float s, const fmat3& a) { return {s * a[0], s * a[1], s * a[2]}; }

GLMC_FN fvec3 operator*(const fmat3& m, fvec3 v) {
    return {m[0][0] * v.x + m[1][0] * v.y + m[2][0] * v.z,
            m[0][1] * v.x + m[1][1] * v.y + m[2][1] * v.z,
            m[0][2] * v.x + m[1][2] * v.y + m[2][2] * v.z};
}

// row vector times matrix: (v^T m)_c = dot(v, m[c])
GLMC_FN fvec3 operator*(fvec3 v, const fmat3& m) {
    return {m[0][0] * v.x + m[0][1] * v.y + m[0][2] * v.z,
            m[1][0] * v.x + m[1][1] * v.y + m[1][2] * v.z,
            m[2][0] * v.x + m[2][1] * v.y + m[2][2] * v.z};
}

GLMC_FN fmat3 operator*(const fmat3& a, const fmat3& b) {
    fmat3 r;
    for (int c = 0; c < 3; ++c) {
        for (int row = 0; row < 3; ++row) {
            r[c][row] = a[0][row] * b[c][0] + a[1][row] * b[c][1] + a[2][row] * b[c][2];
        }
    }
    return r;
}

GLMC_FN fmat3 transpose(const fmat3& m) {
    return {m[0][0], m[1][0], m[2][0],
            m[0][1], m[1][1], m[2][1],
            m[0][2], m[1][2], m[2][2]};
}

GLMC_FN fmat3 outerProduct(fvec3 c, fvec3 r) {
    return {c * r.x, c * r.y, c * r.z};
}

}  // namespace glm
