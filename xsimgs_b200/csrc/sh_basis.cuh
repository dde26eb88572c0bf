// Real spherical-harmonics basis (degree 0..4) and its gradient, and the
// per-warp shared-memory staging of [N, K, 3] coefficient rows, shared by the
// SH kernels (sh.cu, sh_multiview.cu).
#pragma once

#include "common.cuh"

namespace xsg {

// Basis values in the polynomial form of sh_fwd.cu:34-112.
template <int DEG>
__device__ __forceinline__ void sh_basis(float x, float y, float z, float* b) {
    b[0] = 0.2820947917738781f;
    if (DEG < 1) return;
    b[1] = -0.48860251190292f * y;
    b[2] = 0.48860251190292f * z;
    b[3] = -0.48860251190292f * x;
    if (DEG < 2) return;
    const float z2 = z * z;
    const float t0B = -1.092548430592079f * z;
    const float c1 = x * x - y * y, s1 = 2.f * x * y;
    b[4] = 0.5462742152960395f * s1;
    b[5] = t0B * y;
    b[6] = 0.9461746957575601f * z2 - 0.3153915652525201f;
    b[7] = t0B * x;
    b[8] = 0.5462742152960395f * c1;
    if (DEG < 3) return;
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
    if (DEG < 4) return;
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

// Partial derivatives of each basis polynomial in x, y, z (independent).
template <int DEG>
__device__ __forceinline__ void sh_basis_grad(float x, float y, float z, float* bx, float* by, float* bz) {
#pragma unroll
    for (int i = 0; i < 25; ++i) bx[i] = by[i] = bz[i] = 0.f;
    if (DEG < 1) return;
    const float K1 = 0.48860251190292f;
    by[1] = -K1; bz[2] = K1; bx[3] = -K1;
    if (DEG < 2) return;
    const float K4 = 0.5462742152960395f, K5 = -1.092548430592079f, K6 = 0.9461746957575601f;
    bx[4] = K4 * 2.f * y; by[4] = K4 * 2.f * x;
    by[5] = K5 * z; bz[5] = K5 * y;
    bz[6] = 2.f * K6 * z;
    bx[7] = K5 * z; bz[7] = K5 * x;
    bx[8] = K4 * 2.f * x; by[8] = -K4 * 2.f * y;
    if (DEG < 3) return;
    const float K9 = -0.5900435899266435f, KT = 1.445305721320277f;
    const float A = -2.285228997322329f, B = 0.4570457994644658f;
    const float C = 1.865881662950577f, D = -1.119528997770346f;
    const float xx = x * x, yy = y * y, zz = z * z;
    bx[9] = K9 * 6.f * x * y; by[9] = K9 * (3.f * xx - 3.f * yy);
    bx[10] = KT * z * 2.f * y; by[10] = KT * z * 2.f * x; bz[10] = KT * 2.f * x * y;
    by[11] = A * zz + B; bz[11] = 2.f * A * z * y;
    bz[12] = 3.f * C * zz + D;
    bx[13] = A * zz + B; bz[13] = 2.f * A * z * x;
    bx[14] = KT * z * 2.f * x; by[14] = -KT * z * 2.f * y; bz[14] = KT * (xx - yy);
    bx[15] = K9 * (3.f * xx - 3.f * yy); by[15] = K9 * (-6.f * x * y);
    if (DEG < 4) return;
    const float K16 = 0.6258357354491763f, E = -4.683325804901025f, F = 2.007139630671868f;
    const float G = 3.31161143515146f, Hh = -0.47308734787878f, I = -1.770130769779931f;
    bx[16] = K16 * (12.f * xx * y - 4.f * yy * y); by[16] = K16 * (4.f * xx * x - 12.f * x * yy);
    bx[17] = I * z * 6.f * x * y; by[17] = I * z * (3.f * xx - 3.f * yy); bz[17] = I * (3.f * xx * y - yy * y);
    bx[18] = (G * zz + Hh) * 2.f * y; by[18] = (G * zz + Hh) * 2.f * x; bz[18] = 2.f * G * z * 2.f * x * y;
    by[19] = E * zz * z + F * z; bz[19] = (3.f * E * zz + F) * y;
    bz[20] = 1.984313483298443f * (z * (C * zz + D) + z * (3.f * C * zz + D)) - 1.006230589874905f * (2.f * K6 * z);
    bx[21] = E * zz * z + F * z; bz[21] = (3.f * E * zz + F) * x;
    bx[22] = (G * zz + Hh) * 2.f * x; by[22] = -(G * zz + Hh) * 2.f * y; bz[22] = 2.f * G * z * (xx - yy);
    bx[23] = I * z * (3.f * xx - 3.f * yy); by[23] = I * z * (-6.f * x * y); bz[23] = I * (xx * x - 3.f * x * yy);
    bx[24] = K16 * (4.f * xx * x - 12.f * x * yy); by[24] = K16 * (-12.f * xx * y + 4.f * yy * y);
}

// Coefficients of 32 consecutive Gaussians are staged per warp in shared
// memory: [N, K, 3] rows are read (and, in the backward, written) with
// coalesced accesses, and each lane then walks its own row with an odd stride
// (3K + 1 floats) so the per-lane reads do not conflict on banks.  The
// [3, K, N] layout is already coalesced along N and is read directly.
constexpr int kShWarps = 4;
constexpr int kShThreads = kShWarps * 32;

// Copies `total` consecutive floats of global memory into a warp's staging
// rows (row length S, padded row stride S + 1), eight loads in flight per
// lane.  Row/column of element j come from a float reciprocal: (j + 0.5) / S
// is at least 0.5 / S away from an integer, far more than its rounding error.
// Rows of S floats between global memory (dense) and a warp's shared
// staging area (rows padded to S + 1 floats against bank conflicts).  With a
// 16-byte aligned global pointer and S a multiple of 4 the copy moves float4
// words (a word never straddles two rows).
__device__ __forceinline__ bool stage_vec_ok(const float* g, int total, int S) {
    return (reinterpret_cast<uintptr_t>(g) & 15u) == 0 && (S & 3) == 0 && (total & 3) == 0;
}

__device__ __forceinline__ void stage_rows_in(const float* __restrict__ src, int total, int S, float* wb,
                                              int lane) {
    const float invS = 1.0f / float(S);
    if (stage_vec_ok(src, total, S)) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        const int t4 = total >> 2;
        for (int base = 0; base < t4; base += 32 * 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = base + u * 32 + lane;
                v[u] = q < t4 ? s4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = base + u * 32 + lane;
                if (q < t4) {
                    const int j = q << 2;
                    const int row = int((float(j) + 0.5f) * invS);
                    float* d = wb + row * (S + 1) + (j - row * S);
                    d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w;
                }
            }
        }
        return;
    }
    for (int base = 0; base < total; base += 32 * 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = base + u * 32 + lane;
            v[u] = j < total ? src[j] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = base + u * 32 + lane;
            if (j < total) {
                const int row = int((float(j) + 0.5f) * invS);
                wb[row * (S + 1) + (j - row * S)] = v[u];
            }
        }
    }
}

__device__ __forceinline__ void stage_rows_out(float* __restrict__ dst, int total, int S, const float* wb,
                                               int lane) {
    const float invS = 1.0f / float(S);
    if (stage_vec_ok(dst, total, S)) {
        float4* d4 = reinterpret_cast<float4*>(dst);
        const int t4 = total >> 2;
        for (int q = lane; q < t4; q += 32) {
            const int j = q << 2;
            const int row = int((float(j) + 0.5f) * invS);
            const float* sp = wb + row * (S + 1) + (j - row * S);
            d4[q] = make_float4(sp[0], sp[1], sp[2], sp[3]);
        }
        return;
    }
    for (int base = 0; base < total; base += 32 * 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = base + u * 32 + lane;
            if (j < total) {
                const int row = int((float(j) + 0.5f) * invS);
                dst[j] = wb[row * (S + 1) + (j - row * S)];
            }
        }
    }
}

}  // namespace xsg
