// View-dependent colour from real spherical harmonics (degree 0..4), forward
// and backward, for sm_100a.  Semantics: spherical_harmonics_fused_fwd /
// _bwd of the reference (csrc/color/sh_fwd.cu:16-245, sh_bwd.cu:20-376):
// rgb = sum_k Y_k(normalize(pos - origin)) coeff_k + 0.5, no clamp.
//
// One thread per Gaussian evaluates the basis once and all three channels
// (the reference spends one thread per channel); the backward owns each
// Gaussian's gradients outright, so it needs no atomics except the
// per-block partial of d_origin, which a second pass sums deterministically.
#include <mutex>
#include <string>

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

struct ShLayout {
    int64_t n;
    int dim;          // K, bands stored in coeffs
    bool l3kn;        // [3, K, N] else [N, K, 3]
    bool has_dc;      // band 0 kept in coeffs_dc
    // index of (band k, channel ch) in coeffs (band >= 1 when has_dc)
    __device__ __forceinline__ int64_t ci(int64_t i, int k, int ch) const {
        const int kk = has_dc ? k - 1 : k;
        return l3kn ? (int64_t(ch) * dim + kk) * n + i : (i * dim + kk) * 3 + ch;
    }
    __device__ __forceinline__ int64_t di(int64_t i, int ch) const { return l3kn ? int64_t(ch) * n + i : i * 3 + ch; }
};

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
__device__ __forceinline__ void stage_rows_in(const float* __restrict__ src, int total, int S, float* wb,
                                              int lane) {
    const float invS = 1.0f / float(S);
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

template <int DEG, bool kL3KN>
__global__ void __launch_bounds__(kShThreads)
    sh_fwd_kernel(const float* __restrict__ origin, const float* __restrict__ pos, const float* __restrict__ coeffs,
                  const float* __restrict__ dc, const uint32_t* __restrict__ mask, ShLayout L,
                  float* __restrict__ out) {
    constexpr int NB = (DEG + 1) * (DEG + 1);
    extern __shared__ float stage[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t g0 = (int64_t(blockIdx.x) * kShWarps + w) * 32;
    if (g0 >= L.n) return;
    const int cnt = int(min(int64_t(32), L.n - g0));
    const int S = L.dim * 3, SP = S + 1;
    float* wb = stage + w * 32 * SP;
    if constexpr (!kL3KN) {
        stage_rows_in(coeffs + g0 * S, cnt * S, S, wb, lane);
        __syncwarp();
    }
    const int64_t i = g0 + lane;
    if (lane >= cnt) return;
    if (mask && !((mask[i >> 5] >> (i & 31)) & 1u)) return;
    v3 dir = ld3(pos + 3 * i) - mk3(origin[0], origin[1], origin[2]);
    dir = dir * rsqrtf(dot3(dir, dir));
    float b[25];
    sh_basis<DEG>(dir.x, dir.y, dir.z, b);
    const int kb = L.has_dc ? 1 : 0;  // first band held in coeffs
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        auto cf = [&](int k) {
            return kL3KN ? coeffs[(int64_t(ch) * L.dim + (k - kb)) * L.n + i] : wb[lane * SP + (k - kb) * 3 + ch];
        };
        float r = b[0] * (L.has_dc ? dc[L.di(i, ch)] : cf(0));
#pragma unroll
        for (int k = 1; k < NB; ++k) r += b[k] * cf(k);
        out[3 * i + ch] = r + 0.5f;
    }
}

template <int DEG, bool kL3KN>
__global__ void __launch_bounds__(kShThreads)
    sh_bwd_kernel(const float* __restrict__ origin, const float* __restrict__ pos, const float* __restrict__ coeffs,
                  const float* __restrict__ dc, const uint32_t* __restrict__ mask, ShLayout L,
                  const float* __restrict__ d_out, float* __restrict__ d_coeffs, float* __restrict__ d_dc,
                  float* __restrict__ d_pos, float* __restrict__ block_origin) {
    constexpr int NB = (DEG + 1) * (DEG + 1);
    extern __shared__ float stage[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t g0 = (int64_t(blockIdx.x) * kShWarps + w) * 32;
    const int S = L.dim * 3, SP = S + 1;
    float* wb = stage + w * 32 * SP;
    const int cnt = g0 < L.n ? int(min(int64_t(32), L.n - g0)) : 0;
    if constexpr (!kL3KN) {
        if (cnt > 0) stage_rows_in(coeffs + g0 * S, cnt * S, S, wb, lane);
        __syncwarp();
    }
    const int64_t i = g0 + lane;
    const int kb = L.has_dc ? 1 : 0;
    v3 dorig = mk3(0.f, 0.f, 0.f);
    if (lane < cnt) {
        const bool on = !mask || ((mask[i >> 5] >> (i & 31)) & 1u);
        if (!on) {
            // masked Gaussians get zero gradients (outputs are overwritten)
            if constexpr (kL3KN) {
                for (int k = 0; k < L.dim; ++k)
                    for (int ch = 0; ch < 3; ++ch) d_coeffs[(int64_t(ch) * L.dim + k) * L.n + i] = 0.f;
            } else {
                for (int r = 0; r < S; ++r) wb[lane * SP + r] = 0.f;
            }
            if (L.has_dc)
                for (int ch = 0; ch < 3; ++ch) d_dc[L.di(i, ch)] = 0.f;
            st3(d_pos + 3 * i, mk3(0.f, 0.f, 0.f));
        } else {
            const v3 diff = ld3(pos + 3 * i) - mk3(origin[0], origin[1], origin[2]);
            const float il = rsqrtf(dot3(diff, diff));
            const v3 dir = diff * il;
            float b[25], bx[25], by[25], bz[25];
            sh_basis<DEG>(dir.x, dir.y, dir.z, b);
            sh_basis_grad<DEG>(dir.x, dir.y, dir.z, bx, by, bz);
            v3 gd = mk3(0.f, 0.f, 0.f);
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                const float g = d_out[3 * i + ch];
                if (L.has_dc) d_dc[L.di(i, ch)] = b[0] * g;
#pragma unroll
                for (int k = 0; k < NB; ++k) {
                    if (k == 0 && L.has_dc) continue;
                    const int kk = k - kb;
                    float cf;
                    if constexpr (kL3KN) {
                        const int64_t o = (int64_t(ch) * L.dim + kk) * L.n + i;
                        cf = coeffs[o];
                        d_coeffs[o] = b[k] * g;
                    } else {
                        float* e = wb + lane * SP + kk * 3 + ch;
                        cf = *e;
                        *e = b[k] * g;  // the staged row becomes the gradient row
                    }
                    if (k > 0) {
                        const float cg = cf * g;
                        gd.x += bx[k] * cg;
                        gd.y += by[k] * cg;
                        gd.z += bz[k] * cg;
                    }
                }
            }
            // bands stored beyond the degree in use get zero gradient
            for (int kk = NB - kb; kk < L.dim; ++kk)
                for (int ch = 0; ch < 3; ++ch) {
                    if constexpr (kL3KN) d_coeffs[(int64_t(ch) * L.dim + kk) * L.n + i] = 0.f;
                    else wb[lane * SP + kk * 3 + ch] = 0.f;
                }
            // normalize backward: il * g - il^3 (g . v) v
            const float il3 = il * il * il;
            const float gv = dot3(gd, diff);
            const v3 dp = il * gd - (il3 * gv) * diff;
            st3(d_pos + 3 * i, dp);
            dorig = -1.0f * dp;
        }
    }
    if constexpr (!kL3KN) {
        __syncwarp();
        if (cnt > 0) stage_rows_out(d_coeffs + g0 * S, cnt * S, S, wb, lane);
    }
    // per-block partial of d_origin
    __shared__ float s[3][kShWarps];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        dorig.x += __shfl_xor_sync(0xffffffffu, dorig.x, o);
        dorig.y += __shfl_xor_sync(0xffffffffu, dorig.y, o);
        dorig.z += __shfl_xor_sync(0xffffffffu, dorig.z, o);
    }
    if (lane == 0) { s[0][w] = dorig.x; s[1][w] = dorig.y; s[2][w] = dorig.z; }
    __syncthreads();
    if (threadIdx.x < 3) {
        float t = 0.f;
        for (int k = 0; k < kShWarps; ++k) t += s[threadIdx.x][k];
        block_origin[int64_t(blockIdx.x) * 3 + threadIdx.x] = t;
    }
}

__global__ void sum_partials_kernel(const float* __restrict__ p, int64_t nb, float* __restrict__ out) {
    __shared__ float s[3][32];
    float acc[3] = {0.f, 0.f, 0.f};
    for (int64_t b = threadIdx.x; b < nb; b += blockDim.x) {
        acc[0] += p[3 * b]; acc[1] += p[3 * b + 1]; acc[2] += p[3 * b + 2];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        for (int k = 0; k < 3; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0)
        for (int k = 0; k < 3; ++k) s[k][w] = acc[k];
    __syncthreads();
    if (threadIdx.x < 3) {
        float t = 0.f;
        for (int k = 0; k < int(blockDim.x >> 5); ++k) t += s[threadIdx.x][k];
        out[threadIdx.x] = t;
    }
}

static size_t sh_stage_bytes(int dim) { return size_t(kShWarps) * 32 * (3 * dim + 1) * sizeof(float); }

static int sh_check(int degree, int64_t n, int dim, bool has_dc) {
    XSG_REQUIRE(degree >= 0 && degree <= 4, "Unsupported spherical harmonics degree: " + std::to_string(degree));
    XSG_REQUIRE(n >= 0 && dim >= 0, "spherical_harmonics: bad sizes");
    const int req = (degree + 1) * (degree + 1) - (has_dc ? 1 : 0);
    XSG_REQUIRE(dim >= req, "Number of harmonics band in coeffs tensor must be higher or equal than " +
                                std::to_string(req) + " for degree_to_use=" + std::to_string(degree));
    return XSG_OK;
}

}  // namespace xsg

using namespace xsg;

extern "C" {

int xsg_sh_fwd(int degree, const float* origin, const float* pos, const float* coeffs, const float* dc,
               const uint32_t* mask, int layout_3kn, int64_t n, int dim, float* out, xsg_stream_t stream) {
    int rc = sh_check(degree, n, dim, dc != nullptr);
    if (rc != XSG_OK) return rc;
    if (n == 0) return XSG_OK;
    XSG_REQUIRE(origin && pos && out && (coeffs || dim == 0), "spherical_harmonics_fwd: null argument");
    ShLayout L{n, dim, layout_3kn != 0, dc != nullptr};
    cudaStream_t st = as_cuda(stream);
    const unsigned nb = blocks_for(n, kShThreads);
    const size_t sm = layout_3kn ? 0 : sh_stage_bytes(dim);
    int rc2 = XSG_OK;
    auto go = [&](auto kernel) {
        if (sm > 48 * 1024 && cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)) != cudaSuccess)
            rc2 = set_error(XSG_ERR_UNSUPPORTED, "spherical_harmonics_fwd: too many coefficient bands");
        else
            launch(kernel, nb, kShThreads, sm, st, origin, pos, coeffs, dc, mask, L, out);
    };
#define XSG_SHF(D) (layout_3kn ? go(sh_fwd_kernel<D, true>) : go(sh_fwd_kernel<D, false>))
    switch (degree) {
        case 0: XSG_SHF(0); break;
        case 1: XSG_SHF(1); break;
        case 2: XSG_SHF(2); break;
        case 3: XSG_SHF(3); break;
        default: XSG_SHF(4); break;
    }
#undef XSG_SHF
    if (rc2 != XSG_OK) return rc2;
    return check_launch("spherical_harmonics_fwd");
}

size_t xsg_sh_bwd_workspace_size(int64_t n) {
    return Arena::round(size_t(n < 0 ? 0 : (n + kShThreads - 1) / kShThreads + 1) * 3 * sizeof(float));
}

int xsg_sh_bwd(int degree, const float* origin, const float* pos, const float* coeffs, const float* dc,
               const uint32_t* mask, int layout_3kn, int64_t n, int dim, const float* d_out, float* d_coeffs,
               float* d_dc, float* d_pos, float* d_origin, void* workspace, size_t ws_bytes,
               xsg_stream_t stream) {
    int rc = sh_check(degree, n, dim, dc != nullptr);
    if (rc != XSG_OK) return rc;
    XSG_REQUIRE(d_origin, "spherical_harmonics_bwd: null d_origin");
    cudaStream_t st = as_cuda(stream);
    if (n == 0) {
        XSG_CUDA(cudaMemsetAsync(d_origin, 0, 3 * sizeof(float), st));
        return XSG_OK;
    }
    XSG_REQUIRE(origin && pos && d_out && d_coeffs && d_pos && (!dc || d_dc), "spherical_harmonics_bwd: null argument");
    if (!workspace || ws_bytes < xsg_sh_bwd_workspace_size(n))
        return set_error(XSG_ERR_WORKSPACE, "spherical_harmonics_bwd: workspace too small");
    ShLayout L{n, dim, layout_3kn != 0, dc != nullptr};
    const unsigned nb = blocks_for(n, kShThreads);
    float* part = static_cast<float*>(workspace);
    const size_t sm = layout_3kn ? 0 : sh_stage_bytes(dim);
    int rc2 = XSG_OK;
    auto go = [&](auto kernel) {
        if (sm > 48 * 1024 && cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)) != cudaSuccess)
            rc2 = set_error(XSG_ERR_UNSUPPORTED, "spherical_harmonics_bwd: too many coefficient bands");
        else
            launch(kernel, nb, kShThreads, sm, st, origin, pos, coeffs, dc, mask, L, d_out, d_coeffs, d_dc, d_pos,
                   part);
    };
#define XSG_SH_BWD(D) (layout_3kn ? go(sh_bwd_kernel<D, true>) : go(sh_bwd_kernel<D, false>))
    switch (degree) {
        case 0: XSG_SH_BWD(0); break;
        case 1: XSG_SH_BWD(1); break;
        case 2: XSG_SH_BWD(2); break;
        case 3: XSG_SH_BWD(3); break;
        default: XSG_SH_BWD(4); break;
    }
#undef XSG_SH_BWD
    if (rc2 != XSG_OK) return rc2;
    launch(sum_partials_kernel, 1, 1024, 0, st, part, nb, d_origin);
    return check_launch("spherical_harmonics_bwd");
}

}  // extern "C"

// ---------------------------------------------- allocation-free variant --
// xsg_sh_bwd_noalloc: the same spherical-harmonics backward for callers that
// cannot allocate device memory themselves (for example a host runtime that
// hands the library only the tensors it owns, or a process that must not
// call cudaMalloc on a hot path).  Its only scratch, the per-block partial
// sums of d_origin, lives in the fixed device array below, which every GPU
// that loads this library holds until the process exits.
namespace xsg {

constexpr int64_t kShNoAllocMaxGaussians = int64_t(1) << 23;  // 8,388,608
constexpr int64_t kShNoAllocMaxBlocks = (kShNoAllocMaxGaussians + kShThreads - 1) / kShThreads;

// 65,536 blocks x 3 floats = 768 KiB per device.
static __device__ __align__(256) float g_sh_noalloc_partials[kShNoAllocMaxBlocks * 3];

// Device address of the array, looked up once per device (host code may not
// use the symbol itself as a pointer).
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {nullptr};

static int sh_noalloc_scratch(float** out) {
    int dev = -1;
    XSG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(XSG_ERR_UNSUPPORTED, "spherical_harmonics_bwd_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_sh_noalloc_partials);
        if (e != cudaSuccess)
            return set_error(XSG_ERR_CUDA, std::string("spherical_harmonics_bwd_noalloc: cudaGetSymbolAddress: ") +
                                               cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return XSG_OK;
}

}  // namespace xsg

extern "C" {

int64_t xsg_sh_bwd_noalloc_max_gaussians(void) { return xsg::kShNoAllocMaxGaussians; }

int xsg_sh_bwd_noalloc(int degree, const float* origin, const float* pos, const float* coeffs, const float* dc,
                       const uint32_t* mask, int layout_3kn, int64_t n, int dim, const float* d_out,
                       float* d_coeffs, float* d_dc, float* d_pos, float* d_origin, xsg_stream_t stream) {
    int rc = sh_check(degree, n, dim, dc != nullptr);
    if (rc != XSG_OK) return rc;
    XSG_REQUIRE(d_origin, "spherical_harmonics_bwd_noalloc: null d_origin");
    if (n > kShNoAllocMaxGaussians)
        return set_error(XSG_ERR_INVALID_ARGUMENT,
                         "spherical_harmonics_bwd_noalloc: " + std::to_string(n) + " Gaussians exceed the maximum of " +
                             std::to_string(kShNoAllocMaxGaussians) + "; use xsg_sh_bwd with a workspace");
    cudaStream_t st = as_cuda(stream);
    if (n == 0) {
        XSG_CUDA(cudaMemsetAsync(d_origin, 0, 3 * sizeof(float), st));
        return XSG_OK;
    }
    XSG_REQUIRE(origin && pos && d_out && d_coeffs && d_pos && (!dc || d_dc),
                "spherical_harmonics_bwd_noalloc: null argument");
    float* part = nullptr;
    rc = sh_noalloc_scratch(&part);
    if (rc != XSG_OK) return rc;
    // every block writes its own partial before the final sum reads it, so
    // nothing left from an earlier call is read and nothing needs clearing
    ShLayout L{n, dim, layout_3kn != 0, dc != nullptr};
    const unsigned nb = blocks_for(n, kShThreads);
    const size_t sm = layout_3kn ? 0 : sh_stage_bytes(dim);
    int rc2 = XSG_OK;
    auto go = [&](auto kernel) {
        if (sm > 48 * 1024 && cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)) != cudaSuccess)
            rc2 = set_error(XSG_ERR_UNSUPPORTED, "spherical_harmonics_bwd_noalloc: too many coefficient bands");
        else
            launch(kernel, nb, kShThreads, sm, st, origin, pos, coeffs, dc, mask, L, d_out, d_coeffs, d_dc, d_pos,
                   part);
    };
    switch (degree) {
        case 0: layout_3kn ? go(sh_bwd_kernel<0, true>) : go(sh_bwd_kernel<0, false>); break;
        case 1: layout_3kn ? go(sh_bwd_kernel<1, true>) : go(sh_bwd_kernel<1, false>); break;
        case 2: layout_3kn ? go(sh_bwd_kernel<2, true>) : go(sh_bwd_kernel<2, false>); break;
        case 3: layout_3kn ? go(sh_bwd_kernel<3, true>) : go(sh_bwd_kernel<3, false>); break;
        default: layout_3kn ? go(sh_bwd_kernel<4, true>) : go(sh_bwd_kernel<4, false>); break;
    }
    if (rc2 != XSG_OK) return rc2;
    launch(sum_partials_kernel, 1, 1024, 0, st, part, nb, d_origin);
    return check_launch("spherical_harmonics_bwd_noalloc");
}

}  // extern "C"
