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

#include "sh_basis.cuh"

namespace xsg {

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
    ScopedTimer tm("sh_fwd", st);
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
    ScopedTimer tm("sh_bwd", st);
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

// The kernels run on the caller's stream, so the array must be the one on
// that stream's device: a stream of another device is rejected rather than
// handed this device's address.
static int sh_noalloc_scratch(cudaStream_t stream, float** out) {
    int dev = -1;
    XSG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(XSG_ERR_UNSUPPORTED, "spherical_harmonics_bwd_noalloc: device ordinal out of range");
    int stream_dev = dev;
    XSG_CUDA(cudaStreamGetDevice(stream, &stream_dev));
    if (stream_dev != dev)
        return set_error(XSG_ERR_INVALID_ARGUMENT,
                         "spherical_harmonics_bwd_noalloc: the stream belongs to device " + std::to_string(stream_dev) +
                             " but device " + std::to_string(dev) + " is current");
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
    rc = sh_noalloc_scratch(st, &part);
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
