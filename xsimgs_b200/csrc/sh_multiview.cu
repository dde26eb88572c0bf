// Spherical-harmonics backward split for multi-view training (several
// sensors, one process per GPU): the coefficient gradient of a Gaussian,
// summed over views, is  sum_j Y(dir_j) (x) dcolor_j  with dir_j the unit
// vector from view j's origin, so ranks can exchange the 3-float colour
// gradients of their views (and the view origins) instead of the
// 3 x (deg+1)^2-float coefficient gradients, and rebuild the sum locally:
//   xsg_sh_positions_bwd     position gradient of this rank's own views
//                            (needs the coefficients; overwrites d_positions)
//   xsg_sh_coeffs_bwd_multi  coefficient gradient summed over any set of views
//                            (does not read the coefficients)
// Both use the [N, K, 3] coefficient layout with band 0 in `coeffs` and no
// mask; the per-view expressions are those of sh_bwd_kernel (the reference's
// sh_bwd.cu:20-315), so the sums equal the per-view backward summed.
#include <string>
#include <type_traits>

#include "sh_basis.cuh"

namespace xsg {
namespace {

template <int DEG>
__global__ void __launch_bounds__(kShThreads)
    sh_positions_bwd_kernel(int n_views, const float* __restrict__ origins, const float* __restrict__ pos,
                            const float* __restrict__ coeffs, int64_t n, int dim, const float* __restrict__ d_out,
                            float* __restrict__ d_pos) {
    constexpr int NB = (DEG + 1) * (DEG + 1);
    extern __shared__ float stage[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t g0 = (int64_t(blockIdx.x) * kShWarps + w) * 32;
    const int S = dim * 3, SP = S + 1;
    float* wb = stage + w * 32 * SP;
    const int cnt = g0 < n ? int(min(int64_t(32), n - g0)) : 0;
    if (cnt > 0) stage_rows_in(coeffs + g0 * S, cnt * S, S, wb, lane);
    __syncwarp();
    const int64_t i = g0 + lane;
    if (lane >= cnt) return;
    const v3 p = ld3(pos + 3 * i);
    v3 dp = mk3(0.f, 0.f, 0.f);
    for (int j = 0; j < n_views; ++j) {
        const v3 diff = p - ld3(origins + 3 * j);
        const float il = rsqrtf(dot3(diff, diff));
        const v3 dir = diff * il;
        float bx[25], by[25], bz[25];
        sh_basis_grad<DEG>(dir.x, dir.y, dir.z, bx, by, bz);
        v3 gd = mk3(0.f, 0.f, 0.f);
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            const float g = d_out[(int64_t(j) * n + i) * 3 + ch];
#pragma unroll
            for (int k = 1; k < NB; ++k) {
                const float cg = wb[lane * SP + k * 3 + ch] * g;
                gd.x += bx[k] * cg;
                gd.y += by[k] * cg;
                gd.z += bz[k] * cg;
            }
        }
        // normalize backward: il * g - il^3 (g . v) v
        const float il3 = il * il * il;
        dp = dp + (il * gd - (il3 * dot3(gd, diff)) * diff);
    }
    st3(d_pos + 3 * i, dp);
}

template <int DEG>
__global__ void __launch_bounds__(kShThreads)
    sh_coeffs_bwd_multi_kernel(int n_views, const float* __restrict__ origins, const float* __restrict__ pos,
                               int64_t n, int dim, const float* __restrict__ d_out, float* __restrict__ d_coeffs) {
    constexpr int NB = (DEG + 1) * (DEG + 1);
    extern __shared__ float stage[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t g0 = (int64_t(blockIdx.x) * kShWarps + w) * 32;
    const int S = dim * 3, SP = S + 1;
    float* wb = stage + w * 32 * SP;
    const int cnt = g0 < n ? int(min(int64_t(32), n - g0)) : 0;
    const int64_t i = g0 + lane;
    if (lane < cnt) {
        float acc[NB][3];
#pragma unroll
        for (int k = 0; k < NB; ++k) acc[k][0] = acc[k][1] = acc[k][2] = 0.f;
        const v3 p = ld3(pos + 3 * i);
        for (int j = 0; j < n_views; ++j) {
            v3 dir = p - ld3(origins + 3 * j);
            dir = dir * rsqrtf(dot3(dir, dir));
            float b[25];
            sh_basis<DEG>(dir.x, dir.y, dir.z, b);
            const float* go = d_out + (int64_t(j) * n + i) * 3;
            const float g0c = go[0], g1c = go[1], g2c = go[2];
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                acc[k][0] += b[k] * g0c;
                acc[k][1] += b[k] * g1c;
                acc[k][2] += b[k] * g2c;
            }
        }
#pragma unroll
        for (int k = 0; k < NB; ++k)
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) wb[lane * SP + k * 3 + ch] = acc[k][ch];
        // bands stored beyond the degree in use get zero gradient
        for (int k = NB; k < dim; ++k)
            for (int ch = 0; ch < 3; ++ch) wb[lane * SP + k * 3 + ch] = 0.f;
    }
    __syncwarp();
    if (cnt > 0) stage_rows_out(d_coeffs + g0 * S, cnt * S, S, wb, lane);
}

int sh_mv_check(int degree, int n_views, int64_t n, int dim, const char* what) {
    if (degree < 0 || degree > 4 || n_views < 0 || n < 0 || dim < (degree + 1) * (degree + 1) || dim > 64)
        return set_error(XSG_ERR_INVALID_ARGUMENT, std::string(what) + ": bad degree, view count or band count");
    return XSG_OK;
}

size_t stage_bytes(int dim) { return size_t(kShWarps) * 32 * (3 * dim + 1) * sizeof(float); }

template <typename F>
int sh_mv_launch(int degree, F&& go) {
    switch (degree) {
        case 0: return go(std::integral_constant<int, 0>{});
        case 1: return go(std::integral_constant<int, 1>{});
        case 2: return go(std::integral_constant<int, 2>{});
        case 3: return go(std::integral_constant<int, 3>{});
        default: return go(std::integral_constant<int, 4>{});
    }
}

}  // namespace
}  // namespace xsg

using namespace xsg;

extern "C" int xsg_sh_positions_bwd(int degree, int n_views, const float* origins, const float* positions,
                                    const float* coeffs, int64_t n, int dim, const float* d_out, float* d_positions,
                                    xsg_stream_t stream) {
    int rc = sh_mv_check(degree, n_views, n, dim, "spherical_harmonics_positions_bwd");
    if (rc) return rc;
    if (n == 0) return XSG_OK;
    XSG_REQUIRE(origins && positions && coeffs && d_out && d_positions && n_views > 0,
                "spherical_harmonics_positions_bwd: null argument");
    const size_t sm = stage_bytes(dim);
    const unsigned nb = blocks_for(n, kShThreads);
    cudaStream_t st = as_cuda(stream);
    return sh_mv_launch(degree, [&](auto D) {
        auto k = sh_positions_bwd_kernel<decltype(D)::value>;
        if (sm > 48 * 1024) XSG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
        ScopedTimer tm("sh_positions_bwd", st);
        launch(k, nb, kShThreads, sm, st, n_views, origins, positions, coeffs, n, dim, d_out, d_positions);
        return check_launch("spherical_harmonics_positions_bwd");
    });
}

extern "C" int xsg_sh_coeffs_bwd_multi(int degree, int n_views, const float* origins, const float* positions,
                                       int64_t n, int dim, const float* d_out, float* d_coeffs, xsg_stream_t stream) {
    int rc = sh_mv_check(degree, n_views, n, dim, "spherical_harmonics_coeffs_bwd_multi");
    if (rc) return rc;
    if (n == 0) return XSG_OK;
    XSG_REQUIRE(positions && d_coeffs && (n_views == 0 || (origins && d_out)),
                "spherical_harmonics_coeffs_bwd_multi: null argument");
    const size_t sm = stage_bytes(dim);
    const unsigned nb = blocks_for(n, kShThreads);
    cudaStream_t st = as_cuda(stream);
    return sh_mv_launch(degree, [&](auto D) {
        auto k = sh_coeffs_bwd_multi_kernel<decltype(D)::value>;
        if (sm > 48 * 1024) XSG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
        ScopedTimer tm("sh_coeffs_bwd_multi", st);
        launch(k, nb, kShThreads, sm, st, n_views, origins, positions, n, dim, d_out, d_coeffs);
        return check_launch("spherical_harmonics_coeffs_bwd_multi");
    });
}
