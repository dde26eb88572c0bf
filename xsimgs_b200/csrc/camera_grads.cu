// Camera-parameter gradients of the per-pixel rays and pixel times
// (the backward of camera_rays, pixel_time(_delta) and
// pixel_time(_delta)_from_uv) for sm_100a.
//
// Every pixel contributes to the same ~26 pack words, so the work is a
// reduction: a grid of at most kGradMaxBlocks CTAs walks the pixels with a
// grid stride, each thread keeps one register accumulator per pack word, each
// CTA reduces them (warp shuffles, then shared memory) to one row of
// kGradStride floats in the caller's workspace, and a one-CTA pass sums the
// rows in a fixed order into d_pack.  The result is deterministic (no float
// atomics) and d_pack is fully written (zero for words without a gradient:
// the padding word, the lidar table address, the spherical limits).
#include "cameras.cuh"
#include "quat.cuh"

namespace xsg {

constexpr int kGradThreads = 256;
constexpr int kGradWarps = kGradThreads / 32;
constexpr int kGradMaxBlocks = 4 * 148;
constexpr int kGradStride = 48;  // floats per partial row (>= every pack, 36 words at most)

// Reduce the CTA's per-thread accumulators (pack words [off, off + P)) to one
// partial row; words outside that range are written as zero.
template <int P>
__device__ __forceinline__ void block_partials(const float (&acc)[P], int off, float* __restrict__ partial) {
    __shared__ float sm[kGradWarps][P];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int j = 0; j < P; ++j) {
        float v = acc[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sm[warp][j] = v;
    }
    __syncthreads();
    if (threadIdx.x < kGradStride) {
        const int j = int(threadIdx.x) - off;
        float s = 0.0f;
        if (j >= 0 && j < P) {
#pragma unroll
            for (int w = 0; w < kGradWarps; ++w) s += sm[w][j];
        }
        partial[blockIdx.x * kGradStride + threadIdx.x] = s;
    }
}

// d_pack[j] = sum over rows of partial[row][j], one warp per word.
__global__ void sum_partials_kernel(const float* __restrict__ partial, int rows, int words,
                                    float* __restrict__ d_pack) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int j = warp; j < words; j += blockDim.x >> 5) {
        float s = 0.0f;
        for (int r = lane; r < rows; r += 32) s += partial[r * kGradStride + j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) d_pack[j] = s;
    }
}

// sc(theta) = sin(theta/2)/theta and (d sc/d theta)/theta for the rotation
// vector backward.  The forward (axis_angle_quat) switches to the series
// 1/2 - theta^2/48 below 1e-2; the derivative uses the series
// -1/24 + theta^2/960 - theta^4/107520 below 0.3, where the closed form
// (cos(theta/2)/2 - sc)/theta^2 loses digits to cancellation.
__device__ __forceinline__ float aa_dsc_over_theta(float th, float sc, float ch) {
    if (th < 1e-2f) return -1.0f / 24.0f;
    if (th < 0.3f) {
        const float t2 = th * th;
        return -1.0f / 24.0f + t2 * (1.0f / 960.0f - t2 * (1.0f / 107520.0f));
    }
    return (0.5f * ch - sc) / (th * th);
}

// Backward of one world-space ray (camera_ray_backward_kernel_cuda,
// include/cameras/ray_kernels.h:61-123):
//   ray_o = t0 + v dt,  ray_d = R(q_aa(w dt) (x) std(q0)) n(ray_cs(uv)),
//   dt = trigger + uv . rolling - pose.
template <typename Cam, int P>
__device__ __forceinline__ v3 world_ray_bwd(const Cam& k, Q q0raw, Q q0s, float2 uv, v3 ray, int normalized,
                                            v3 g_o, v3 g_d, float (&acc)[P]) {
    const float dt = k.pixel_time(uv.x, uv.y) - k.pose;
    acc[4] += g_o.x; acc[5] += g_o.y; acc[6] += g_o.z;
    acc[7] += dt * g_o.x; acc[8] += dt * g_o.y; acc[9] += dt * g_o.z;
    float d_dt = dot3(g_o, k.v);

    const v3 nray = normalized ? ray * rsqrtf(dot3(ray, ray)) : ray;
    // q_aa = (cos(th/2), sc(th) a), a = w dt, th = |w| |dt|
    const float wn = sqrtf(dot3(k.w, k.w));
    const float th = wn * fabsf(dt);
    float sh, ch;
    sincosf(0.5f * th, &sh, &ch);
    const float sc = (th < 1e-2f) ? 0.5f - th * th * (1.0f / 48.0f) : sh / th;
    const v3 a = k.w * dt;
    const Q qa{ch, sc * a.x, sc * a.y, sc * a.z};
    const Q q = qmul(qa, q0s);

    const Q gq = rot_bwd_q(q, nray, g_d);
    const v3 d_nray = rot(conj(q), g_d);

    // (qa (x) q0s) backward
    const v3 av = vec(qa), bv = vec(q0s), gv = vec(gq);
    const float d_aw = gq.w * q0s.w + dot3(gv, bv);
    const v3 d_av = (q0s.w * gv - gq.w * bv) + cross3(bv, gv);
    const float d_bw = gq.w * qa.w + dot3(gv, av);
    const v3 d_bv = (qa.w * gv - gq.w * av) + cross3(gv, av);

    // rotation vector backward
    const v3 ga = (-0.5f * sc * d_aw) * a + sc * d_av + (dot3(a, d_av) * aa_dsc_over_theta(th, sc, ch)) * a;
    acc[10] += dt * ga.x; acc[11] += dt * ga.y; acc[12] += dt * ga.z;
    d_dt += dot3(k.w, ga);

    const Q d0 = qstd_bwd(q0raw, Q{d_bw, d_bv.x, d_bv.y, d_bv.z});
    acc[0] += d0.w; acc[1] += d0.x; acc[2] += d0.y; acc[3] += d0.z;

    acc[14] += d_dt * uv.x;
    acc[15] += d_dt * uv.y;
    acc[16] += d_dt;
    acc[17] -= d_dt;
    return d_nray;
}

__device__ __forceinline__ v3 normalize_bwd(v3 r, v3 g) {
    const float il = rsqrtf(dot3(r, r));
    const v3 n = r * il;
    return (g - dot3(n, g) * n) * il;
}

template <typename Cam>
__global__ void __launch_bounds__(kGradThreads)
    rays_bwd_kernel(const float* __restrict__ pack, int W, int H, int world, int normalized,
                    const float* __restrict__ d_ray_o, const float* __restrict__ d_ray_d,
                    float* __restrict__ partial) {
    constexpr int P = Cam::kWords;
    Cam k;
    k.load(pack);
    const Q q0raw{k.qw, k.qx, k.qy, k.qz};
    const Q q0s = qstd(q0raw);
    float acc[P];
#pragma unroll
    for (int j = 0; j < P; ++j) acc[j] = 0.0f;
    const int64_t n = int64_t(W) * H;
    for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const float2 uv = k.pixel_to_uv(int(idx % W), int(idx / W), W, H);
        const v3 ray = k.ray_cs(uv);
        const v3 g_d = ld3(d_ray_d + 3 * idx);
        v3 d_ray;
        if (world) {
            const v3 g_o = d_ray_o ? ld3(d_ray_o + 3 * idx) : mk3(0.f, 0.f, 0.f);
            d_ray = world_ray_bwd(k, q0raw, q0s, uv, ray, normalized, g_o, g_d, acc);
        } else {
            d_ray = g_d;
        }
        if (normalized) d_ray = normalize_bwd(ray, d_ray);
        k.ray_cs_bwd(uv, d_ray, acc);
    }
    block_partials(acc, 0, partial);
}

// pixel_time(_delta)_bwd_kernel and the _from_uv variants,
// include/cameras/time_kernels.h:115-300: t = trigger + uv . rolling
// (- pose for the delta variants); d_uv = grad * rolling for uv input.
template <typename Cam>
__global__ void __launch_bounds__(kGradThreads)
    time_bwd_kernel(const float* __restrict__ pack, int W, int H, const float* __restrict__ uv_in, int64_t n,
                    int delta, const float* __restrict__ grad, float* __restrict__ d_uv,
                    float* __restrict__ partial) {
    Cam k;
    k.load(pack);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rolling.x, rolling.y, trigger, pose
    for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
         idx += int64_t(gridDim.x) * blockDim.x) {
        float2 uv;
        if (uv_in) uv = reinterpret_cast<const float2*>(uv_in)[idx];
        else uv = k.pixel_to_uv(int(idx % W), int(idx / W), W, H);
        const float g = grad[idx];
        acc[0] += g * uv.x;
        acc[1] += g * uv.y;
        acc[2] += g;
        if (delta) acc[3] -= g;
        if (d_uv) reinterpret_cast<float2*>(d_uv)[idx] = make_float2(g * k.rolling.x, g * k.rolling.y);
    }
    block_partials(acc, 14, partial);
}

int grad_blocks(int64_t n) {
    const int64_t b = (n + kGradThreads - 1) / kGradThreads;
    return int(b < 1 ? 1 : (b > kGradMaxBlocks ? kGradMaxBlocks : b));
}

}  // namespace xsg

using namespace xsg;

extern "C" {

size_t xsg_camera_grad_workspace_size(void) { return size_t(kGradMaxBlocks) * kGradStride * sizeof(float); }

int xsg_camera_rays_bwd(int type, const float* pack, int W, int H, int world, int normalized,
                        const float* d_ray_o, const float* d_ray_d, float* d_pack, void* workspace,
                        size_t workspace_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(pack && d_ray_d && d_pack && W > 0 && H > 0, "camera_rays_bwd: bad arguments");
    if (!workspace || workspace_bytes < xsg_camera_grad_workspace_size())
        return set_error(XSG_ERR_WORKSPACE, "camera_rays_bwd: workspace too small");
    const int64_t n = int64_t(W) * H;
    const int nb = grad_blocks(n);
    float* partial = static_cast<float*>(workspace);
    const int words = xsg_camera_pack_words(type);
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        launch(rays_bwd_kernel<Cam>, nb, kGradThreads, 0, as_cuda(stream), pack, W, H, world, normalized,
               d_ray_o, d_ray_d, partial);
    });
    if (rc != XSG_OK) return rc;
    launch(sum_partials_kernel, 1, 1024, 0, as_cuda(stream), static_cast<const float*>(partial), nb, words, d_pack);
    return check_launch("camera_rays_bwd");
}

static int time_bwd(const char* what, int type, const float* pack, int W, int H, const float* uv, int64_t n,
                    int delta, const float* grad, float* d_pack, float* d_uv, void* workspace,
                    size_t workspace_bytes, xsg_stream_t stream) {
    if (!workspace || workspace_bytes < xsg_camera_grad_workspace_size())
        return set_error(XSG_ERR_WORKSPACE, std::string(what) + ": workspace too small");
    const int nb = grad_blocks(n);
    float* partial = static_cast<float*>(workspace);
    const int words = xsg_camera_pack_words(type);
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        launch(time_bwd_kernel<Cam>, nb, kGradThreads, 0, as_cuda(stream), pack, W, H, uv, n, delta, grad, d_uv,
               partial);
    });
    if (rc != XSG_OK) return rc;
    launch(sum_partials_kernel, 1, 1024, 0, as_cuda(stream), static_cast<const float*>(partial), nb, words, d_pack);
    return check_launch(what);
}

int xsg_pixel_time_bwd(int type, const float* pack, int W, int H, int delta, const float* grad, float* d_pack,
                       void* workspace, size_t workspace_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(pack && grad && d_pack && W > 0 && H > 0, "pixel_time_bwd: bad arguments");
    return time_bwd("pixel_time_bwd", type, pack, W, H, nullptr, int64_t(W) * H, delta, grad, d_pack, nullptr,
                    workspace, workspace_bytes, stream);
}

int xsg_pixel_time_from_uv_bwd(int type, const float* pack, const float* uv, int64_t n, int delta,
                               const float* grad, float* d_pack, float* d_uv, void* workspace,
                               size_t workspace_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(pack && d_pack && n >= 0 && (n == 0 || (uv && grad)), "pixel_time_from_uv_bwd: bad arguments");
    XSG_REQUIRE(reinterpret_cast<uintptr_t>(uv) % 8 == 0 && reinterpret_cast<uintptr_t>(d_uv) % 8 == 0,
                "pixel_time_from_uv_bwd: uv and d_uv must be 8-byte aligned");
    return time_bwd("pixel_time_from_uv_bwd", type, pack, 1, 1, uv, n, delta, grad, d_pack, d_uv, workspace,
                    workspace_bytes, stream);
}

}  // extern "C"
