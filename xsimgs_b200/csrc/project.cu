// Camera rays, pixel times, point projection and the unscented-transform
// Gaussian projection (plain and phase-modelled) for sm_100a.
//
// One thread per pixel / point / Gaussian; all inputs are read once with
// coalesced loads and every output element is written (no pre-zeroing pass).
#include "cameras.cuh"
#include "ut_device.cuh"

namespace xsg {

constexpr int kThreads = 256;

// ------------------------------------------------------------------ rays --
// ray_kernels.h:8-59 / camera.h:125-131
template <typename Cam>
__global__ void __launch_bounds__(kThreads) rays_kernel(const float* __restrict__ pack, int W, int H,
                                                        int world, int normalized, float* ray_o,
                                                        float* __restrict__ ray_d, uint8_t* valid) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(W) * H) return;
    Cam k;
    k.load(pack);
    const int px = int(idx % W), py = int(idx / W);
    const float2 uv = k.pixel_to_uv(px, py, W, H);
    v3 r = k.ray_cs(uv);
    if (normalized) r = r * rsqrtf(dot3(r, r));
    v3 o = mk3(0.f, 0.f, 0.f), d = r;
    if (world) {
        const float dt = k.pixel_time(uv.x, uv.y) - k.pose;
        // toast q0.std(): unit length, non-negative real part
        float n = rsqrtf(k.qw * k.qw + k.qx * k.qx + k.qy * k.qy + k.qz * k.qz);
        if (k.qw < 0.0f) n = -n;
        float rw;
        v3 rv;
        pose_rotation(k, k.qw * n, mk3(k.qx * n, k.qy * n, k.qz * n), dt, rw, rv);
        o = k.t0 + k.v * dt;
        d = quat_rotate(rw, rv, r);
    }
    if (ray_o) st3(ray_o + 3 * idx, o);
    st3(ray_d + 3 * idx, d);
    if (valid) valid[idx] = k.ray_valid(uv) ? 1 : 0;
}

// time_kernels.h:5-112
template <typename Cam>
__global__ void pixel_time_kernel(const float* __restrict__ pack, int W, int H, const float* uv_in,
                                  int64_t n, int delta, float* __restrict__ out) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    Cam k;
    k.load(pack);
    float2 uv;
    if (uv_in) uv = make_float2(uv_in[2 * idx], uv_in[2 * idx + 1]);
    else uv = k.pixel_to_uv(int(idx % W), int(idx / W), W, H);
    const float t = k.pixel_time(uv.x, uv.y);
    out[idx] = delta ? t - k.pose : t;
}

// undistort_map, distortion.h:33-56 (the reference maps to [-1, 1] when
// normalized_range is false)
__global__ void undistort_map_kernel(const float* __restrict__ pack, int W, int H, int normalized_range,
                                     float2* __restrict__ out) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(W) * H) return;
    Distorted k;
    k.load(pack);
    const float2 r = k.distort_uv(k.pixel_to_uv(int(idx % W), int(idx / W), W, H));
    out[idx] = normalized_range ? r : make_float2(r.x * 2.0f - 1.0f, r.y * 2.0f - 1.0f);
}

// camera_projection_fwd, projection_kernels.h:259-309
template <typename Cam, bool kJac>
__global__ void projection_kernel(const float* __restrict__ pack, const float* __restrict__ pts,
                                  const float* __restrict__ vel, int64_t n, float thr, float max_res,
                                  float margin, int mode, float4* __restrict__ uvdt,
                                  uint8_t* __restrict__ mask) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    Cam k;
    k.load(pack);
    const v3 P = ld3(pts + 3 * i);
    const v3 V = vel ? ld3(vel + 3 * i) : mk3(0.f, 0.f, 0.f);
    bool m = true;
    float4 u;
    project_point<Cam, kJac>(k, P, V, thr, max_res, margin, mode, u, m);
    u.w += k.pose;
    uvdt[i] = u;
    m = m && (u.x >= 0.0f && u.y >= 0.0f) && (u.x <= 1.0f && u.y <= 1.0f);
    mask[i] = m ? 1 : 0;
}

// unscented_transform_kernel (ut_kernels.h:192-246) and, with kPhm,
// unscented_transform_phm_kernel (ut_phm_kernels.h:13-114).
template <typename Cam, bool kPhm>
__global__ void __launch_bounds__(kThreads)
    utgs_kernel(const float* __restrict__ pack, UTParams p, const float* __restrict__ pts,
                const float* __restrict__ vel, const float* __restrict__ scales,
                const float4* __restrict__ quats, const float* __restrict__ opacity, int64_t n,
                uint8_t* __restrict__ flags, float2* __restrict__ radii, float2* __restrict__ means2d,
                float* __restrict__ depths) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint8_t fl = 0;
    float2 r_out = make_float2(0.f, 0.f), m_out = make_float2(0.f, 0.f);
    float d_out = 0.f;
    const float o = opacity ? opacity[i] : 1.0f;
    if (!(o < 1.0f / 255.0f)) {
        Cam k;
        k.load(pack);
        const v3 P = ld3(pts + 3 * i);
        const v3 V = vel ? ld3(vel + 3 * i) : mk3(0.f, 0.f, 0.f);
        v3 d[3];
        ut_deltas(p.sq, quats[i], ld3(scales + 3 * i), d);
        float2 m, r;
        float dep, ud;
        if constexpr (!kPhm) {
            if (ut_project(k, p, MODE_CENTRAL, P, V, o, d, m, r, dep, ud)) {
                fl = 1; r_out = r; m_out = m; d_out = dep;
            }
        } else {
            bool res = ut_project(k, p, MODE_CENTRAL, P, V, o, d, m, r, dep, ud);
            if (res) {
                const float u_pi = float(M_PI) * p.img_w / fabsf(k.phi_range);
                const int rc = int(res) * (int(ud > u_pi) + 1);
                float2 ml, rl, mr, rr;
                float dl, dr;
                res = ut_project(k, p, MODE_NEG, P, V, o, d, ml, rl, dl, ud);
                const int rL = int(res) * (int(ud > u_pi) + 1);
                res = ut_project(k, p, MODE_POS, P, V, o, d, mr, rr, dr, ud);
                const int rR = int(res) * (int(ud > u_pi) + 1);
                if (rL == 1 && rR == 1) {
                    fl = 2; r_out = rl; m_out = ml; d_out = dl;
                } else if (rc == 1) {
                    fl = 1; r_out = r; m_out = m; d_out = dep;
                } else if (!(rL != 1 && rR != 1)) {
                    const bool use_left = rL != 1;
                    fl = 1;
                    r_out = use_left ? rl : rr;
                    m_out = use_left ? ml : mr;
                    d_out = use_left ? dl : dr;
                }
            }
        }
    }
    flags[i] = fl;
    radii[i] = r_out;
    means2d[i] = m_out;
    depths[i] = d_out;
}

// mask_radii.cu:10-58
__global__ void mask_radii_kernel(const uint8_t* __restrict__ mask, const uint32_t* __restrict__ packed,
                                  int64_t n, float2* __restrict__ radii) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const bool keep = mask ? (mask[i] != 0) : (((packed[i >> 5] >> (i & 31)) & 1u) != 0);
    if (!keep) radii[i] = make_float2(0.f, 0.f);
}

}  // namespace xsg

using namespace xsg;

extern "C" {

int xsg_camera_pack_words(int type) {
    switch (type) {
        case XSG_CAM_PINHOLE: return Pinhole::kWords;
        case XSG_CAM_FISHEYE: return Fisheye::kWords;
        case XSG_CAM_SPHERICAL: return Spherical<false>::kWords;
        case XSG_CAM_LIDAR: return Spherical<true>::kWords;
        case XSG_CAM_DISTORTED: return Distorted::kWords;
        default: return -1;
    }
}

int xsg_camera_intrinsics_word(int type) {
    switch (type) {
        case XSG_CAM_FISHEYE:
        case XSG_CAM_DISTORTED: return 20;
        case XSG_CAM_PINHOLE:
        case XSG_CAM_SPHERICAL:
        case XSG_CAM_LIDAR: return 18;
        default: return -1;
    }
}

int xsg_camera_rays(int type, const float* pack, int W, int H, int world, int normalized,
                    float* ray_o, float* ray_d, uint8_t* valid, xsg_stream_t stream) {
    XSG_REQUIRE(pack && ray_d && W > 0 && H > 0, "camera_rays: bad arguments");
    const int64_t n = int64_t(W) * H;
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        launch(rays_kernel<Cam>, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
            pack, W, H, world, normalized, ray_o, ray_d, valid);
    });
    if (rc != XSG_OK) return rc;
    return check_launch("camera_rays");
}

int xsg_pixel_time(int type, const float* pack, int W, int H, int delta, float* out,
                   xsg_stream_t stream) {
    XSG_REQUIRE(pack && out && W > 0 && H > 0, "pixel_time: bad arguments");
    const int64_t n = int64_t(W) * H;
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        launch(pixel_time_kernel<Cam>, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
            pack, W, H, nullptr, n, delta, out);
    });
    if (rc != XSG_OK) return rc;
    return check_launch("pixel_time");
}

int xsg_pixel_time_from_uv(int type, const float* pack, const float* uv, int64_t n, int delta,
                           float* out, xsg_stream_t stream) {
    XSG_REQUIRE(pack && n >= 0 && (n == 0 || (uv && out)), "pixel_time_from_uv: bad arguments");
    if (n == 0) return XSG_OK;
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        launch(pixel_time_kernel<Cam>, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
            pack, 1, 1, uv, n, delta, out);
    });
    if (rc != XSG_OK) return rc;
    return check_launch("pixel_time_from_uv");
}

int xsg_undistort_map(int type, const float* pack, int W, int H, int normalized_range, float* out,
                      xsg_stream_t stream) {
    XSG_REQUIRE(pack && out && W > 0 && H > 0, "undistort_map: bad arguments");
    if (type != XSG_CAM_DISTORTED) return set_error(XSG_ERR_UNSUPPORTED, "undistort_map: camera has no distortion");
    const int64_t n = int64_t(W) * H;
    launch(undistort_map_kernel, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), pack, W, H,
           normalized_range, reinterpret_cast<float2*>(out));
    return check_launch("undistort_map");
}

int xsg_projection(int type, const float* pack, const float* pts, const float* vel, int64_t n,
                   float thr, float max_res, float margin, int mode, int force_nojac, float* uvdt,
                   uint8_t* mask, xsg_stream_t stream) {
    XSG_REQUIRE(pack && n >= 0 && (n == 0 || (pts && uvdt && mask)), "projection: bad arguments");
    XSG_REQUIRE(mode >= 0 && mode <= 2, "projection: bad projection mode");
    if (n == 0) return XSG_OK;
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        if (force_nojac)
            launch(projection_kernel<Cam, false>, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
                pack, pts, vel, n, thr, max_res, margin, mode, reinterpret_cast<float4*>(uvdt), mask);
        else
            launch(projection_kernel<Cam, true>, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
                pack, pts, vel, n, thr, max_res, margin, mode, reinterpret_cast<float4*>(uvdt), mask);
    });
    if (rc != XSG_OK) return rc;
    return check_launch("projection");
}

int xsg_projection_utgs(int type, const float* pack, const float* pts, const float* vel,
                        const float* scales, const float* quats, const float* opacity, int64_t n,
                        float W, float H, float ua, float ub, float uk, float thr, float max_res,
                        float margin, int phm, uint8_t* flags, float* radii, float* means2d,
                        float* depths, xsg_stream_t stream) {
    XSG_REQUIRE(pack && n >= 0 && (n == 0 || (pts && scales && quats && flags && radii && means2d && depths)),
                "projection_utgs: bad arguments");
    XSG_REQUIRE(reinterpret_cast<uintptr_t>(quats) % 16 == 0, "projection_utgs: quats must be 16-byte aligned");
    if (n == 0) return XSG_OK;
    if (phm && type != XSG_CAM_SPHERICAL && type != XSG_CAM_LIDAR)
        return set_error(XSG_ERR_UNSUPPORTED, "projection_utgs_phm: only spherical and lidar cameras");
    const UTParams p = ut_params(ua, ub, uk, thr, max_res, margin, W, H);
    ScopedTimer tm(phm ? "projection_utgs_phm" : "projection_utgs", as_cuda(stream));
    int rc = dispatch_camera(type, [&](auto cam) {
        using Cam = decltype(cam);
        auto* f4q = reinterpret_cast<const float4*>(quats);
        auto* r2 = reinterpret_cast<float2*>(radii);
        auto* m2 = reinterpret_cast<float2*>(means2d);
        if constexpr (Cam::kType == XSG_CAM_SPHERICAL || Cam::kType == XSG_CAM_LIDAR) {
            if (phm) {
                launch(utgs_kernel<Cam, true>, blocks_for(n, kThreads / 2), kThreads / 2, 0, as_cuda(stream), 
                    pack, p, pts, vel, scales, f4q, opacity, n, flags, r2, m2, depths);
                return;
            }
        }
        launch(utgs_kernel<Cam, false>, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
            pack, p, pts, vel, scales, f4q, opacity, n, flags, r2, m2, depths);
    });
    if (rc != XSG_OK) return rc;
    return check_launch("projection_utgs");
}

int xsg_mask_radii(const uint8_t* mask, const uint32_t* packed, int64_t n, float* radii,
                   xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0, "mask_radii: bad arguments");
    if (n == 0) return XSG_OK;
    XSG_REQUIRE((mask == nullptr) != (packed == nullptr), "mask_radii: pass exactly one mask");
    XSG_REQUIRE(radii, "mask_radii: bad arguments");
    launch(mask_radii_kernel, blocks_for(n, kThreads), kThreads, 0, as_cuda(stream), 
        mask, packed, n, reinterpret_cast<float2*>(radii));
    return check_launch("mask_radii");
}

}  // extern "C"
