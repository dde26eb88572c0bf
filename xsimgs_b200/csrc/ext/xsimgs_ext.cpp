// xsimgs_b200._C — the PyTorch extension with the reference's `xsimgs._C`
// operator surface (csrc/ext.cpp:12-20 and the bind_* functions it calls):
// the same function and class names, keyword arguments, defaults, tensor
// layouts and error wording.  Each op checks its tensors, allocates outputs
// and scratch with the caching allocator and calls the C ABI of
// libxsimgs_b200.so (include/xsimgs_b200.h) on the current CUDA stream.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <optional>
#include <string>
#include <vector>

#include "xsimgs_b200.h"

namespace py = pybind11;
using at::Tensor;
using OptT = std::optional<Tensor>;

namespace {

void check(int rc) {
    if (rc != XSG_OK) throw std::runtime_error(xsg_last_error());
}

xsg_stream_t stream() { return reinterpret_cast<xsg_stream_t>(c10::cuda::getCurrentCUDAStream().stream()); }

void require_cuda(const Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

void require_contig(const Tensor& t, const char* name) {
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void require_f32(const Tensor& t, const char* name) {
    TORCH_CHECK(t.scalar_type() == at::kFloat, name, " must be float32");
}

void check_tensor(const Tensor& t, const char* name, const Tensor& ref) {
    require_cuda(t, name);
    require_contig(t, name);
    TORCH_CHECK(t.device() == ref.device(), name, " must be on the same device as the other inputs");
}

const float* fptr(const Tensor& t) { return t.data_ptr<float>(); }
const float* fptr(const OptT& t) { return t.has_value() && t->defined() ? t->data_ptr<float>() : nullptr; }
float* fptr_mut(const Tensor& t) { return t.data_ptr<float>(); }

Tensor workspace(size_t bytes, const Tensor& like) {
    return at::empty({static_cast<int64_t>(bytes > 0 ? bytes : 1)}, like.options().dtype(at::kByte));
}

bool has(const OptT& t) { return t.has_value() && t->defined(); }

py::object opt(const Tensor& t) { return t.defined() ? py::cast(t) : py::none(); }

// -------------------------------------------------------------- cameras --
enum class ProjectionMode : int { Central = 0, NegativeDelta = 1, PositiveDelta = 2 };

constexpr float kResidualEarlyStop = 1e-4f;  // include/cameras/bind.h:17-20
constexpr float kResidualMax = 0.002f;
constexpr float kMaxMargin = 1.0f;

struct CameraSpec {
    int type;
    const char* name;
    std::vector<int> impl_dims;  // last dims of the intrinsics tensors
};

const std::vector<int> kBaseDims = {4, 3, 3, 3, 2, 1, 1};  // camera.h:144

// Camera tensors -> one [1, P] float pack (layout in xsimgs_b200.h); built
// from differentiable ATen ops, so gradients reach the camera tensors.
Tensor camera_pack(const CameraSpec& spec, const std::vector<Tensor>& tensors) {
    const size_t total = kBaseDims.size() + spec.impl_dims.size();
    if (tensors.size() != total)
        throw std::runtime_error("Tensor list size mismatch. Expected " + std::to_string(total) +
                                 ", but found: " + std::to_string(tensors.size()));
    std::vector<Tensor> parts;
    for (size_t i = 0; i < tensors.size(); ++i) {
        const Tensor& t = tensors[i];
        TORCH_CHECK(t.scalar_type() == at::kFloat, "Camera tensors must be float32");
        const int want = i < kBaseDims.size() ? kBaseDims[i] : spec.impl_dims[i - kBaseDims.size()];
        TORCH_CHECK(t.dim() >= 1 && t.size(-1) == want, "Camera tensor ", i, " must have last dimension ", want);
        TORCH_CHECK(t.numel() == want, "Only single camera is currently supported");
        TORCH_CHECK(t.device() == tensors[0].device(), "Camera tensors must be on the same device");
        parts.push_back(t.reshape({want}));
        if (i == 3) parts.push_back(at::zeros({1}, t.options()));  // padding word 13
        // the intrinsics start where the reference's Camera<Impl> struct puts
        // them: word 20 for impls holding a float4 (16-byte aligned)
        if (i + 1 == kBaseDims.size() && xsg_camera_intrinsics_word(spec.type) > 18)
            parts.push_back(at::zeros({xsg_camera_intrinsics_word(spec.type) - 18}, t.options()));
    }
    Tensor pack = at::cat(parts);
    const int64_t words = xsg_camera_pack_words(spec.type);
    if (pack.numel() < words) pack = at::cat({pack, at::zeros({words - pack.numel()}, pack.options())});
    return pack.view({1, -1});
}

void validate_pack(const CameraSpec& spec, const Tensor& pack) {
    TORCH_CHECK(pack.numel() == xsg_camera_pack_words(spec.type), "Only single camera is currently supported");
    TORCH_CHECK(pack.scalar_type() == at::kFloat, "Camera type must be float32");
    TORCH_CHECK(pack.is_contiguous(), "Camera pack must be contiguous tensor");
    require_cuda(pack, "camera pack");
}

using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

Tensor grad_workspace(const Tensor& like) { return workspace(xsg_camera_grad_workspace_size(), like); }

// camera_rays with the camera-parameter gradient (CameraRaysFunction,
// include/cameras/ray_kernels.h:158-223): backward returns d_pack only.
struct CameraRaysFn : public torch::autograd::Function<CameraRaysFn> {
    static variable_list forward(AutogradContext* ctx, const Tensor& pack, int64_t type, int64_t width,
                                 int64_t height, bool world_space, bool normalized, bool return_origins,
                                 bool return_valid) {
        c10::cuda::CUDAGuard g(pack.device());
        auto opt = pack.options();
        // Outputs not asked for are empty tensors (autograd outputs must be
        // defined); camera_rays() hands them to Python as None / drops them.
        Tensor ray_o = at::empty(return_origins ? at::IntArrayRef{height, width, 3} : at::IntArrayRef{0}, opt);
        Tensor ray_d = at::empty({height, width, 3}, opt);
        Tensor valid = at::empty(return_valid ? at::IntArrayRef{height, width} : at::IntArrayRef{0},
                                 opt.dtype(at::kBool));
        check(xsg_camera_rays(int(type), fptr(pack), int(width), int(height), world_space, normalized,
                              return_origins ? fptr_mut(ray_o) : nullptr, fptr_mut(ray_d),
                              return_valid ? reinterpret_cast<uint8_t*>(valid.data_ptr()) : nullptr, stream()));
        ctx->save_for_backward({pack});
        ctx->saved_data["type"] = type;
        ctx->saved_data["width"] = width;
        ctx->saved_data["height"] = height;
        ctx->saved_data["world_space"] = world_space;
        ctx->saved_data["normalized"] = normalized;
        ctx->set_materialize_grads(false);
        ctx->mark_non_differentiable({valid});
        return {ray_o, ray_d, valid};
    }
    static variable_list backward(AutogradContext* ctx, variable_list grads) {
        const Tensor pack = ctx->get_saved_variables()[0];
        c10::cuda::CUDAGuard g(pack.device());
        const int64_t W = ctx->saved_data["width"].toInt(), H = ctx->saved_data["height"].toInt();
        Tensor d_pack = at::empty(pack.sizes(), pack.options());
        Tensor go = (grads[0].defined() && grads[0].numel() == H * W * 3) ? grads[0].contiguous() : Tensor();
        Tensor gd = grads[1].defined() ? grads[1].contiguous() : at::zeros({H, W, 3}, pack.options());
        Tensor ws = grad_workspace(pack);
        check(xsg_camera_rays_bwd(int(ctx->saved_data["type"].toInt()), fptr(pack), int(W), int(H),
                                  ctx->saved_data["world_space"].toBool(), ctx->saved_data["normalized"].toBool(),
                                  go.defined() ? fptr(go) : nullptr, fptr(gd), fptr_mut(d_pack), ws.data_ptr(),
                                  size_t(ws.nbytes()), stream()));
        return {d_pack, Tensor(), Tensor(), Tensor(), Tensor(), Tensor(), Tensor(), Tensor()};
    }
};

py::object camera_rays(const CameraSpec& spec, const Tensor& pack, int64_t width, int64_t height,
                       bool world_space, bool normalized, bool return_origins, bool return_valid) {
    validate_pack(spec, pack);
    TORCH_CHECK(width > 0 && height > 0, "camera_rays: width and height must be positive");
    variable_list out = CameraRaysFn::apply(pack, int64_t(spec.type), width, height, world_space, normalized,
                                            return_origins, return_valid);
    py::list res;
    res.append(return_origins ? py::cast(out[0]) : py::none());
    res.append(py::cast(out[1]));
    if (return_valid) res.append(py::cast(out[2]));
    return std::move(res);
}

// pixel_time / pixel_time_delta with their backward (CameraPixelTimeFunction
// and CameraPixelTimeDeltaFunction, include/cameras/time_kernels.h:364-460).
struct PixelTimeFn : public torch::autograd::Function<PixelTimeFn> {
    static Tensor forward(AutogradContext* ctx, const Tensor& pack, int64_t type, int64_t width, int64_t height,
                          bool delta) {
        c10::cuda::CUDAGuard g(pack.device());
        Tensor out = at::empty({height, width}, pack.options());
        check(xsg_pixel_time(int(type), fptr(pack), int(width), int(height), delta, fptr_mut(out), stream()));
        ctx->save_for_backward({pack});
        ctx->saved_data["type"] = type;
        ctx->saved_data["delta"] = delta;
        return out;
    }
    static variable_list backward(AutogradContext* ctx, variable_list grads) {
        const Tensor pack = ctx->get_saved_variables()[0];
        c10::cuda::CUDAGuard g(pack.device());
        Tensor grad = grads[0].contiguous();
        Tensor d_pack = at::empty(pack.sizes(), pack.options());
        Tensor ws = grad_workspace(pack);
        check(xsg_pixel_time_bwd(int(ctx->saved_data["type"].toInt()), fptr(pack), int(grad.size(1)),
                                 int(grad.size(0)), ctx->saved_data["delta"].toBool(), fptr(grad), fptr_mut(d_pack),
                                 ws.data_ptr(), size_t(ws.nbytes()), stream()));
        return {d_pack, Tensor(), Tensor(), Tensor(), Tensor()};
    }
};

// The uv variants (CameraPixelTimeFromUVFunction and
// CameraPixelTimeDeltaFromUVFunction, time_kernels.h:398-492): gradients for
// the pack and for uv.
struct PixelTimeFromUVFn : public torch::autograd::Function<PixelTimeFromUVFn> {
    static Tensor forward(AutogradContext* ctx, const Tensor& pack, const Tensor& uv, int64_t type, bool delta) {
        c10::cuda::CUDAGuard g(pack.device());
        Tensor u = uv.contiguous();
        auto sizes = u.sizes().vec();
        sizes.pop_back();
        Tensor out = at::empty(sizes, u.options());
        check(xsg_pixel_time_from_uv(int(type), fptr(pack), fptr(u), u.numel() / 2, delta, fptr_mut(out), stream()));
        ctx->save_for_backward({pack, u});
        ctx->saved_data["type"] = type;
        ctx->saved_data["delta"] = delta;
        return out;
    }
    static variable_list backward(AutogradContext* ctx, variable_list grads) {
        const auto saved = ctx->get_saved_variables();
        const Tensor pack = saved[0], u = saved[1];
        c10::cuda::CUDAGuard g(pack.device());
        Tensor grad = grads[0].contiguous();
        Tensor d_pack = at::empty(pack.sizes(), pack.options());
        Tensor d_uv = ctx->needs_input_grad(1) ? at::empty_like(u) : Tensor();
        Tensor ws = grad_workspace(pack);
        check(xsg_pixel_time_from_uv_bwd(int(ctx->saved_data["type"].toInt()), fptr(pack), fptr(u), u.numel() / 2,
                                         ctx->saved_data["delta"].toBool(), fptr(grad), fptr_mut(d_pack),
                                         d_uv.defined() ? fptr_mut(d_uv) : nullptr, ws.data_ptr(),
                                         size_t(ws.nbytes()), stream()));
        return {d_pack, d_uv, Tensor(), Tensor()};
    }
};

Tensor pixel_time(const CameraSpec& spec, const Tensor& pack, int64_t width, int64_t height, bool delta) {
    validate_pack(spec, pack);
    TORCH_CHECK(width > 0 && height > 0, "pixel_time: width and height must be positive");
    return PixelTimeFn::apply(pack, int64_t(spec.type), width, height, delta);
}

Tensor pixel_time_from_uv(const CameraSpec& spec, const Tensor& pack, const Tensor& uv, bool delta) {
    validate_pack(spec, pack);
    TORCH_CHECK(uv.size(-1) == 2, "UV coordinates last dimension must be 2");
    TORCH_CHECK(uv.device() == pack.device(), "Camera and UV-s must be on the same device");
    TORCH_CHECK(uv.scalar_type() == at::kFloat, "UV coordinates must be float32 tensor");
    return PixelTimeFromUVFn::apply(pack, uv, int64_t(spec.type), delta);
}

std::tuple<Tensor, Tensor> projection(const CameraSpec& spec, bool nojac, const Tensor& pack, const Tensor& points,
                                      const OptT& vel, float thr, float max_res, float margin, ProjectionMode mode) {
    validate_pack(spec, pack);
    check_tensor(points, "points", pack);
    if (has(vel)) check_tensor(*vel, "points_velocity", pack);
    c10::cuda::CUDAGuard g(pack.device());
    const int64_t n = points.size(0);
    Tensor uvdt = at::empty({n, 4}, pack.options());
    Tensor mask = at::empty({n}, pack.options().dtype(at::kBool));
    check(xsg_projection(spec.type, fptr(pack), fptr(points), fptr(vel), n, thr, max_res, margin, int(mode), nojac,
                         fptr_mut(uvdt), reinterpret_cast<uint8_t*>(mask.data_ptr()), stream()));
    return {uvdt, mask};
}

std::tuple<Tensor, Tensor, Tensor, Tensor> projection_utgs(const CameraSpec& spec, bool phm, const Tensor& pack,
                                                           const Tensor& points, const OptT& vel,
                                                           const Tensor& scales, const Tensor& quats,
                                                           const OptT& opacity, float width, float height, float ua,
                                                           float ub, float uk, float thr, float max_res,
                                                           float margin) {
    validate_pack(spec, pack);
    check_tensor(points, "points", pack);
    check_tensor(scales, "scales", pack);
    check_tensor(quats, "quats", pack);
    if (has(vel)) check_tensor(*vel, "points_velocity", pack);
    if (has(opacity)) check_tensor(*opacity, "opacity", pack);
    c10::cuda::CUDAGuard g(pack.device());
    const int64_t n = points.size(0);
    auto opt = points.options();
    Tensor flags = at::empty({n}, opt.dtype(at::kByte));
    Tensor radii = at::empty({n, 2}, opt);
    Tensor means2d = at::empty({n, 2}, opt);
    Tensor depths = at::empty({n}, opt);
    check(xsg_projection_utgs(spec.type, fptr(pack), fptr(points), fptr(vel), fptr(scales), fptr(quats),
                              fptr(opacity), n, width, height, ua, ub, uk, thr, max_res, margin, phm,
                              flags.data_ptr<uint8_t>(), fptr_mut(radii), fptr_mut(means2d), fptr_mut(depths),
                              stream()));
    return {flags, radii, means2d, depths};
}

template <typename Cls>
py::class_<Cls> bind_camera(py::module& m, const char* name, CameraSpec spec, bool with_phm) {
    auto cls = py::class_<Cls>(m, name);
    cls.def_static("pack", [spec](const std::vector<Tensor>& tensors) { return camera_pack(spec, tensors); },
                   py::arg("tensors"));
    cls.def_static("camera_rays",
                   [spec](const Tensor& pack, int64_t width, int64_t height, bool world_space, bool normalized,
                          bool return_origins, bool return_valid) {
                       return camera_rays(spec, pack, width, height, world_space, normalized, return_origins,
                                          return_valid);
                   },
                   py::arg("pack"), py::arg("width"), py::arg("height"), py::arg("world_space") = true,
                   py::arg("normalized") = true, py::arg("return_origins") = true, py::arg("return_valid") = false);
    cls.def_static("pixel_time",
                   [spec](const Tensor& pack, int64_t w, int64_t h) { return pixel_time(spec, pack, w, h, false); },
                   py::arg("pack"), py::arg("width"), py::arg("height"));
    cls.def_static("pixel_time_delta",
                   [spec](const Tensor& pack, int64_t w, int64_t h) { return pixel_time(spec, pack, w, h, true); },
                   py::arg("pack"), py::arg("width"), py::arg("height"));
    cls.def_static("pixel_time_from_uv",
                   [spec](const Tensor& pack, const Tensor& uv) { return pixel_time_from_uv(spec, pack, uv, false); },
                   py::arg("pack"), py::arg("uvs"));
    cls.def_static("pixel_time_delta_from_uv",
                   [spec](const Tensor& pack, const Tensor& uv) { return pixel_time_from_uv(spec, pack, uv, true); },
                   py::arg("pack"), py::arg("uvs"));
    for (int nojac = 0; nojac < 2; ++nojac) {
        cls.def_static(nojac ? "projection_nojac" : "projection",
                       [spec, nojac](const Tensor& pack, const Tensor& points, const OptT& vel, float thr,
                                     float max_res, float margin, ProjectionMode mode) {
                           return projection(spec, nojac != 0, pack, points, vel, thr, max_res, margin, mode);
                       },
                       py::arg("pack"), py::arg("points"), py::arg("points_velocity") = py::none(),
                       py::arg("residual_thr_early_stop") = kResidualEarlyStop,
                       py::arg("max_residual") = kResidualMax, py::arg("max_margin") = kMaxMargin,
                       py::arg("projection_mode") = ProjectionMode::Central);
    }
    for (int phm = 0; phm < (with_phm ? 2 : 1); ++phm) {
        cls.def_static(phm ? "projection_utgs_phm" : "projection_utgs",
                       [spec, phm](const Tensor& pack, const Tensor& points, const OptT& vel, const Tensor& scales,
                                   const Tensor& quats, const OptT& opacity, float width, float height, float ua,
                                   float ub, float uk, float thr, float max_res, float margin) {
                           return projection_utgs(spec, phm != 0, pack, points, vel, scales, quats, opacity, width,
                                                  height, ua, ub, uk, thr, max_res, margin);
                       },
                       py::arg("pack"), py::arg("points"), py::arg("points_velocity"), py::arg("scales"),
                       py::arg("quats"), py::arg("opacity"), py::arg("width"), py::arg("height"),
                       py::arg("ut_alpha") = 0.1f, py::arg("ut_beta") = 2.0f, py::arg("ut_kappa") = 0.0f,
                       py::arg("residual_thr_early_stop") = kResidualEarlyStop,
                       py::arg("max_residual") = kResidualMax, py::arg("max_margin") = kMaxMargin);
    }
    return cls;
}

struct PerspectiveCamera {};
struct OpenCVFisheyeCamera {};
struct SphericalCamera {};
struct LidarCamera {};
struct DistortedPerspectiveCamera {};

Tensor undistort_map(const CameraSpec& spec, const Tensor& pack, int64_t width, int64_t height,
                     bool normalized_range) {
    validate_pack(spec, pack);
    TORCH_CHECK(width > 0 && height > 0, "undistort_map: width and height must be positive");
    c10::cuda::CUDAGuard g(pack.device());
    Tensor out = at::empty({height, width, 2}, pack.options());
    check(xsg_undistort_map(spec.type, fptr(pack), int(width), int(height), normalized_range, fptr_mut(out),
                            stream()));
    return out;
}

// --------------------------------------------------------------- tiling --
std::tuple<Tensor, Tensor, Tensor> isect_regular_tiles(const Tensor& means2d, const Tensor& radii,
                                                       const Tensor& depths, int64_t img_width, int64_t img_height,
                                                       int64_t tile_size_x, int64_t tile_size_y, bool sort,
                                                       bool /*double_buffer*/) {
    check_tensor(means2d, "means2d", means2d);
    check_tensor(radii, "radii", means2d);
    check_tensor(depths, "depth", means2d);
    c10::cuda::CUDAGuard g(means2d.device());
    const int64_t n = means2d.numel() / 2;
    auto opt = depths.options();
    Tensor tiles_per_gauss = at::empty_like(depths, opt.dtype(at::kInt));
    Tensor ws = workspace(xsg_isect_workspace_size(n, 0), means2d);
    int64_t n_isects = 0;
    check(xsg_isect_regular_count(fptr(means2d), fptr(radii), n, int(img_width), int(img_height), int(tile_size_x),
                                  int(tile_size_y), tiles_per_gauss.data_ptr<int32_t>(), &n_isects,
                                  ws.data_ptr(), size_t(ws.numel()), stream()));
    Tensor isect_ids = at::empty({n_isects}, opt.dtype(at::kLong));
    Tensor flatten_ids = at::empty({n_isects}, opt.dtype(at::kInt));
    if (n_isects == 0) return {tiles_per_gauss, isect_ids, flatten_ids};
    const size_t need = xsg_isect_workspace_size(n, sort ? n_isects : 0);
    if (size_t(ws.numel()) < need) ws = workspace(need, means2d);
    check(xsg_isect_regular_emit(fptr(means2d), fptr(radii), fptr(depths), n, int(img_width), int(img_height),
                                 int(tile_size_x), int(tile_size_y), sort, tiles_per_gauss.data_ptr<int32_t>(),
                                 n_isects, isect_ids.data_ptr<int64_t>(), flatten_ids.data_ptr<int32_t>(),
                                 ws.data_ptr(), size_t(ws.numel()), stream()));
    return {tiles_per_gauss, isect_ids, flatten_ids};
}

// Capacity-sized regular tiling with no host synchronisation: returns
// (tiles_per_gauss, isect_ids[capacity], flatten_ids[capacity],
// offsets[tiles_h, tiles_w], counts int64[2] = {total, written}).  Lists
// match isect_regular_tiles + isect_offset_encode when total <= capacity.
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> isect_regular_tiles_async(
    const Tensor& means2d, const Tensor& radii, const Tensor& depths, int64_t img_width, int64_t img_height,
    int64_t tile_size_x, int64_t tile_size_y, int64_t capacity, const OptT& workspace_in) {
    check_tensor(means2d, "means2d", means2d);
    check_tensor(radii, "radii", means2d);
    check_tensor(depths, "depth", means2d);
    TORCH_CHECK(capacity > 0, "isect_regular_tiles_async: capacity must be positive");
    c10::cuda::CUDAGuard g(means2d.device());
    const int64_t n = means2d.numel() / 2;
    auto opt = depths.options();
    const int64_t ntx = (img_width + tile_size_x - 1) / tile_size_x, nty = (img_height + tile_size_y - 1) / tile_size_y;
    Tensor tiles_per_gauss = at::empty_like(depths, opt.dtype(at::kInt));
    Tensor isect_ids = at::empty({capacity}, opt.dtype(at::kLong));
    Tensor flatten_ids = at::empty({capacity}, opt.dtype(at::kInt));
    Tensor offsets = at::empty({nty, ntx}, opt.dtype(at::kInt));
    Tensor counts = at::empty({2}, opt.dtype(at::kLong));
    const size_t need = xsg_isect_workspace_size(n, capacity);
    Tensor ws;
    if (has(workspace_in) && size_t(workspace_in->nbytes()) >= need) {
        check_tensor(*workspace_in, "workspace", means2d);
        ws = *workspace_in;
    } else {
        ws = workspace(need, means2d);
    }
    check(xsg_isect_regular_tiles_async(fptr(means2d), fptr(radii), fptr(depths), n, int(img_width), int(img_height),
                                        int(tile_size_x), int(tile_size_y), capacity,
                                        tiles_per_gauss.data_ptr<int32_t>(), isect_ids.data_ptr<int64_t>(),
                                        flatten_ids.data_ptr<int32_t>(), offsets.data_ptr<int32_t>(),
                                        counts.data_ptr<int64_t>(), ws.data_ptr(), size_t(ws.nbytes()), stream()));
    return {tiles_per_gauss, isect_ids, flatten_ids, offsets, counts};
}

std::tuple<Tensor, Tensor, Tensor> isect_range_tiles(bool lidar, const Tensor& pack, const Tensor& points,
                                                     const OptT& vel, const Tensor& scale, const Tensor& quat,
                                                     const OptT& opacity, const Tensor& flag, const Tensor& means2d,
                                                     const Tensor& radii, const Tensor& depths, const OptT& elev,
                                                     int64_t tsx, int64_t tsy, float W, float H, float ua, float ub,
                                                     float uk, bool sort) {
    TORCH_CHECK(pack.is_cuda(), "camera_pack must be CUDA tensor");
    for (auto* t : {&pack, &points, &scale, &quat, &flag, &means2d, &radii, &depths}) check_tensor(*t, "input", pack);
    if (has(vel)) check_tensor(*vel, "points_velocity", pack);
    if (has(opacity)) check_tensor(*opacity, "opacity", pack);
    if (lidar) check_tensor(*elev, "elev_boundaries", pack);
    TORCH_CHECK(pack.numel() == xsg_camera_pack_words(lidar ? XSG_CAM_LIDAR : XSG_CAM_SPHERICAL),
                "Only single camera is currently supported");
    c10::cuda::CUDAGuard g(pack.device());
    const int64_t n = means2d.numel() / 2;
    auto opt = depths.options();
    Tensor tiles_per_gauss = at::zeros_like(depths, opt.dtype(at::kInt));
    const float* eb = lidar ? fptr(*elev) : nullptr;
    const int n_elev = lidar ? int(elev->size(0)) : 0;
    Tensor ws = workspace(xsg_isect_workspace_size(n, 0), means2d);
    int64_t n_isects = 0;
    check(xsg_isect_spherical_count(lidar, fptr(pack), fptr(points), fptr(vel), fptr(scale), fptr(quat), fptr(opacity),
                                    flag.data_ptr<uint8_t>(), fptr(means2d), fptr(radii), fptr(depths), eb, n_elev, n,
                                    int(tsx), int(tsy), W, H, ua, ub, uk, tiles_per_gauss.data_ptr<int32_t>(),
                                    &n_isects, ws.data_ptr(), size_t(ws.numel()), stream()));
    Tensor isect_ids = at::empty({n_isects}, opt.dtype(at::kLong));
    Tensor flatten_ids = at::empty({n_isects}, opt.dtype(at::kInt));
    if (n_isects == 0) return {tiles_per_gauss, isect_ids, flatten_ids};
    const size_t need = xsg_isect_workspace_size(n, sort ? n_isects : 0);
    if (size_t(ws.numel()) < need) ws = workspace(need, means2d);
    check(xsg_isect_spherical_emit(lidar, fptr(pack), fptr(points), fptr(vel), fptr(scale), fptr(quat), fptr(opacity),
                                   flag.data_ptr<uint8_t>(), fptr(means2d), fptr(radii), fptr(depths), eb, n_elev, n,
                                   int(tsx), int(tsy), W, H, ua, ub, uk, sort, tiles_per_gauss.data_ptr<int32_t>(),
                                   n_isects, isect_ids.data_ptr<int64_t>(), flatten_ids.data_ptr<int32_t>(),
                                   ws.data_ptr(), size_t(ws.numel()), stream()));
    return {tiles_per_gauss, isect_ids, flatten_ids};
}

Tensor isect_offset_encode(const Tensor& isect_ids, int64_t tile_width, int64_t tile_height) {
    TORCH_CHECK(isect_ids.is_cuda() && isect_ids.is_contiguous(), "isect_ids must be contiguous cuda tensor");
    c10::cuda::CUDAGuard g(isect_ids.device());
    const int64_t n = isect_ids.size(0);
    Tensor offsets = at::empty({tile_height, tile_width}, isect_ids.options().dtype(at::kInt));
    check(xsg_isect_offset_encode(n ? isect_ids.data_ptr<int64_t>() : nullptr, n, int(tile_width), int(tile_height),
                                  offsets.data_ptr<int32_t>(), stream()));
    return offsets;
}

void mask_radii(const Tensor& mask, const Tensor& radii) {
    if (radii.size(-1) != 2) throw std::runtime_error("radii must be [..., 2] tensor");
    TORCH_CHECK(mask.scalar_type() == at::kBool, "Mask must be torch.bool tensor");
    const int64_t n = radii.numel() / 2;
    TORCH_CHECK(mask.numel() == n, "Mask size mismatch with radii");
    check_tensor(mask, "mask", radii);
    check_tensor(radii, "radii", radii);
    c10::cuda::CUDAGuard g(radii.device());
    check(xsg_mask_radii(reinterpret_cast<const uint8_t*>(mask.data_ptr()), nullptr, n, fptr_mut(radii), stream()));
}

void mask_radii_packed(const Tensor& packed_mask, const Tensor& radii) {
    if (radii.size(-1) != 2) throw std::runtime_error("radii must be [..., 2] tensor");
    TORCH_CHECK(packed_mask.element_size() == 4 && !packed_mask.is_floating_point(),
                "Packed mask must be UInt32 tensor");
    const int64_t n = radii.numel() / 2;
    TORCH_CHECK(packed_mask.numel() * 32 >= n, "Packed mask size mismatch with radii");
    check_tensor(packed_mask, "packed_mask", radii);
    check_tensor(radii, "radii", radii);
    c10::cuda::CUDAGuard g(radii.device());
    check(xsg_mask_radii(nullptr, reinterpret_cast<const uint32_t*>(packed_mask.data_ptr()), n, fptr_mut(radii),
                         stream()));
}

// ---------------------------------------------------------- rasteriser ---
// The device-side list length of a capacity-sized intersection list
// (isect_regular_tiles_async), or null: the list is then flatten_ids whole.
const int64_t* n_isects_ptr(const OptT& n_dev, const Tensor& like) {
    if (!has(n_dev)) return nullptr;
    check_tensor(*n_dev, "n_isects", like);
    TORCH_CHECK(n_dev->scalar_type() == at::kLong && n_dev->numel() >= 1, "n_isects must be an int64 device tensor");
    return n_dev->data_ptr<int64_t>();
}

std::vector<int64_t> eval3d_supported_ndims() {
    int buf[64];
    const int n = xsg_raster_supported_channels(buf, 64);
    return std::vector<int64_t>(buf, buf + n);
}

std::tuple<Tensor, Tensor, Tensor, Tensor> raster_fwd(const Tensor& means, const OptT& velocity, const Tensor& quats,
                                                      const Tensor& scales, const OptT& colors,
                                                      const Tensor& opacities, int64_t W, int64_t H, int64_t tsx,
                                                      int64_t tsy, const Tensor& ray_o, const Tensor& ray_d,
                                                      const OptT& ray_t, const Tensor& tile_offsets,
                                                      const Tensor& flatten_ids, const OptT& workspace_in,
                                                      const OptT& n_isects_dev) {
    for (auto* t : {&means, &quats, &scales, &opacities, &ray_o, &ray_d, &tile_offsets, &flatten_ids})
        check_tensor(*t, "rasterize input", means);
    if (has(colors)) check_tensor(*colors, "colors", means);
    if (has(velocity)) check_tensor(*velocity, "velocity", means);
    if (has(ray_t)) check_tensor(*ray_t, "ray_time_delta", means);
    c10::cuda::CUDAGuard g(means.device());
    const int64_t channels = has(colors) ? colors->size(-1) : 0;
    const int64_t n = means.numel() / 3;
    auto opt = means.options();
    Tensor renders = at::empty({H, W, channels}, opt);
    Tensor depths = at::empty({H, W}, opt);
    Tensor alphas = at::empty({H, W}, opt);
    Tensor last_ids = at::empty({H, W}, opt.dtype(at::kInt));
    const size_t ws_need = xsg_rasterize_workspace_size(n, int(channels), 0, 0, 0);
    Tensor ws;
    if (has(workspace_in)) {
        check_tensor(*workspace_in, "workspace", means);
        TORCH_CHECK(size_t(workspace_in->nbytes()) >= ws_need, "workspace too small: need ", ws_need, " bytes");
        ws = *workspace_in;
    } else {
        ws = workspace(ws_need, means);
    }
    check(xsg_rasterize_fwd(fptr(means), fptr(velocity), fptr(quats), fptr(scales), fptr(colors), int(channels),
                            fptr(opacities), n, int(W), int(H), int(tsx), int(tsy), fptr(ray_o), fptr(ray_d),
                            fptr(ray_t), tile_offsets.data_ptr<int32_t>(), int(tile_offsets.size(-1)),
                            int(tile_offsets.size(-2)), flatten_ids.data_ptr<int32_t>(), flatten_ids.numel(),
                            channels ? fptr_mut(renders) : nullptr, fptr_mut(depths), fptr_mut(alphas),
                            last_ids.data_ptr<int32_t>(), ws.data_ptr(), size_t(ws.nbytes()), stream(),
                            n_isects_ptr(n_isects_dev, means)));
    return {renders, depths, alphas, last_ids};
}

struct BwdOut {
    Tensor v_points, v_velocity, v_quat, v_scale, v_opacity;
    OptT v_colors;
    Tensor v_ray_o, v_ray_d, v_time;
};

BwdOut raster_bwd(const Tensor& points, const OptT& velocity, const Tensor& scale, const Tensor& quat,
                  const Tensor& opacity, const OptT& colors, const Tensor& ray_o, const Tensor& ray_d,
                  const OptT& ray_t, int64_t tsx, int64_t tsy, const Tensor& tile_offsets, const Tensor& flatten_ids,
                  const Tensor& render_alpha, const Tensor& last_ids, const OptT& v_colors_in, const Tensor& v_depth,
                  const Tensor& v_alpha, bool ray_grads, const OptT& fwd_ws, const OptT& n_isects_dev) {
    if (has(v_colors_in) && !v_colors_in->is_contiguous())
        throw std::runtime_error("v_render_colors must be contiguous");
    for (auto* t : {&points, &scale, &quat, &opacity, &ray_o, &ray_d, &tile_offsets, &flatten_ids, &render_alpha,
                    &last_ids, &v_depth, &v_alpha})
        check_tensor(*t, "rasterize_bwd input", points);
    if (has(colors)) check_tensor(*colors, "colors", points);
    if (has(velocity)) check_tensor(*velocity, "velocity", points);
    c10::cuda::CUDAGuard g(points.device());
    const int64_t H = ray_o.size(0), W = ray_o.size(1);
    const int64_t n = points.numel() / 3;
    const int64_t cdim = has(colors) ? colors->size(1) : 0;
    BwdOut o;
    o.v_points = at::empty_like(points);
    o.v_scale = at::empty_like(scale);
    o.v_quat = at::empty_like(quat);
    o.v_opacity = at::empty_like(opacity);
    if (has(colors)) o.v_colors = at::empty_like(*colors);
    if (ray_grads) {
        o.v_ray_o = at::empty_like(ray_o);
        o.v_ray_d = at::empty_like(ray_d);
    }
    const bool dyn = has(velocity);
    if (dyn) {
        o.v_velocity = at::empty_like(*velocity);
        if (ray_grads) o.v_time = at::empty_like(*ray_t);
    }
    const size_t ws_need = xsg_rasterize_workspace_size(n, int(cdim), 0, 0, 0);
    Tensor ws;
    if (has(fwd_ws)) {
        check_tensor(*fwd_ws, "forward_workspace", points);
        TORCH_CHECK(size_t(fwd_ws->nbytes()) >= ws_need, "forward_workspace too small: need ", ws_need, " bytes");
        ws = *fwd_ws;
    } else {
        ws = workspace(ws_need, points);
    }
    check(xsg_rasterize_bwd(fptr(points), fptr(velocity), fptr(quat), fptr(scale), fptr(colors), int(cdim),
                            fptr(opacity), n, int(W), int(H), int(tsx), int(tsy), fptr(ray_o), fptr(ray_d),
                            fptr(ray_t), tile_offsets.data_ptr<int32_t>(), int(tile_offsets.size(1)),
                            int(tile_offsets.size(0)), flatten_ids.data_ptr<int32_t>(), flatten_ids.numel(),
                            fptr(render_alpha), last_ids.data_ptr<int32_t>(), fptr(v_colors_in), fptr(v_depth),
                            fptr(v_alpha), fptr_mut(o.v_points), dyn ? fptr_mut(o.v_velocity) : nullptr,
                            fptr_mut(o.v_quat), fptr_mut(o.v_scale), has(colors) ? fptr_mut(*o.v_colors) : nullptr,
                            fptr_mut(o.v_opacity), ray_grads ? fptr_mut(o.v_ray_o) : nullptr,
                            ray_grads ? fptr_mut(o.v_ray_d) : nullptr, dyn && ray_grads ? fptr_mut(o.v_time) : nullptr,
                            ws.data_ptr(), size_t(ws.nbytes()), has(fwd_ws) ? 1 : 0, stream(),
                            n_isects_ptr(n_isects_dev, points)));
    return o;
}

// ------------------------------------------------------------- exchange ---
// Multi-GPU gradient exchange on symmetric buffers (no reference
// counterpart); addresses are device / multicast virtual addresses as ints.
void exchange_barrier(uint64_t peer_flags_dev, int64_t rank, int64_t world, int64_t epoch, double timeout_s,
                      const Tensor& err) {
    TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.numel() >= 1, "err must be a CUDA int32 tensor");
    c10::cuda::CUDAGuard g(err.device());
    check(xsg_exchange_barrier(reinterpret_cast<uint32_t* const*>(peer_flags_dev), int(rank), int(world),
                               uint32_t(epoch), timeout_s, err.data_ptr<int32_t>(), stream()));
}

void nvls_allreduce_sum(uint64_t mc_addr, int64_t n, int64_t rank, int64_t world, const Tensor& like) {
    TORCH_CHECK(like.is_cuda(), "nvls_allreduce: a CUDA tensor names the device");
    c10::cuda::CUDAGuard g(like.device());
    check(xsg_nvls_allreduce_sum_f32(mc_addr, n, int(rank), int(world), stream()));
}

void nvls_broadcast(const Tensor& src, uint64_t mc_dst) {
    check_tensor(src, "src", src);
    TORCH_CHECK(src.scalar_type() == at::kFloat, "nvls_broadcast: float32 source");
    c10::cuda::CUDAGuard g(src.device());
    check(xsg_nvls_broadcast_f32(fptr(src), mc_dst, src.numel(), stream()));
}

// ------------------------------------------------------------------ SH ---
Tensor sh_fwd(int64_t degree, const Tensor& origin, const Tensor& positions, const Tensor& coeffs, const OptT& mask,
              bool layout_3kn, const OptT& coeffs_dc, const OptT& output) {
    for (auto* t : {&origin, &positions, &coeffs}) check_tensor(*t, "spherical harmonics input", positions);
    if (has(mask)) check_tensor(*mask, "mask", positions);
    if (has(coeffs_dc)) check_tensor(*coeffs_dc, "coeffs_dc", positions);
    if (has(output)) check_tensor(*output, "output", positions);
    TORCH_CHECK(coeffs.dim() == 3 && coeffs.size(layout_3kn ? 0 : 2) == 3,
                "coeffs tensor must be [3, K, N] if layout_3kn else [N, K, 3]");
    const int64_t n = layout_3kn ? coeffs.size(2) : coeffs.size(0);
    const int64_t dim = coeffs.size(1);
    if (has(coeffs_dc)) {
        const auto dd = coeffs_dc->dim();
        TORCH_CHECK(dd == 2 || dd == 3, "coeffs_dc must be 2D or 3D");
        const int64_t ch_axis = layout_3kn ? 0 : dd - 1, n_axis = layout_3kn ? dd - 1 : 0;
        TORCH_CHECK(coeffs_dc->size(ch_axis) == 3 && coeffs_dc->size(n_axis) == n && coeffs_dc->numel() == 3 * n,
                    "coeffs_dc must hold a single SH band: [N, 3] or [N, 1, 3] if !layout_3kn else [3, N] or [3, 1, N]");
    }
    c10::cuda::CUDAGuard g(positions.device());
    Tensor out = has(output) ? *output : at::zeros({n, 3}, positions.options());
    check(xsg_sh_fwd(int(degree), fptr(origin), fptr(positions), fptr(coeffs), fptr(coeffs_dc),
                     has(mask) ? reinterpret_cast<const uint32_t*>(mask->data_ptr()) : nullptr, layout_3kn, n, int(dim),
                     fptr_mut(out), stream()));
    return out;
}

std::tuple<Tensor, Tensor, Tensor, Tensor> sh_bwd(int64_t degree, const Tensor& origin, const Tensor& positions,
                                                  const Tensor& coeffs, const OptT& mask, bool layout_3kn,
                                                  const Tensor& d_output, const OptT& coeffs_dc) {
    TORCH_CHECK(d_output.is_contiguous(), "d_output must be contiguous");
    for (auto* t : {&origin, &positions, &coeffs, &d_output}) check_tensor(*t, "spherical harmonics input", positions);
    if (has(mask)) check_tensor(*mask, "mask", positions);
    if (has(coeffs_dc)) check_tensor(*coeffs_dc, "coeffs_dc", positions);
    c10::cuda::CUDAGuard g(positions.device());
    const int64_t n = layout_3kn ? coeffs.size(2) : coeffs.size(0);
    const int64_t dim = coeffs.size(1);
    Tensor d_coeffs = at::empty_like(coeffs);
    Tensor d_dc = has(coeffs_dc) ? at::empty_like(*coeffs_dc) : at::empty({0}, coeffs.options());
    Tensor d_pos = at::empty_like(positions);
    Tensor d_origin = at::empty({3}, origin.options());
    Tensor ws = workspace(xsg_sh_bwd_workspace_size(n), positions);
    check(xsg_sh_bwd(int(degree), fptr(origin), fptr(positions), fptr(coeffs), fptr(coeffs_dc),
                     has(mask) ? reinterpret_cast<const uint32_t*>(mask->data_ptr()) : nullptr, layout_3kn, n, int(dim),
                     fptr(d_output), fptr_mut(d_coeffs), has(coeffs_dc) ? fptr_mut(d_dc) : nullptr, fptr_mut(d_pos),
                     fptr_mut(d_origin), ws.data_ptr(), size_t(ws.numel()), stream()));
    return {d_coeffs, d_dc, d_pos, d_origin};
}

// ------------------------------------------------- multi-view SH split --
// Not in the reference: the SH backward split used by the multi-GPU step
// (xsimgs_b200.multiview), [N, K, 3] coefficients, no mask.
Tensor sh_positions_bwd(int64_t degree, const Tensor& origins, const Tensor& positions, const Tensor& coeffs,
                        const Tensor& d_outputs) {
    for (auto* t : {&origins, &positions, &coeffs, &d_outputs}) check_tensor(*t, "spherical harmonics input", positions);
    TORCH_CHECK(coeffs.dim() == 3 && coeffs.size(2) == 3, "coeffs must be [N, K, 3]");
    const int64_t n = positions.size(0), views = origins.size(0);
    TORCH_CHECK(d_outputs.numel() == views * n * 3, "d_outputs must be [views, N, 3]");
    c10::cuda::CUDAGuard g(positions.device());
    Tensor d_pos = at::empty_like(positions);
    check(xsg_sh_positions_bwd(int(degree), int(views), fptr(origins), fptr(positions), fptr(coeffs), n,
                               int(coeffs.size(1)), fptr(d_outputs), fptr_mut(d_pos), stream()));
    return d_pos;
}

Tensor sh_coeffs_bwd_multi(int64_t degree, const Tensor& origins, const Tensor& positions, const Tensor& d_outputs,
                           int64_t dim) {
    for (auto* t : {&origins, &positions, &d_outputs}) check_tensor(*t, "spherical harmonics input", positions);
    const int64_t n = positions.size(0), views = origins.size(0);
    TORCH_CHECK(d_outputs.numel() == views * n * 3, "d_outputs must be [views, N, 3]");
    c10::cuda::CUDAGuard g(positions.device());
    Tensor d_coeffs = at::empty({n, dim, 3}, positions.options());
    check(xsg_sh_coeffs_bwd_multi(int(degree), int(views), fptr(origins), fptr(positions), n, int(dim),
                                  fptr(d_outputs), fptr_mut(d_coeffs), stream()));
    return d_coeffs;
}

// ----------------------------------------------------------------- SMPL --
// csrc/nodes/smpl_local_to_global.cu:91-337, smpl_lbs_skinning.cu:94-352,
// smpl.cu:52-95.  Id tensors are 32-bit (int32 or uint32), read as uint32.
const uint32_t* u32ptr(const Tensor& t, const char* name) {
    TORCH_CHECK(t.element_size() == 4 && !t.is_floating_point(), name, " must be a 32-bit integer tensor");
    return reinterpret_cast<const uint32_t*>(t.data_ptr());
}

std::tuple<Tensor, Tensor> smpl_local_to_global_fwd(const Tensor& ids, const Tensor& local_q, const Tensor& joints,
                                                    const Tensor& a0q, const Tensor& a0t) {
    for (auto* t : {&ids, &local_q, &joints, &a0q, &a0t}) check_tensor(*t, "smpl_local_to_global_fwd input", local_q);
    for (auto* t : {&local_q, &joints, &a0q, &a0t}) require_f32(*t, "smpl_local_to_global_fwd input");
    TORCH_CHECK(local_q.dim() == 3 && local_q.size(1) == 24 && local_q.size(2) == 4, "local_q must be [N, 24, 4]");
    c10::cuda::CUDAGuard g(local_q.device());
    const int64_t b = ids.numel();
    Tensor out_q = at::empty({b, 24, 4}, local_q.options());
    Tensor out_t = at::empty({b, 24, 3}, local_q.options());
    check(xsg_smpl_local_to_global_fwd(u32ptr(ids, "local_q_ids"), b, fptr(local_q), fptr(joints), fptr(a0q),
                                       fptr(a0t), local_q.size(0), fptr_mut(out_q), fptr_mut(out_t), stream()));
    return {out_q, out_t};
}

std::tuple<Tensor, Tensor, Tensor> smpl_local_to_global_bwd(const Tensor& ids, const Tensor& local_q,
                                                            const Tensor& joints, const Tensor& a0q,
                                                            const Tensor& a0t, const Tensor& out_q,
                                                            const Tensor& out_t, const Tensor& gq, const Tensor& gt) {
    for (auto* t : {&ids, &local_q, &joints, &a0q, &a0t, &gq, &gt})
        check_tensor(*t, "smpl_local_to_global_bwd input", local_q);
    TORCH_CHECK(gq.numel() == ids.numel() * 96 && gt.numel() == ids.numel() * 72,
                "grad_output_q / grad_output_t must be [B, 24, 4] / [B, 24, 3]");
    c10::cuda::CUDAGuard g(local_q.device());
    Tensor d_local_q = at::zeros_like(local_q);
    Tensor d_a0q = at::zeros_like(a0q);
    Tensor d_a0t = at::zeros_like(a0t);
    check(xsg_smpl_local_to_global_bwd(u32ptr(ids, "local_q_ids"), ids.numel(), fptr(local_q), fptr(joints),
                                       fptr(a0q), fptr(a0t), local_q.size(0), fptr(gq), fptr(gt),
                                       fptr_mut(d_local_q), fptr_mut(d_a0q), fptr_mut(d_a0t), stream()));
    return {d_local_q, d_a0q, d_a0t};
}

void smpl_lbs_skinning_fwd(const Tensor& valid_ids, const Tensor& global_q, const Tensor& global_t,
                           const Tensor& vertices, const Tensor& quats, const Tensor& weights,
                           const Tensor& instance_ids, const Tensor& instance_t, const Tensor& instance_v,
                           int64_t global_offset, const Tensor& out_positions, const Tensor& out_rotations,
                           const OptT& out_velocities, const OptT& out_mask) {
    for (auto* t : {&valid_ids, &global_q, &global_t, &vertices, &quats, &weights, &instance_ids, &instance_t,
                    &instance_v, &out_positions, &out_rotations})
        check_tensor(*t, "smpl_lbs_skinning input", vertices);
    TORCH_CHECK(vertices.dim() == 3 && vertices.size(2) == 3, "vertices must be [N, V, 3]");
    TORCH_CHECK(weights.dim() == 3 && weights.size(1) == 24 && weights.size(2) == vertices.size(1),
                "weights must be [N, 24, V]");
    if (has(out_velocities)) check_tensor(*out_velocities, "out_velocities", vertices);
    if (has(out_mask)) {
        check_tensor(*out_mask, "out_mask", vertices);
        TORCH_CHECK(out_mask->element_size() == 1, "out_mask must be a bool or uint8 tensor");
    }
    c10::cuda::CUDAGuard g(vertices.device());
    check(xsg_smpl_lbs_skinning_fwd(
        u32ptr(valid_ids, "valid_ids"), valid_ids.numel(), fptr(global_q), fptr(global_t), fptr(vertices),
        fptr(quats), fptr(weights), vertices.size(0), vertices.size(1), u32ptr(instance_ids, "instance_ids"),
        fptr(instance_t), fptr(instance_v), instance_t.size(0), global_offset, out_positions.size(0),
        fptr_mut(out_positions), fptr_mut(out_rotations), has(out_velocities) ? fptr_mut(*out_velocities) : nullptr,
        has(out_mask) ? reinterpret_cast<uint8_t*>(out_mask->data_ptr()) : nullptr, stream()));
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> smpl_lbs_skinning_bwd(
    const Tensor& valid_ids, const Tensor& instance_ids, const Tensor& global_q, const Tensor& global_t,
    const Tensor& vertices, const Tensor& quats, const Tensor& weights, int64_t global_offset, int64_t num_instances,
    const Tensor& grad_pos, const Tensor& grad_rot, const OptT& grad_vel) {
    for (auto* t : {&valid_ids, &instance_ids, &global_q, &global_t, &vertices, &quats, &weights, &grad_pos,
                    &grad_rot})
        check_tensor(*t, "smpl_lbs_skinning_bwd input", vertices);
    if (has(grad_vel)) check_tensor(*grad_vel, "grad_out_velocities", vertices);
    c10::cuda::CUDAGuard g(vertices.device());
    Tensor d_global_q = at::zeros_like(global_q);
    Tensor d_global_t = at::zeros_like(global_t);
    Tensor d_vertices = at::zeros_like(vertices);
    Tensor d_quats = at::zeros_like(quats);
    Tensor d_weights = at::zeros_like(weights);
    Tensor d_instance_v = at::zeros({num_instances, 3}, global_q.options());
    Tensor d_instance_t = at::zeros({num_instances, 3}, global_q.options());
    check(xsg_smpl_lbs_skinning_bwd(
        u32ptr(valid_ids, "valid_ids"), valid_ids.numel(), u32ptr(instance_ids, "instance_ids"), fptr(global_q),
        fptr(global_t), fptr(vertices), fptr(quats), fptr(weights), vertices.size(0), vertices.size(1),
        num_instances, global_offset, grad_pos.size(0), fptr(grad_pos), fptr(grad_rot),
        has(grad_vel) ? fptr(*grad_vel) : nullptr, fptr_mut(d_global_q), fptr_mut(d_global_t), fptr_mut(d_vertices),
        fptr_mut(d_quats), fptr_mut(d_weights), has(grad_vel) ? fptr_mut(d_instance_v) : nullptr,
        fptr_mut(d_instance_t), stream()));
    return {d_global_q, d_global_t, d_vertices, d_quats, d_weights, d_instance_v, d_instance_t};
}

Tensor smpl_ids_compaction(const Tensor& instance_ids, const Tensor& instance_mask) {
    check_tensor(instance_ids, "instance_ids", instance_ids);
    check_tensor(instance_mask, "instance_mask", instance_ids);
    TORCH_CHECK(instance_mask.element_size() == 1, "instance_mask must be a bool or uint8 tensor");
    c10::cuda::CUDAGuard g(instance_ids.device());
    Tensor out = at::empty({instance_ids.numel()}, instance_ids.options());
    Tensor count = at::empty({1}, instance_ids.options().dtype(at::kLong));
    int64_t n_out = 0;
    check(xsg_smpl_ids_compaction(u32ptr(instance_ids, "instance_ids"), instance_ids.numel(),
                                  reinterpret_cast<const uint8_t*>(instance_mask.data_ptr()), instance_mask.numel(),
                                  reinterpret_cast<uint32_t*>(out.data_ptr()), count.data_ptr<int64_t>(), &n_out,
                                  stream()));
    return out.slice(0, 0, n_out);
}

// -------------------------------------------------------- scene nodes --
// csrc/nodes/container.cu:157-301, gs_masking.cu:27-48,
// smpl_interpolate.cu:60-248.
const uint32_t* opt_u32(const OptT& t, const char* name) { return has(t) ? u32ptr(*t, name) : nullptr; }

void rigid_transform_fwd(const Tensor& positions, const Tensor& rotations, const Tensor& instance_id,
                         const Tensor& inst_q, const Tensor& inst_t, const Tensor& inst_v, const Tensor& inst_w,
                         const Tensor& inst_mask, const Tensor& out_positions, const Tensor& out_rotations,
                         const OptT& out_velocities, const OptT& out_mask, int64_t buffer_offset,
                         const OptT& per_instance_offsets, const OptT& gs_inst_offsets) {
    for (auto* t : {&positions, &rotations, &instance_id, &inst_q, &inst_t, &inst_v, &inst_w, &inst_mask,
                    &out_positions, &out_rotations})
        check_tensor(*t, "copy_gs_rigid_transform_fwd input", positions);
    if (has(out_velocities)) check_tensor(*out_velocities, "out_velocities", positions);
    if (has(out_mask)) check_tensor(*out_mask, "out_mask", positions);
    c10::cuda::CUDAGuard g(positions.device());
    check(xsg_rigid_transform_fwd(
        positions.size(0), fptr(positions), fptr(rotations), u32ptr(instance_id, "instance_id"), fptr(inst_q),
        fptr(inst_t), fptr(inst_v), fptr(inst_w), reinterpret_cast<const uint8_t*>(inst_mask.data_ptr()),
        inst_q.size(0), buffer_offset, opt_u32(per_instance_offsets, "per_instance_offsets"),
        opt_u32(gs_inst_offsets, "gs_inst_offsets"), out_positions.size(0), fptr_mut(out_positions),
        fptr_mut(out_rotations), has(out_velocities) ? fptr_mut(*out_velocities) : nullptr,
        has(out_mask) ? reinterpret_cast<uint8_t*>(out_mask->data_ptr()) : nullptr, stream()));
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> rigid_transform_bwd(
    const Tensor& positions, const Tensor& rotations, const Tensor& instance_id, const Tensor& inst_q,
    const Tensor& inst_w, const Tensor& inst_mask, int64_t buffer_offset, const OptT& per_instance_offsets,
    const OptT& gs_inst_offsets, const Tensor& v_positions, const Tensor& v_rotations, const OptT& v_velocities) {
    for (auto* t : {&positions, &rotations, &instance_id, &inst_q, &inst_w, &inst_mask, &v_positions, &v_rotations})
        check_tensor(*t, "copy_gs_rigid_transform_bwd input", positions);
    if (has(v_velocities)) check_tensor(*v_velocities, "v_velocities", positions);
    c10::cuda::CUDAGuard g(positions.device());
    Tensor gp = at::zeros_like(positions), gr = at::zeros_like(rotations);
    Tensor gq = at::zeros_like(inst_q), gt = at::zeros_like(inst_w), gv = at::zeros_like(inst_w),
           gw = at::zeros_like(inst_w);
    check(xsg_rigid_transform_bwd(
        positions.size(0), fptr(positions), fptr(rotations), u32ptr(instance_id, "instance_id"), fptr(inst_q),
        fptr(inst_w), reinterpret_cast<const uint8_t*>(inst_mask.data_ptr()), inst_q.size(0), buffer_offset,
        opt_u32(per_instance_offsets, "per_instance_offsets"), opt_u32(gs_inst_offsets, "gs_inst_offsets"),
        v_positions.size(0), fptr(v_positions), fptr(v_rotations), has(v_velocities) ? fptr(*v_velocities) : nullptr,
        fptr_mut(gp), fptr_mut(gr), fptr_mut(gq), fptr_mut(gt), fptr_mut(gv), fptr_mut(gw), stream()));
    return {gp, gr, gq, gt, gv, gw};
}

// image_to_*_byte, csrc/nodes/img_layout.cu:57-115: the same checks and
// messages; a non-contiguous image is made contiguous first.
Tensor image_to_bytes(const Tensor& image_in, int layout) {
    if (!image_in.is_cuda()) throw std::runtime_error("image is not a CUDA tensor");
    if (image_in.dim() != 3) throw std::runtime_error("image must have dimensions [H, W, 3]");
    if (image_in.scalar_type() != at::kFloat) throw std::runtime_error("image must have float32 dtype");
    if (image_in.size(-1) != 3) throw std::runtime_error("image must have dimensions [H, W, 3]");
    Tensor image = image_in.contiguous();
    c10::cuda::CUDAGuard g(image.device());
    const int64_t H = image.size(0), W = image.size(1);
    auto opt = image.options().dtype(at::kByte);
    Tensor out = layout == XSG_IMG_CHW_RGB ? at::empty({3, H, W}, opt)
                                           : at::empty({H, W, layout == XSG_IMG_HWC_RGBA ? 4 : 3}, opt);
    check(xsg_image_to_bytes(layout, fptr(image), H * W, out.data_ptr<uint8_t>(), stream()));
    return out;
}

Tensor packed_mask_from_instances(const Tensor& instance_ids, const Tensor& instance_mask) {
    check_tensor(instance_ids, "instance_ids", instance_ids);
    check_tensor(instance_mask, "instance_mask", instance_ids);
    TORCH_CHECK(instance_ids.element_size() == 4 && !instance_ids.is_floating_point(),
                "instance_ids must be a 32-bit integer tensor");
    TORCH_CHECK(instance_mask.element_size() == 1, "instance_mask must be a bool or uint8 tensor");
    c10::cuda::CUDAGuard g(instance_ids.device());
    const int64_t n = instance_ids.numel();
    Tensor out = at::empty({(n + 31) / 32}, instance_ids.options().dtype(at::kUInt32));
    check(xsg_packed_mask_from_instances(reinterpret_cast<const int32_t*>(instance_ids.data_ptr()), n,
                                         reinterpret_cast<const uint8_t*>(instance_mask.data_ptr()),
                                         instance_mask.numel(), reinterpret_cast<uint32_t*>(out.data_ptr()),
                                         stream()));
    return out;
}

Tensor interpolate_smpl_fwd(const Tensor& poses, const Tensor& times, const Tensor& root_q, const Tensor& inst_ids,
                            const Tensor& query_time) {
    for (auto* t : {&poses, &times, &root_q, &inst_ids, &query_time})
        check_tensor(*t, "interpolate_smpl_poses_fwd input", poses);
    TORCH_CHECK(poses.dim() == 4 && poses.size(3) == 4, "smpl_poses must be [N, frames, joints, 4]");
    TORCH_CHECK(poses.size(2) == 24, "num_joints only 24 supported now");
    c10::cuda::CUDAGuard g(poses.device());
    Tensor out = at::empty({poses.size(0), poses.size(2), 4}, poses.options());
    check(xsg_interpolate_smpl_poses_fwd(poses.size(0), int(poses.size(1)), int(poses.size(2)), fptr(query_time),
                                         fptr(poses), fptr(times), fptr(root_q), u32ptr(inst_ids, "instance_ids"),
                                         root_q.size(0), fptr_mut(out), stream()));
    return out;
}

std::tuple<Tensor, Tensor, Tensor> interpolate_smpl_bwd(const Tensor& poses, const Tensor& times,
                                                        const Tensor& root_q, const Tensor& inst_ids,
                                                        const Tensor& query_time, const Tensor& grad_out) {
    for (auto* t : {&poses, &times, &root_q, &inst_ids, &query_time, &grad_out})
        check_tensor(*t, "interpolate_smpl_poses_bwd input", poses);
    TORCH_CHECK(poses.size(2) == 24, "num_joints only 24 supported now");
    c10::cuda::CUDAGuard g(poses.device());
    Tensor d_poses = at::zeros_like(poses), d_root = at::zeros_like(root_q), d_q = at::zeros_like(query_time);
    check(xsg_interpolate_smpl_poses_bwd(poses.size(0), int(poses.size(1)), int(poses.size(2)), fptr(query_time),
                                         fptr(poses), fptr(times), u32ptr(inst_ids, "instance_ids"), root_q.size(0),
                                         fptr(grad_out), fptr_mut(d_poses), fptr_mut(d_root), fptr_mut(d_q),
                                         stream()));
    return {d_poses, d_root, d_q};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "xsimgs-b200: B200-native kernels behind the xsimgs._C operator surface";
    m.def("version", []() { return std::string(xsg_version()); });

    py::enum_<ProjectionMode>(m, "ProjectionMode")
        .value("Central", ProjectionMode::Central)
        .value("NegativeDelta", ProjectionMode::NegativeDelta)
        .value("PositiveDelta", ProjectionMode::PositiveDelta);

    bind_camera<PerspectiveCamera>(m, "PerspectiveCamera", {XSG_CAM_PINHOLE, "PerspectiveCamera", {4}}, false);
    bind_camera<OpenCVFisheyeCamera>(m, "OpenCVFisheyeCamera", {XSG_CAM_FISHEYE, "OpenCVFisheyeCamera", {4, 4}}, false);
    bind_camera<SphericalCamera>(m, "SphericalCamera", {XSG_CAM_SPHERICAL, "SphericalCamera", {4}}, true);
    bind_camera<LidarCamera>(m, "LidarCamera", {XSG_CAM_LIDAR, "LidarCamera", {4, 2}}, true);
    {
        const CameraSpec spec{XSG_CAM_DISTORTED, "DistortedPerspectiveCamera", {4, 8, 1}};
        bind_camera<DistortedPerspectiveCamera>(m, "DistortedPerspectiveCamera", spec, false)
            .def_static("undistort_map",
                        [spec](const Tensor& pack, int64_t width, int64_t height, bool normalized_range) {
                            return undistort_map(spec, pack, width, height, normalized_range);
                        },
                        py::arg("pack"), py::arg("width"), py::arg("height"), py::arg("normalized_range") = false);
    }

    m.def("isect_regular_tiles", &isect_regular_tiles, py::arg("means2d"), py::arg("radii"), py::arg("depth"),
          py::arg("img_width"), py::arg("img_height"), py::arg("tile_size_x"), py::arg("tile_size_y"),
          py::arg("sort") = true, py::arg("double_buffer") = true);
    m.def("isect_regular_tiles_async", &isect_regular_tiles_async, py::arg("means2d"), py::arg("radii"),
          py::arg("depth"), py::arg("img_width"), py::arg("img_height"), py::arg("tile_size_x"),
          py::arg("tile_size_y"), py::arg("capacity"), py::arg("workspace") = py::none());
    m.def("isect_lidar_tiles",
          [](const Tensor& pack, const Tensor& points, const OptT& vel, const Tensor& scale, const Tensor& quat,
             const OptT& opacity, const Tensor& flag, const Tensor& means2d, const Tensor& radii, const Tensor& depths,
             const Tensor& elev_boundaries, int64_t tile_size_x, float img_width, float img_height, float ua, float ub,
             float uk, bool sort, bool /*double_buffer*/) {
              return isect_range_tiles(true, pack, points, vel, scale, quat, opacity, flag, means2d, radii, depths,
                                       elev_boundaries, tile_size_x, 1, img_width, img_height, ua, ub, uk, sort);
          },
          py::arg("camera_pack"), py::arg("points"), py::arg("points_velocity"), py::arg("scale"), py::arg("quat"),
          py::arg("opacity"), py::arg("flag"), py::arg("means2d"), py::arg("radii"), py::arg("depths"),
          py::arg("elev_boundaries"), py::arg("tile_size_x"), py::arg("img_width"), py::arg("img_height"),
          py::arg("ut_alpha") = 0.1f, py::arg("ut_beta") = 2.0f, py::arg("ut_kappa") = 0.0f, py::arg("sort") = true,
          py::arg("double_buffer") = true);
    m.def("isect_spherical_tiles",
          [](const Tensor& pack, const Tensor& points, const OptT& vel, const Tensor& scale, const Tensor& quat,
             const OptT& opacity, const Tensor& flag, const Tensor& means2d, const Tensor& radii, const Tensor& depths,
             int64_t tile_size_x, int64_t tile_size_y, float img_width, float img_height, float ua, float ub, float uk,
             bool sort, bool /*double_buffer*/) {
              return isect_range_tiles(false, pack, points, vel, scale, quat, opacity, flag, means2d, radii, depths,
                                       std::nullopt, tile_size_x, tile_size_y, img_width, img_height, ua, ub, uk,
                                       sort);
          },
          py::arg("camera_pack"), py::arg("points"), py::arg("points_velocity"), py::arg("scale"), py::arg("quat"),
          py::arg("opacity"), py::arg("flag"), py::arg("means2d"), py::arg("radii"), py::arg("depths"),
          py::arg("tile_size_x"), py::arg("tile_size_y"), py::arg("img_width"), py::arg("img_height"),
          py::arg("ut_alpha") = 0.1f, py::arg("ut_beta") = 2.0f, py::arg("ut_kappa") = 0.0f, py::arg("sort") = true,
          py::arg("double_buffer") = true);
    m.def("isect_offset_encode", &isect_offset_encode, py::arg("isect_ids"), py::arg("tile_width"),
          py::arg("tile_height"));
    m.def("mask_radii_packed", &mask_radii_packed, py::arg("packed_mask"), py::arg("radii"));
    m.def("mask_radii", &mask_radii, py::arg("mask"), py::arg("radii"));

    m.def("eval3d_supported_ndims", &eval3d_supported_ndims);
    // bytes of the scratch a rasterize call uses: a caller that passes the
    // forward's `workspace` on to the backward as `forward_workspace` lets
    // the backward reuse the forward's packed records and, when the size
    // was asked with the intersection and tile counts, its per-warp
    // contributor masks (not in the reference)
    m.def("rasterize_workspace_size",
          [](int64_t n_gauss, int64_t channels, int64_t n_isects, int64_t n_tiles, int64_t tile_pixels) {
              return int64_t(xsg_rasterize_workspace_size(n_gauss, int(channels), n_isects, n_tiles, int(tile_pixels)));
          },
          py::arg("n_gauss"), py::arg("channels"), py::arg("n_isects") = 0, py::arg("n_tiles") = 0,
          py::arg("tile_pixels") = 256);
    m.def("rasterize_eval3d_fwd",
          [](const Tensor& means, const Tensor& quats, const Tensor& scales, const OptT& colors, const Tensor& opac,
             int64_t W, int64_t H, int64_t tsx, int64_t tsy, const Tensor& ray_o, const Tensor& ray_d,
             const Tensor& offsets, const Tensor& flatten, const OptT& ws, const OptT& n_isects) {
              return raster_fwd(means, std::nullopt, quats, scales, colors, opac, W, H, tsx, tsy, ray_o, ray_d,
                                std::nullopt, offsets, flatten, ws, n_isects);
          },
          py::arg("means"), py::arg("quats"), py::arg("scales"), py::arg("colors"), py::arg("opacities"),
          py::arg("image_width"), py::arg("image_height"), py::arg("tile_size_width"), py::arg("tile_size_height"),
          py::arg("ray_origs"), py::arg("ray_dirs"), py::arg("tile_offsets"), py::arg("flatten_ids"),
          py::arg("workspace") = py::none(), py::arg("n_isects") = py::none());
    m.def("rasterize_eval3d_dynamic_fwd",
          [](const Tensor& means, const OptT& vel, const Tensor& quats, const Tensor& scales, const OptT& colors,
             const Tensor& opac, int64_t W, int64_t H, int64_t tsx, int64_t tsy, const Tensor& ray_o,
             const Tensor& ray_d, const OptT& ray_t, const Tensor& offsets, const Tensor& flatten, const OptT& ws,
             const OptT& n_isects) {
              return raster_fwd(means, vel, quats, scales, colors, opac, W, H, tsx, tsy, ray_o, ray_d, ray_t,
                                offsets, flatten, ws, n_isects);
          },
          py::arg("means"), py::arg("velocity"), py::arg("quats"), py::arg("scales"), py::arg("colors"),
          py::arg("opacities"), py::arg("image_width"), py::arg("image_height"), py::arg("tile_size_width"),
          py::arg("tile_size_height"), py::arg("ray_origs"), py::arg("ray_dirs"), py::arg("ray_time_delta"),
          py::arg("tile_offsets"), py::arg("flatten_ids"), py::arg("workspace") = py::none(),
          py::arg("n_isects") = py::none());
    m.def("rasterize_eval3d_bwd",
          [](const Tensor& points, const Tensor& scale, const Tensor& quat, const Tensor& opacity, const OptT& colors,
             const Tensor& ray_o, const Tensor& ray_d, int64_t tsx, int64_t tsy, const Tensor& offsets,
             const Tensor& flatten, const Tensor& render_alpha, const Tensor& last_ids, const OptT& v_colors,
             const Tensor& v_depth, const Tensor& v_alpha, bool ray_grads, const OptT& fwd_ws,
             const OptT& n_isects) {
              BwdOut o = raster_bwd(points, std::nullopt, scale, quat, opacity, colors, ray_o, ray_d, std::nullopt,
                                    tsx, tsy, offsets, flatten, render_alpha, last_ids, v_colors, v_depth, v_alpha,
                                    ray_grads, fwd_ws, n_isects);
              return py::make_tuple(o.v_points, o.v_quat, o.v_scale, o.v_opacity,
                                    o.v_colors.has_value() ? py::cast(*o.v_colors) : py::none(), opt(o.v_ray_o),
                                    opt(o.v_ray_d));
          },
          py::arg("points"), py::arg("scale"), py::arg("quat"), py::arg("opacity"), py::arg("colors"),
          py::arg("ray_origins"), py::arg("ray_directions"), py::arg("tile_size_x"), py::arg("tile_size_y"),
          py::arg("tile_offsets"), py::arg("flatten_ids"), py::arg("render_alpha"), py::arg("last_ids"),
          py::arg("v_render_colors"), py::arg("v_render_depth"), py::arg("v_render_alpha"),
          py::arg("ray_grads") = true, py::arg("forward_workspace") = py::none(), py::arg("n_isects") = py::none());
    m.def("rasterize_eval3d_dynamic_bwd",
          [](const Tensor& points, const Tensor& vel, const Tensor& scale, const Tensor& quat, const Tensor& opacity,
             const OptT& colors, const Tensor& ray_o, const Tensor& ray_d, const Tensor& ray_t, int64_t tsx,
             int64_t tsy, const Tensor& offsets, const Tensor& flatten, const Tensor& render_alpha,
             const Tensor& last_ids, const OptT& v_colors, const Tensor& v_depth, const Tensor& v_alpha,
             bool ray_grads, const OptT& fwd_ws, const OptT& n_isects) {
              check_tensor(vel, "velocity", points);
              check_tensor(ray_t, "ray_time_delta", points);
              BwdOut o = raster_bwd(points, vel, scale, quat, opacity, colors, ray_o, ray_d, ray_t, tsx, tsy, offsets,
                                    flatten, render_alpha, last_ids, v_colors, v_depth, v_alpha, ray_grads, fwd_ws,
                                    n_isects);
              return py::make_tuple(o.v_points, o.v_velocity, o.v_quat, o.v_scale, o.v_opacity,
                                    o.v_colors.has_value() ? py::cast(*o.v_colors) : py::none(), opt(o.v_ray_o),
                                    opt(o.v_ray_d), opt(o.v_time));
          },
          py::arg("points"), py::arg("velocity"), py::arg("scale"), py::arg("quat"), py::arg("opacity"),
          py::arg("colors"), py::arg("ray_origins"), py::arg("ray_directions"), py::arg("ray_time_delta"),
          py::arg("tile_size_x"), py::arg("tile_size_y"), py::arg("tile_offsets"), py::arg("flatten_ids"),
          py::arg("render_alpha"), py::arg("last_ids"), py::arg("v_render_colors"), py::arg("v_render_depth"),
          py::arg("v_render_alpha"), py::arg("ray_grads") = true, py::arg("forward_workspace") = py::none(),
          py::arg("n_isects") = py::none());

    m.def("exchange_barrier", &exchange_barrier, py::arg("peer_flags"), py::arg("rank"), py::arg("world"),
          py::arg("epoch"), py::arg("timeout_s"), py::arg("err"));
    m.def("nvls_allreduce_sum", &nvls_allreduce_sum, py::arg("mc_addr"), py::arg("n"), py::arg("rank"),
          py::arg("world"), py::arg("like"));
    m.def("nvls_broadcast", &nvls_broadcast, py::arg("src"), py::arg("mc_dst"));
    m.def("exchange_set_max_ctas", [](int64_t n) { xsg_exchange_set_max_ctas(int(n)); }, py::arg("n"));
    m.def("spherical_harmonics_fused_fwd", &sh_fwd, py::arg("degree_to_use"), py::arg("origin"),
          py::arg("positions"), py::arg("coeffs"), py::arg("mask"), py::arg("layout_3kn"),
          py::arg("coeffs_dc") = py::none(), py::arg("output") = py::none());
    m.def("spherical_harmonics_fused_bwd", &sh_bwd, py::arg("degree_to_use"), py::arg("origin"),
          py::arg("positions"), py::arg("coeffs"), py::arg("mask"), py::arg("layout_3kn"), py::arg("d_output"),
          py::arg("coeffs_dc") = py::none());
    m.def("spherical_harmonics_positions_bwd", &sh_positions_bwd, py::arg("degree_to_use"), py::arg("origins"),
          py::arg("positions"), py::arg("coeffs"), py::arg("d_outputs"));
    m.def("spherical_harmonics_coeffs_bwd_multi", &sh_coeffs_bwd_multi, py::arg("degree_to_use"), py::arg("origins"),
          py::arg("positions"), py::arg("d_outputs"), py::arg("dim"));
    m.def("smpl_local_to_global_fwd", &smpl_local_to_global_fwd, py::arg("local_q_ids"), py::arg("local_q"),
          py::arg("joints"), py::arg("a0_inv_q"), py::arg("a0_inv_t"));
    m.def("smpl_local_to_global_bwd", &smpl_local_to_global_bwd, py::arg("local_q_ids"), py::arg("local_q"),
          py::arg("joints"), py::arg("a0_inv_q"), py::arg("a0_inv_t"), py::arg("output_q"), py::arg("output_t"),
          py::arg("grad_output_q"), py::arg("grad_output_t"));
    m.def("smpl_lbs_skinning", &smpl_lbs_skinning_fwd, py::arg("valid_ids"), py::arg("global_q"),
          py::arg("global_t"), py::arg("vertices"), py::arg("quats"), py::arg("weights"), py::arg("instance_ids"),
          py::arg("instance_t"), py::arg("instance_v"), py::arg("global_offset"), py::arg("out_positions"),
          py::arg("out_rotations"), py::arg("out_velocities"), py::arg("out_mask"));
    m.def("smpl_lbs_skinning_bwd", &smpl_lbs_skinning_bwd, py::arg("valid_ids"), py::arg("instance_ids"),
          py::arg("global_q"), py::arg("global_t"), py::arg("vertices"), py::arg("quats"), py::arg("weights"),
          py::arg("global_offset"), py::arg("num_instances"), py::arg("grad_out_vertices"),
          py::arg("grad_out_quats"), py::arg("grad_out_velocities") = py::none());
    m.def("smpl_ids_compaction", &smpl_ids_compaction, py::arg("instance_ids"), py::arg("instance_mask"));
    m.def("copy_gs_rigid_transform_fwd", &rigid_transform_fwd, py::arg("positions"), py::arg("rotations"),
          py::arg("instance_id"), py::arg("inst_q"), py::arg("inst_t"), py::arg("inst_v"), py::arg("inst_w"),
          py::arg("inst_mask"), py::arg("out_positions"), py::arg("out_rotations"), py::arg("out_velocities"),
          py::arg("out_mask"), py::arg("buffer_offset"), py::arg("per_instance_offsets") = py::none(),
          py::arg("gs_inst_offsets") = py::none());
    m.def("copy_gs_rigid_transform_bwd", &rigid_transform_bwd, py::arg("positions"), py::arg("rotations"),
          py::arg("instance_id"), py::arg("inst_q"), py::arg("inst_w"), py::arg("inst_mask"),
          py::arg("buffer_offset"), py::arg("per_instance_offsets"), py::arg("gs_inst_offsets"),
          py::arg("v_positions"), py::arg("v_rotations"), py::arg("v_velocities"));
    m.def("image_to_hwc_rgb_byte", [](const Tensor& image) { return image_to_bytes(image, XSG_IMG_HWC_RGB); },
          py::arg("image"));
    m.def("image_to_hwc_rgba_byte", [](const Tensor& image) { return image_to_bytes(image, XSG_IMG_HWC_RGBA); },
          py::arg("image"));
    m.def("image_to_chw_rgb_byte", [](const Tensor& image) { return image_to_bytes(image, XSG_IMG_CHW_RGB); },
          py::arg("image"));
    m.def("packed_mask_from_instances", &packed_mask_from_instances, py::arg("instance_ids"),
          py::arg("instance_mask"));
    m.def("interpolate_smpl_poses_fwd", &interpolate_smpl_fwd, py::arg("smpl_poses"), py::arg("smpl_poses_time"),
          py::arg("root_q"), py::arg("instance_ids"), py::arg("query_time"));
    m.def("interpolate_smpl_poses_bwd", &interpolate_smpl_bwd, py::arg("smpl_poses"), py::arg("smpl_poses_time"),
          py::arg("root_q"), py::arg("instance_ids"), py::arg("query_time"), py::arg("grad_out_quats"));
}
