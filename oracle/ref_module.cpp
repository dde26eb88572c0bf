// Test infrastructure: the Python module of the GPU test oracle built from
// the reference's own CUDA sources (oracle/build_ref.py).  It only calls the
// reference's bind_* functions, so the module exposes the reference's op
// names and keyword arguments (csrc/ext.cpp:12-20 binds the same functions).
// Nothing in the shipped library imports or links it.
#include <torch/csrc/utils/pybind.h>

void bind_rasterization_eval3d(py::module& m);
void bind_common_tiling(py::module_& m);
void bind_regular_tiling(py::module_& m);
void bind_mask_radii(py::module_& m);
void bind_sh(py::module_& m);
void bind_perspective(py::module_& m);
void bind_distorted_perspective(py::module_& m);
void bind_fisheye(py::module_& m);
void bind_spherical(py::module_& m);
void bind_lidar_tiling(py::module_& m);
void bind_spherical_tiling(py::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    bind_rasterization_eval3d(m);
    bind_common_tiling(m);
    bind_regular_tiling(m);
    bind_mask_radii(m);
    bind_sh(m);
    bind_perspective(m);
    bind_distorted_perspective(m);
    bind_fisheye(m);
    bind_spherical(m);
    bind_lidar_tiling(m);
    bind_spherical_tiling(m);
}
