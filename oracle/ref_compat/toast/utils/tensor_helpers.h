// Test infrastructure: a minimal stand-in for pytoast's
// <toast/utils/tensor_helpers.h> (see vector_math.h in this folder for why):
// argument checks that raise the usual torch errors; it brings in the ATen
// operator declarations (at::empty, at::zeros, ...) the sources call.
#pragma once

#include <ATen/ATen.h>
#include <c10/util/Exception.h>

inline void xsg_ref_check_contiguous(const at::Tensor& t) {
    TORCH_CHECK(t.is_contiguous(), "all tensors must be contiguous");
}

template <typename... Ts>
inline void all_contiguous(const Ts&... ts) {
    (xsg_ref_check_contiguous(ts), ...);
}

inline void xsg_ref_check_device(const at::Tensor& a, const at::Tensor& b) {
    TORCH_CHECK(a.device() == b.device(), "all tensors must be on the same device");
}

template <typename T0, typename... Ts>
inline void check_same_device(const T0& t0, const Ts&... ts) {
    (xsg_ref_check_device(t0, ts), ...);
}

inline void check_same_device(const std::vector<at::Tensor>& ts) {
    for (const auto& t : ts) xsg_ref_check_device(ts.front(), t);
}

inline void check_dtypes(at::ScalarType dtype, const std::vector<at::Tensor>& ts) {
    for (const auto& t : ts) TORCH_CHECK(t.scalar_type() == dtype, "unexpected tensor dtype ", t.scalar_type());
}

template <typename Dims>
inline void check_operand_last_dims(const std::vector<at::Tensor>& ts, const Dims& dims) {
    TORCH_CHECK(ts.size() == dims.size(), "expected ", dims.size(), " tensors, got ", ts.size());
    for (size_t i = 0; i < ts.size(); ++i) {
        TORCH_CHECK(ts[i].dim() > 0 && ts[i].size(-1) == dims[i], "tensor ", i, ": last dimension must be ",
                    dims[i], ", got ", ts[i].sizes());
    }
}

// A device tensor holding the data addresses of `ts` (int64 words), for
// kernels that gather from several tensors through one pointer table.
inline at::Tensor make_ptr_tensor(const std::vector<at::Tensor>& ts) {
    std::vector<int64_t> ptrs;
    ptrs.reserve(ts.size());
    for (const auto& t : ts) {
        xsg_ref_check_contiguous(t);
        ptrs.push_back(reinterpret_cast<int64_t>(t.data_ptr()));
    }
    auto host = at::tensor(ptrs, at::TensorOptions().dtype(at::kLong));
    return host.to(ts.front().device());
}
