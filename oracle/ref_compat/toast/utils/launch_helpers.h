// Test infrastructure: a minimal stand-in for pytoast's
// <toast/utils/launch_helpers.h> (see vector_math.h in this folder for why).
// launch_kernel_cuda<THREADS>(n, device, kernel, args...) launches
// ceil(n / THREADS) blocks of THREADS threads on the device's current
// stream (nothing when n is 0) and checks the launch.
// CUDA_DEFAULT_NUM_THREADS is 1024: the reference's block reductions
// (include/utils/reduce_helpers.cuh:5-6) only compile with that value.
// INLINE_KERNEL(n, device, { body }) runs `body` once per index idx < n in a
// device lambda that captures the enclosing scope by value.
#pragma once

#include <ATen/core/Tensor.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#ifndef CUDA_DEFAULT_NUM_THREADS
#define CUDA_DEFAULT_NUM_THREADS 1024
#endif

template <unsigned THREADS = CUDA_DEFAULT_NUM_THREADS, typename Kernel, typename... Args>
inline void launch_kernel_cuda(size_t n, const c10::Device& device, Kernel kernel, Args&&... args) {
    if (n == 0) return;
    const c10::cuda::OptionalCUDAGuard guard(device);
    const unsigned blocks = static_cast<unsigned>((n + THREADS - 1) / THREADS);
    kernel<<<blocks, THREADS, 0, c10::cuda::getCurrentCUDAStream()>>>(std::forward<Args>(args)...);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <typename F>
__global__ void xsg_ref_inline_kernel(unsigned n, F f) {
    const unsigned idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < n) f(idx);
}

template <typename F>
inline void xsg_ref_launch_inline(size_t n, const c10::Device& device, F f) {
    if (n == 0) return;
    const c10::cuda::OptionalCUDAGuard guard(device);
    constexpr unsigned threads = CUDA_DEFAULT_NUM_THREADS;
    const unsigned blocks = static_cast<unsigned>((n + threads - 1) / threads);
    xsg_ref_inline_kernel<<<blocks, threads, 0, c10::cuda::getCurrentCUDAStream()>>>(static_cast<unsigned>(n), f);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
}

#define INLINE_KERNEL(N_, DEVICE_, ...) \
    xsg_ref_launch_inline((N_), (DEVICE_), [=] __device__ (const unsigned idx) __VA_ARGS__);
