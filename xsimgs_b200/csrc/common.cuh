// Shared host/device helpers for the xsimgs-b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/xsimgs_b200.h"

namespace xsg {

// --------------------------------------------------------------- status --
// Sets the thread-local error message and returns `code`.
int set_error(int code, const std::string& msg);
int check_launch(const char* what);

#define XSG_REQUIRE(cond, msg)                                              \
    do {                                                                    \
        if (!(cond)) return ::xsg::set_error(XSG_ERR_INVALID_ARGUMENT, msg); \
    } while (0)

#define XSG_CUDA(call)                                                        \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess)                                                \
            return ::xsg::set_error(XSG_ERR_CUDA, std::string(#call) + ": " + \
                                                  cudaGetErrorString(e_));    \
    } while (0)

inline cudaStream_t as_cuda(xsg_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Every kernel launch of the library goes through launch(): it counts the
// launch (xsg_launch_count) before issuing it with <<<>>>.
void count_launch();
template <typename K, typename... A>
inline void launch(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args) {
    count_launch();
    kernel<<<grid, block, smem, st>>>(args...);
}

// Programmatic dependent launch (sm_90+): the kernel may be scheduled while
// its predecessor in the stream is still finishing its last CTAs; it must
// call pdl_wait() before its first global memory access (read or write), which
// returns once the predecessor has completed and its writes are visible.
// Chains of short dependent kernels (scans, sort passes) so lose the launch
// gap and the predecessor's tail.  Kernels launched this way call
// pdl_trigger() to let their own dependents be scheduled; the trigger takes
// effect once every CTA of the grid has issued it or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... P, typename... A>
inline void launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args) {
    count_launch();
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    (void)cudaLaunchKernelEx(&cfg, kernel, static_cast<P>(args)...);  // errors surface in check_launch
}

// Optional per-kernel device timing (xsg_timing_enable): records a CUDA event
// pair on `st` around the scope when enabled.
struct ScopedTimer {
    int slot = -1;
    cudaStream_t st;
    ScopedTimer(const char* name, cudaStream_t stream);
    ~ScopedTimer();
};

inline unsigned blocks_for(int64_t n, int threads) {
    return static_cast<unsigned>((n + threads - 1) / threads);
}

// Bump-allocates 256-byte aligned slices out of a caller workspace.
struct Arena {
    char* base;
    size_t cap;
    size_t used = 0;
    Arena(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
    static size_t round(size_t n) { return (n + 255) & ~size_t(255); }
    template <typename T>
    T* take(size_t count) {
        const size_t bytes = round(count * sizeof(T));
        if (used + bytes > cap) return nullptr;
        T* p = reinterpret_cast<T*>(base + used);
        used += bytes;
        return p;
    }
};

// ---------------------------------------------------------- vector math --
struct v3 {
    float x, y, z;
};
__host__ __device__ __forceinline__ v3 mk3(float x, float y, float z) { return {x, y, z}; }
__host__ __device__ __forceinline__ v3 operator+(v3 a, v3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
__host__ __device__ __forceinline__ v3 operator-(v3 a, v3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
__host__ __device__ __forceinline__ v3 operator*(float s, v3 a) { return {s * a.x, s * a.y, s * a.z}; }
__host__ __device__ __forceinline__ v3 operator*(v3 a, float s) { return {a.x * s, a.y * s, a.z * s}; }
__host__ __device__ __forceinline__ float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
// component order as glm::cross
__host__ __device__ __forceinline__ v3 cross3(v3 a, v3 b) {
    return {a.y * b.z - b.y * a.z, a.z * b.x - b.z * a.x, a.x * b.y - b.x * a.y};
}

__device__ __forceinline__ v3 ld3(const float* p) { return {p[0], p[1], p[2]}; }
__device__ __forceinline__ void st3(float* p, v3 v) { p[0] = v.x; p[1] = v.y; p[2] = v.z; }

// Vector reduction into global memory (sm_90+): one instruction, four floats.
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

}  // namespace xsg
