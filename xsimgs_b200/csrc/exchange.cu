// Gradient exchange of the multi-GPU render step over NVLink / NVSwitch,
// written as plain kernels on the compute stream (no reference counterpart:
// the reference renders on one GPU).
//
// Buffers are symmetric: every rank allocated the same-sized buffer and the
// NVSwitch maps all copies behind one multicast address (NVLink SHARP).
//   * multimem.ld_reduce at a multicast address returns the sum of the value
//     over every rank's copy (the switch reads and adds them);
//   * multimem.st at a multicast address writes the value into every copy.
// So an all-reduce is: every rank sums its 1/world slice with ld_reduce and
// stores the sum back to all copies with st (each rank's link carries its
// slice once each way); an all-gather is every rank storing its own slice
// into all copies.  A barrier over per-rank flag words (written over NVLink
// with release semantics, polled locally with acquire semantics) brackets
// each exchange: on entry every rank's inputs are written and every rank has
// finished reading the buffer's previous contents; on exit every store has
// landed.  Waits are bounded by a timeout on the global timer, after which the
// kernel records an error (read by the host) and returns.
#include <algorithm>

#include "common.cuh"

namespace xsg {

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// flags[r] points at rank r's flag words (world of them); word s of rank r
// holds the last barrier epoch rank s reached.  Epochs grow by one per
// barrier on every rank, so a word is only ever raised.
__global__ void exchange_barrier_kernel(uint32_t* const* __restrict__ flags, int rank, int world, uint32_t epoch,
                                        uint64_t timeout_ns, int* __restrict__ err) {
    const int t = threadIdx.x;
    if (t >= world) return;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(flags[t] + rank, epoch);
    const uint32_t* mine = flags[rank] + t;
    const uint64_t t0 = global_ns();
    while (int32_t(ld_acquire_sys(mine) - epoch) < 0) {
        if (global_ns() - t0 > timeout_ns) {
            atomicMax(err, 1 + t);  // rank t never arrived
            break;
        }
        __nanosleep(128);
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ float4 mm_ld_reduce_add(uint64_t a) {
    float4 s;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(s.x), "=f"(s.y), "=f"(s.z), "=f"(s.w)
                 : "l"(a)
                 : "memory");
    return s;
}

__device__ __forceinline__ void mm_st(uint64_t a, float4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void mm_st1(uint64_t a, float v) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(a), "f"(v) : "memory");
}

// Rank `rank` reduces 16-byte vectors [v0, v1) of the buffer: four
// ld_reduce in flight per thread, then their stores.
constexpr int kExUnroll = 4;
__global__ void __launch_bounds__(512) nvls_allreduce_kernel(uint64_t mc, int64_t v0, int64_t v1) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t v = v0 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < v1; v += kExUnroll * stride) {
        float4 s[kExUnroll];
#pragma unroll
        for (int u = 0; u < kExUnroll; ++u)
            if (v + u * stride < v1) s[u] = mm_ld_reduce_add(mc + 16 * uint64_t(v + u * stride));
#pragma unroll
        for (int u = 0; u < kExUnroll; ++u)
            if (v + u * stride < v1) mm_st(mc + 16 * uint64_t(v + u * stride), s[u]);
    }
}

// Local src -> every rank's copy at the multicast address dst.
__global__ void __launch_bounds__(512) nvls_broadcast_v4_kernel(const float4* __restrict__ src, uint64_t dst,
                                                                int64_t n_vec) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < n_vec; v += kExUnroll * stride) {
        float4 x[kExUnroll];
#pragma unroll
        for (int u = 0; u < kExUnroll; ++u)
            if (v + u * stride < n_vec) x[u] = src[v + u * stride];
#pragma unroll
        for (int u = 0; u < kExUnroll; ++u)
            if (v + u * stride < n_vec) mm_st(dst + 16 * uint64_t(v + u * stride), x[u]);
    }
}

__global__ void __launch_bounds__(512) nvls_broadcast_f32_kernel(const float* __restrict__ src, uint64_t dst,
                                                                 int64_t n) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        mm_st1(dst + 4 * uint64_t(i), src[i]);
}

static int g_exchange_ctas = 0;  // 0: up to 4 per SM

static unsigned exchange_grid(int64_t work) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t cap = g_exchange_ctas > 0 ? g_exchange_ctas : int64_t(sms) * 4;
    const int64_t want = (work + 511) / 512;
    return unsigned(std::max<int64_t>(1, std::min<int64_t>(want, cap)));
}

}  // namespace xsg

using namespace xsg;

extern "C" {

void xsg_exchange_set_max_ctas(int n) { g_exchange_ctas = n > 0 ? n : 0; }

int xsg_exchange_barrier(uint32_t* const* peer_flags, int rank, int world, uint32_t epoch, double timeout_s,
                         int* err, xsg_stream_t stream) {
    XSG_REQUIRE(peer_flags && err && world >= 1 && world <= 64 && rank >= 0 && rank < world && timeout_s > 0,
                "exchange_barrier: bad arguments");
    launch(exchange_barrier_kernel, 1, 64, 0, as_cuda(stream), peer_flags, rank, world, epoch,
           uint64_t(timeout_s * 1e9), err);
    return check_launch("exchange_barrier");
}

int xsg_nvls_allreduce_sum_f32(uint64_t mc_addr, int64_t n, int rank, int world, xsg_stream_t stream) {
    XSG_REQUIRE(mc_addr && mc_addr % 16 == 0 && n >= 0 && n % 4 == 0 && world >= 1 && rank >= 0 && rank < world,
                "nvls_allreduce: the multicast address must be 16-byte aligned and n a multiple of 4");
    const int64_t nv = n / 4;
    const int64_t per = (nv + world - 1) / world;
    const int64_t v0 = std::min<int64_t>(nv, per * rank), v1 = std::min<int64_t>(nv, v0 + per);
    if (v1 > v0)
        launch(nvls_allreduce_kernel, exchange_grid((v1 - v0 + kExUnroll - 1) / kExUnroll), 512, 0,
               as_cuda(stream), mc_addr, v0, v1);
    return check_launch("nvls_allreduce");
}

int xsg_nvls_broadcast_f32(const float* src, uint64_t mc_dst, int64_t n, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && (n == 0 || (src && mc_dst && mc_dst % 4 == 0)), "nvls_broadcast: bad arguments");
    if (n == 0) return XSG_OK;
    cudaStream_t st = as_cuda(stream);
    if (n % 4 == 0 && mc_dst % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0)
        launch(nvls_broadcast_v4_kernel, exchange_grid((n / 4 + kExUnroll - 1) / kExUnroll), 512, 0, st,
               reinterpret_cast<const float4*>(src), mc_dst, n / 4);
    else
        launch(nvls_broadcast_f32_kernel, exchange_grid(n), 512, 0, st, src, mc_dst, n);
    return check_launch("nvls_broadcast");
}

}  // extern "C"
