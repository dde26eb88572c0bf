// Error reporting of the C ABI (a thread-local message per failing call),
// the launch counter and the optional per-kernel device timers.
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace xsg {

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(XSG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return XSG_OK;
}

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

struct TimerRec {
    std::string name;
    cudaEvent_t a, b;
};
static std::mutex g_tmu;
static bool g_timing = false;
static std::vector<TimerRec> g_timers;

ScopedTimer::ScopedTimer(const char* name, cudaStream_t stream) : st(stream) {
    std::lock_guard<std::mutex> lk(g_tmu);
    if (!g_timing) return;
    TimerRec r{name, nullptr, nullptr};
    if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return;
    cudaEventRecord(r.a, st);
    g_timers.push_back(r);
    slot = int(g_timers.size()) - 1;
}

ScopedTimer::~ScopedTimer() {
    if (slot < 0) return;
    std::lock_guard<std::mutex> lk(g_tmu);
    if (slot < int(g_timers.size())) cudaEventRecord(g_timers[slot].b, st);
}

}  // namespace xsg

extern "C" {

long long xsg_launch_count(void) { return xsg::g_launches.load(); }

void xsg_timing_enable(int on) {
    std::lock_guard<std::mutex> lk(xsg::g_tmu);
    xsg::g_timing = on != 0;
}

void xsg_timing_reset(void) {
    std::lock_guard<std::mutex> lk(xsg::g_tmu);
    for (auto& r : xsg::g_timers) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    xsg::g_timers.clear();
}

int xsg_timing_query(const char* name, double* total_ms, long long* launches) {
    std::lock_guard<std::mutex> lk(xsg::g_tmu);
    double tot = 0.0;
    long long cnt = 0;
    for (auto& r : xsg::g_timers) {
        if (r.name != name) continue;
        if (cudaEventSynchronize(r.b) != cudaSuccess) return xsg::set_error(XSG_ERR_CUDA, "timing: event sync failed");
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess)
            return xsg::set_error(XSG_ERR_CUDA, "timing: elapsed time failed");
        tot += ms;
        ++cnt;
    }
    if (total_ms) *total_ms = tot;
    if (launches) *launches = cnt;
    return XSG_OK;
}

const char* xsg_last_error(void) { return xsg::g_last_error.c_str(); }

const char* xsg_version(void) { return "xsimgs-b200 0.1 (sm_100a)"; }

}  // extern "C"

// ------------------------------------------------------------ FP32 probe --
// Peak FP32 FMA throughput of this GPU at its current clocks: every thread
// runs 8 independent FMA chains (enough to cover the FMA latency), so the
// kernel is issue-bound on the FP32 pipe.  Used as the roofline denominator
// of the compositing kernels, which are FP32/MUFU-bound, not HBM-bound.
namespace xsg {
__global__ void __launch_bounds__(512) fma_probe_kernel(float* out, int iters, float s) {
    float a0 = threadIdx.x * 1e-7f, a1 = a0 + 1e-3f, a2 = a0 + 2e-3f, a3 = a0 + 3e-3f;
    float a4 = a0 + 4e-3f, a5 = a0 + 5e-3f, a6 = a0 + 6e-3f, a7 = a0 + 7e-3f;
    const float m = 0.999999f;
#pragma unroll 1
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            a0 = fmaf(a0, m, s); a1 = fmaf(a1, m, s); a2 = fmaf(a2, m, s); a3 = fmaf(a3, m, s);
            a4 = fmaf(a4, m, s); a5 = fmaf(a5, m, s); a6 = fmaf(a6, m, s); a7 = fmaf(a7, m, s);
        }
    }
    const float r = a0 + a1 + a2 + a3 + a4 + a5 + a6 + a7;
    if (r == 1234.5f) out[threadIdx.x] = r;  // keeps the chains alive
}
}  // namespace xsg

extern "C" int xsg_fp32_probe(float* out, int iters, int blocks, xsg_stream_t stream, double* flops) {
    XSG_REQUIRE(out && iters > 0 && blocks > 0, "fp32_probe: bad arguments");
    const int threads = 512;
    xsg::launch(xsg::fma_probe_kernel, blocks, threads, 0, xsg::as_cuda(stream), out, iters, 1e-6f);
    if (flops) *flops = double(blocks) * threads * double(iters) * 16 * 8 * 2;
    return xsg::check_launch("fp32_probe");
}
