// Device-wide exclusive scan and stable counting-sort passes of (u32 key,
// u32 value) pairs, written for this library (no CUB).  Used by tile
// intersection: a depth presort of the visible Gaussians and a stable bucket
// sort of intersections by tile.
#pragma once

#include "common.cuh"

namespace xsg {

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;                         // per thread
constexpr int kScanChunk = kScanThreads * kScanItems;  // per block

__device__ __forceinline__ int64_t warp_incl_scan(int64_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total to *total.
__device__ __forceinline__ int64_t block_excl_scan(int64_t v, int64_t* total) {
    __shared__ int64_t warp_sums[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    const int64_t inc = warp_incl_scan(v);
    if (lane == 31) warp_sums[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        int64_t s = lane < nw ? warp_sums[lane] : 0;
        s = warp_incl_scan(s);
        if (lane < nw) warp_sums[lane] = s;
    }
    __syncthreads();
    const int64_t base = wid > 0 ? warp_sums[wid - 1] : 0;
    *total = warp_sums[nw - 1];
    __syncthreads();
    return base + inc - v;
}

// Phase 1: per-block sums of `in` (T = int32 or int64), optionally of a
// predicate (in[i] > 0).
// n_dev (optional) holds the element count on the device; the grid is then
// sized for its upper bound n.
template <typename T, bool kPred>
__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const T* __restrict__ in, int64_t n,
                                                                   int64_t* __restrict__ block_sums,
                                                                   const int64_t* __restrict__ n_dev) {
    pdl_wait();
    pdl_trigger();
    if (n_dev) n = *n_dev;
    const int64_t base = int64_t(blockIdx.x) * kScanChunk;
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + int64_t(k) * kScanThreads + threadIdx.x;
        if (i < n) s += kPred ? (in[i] > 0 ? 1 : 0) : int64_t(in[i]);
    }
    int64_t total;
    block_excl_scan(s, &total);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// Phase 3: exclusive scan inside each block plus the block offset.
// Items are processed in blocked order (thread t owns kScanItems
// consecutive elements).  out may alias nothing.  If total != nullptr the
// grand total is written by the last block.
template <typename T, bool kPred>
__global__ void __launch_bounds__(kScanThreads)
    scan_apply_kernel(const T* __restrict__ in, int64_t n, const int64_t* __restrict__ block_offsets,
                      int64_t* __restrict__ out, int64_t* __restrict__ total, const int64_t* __restrict__ n_dev) {
    pdl_wait();
    pdl_trigger();
    if (n_dev) n = *n_dev;
    const int64_t base = int64_t(blockIdx.x) * kScanChunk + int64_t(threadIdx.x) * kScanItems;
    int64_t vals[kScanItems];
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k;
        vals[k] = (i < n) ? (kPred ? (in[i] > 0 ? 1 : 0) : int64_t(in[i])) : 0;
        s += vals[k];
    }
    int64_t btotal;
    int64_t run = block_excl_scan(s, &btotal) + block_offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k;
        if (i < n) out[i] = run;
        run += vals[k];
    }
    if (total && blockIdx.x == gridDim.x - 1 && threadIdx.x == blockDim.x - 1) *total = run;
}

// Single-block exclusive scan of up to any length (loops in chunks).
__global__ void __launch_bounds__(1024) scan_small_kernel(int64_t* __restrict__ v, int64_t n) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const int64_t x = i < n ? v[i] : 0;
        int64_t total;
        const int64_t ex = block_excl_scan(x, &total);
        const int64_t c = carry;
        if (i < n) v[i] = ex + c;
        __syncthreads();
        if (threadIdx.x == 0) carry = c + total;
        __syncthreads();
    }
}

inline size_t scan_workspace_bytes(int64_t n) {
    const int64_t nb = (n + kScanChunk - 1) / kScanChunk;
    return Arena::round(size_t(nb + 1) * sizeof(int64_t));
}

// Exclusive scan of n values into out (int64).  `total` (device, may be
// null) receives the sum.  tmp needs scan_workspace_bytes(n).
// With n_dev the count is read on the device (at most n; out is written
// for the first *n_dev elements only).
template <typename T, bool kPred = false>
int exclusive_scan(const T* in, int64_t n, int64_t* out, int64_t* total, void* tmp,
                   cudaStream_t st, const int64_t* n_dev = nullptr) {
    if (n == 0) {
        if (total) XSG_CUDA(cudaMemsetAsync(total, 0, sizeof(int64_t), st));
        return XSG_OK;
    }
    const int64_t nb = (n + kScanChunk - 1) / kScanChunk;
    int64_t* bs = static_cast<int64_t*>(tmp);
    launch_pdl(scan_reduce_kernel<T, kPred>, unsigned(nb), kScanThreads, 0, st, in, n, bs, n_dev);
    launch_pdl(scan_small_kernel, 1, 1024, 0, st, bs, nb);
    launch_pdl(scan_apply_kernel<T, kPred>, unsigned(nb), kScanThreads, 0, st, in, n, static_cast<const int64_t*>(bs),
           out, total, n_dev);
    return check_launch("exclusive_scan");
}

// Output mode of the final scatter of the tile sort: keys become the
// reference's 64-bit isect ids (tile << 32 | sign-extended depth bits).
struct IsectEpilogue {
    const float* depths;     // per Gaussian
    int64_t* isect_ids;      // out
    int32_t* flatten_ids;    // out
};

// ------------------------------------------------------ counting pass --
// One stable counting-sort pass of (u32 key, u32 value) pairs on a digit of
// the key (at most kCsMaxBins values).  Warp w (one warp per CTA) owns the
// contiguous input range [w * per, (w + 1) * per):
//   1. hist:    it counts its digits in its own shared-memory bins;
//   2. offsets: every (bin, warp) gets its first output position;
//   3. scatter: the warp walks its range 32 keys at a time, in order: lanes
//               with equal digits are grouped with a match and ranked by
//               lane, and the group's leader advances the bin's cursor.
// Ranges are visited in order inside every bin, so the pass is stable.
// Narrow digits (<= kCsNarrowBins values) use many short ranges and a
// bin-major count array scanned as a whole; wide digits use fewer, longer
// ranges, a warp-major array, a column scan per bin and a scan of the bin
// totals.  The element count may live on the device (n_dev, at most n).
constexpr int kCsMaxBins = 8192;
constexpr int kCsNarrowBins = 256;

struct CsPlan {
    int max_warps, min_per;
};
__host__ __device__ constexpr CsPlan cs_plan(int nbins) {
    return nbins <= kCsNarrowBins ? CsPlan{148 * 32, 512} : CsPlan{4 * 148, 2048};
}

struct CsDigit {
    int shift;
    uint32_t mask;
    __device__ __forceinline__ int operator()(uint32_t k) const { return int((k >> shift) & mask); }
};

__device__ __forceinline__ void cs_range(int64_t n, int64_t& i0, int64_t& i1) {
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    i0 = int64_t(blockIdx.x) * per;
    i1 = min(n, i0 + per);
}

// counts[b * G + w] (bin-major) or counts[w * nbins + b] (warp-major)
template <bool kBinMajor>
__global__ void __launch_bounds__(32)
    cs_hist_kernel(const uint2* __restrict__ kv, int64_t n, const int64_t* __restrict__ n_dev, CsDigit dg,
                   int nbins, int32_t* __restrict__ counts) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ int32_t h[];
    const int lane = threadIdx.x;
    if (n_dev) n = *n_dev;
    for (int b = lane; b < nbins; b += 32) h[b] = 0;
    __syncwarp();
    int64_t i0, i1;
    cs_range(n, i0, i1);
    for (int64_t i = i0 + lane; i < i1; i += 32) atomicAdd(h + dg(kv[i].x), 1);
    __syncwarp();
    for (int b = lane; b < nbins; b += 32)
        counts[kBinMajor ? int64_t(b) * gridDim.x + blockIdx.x : int64_t(blockIdx.x) * nbins + b] = h[b];
}

// Wide digits: block (32 bins) x (32 warp groups); thread (g, c) owns warps
// [g R, (g + 1) R) of bin b0 + c (coalesced across c), sums them, the 32
// group sums of a bin are scanned in shared memory, then the warps' offsets
// inside the bin (offs, warp-major) and the bin totals are written.
constexpr int kCsColRows = (4 * 148 + 31) / 32;
__global__ void __launch_bounds__(1024)
    cs_colscan_kernel(const int32_t* __restrict__ counts, int G, int nbins, int32_t* __restrict__ offs,
                      int64_t* __restrict__ totals) {
    pdl_wait();
    pdl_trigger();
    __shared__ int32_t part[32][33];
    const int c = threadIdx.x & 31, g = threadIdx.x >> 5;
    const int b = blockIdx.x * 32 + c;
    const int R = (G + 31) / 32;
    const int w0 = g * R, w1 = min(G, w0 + R);
    int32_t v[kCsColRows];
    int32_t sum = 0;
#pragma unroll
    for (int r = 0; r < kCsColRows; ++r) {
        const int w = w0 + r;
        v[r] = (r < R && w < w1 && b < nbins) ? counts[int64_t(w) * nbins + b] : 0;
        sum += v[r];
    }
    part[g][c] = sum;
    __syncthreads();
    if (g == 0) {
        int32_t run = 0;
        for (int k = 0; k < 32; ++k) {
            const int32_t t = part[k][c];
            part[k][c] = run;
            run += t;
        }
        if (b < nbins) totals[b] = run;
    }
    __syncthreads();
    int32_t run = part[g][c];
#pragma unroll
    for (int r = 0; r < kCsColRows; ++r) {
        const int w = w0 + r;
        if (r < R && w < w1 && b < nbins) offs[int64_t(w) * nbins + b] = run;
        run += v[r];
    }
}

// starts[b] = totals[< b]; one CTA.
__global__ void __launch_bounds__(1024) cs_starts_kernel(const int64_t* __restrict__ totals, int nbins,
                                                         int64_t* __restrict__ starts) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < nbins; base += blockDim.x) {
        const int b = base + threadIdx.x;
        int64_t tot;
        const int64_t ex = block_excl_scan(b < nbins ? totals[b] : 0, &tot);
        const int64_t c = carry;
        if (b < nbins) starts[b] = c + ex;
        __syncthreads();
        if (threadIdx.x == 0) carry = c + tot;
        __syncthreads();
    }
}

// Cursor of (bin b, this warp): pos0[b * G + w] (narrow digits) or
// starts[b] + offs[w * nbins + b] (wide digits).
template <bool kBinMajor, bool kIsect>
__global__ void __launch_bounds__(32)
    cs_scatter_kernel(const uint2* __restrict__ kv, int64_t n, const int64_t* __restrict__ n_dev, CsDigit dg,
                      int nbins, const int64_t* __restrict__ pos0, const int32_t* __restrict__ offs,
                      const int64_t* __restrict__ starts, uint2* __restrict__ kv_out, IsectEpilogue ep) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ int32_t cur[];  // positions < n < 2^31
    const int lane = threadIdx.x;
    if (n_dev) n = *n_dev;
    for (int b = lane; b < nbins; b += 32)
        cur[b] = kBinMajor ? int32_t(pos0[int64_t(b) * gridDim.x + blockIdx.x])
                           : int32_t(starts[b]) + offs[int64_t(blockIdx.x) * nbins + b];
    __syncwarp();
    int64_t i0, i1;
    cs_range(n, i0, i1);
    const unsigned lt = (1u << lane) - 1u;
    constexpr int kB = 16;  // rounds whose loads are issued together
    for (int64_t base = i0; base < i1; base += 32 * kB) {
        uint32_t kk[kB], vv[kB];
        float dd[kB];
#pragma unroll
        for (int r = 0; r < kB; ++r) {
            const int64_t i = base + 32 * r + lane;
            const uint2 e = i < i1 ? kv[i] : make_uint2(0u, 0u);
            kk[r] = e.x;
            vv[r] = e.y;
        }
        if constexpr (kIsect) {
#pragma unroll
            for (int r = 0; r < kB; ++r) dd[r] = (base + 32 * r + lane < i1) ? ep.depths[vv[r]] : 0.f;
        }
#pragma unroll
        for (int r = 0; r < kB; ++r) {
            const bool ok = base + 32 * r + lane < i1;
            const int d = ok ? dg(kk[r]) : nbins;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            const int leader = __ffs(peers) - 1;
            int32_t p0 = 0;
            if (ok && lane == leader) {
                p0 = cur[d];
                cur[d] = p0 + __popc(peers);
            }
            p0 = __shfl_sync(0xffffffffu, p0, leader);
            __syncwarp();
            if (ok) {
                const int32_t pos = p0 + __popc(peers & lt);
                if constexpr (kIsect) {
                    const int32_t bits = __float_as_int(dd[r]);
                    const uint64_t hi = bits < 0 ? 0xFFFFFFFF00000000ull : (uint64_t(kk[r]) << 32);
                    ep.isect_ids[pos] = int64_t(hi | uint64_t(uint32_t(bits)));
                    ep.flatten_ids[pos] = int32_t(vv[r]);
                } else {
                    kv_out[pos] = make_uint2(kk[r], vv[r]);
                }
            }
        }
    }
}

inline int cs_warps(int64_t n, int nbins) {
    const CsPlan pl = cs_plan(nbins);
    const int64_t want = (n + pl.min_per - 1) / pl.min_per;
    return int(want < 1 ? 1 : (want > pl.max_warps ? pl.max_warps : want));
}

// Scratch of a pass over at most n keys with nbins bins.
inline size_t cs_workspace_bytes(int64_t n, int nbins) {
    const int64_t mat = int64_t(cs_warps(n, nbins)) * nbins;
    if (nbins <= kCsNarrowBins)
        return Arena::round(size_t(mat) * sizeof(int32_t)) + Arena::round(size_t(mat + 1) * sizeof(int64_t)) +
               scan_workspace_bytes(mat);
    return 2 * Arena::round(size_t(mat) * sizeof(int32_t)) + 2 * Arena::round(size_t(nbins + 1) * sizeof(int64_t));
}

// One stable pass of `n` (upper bound; the count itself at n_dev when given)
// (key, value) pairs, stored interleaved (one 8-byte word each, so a scatter
// is one store per pair), on digit dg with nbins values into kv_out, or with
// `ep` into the 64-bit isect ids and flatten ids.
inline int counting_pass(const uint2* kv, uint2* kv_out, int64_t n, const int64_t* n_dev, CsDigit dg, int nbins,
                         void* tmp, size_t tmp_bytes, cudaStream_t st, const IsectEpilogue* ep) {
    if (n <= 0) return XSG_OK;
    if (nbins > kCsMaxBins) return set_error(XSG_ERR_UNSUPPORTED, "counting pass: too many bins");
    static bool attrs_set[64] = {};
    int dev = 0;
    XSG_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !attrs_set[dev]) {
        const int sm = int(kCsMaxBins * sizeof(int32_t));
        XSG_CUDA(cudaFuncSetAttribute(cs_hist_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
        XSG_CUDA(cudaFuncSetAttribute(cs_scatter_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      sm));
        XSG_CUDA(cudaFuncSetAttribute(cs_scatter_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      sm));
        attrs_set[dev] = true;
    }
    const int G = cs_warps(n, nbins);
    const int64_t mat = int64_t(G) * nbins;
    const size_t smem = size_t(nbins) * sizeof(int32_t);
    Arena a(tmp, tmp_bytes);
    IsectEpilogue none{};
    const IsectEpilogue& e = ep ? *ep : none;
    int32_t* counts = a.take<int32_t>(size_t(mat));
    if (nbins <= kCsNarrowBins) {
        int64_t* pos0 = a.take<int64_t>(size_t(mat + 1));
        void* stmp = a.take<char>(scan_workspace_bytes(mat));
        if (!counts || !pos0 || !stmp) return set_error(XSG_ERR_WORKSPACE, "counting pass: workspace too small");
        launch_pdl(cs_hist_kernel<true>, G, 32, smem, st, kv, n, n_dev, dg, nbins, counts);
        int rc = exclusive_scan<int32_t>(counts, mat, pos0, nullptr, stmp, st);
        if (rc != XSG_OK) return rc;
        const int64_t* p0 = pos0;
        launch_pdl(ep ? cs_scatter_kernel<true, true> : cs_scatter_kernel<true, false>, G, 32, smem, st, kv, n,
                   n_dev, dg, nbins, p0, static_cast<const int32_t*>(nullptr), static_cast<const int64_t*>(nullptr),
                   ep ? nullptr : kv_out, e);
        return check_launch("counting_pass");
    }
    int32_t* offs = a.take<int32_t>(size_t(mat));
    int64_t* totals = a.take<int64_t>(size_t(nbins + 1));
    int64_t* starts = a.take<int64_t>(size_t(nbins + 1));
    if (!counts || !offs || !totals || !starts) return set_error(XSG_ERR_WORKSPACE, "counting pass: workspace too small");
    launch_pdl(cs_hist_kernel<false>, G, 32, smem, st, kv, n, n_dev, dg, nbins, counts);
    launch_pdl(cs_colscan_kernel, unsigned((nbins + 31) / 32), 1024, 0, st, static_cast<const int32_t*>(counts), G,
           nbins, offs, totals);
    launch_pdl(cs_starts_kernel, 1, 1024, 0, st, static_cast<const int64_t*>(totals), nbins, starts);
    const int32_t* of = offs;
    const int64_t* sts = starts;
    launch_pdl(ep ? cs_scatter_kernel<false, true> : cs_scatter_kernel<false, false>, G, 32, smem, st, kv, n, n_dev,
               dg, nbins, static_cast<const int64_t*>(nullptr), of, sts, ep ? nullptr : kv_out, e);
    return check_launch("counting_pass");
}

}  // namespace xsg
