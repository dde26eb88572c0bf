// Device-wide exclusive scan and a stable LSD radix sort of (u32 key, u32
// value) pairs, written for this library (no CUB).  Used by tile
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
template <typename T, bool kPred>
__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const T* __restrict__ in, int64_t n,
                                                                   int64_t* __restrict__ block_sums) {
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
                      int64_t* __restrict__ out, int64_t* __restrict__ total) {
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
template <typename T, bool kPred = false>
int exclusive_scan(const T* in, int64_t n, int64_t* out, int64_t* total, void* tmp,
                   cudaStream_t st) {
    if (n == 0) {
        if (total) XSG_CUDA(cudaMemsetAsync(total, 0, sizeof(int64_t), st));
        return XSG_OK;
    }
    const int64_t nb = (n + kScanChunk - 1) / kScanChunk;
    int64_t* bs = static_cast<int64_t*>(tmp);
    launch(scan_reduce_kernel<T, kPred>, unsigned(nb), kScanThreads, 0, st, in, n, bs);
    launch(scan_small_kernel, 1, 1024, 0, st, bs, nb);
    launch(scan_apply_kernel<T, kPred>, unsigned(nb), kScanThreads, 0, st, in, n, bs, out, total);
    return check_launch("exclusive_scan");
}

// ---------------------------------------------------------------- radix --
// Stable LSD radix sort, 8-bit digits, warp-granular: the input is cut into
// warp chunks of 32 x R consecutive keys (R = 16 or 64).  Per pass:
//   1. hist:     every warp counts the digits of its chunk in its own
//                shared-memory counters -> counts[digit][chunk];
//   2. row scan: one CTA per digit scans its row over the chunks ->
//                offsets[digit][chunk] (within the digit) and totals[digit];
//   3. scatter:  every warp walks its chunk in order, 32 keys at a time,
//                ranks equal digits among its lanes and keeps its own
//                per-digit cursor in shared memory; the digit bases come
//                from a scan of the 256 totals.  No block-wide barrier
//                inside the loop; keys are prefetched 16 rounds at a time.
// Warp chunks are processed in input order inside each digit, so the sort
// is stable.
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kRadixBits = 8;
constexpr int kRadixBins = 1 << kRadixBits;
constexpr int kRxBatch = 16;  // rounds prefetched together

inline int sort_rounds(int64_t n) { return n > (int64_t(4) << 20) ? 64 : 16; }
inline int64_t sort_chunks(int64_t n) {
    const int64_t per = int64_t(32) * sort_rounds(n);
    return (n + per - 1) / per;
}

// Lanes of the warp holding the same digit (0..255, or 256 for a lane past
// the end): nine ballots, constant time whatever the digits are.
__device__ __forceinline__ unsigned match_digit(int digit) {
    unsigned m = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < kRadixBits + 1; ++b) {
        const bool bit = (digit >> b) & 1;
        const unsigned bal = __ballot_sync(0xffffffffu, bit);
        m &= bit ? bal : ~bal;
    }
    return m;
}

__global__ void __launch_bounds__(kSortThreads)
    radix_hist_kernel(const uint32_t* __restrict__ keys, int64_t n, int shift, int rounds,
                      int32_t* __restrict__ counts, int64_t nchunks) {
    __shared__ int32_t h[kSortWarps][kRadixBins];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t c = int64_t(blockIdx.x) * kSortWarps + w;
    if (c >= nchunks) return;  // warp-uniform; no block barrier below
#pragma unroll
    for (int k = 0; k < kRadixBins / 32; ++k) h[w][lane + 32 * k] = 0;
    __syncwarp();
    const int64_t base = c * 32 * rounds;
    for (int b = 0; b < rounds; b += kRxBatch) {
        int dg[kRxBatch];
#pragma unroll
        for (int r = 0; r < kRxBatch; ++r) {
            const int64_t i = base + int64_t(b + r) * 32 + lane;
            dg[r] = i < n ? int((keys[i] >> shift) & (kRadixBins - 1)) : kRadixBins;
        }
#pragma unroll
        for (int r = 0; r < kRxBatch; ++r) {
            const unsigned peers = match_digit(dg[r]);
            if (dg[r] < kRadixBins && lane == __ffs(peers) - 1) h[w][dg[r]] += __popc(peers);
            __syncwarp();
        }
    }
#pragma unroll
    for (int k = 0; k < kRadixBins / 32; ++k) {
        const int d = lane + 32 * k;
        counts[int64_t(d) * nchunks + c] = h[w][d];
    }
}

// One CTA per digit: exclusive scan of counts[d][*] -> offsets[d][*], eight
// consecutive chunks per thread.
constexpr int kRowItems = 8;
__global__ void __launch_bounds__(1024)
    radix_rowscan_kernel(const int32_t* __restrict__ counts, int64_t nchunks, int32_t* __restrict__ offsets,
                         int64_t* __restrict__ totals) {
    __shared__ int64_t carry;
    const int64_t d = blockIdx.x;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int32_t* row = counts + d * nchunks;
    int32_t* orow = offsets + d * nchunks;
    const int64_t span = int64_t(blockDim.x) * kRowItems;
    for (int64_t b = 0; b < nchunks; b += span) {
        const int64_t i0 = b + int64_t(threadIdx.x) * kRowItems;
        int32_t v[kRowItems];
        int64_t s = 0;
#pragma unroll
        for (int k = 0; k < kRowItems; ++k) {
            v[k] = (i0 + k < nchunks) ? row[i0 + k] : 0;
            s += v[k];
        }
        int64_t tot;
        int64_t run = block_excl_scan(s, &tot) + carry;
#pragma unroll
        for (int k = 0; k < kRowItems; ++k) {
            if (i0 + k < nchunks) orow[i0 + k] = int32_t(run);
            run += v[k];
        }
        __syncthreads();
        if (threadIdx.x == 0) carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) totals[d] = carry;
}

// Output mode of the final scatter of the tile sort: keys become the
// reference's 64-bit isect ids (tile << 32 | sign-extended depth bits).
struct IsectEpilogue {
    const float* depths;     // per Gaussian
    int64_t* isect_ids;      // out
    int32_t* flatten_ids;    // out
};

template <bool kIsect>
__global__ void __launch_bounds__(kSortThreads)
    radix_scatter_kernel(const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in, int64_t n,
                         int shift, int rounds, const int32_t* __restrict__ offsets,
                         const int64_t* __restrict__ totals, int64_t nchunks, uint32_t* __restrict__ keys_out,
                         uint32_t* __restrict__ vals_out, IsectEpilogue ep) {
    __shared__ int64_t dbase[kRadixBins];
    __shared__ int64_t cur[kSortWarps][kRadixBins];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    // digit bases: exclusive scan of the 256 digit totals (one per thread)
    {
        int64_t tot;
        dbase[threadIdx.x] = block_excl_scan(totals[threadIdx.x], &tot);
    }
    __syncthreads();
    const int64_t c = int64_t(blockIdx.x) * kSortWarps + w;
    if (c >= nchunks) return;  // warp-uniform; no block barrier below
#pragma unroll
    for (int k = 0; k < kRadixBins / 32; ++k) {
        const int d = lane + 32 * k;
        cur[w][d] = dbase[d] + offsets[int64_t(d) * nchunks + c];
    }
    __syncwarp();
    const unsigned lt = (1u << lane) - 1u;
    const int64_t base = c * 32 * rounds;
    for (int b = 0; b < rounds; b += kRxBatch) {
        uint32_t kk[kRxBatch], vv[kRxBatch];
#pragma unroll
        for (int r = 0; r < kRxBatch; ++r) {
            const int64_t i = base + int64_t(b + r) * 32 + lane;
            kk[r] = i < n ? keys_in[i] : 0u;
            vv[r] = i < n ? vals_in[i] : 0u;
        }
#pragma unroll
        for (int r = 0; r < kRxBatch; ++r) {
            const int64_t i = base + int64_t(b + r) * 32 + lane;
            const bool ok = i < n;
            const int digit = ok ? int((kk[r] >> shift) & (kRadixBins - 1)) : kRadixBins;
            const unsigned peers = match_digit(digit);
            const int leader = __ffs(peers) - 1;
            int64_t p0 = 0;
            if (ok && lane == leader) p0 = cur[w][digit];
            p0 = __shfl_sync(0xffffffffu, p0, leader);
            if (ok && lane == leader) cur[w][digit] = p0 + __popc(peers);
            __syncwarp();
            if (ok) {
                const int64_t pos = p0 + __popc(peers & lt);
                if constexpr (kIsect) {
                    const int32_t bits = __float_as_int(ep.depths[vv[r]]);
                    // negative depths: the sign extension fills the tile bits
                    const uint64_t hi = bits < 0 ? 0xFFFFFFFF00000000ull : (uint64_t(kk[r]) << 32);
                    ep.isect_ids[pos] = int64_t(hi | uint64_t(uint32_t(bits)));
                    ep.flatten_ids[pos] = int32_t(vv[r]);
                } else {
                    keys_out[pos] = kk[r];
                    vals_out[pos] = vv[r];
                }
            }
        }
    }
}

// largest chunk count of any sort of at most n keys
inline int64_t sort_chunks_max(int64_t n) {
    const int64_t small = n < (int64_t(4) << 20) ? n : (int64_t(4) << 20);
    const int64_t a = sort_chunks(n), b = sort_chunks(small);
    return a > b ? a : b;
}

inline size_t radix_workspace_bytes(int64_t n) {
    const int64_t nc = sort_chunks_max(n);
    return 2 * Arena::round(size_t(nc) * kRadixBins * sizeof(int32_t)) +
           Arena::round(size_t(kRadixBins) * sizeof(int64_t));
}

// Stable ascending sort of (key, value) pairs on key bits [0, bits).
// keys/vals and keys_alt/vals_alt are ping-pong buffers; the sorted result
// is returned in *keys_res / *vals_res (one of the two).  With `ep` given the
// final pass writes 64-bit isect ids and flatten ids instead.
inline int radix_sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* keys_alt, uint32_t* vals_alt,
                            int64_t n, int bits, void* tmp, size_t tmp_bytes, cudaStream_t st,
                            const IsectEpilogue* ep, uint32_t** keys_res, uint32_t** vals_res) {
    if (keys_res) *keys_res = keys;
    if (vals_res) *vals_res = vals;
    if (n == 0) return XSG_OK;
    if (n >= (int64_t(1) << 31)) return set_error(XSG_ERR_UNSUPPORTED, "radix sort: 2^31 or more keys");
    const int64_t nc = sort_chunks(n);
    const int rounds = sort_rounds(n);
    Arena a(tmp, tmp_bytes);
    int32_t* counts = a.take<int32_t>(size_t(nc) * kRadixBins);
    int32_t* offs = a.take<int32_t>(size_t(nc) * kRadixBins);
    int64_t* totals = a.take<int64_t>(kRadixBins);
    if (!counts || !offs || !totals) return set_error(XSG_ERR_WORKSPACE, "radix sort: workspace too small");
    const unsigned grid = unsigned((nc + kSortWarps - 1) / kSortWarps);
    const int passes = (bits + kRadixBits - 1) / kRadixBits;
    IsectEpilogue none{};
    for (int p = 0; p < passes; ++p) {
        const int shift = p * kRadixBits;
        launch(radix_hist_kernel, grid, kSortThreads, 0, st, keys, n, shift, rounds, counts, nc);
        launch(radix_rowscan_kernel, kRadixBins, 1024, 0, st, counts, nc, offs, totals);
        const bool last = (p == passes - 1);
        if (last && ep) {
            launch(radix_scatter_kernel<true>, grid, kSortThreads, 0, st, keys, vals, n, shift, rounds, offs,
                   totals, nc, nullptr, nullptr, *ep);
        } else {
            launch(radix_scatter_kernel<false>, grid, kSortThreads, 0, st, keys, vals, n, shift, rounds, offs,
                   totals, nc, keys_alt, vals_alt, none);
            uint32_t* t = keys; keys = keys_alt; keys_alt = t;
            t = vals; vals = vals_alt; vals_alt = t;
        }
    }
    if (keys_res) *keys_res = keys;
    if (vals_res) *vals_res = vals;
    return check_launch("radix_sort_pairs");
}

}  // namespace xsg
