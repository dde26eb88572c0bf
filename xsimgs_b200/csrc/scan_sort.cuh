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
constexpr int kSortThreads = 256;
constexpr int kSortRounds = 16;
constexpr int kSortChunk = kSortThreads * kSortRounds;  // items per block
constexpr int kRadixBits = 8;
constexpr int kRadixBins = 1 << kRadixBits;

inline int64_t sort_blocks(int64_t n) { return (n + kSortChunk - 1) / kSortChunk; }

__global__ void __launch_bounds__(kSortThreads)
    radix_hist_kernel(const uint32_t* __restrict__ keys, int64_t n, int shift, int32_t* __restrict__ counts,
                      int64_t nblocks) {
    __shared__ int32_t h[kRadixBins];
    h[threadIdx.x] = 0;
    __syncthreads();
    const int64_t base = int64_t(blockIdx.x) * kSortChunk;
#pragma unroll 4
    for (int r = 0; r < kSortRounds; ++r) {
        const int64_t i = base + int64_t(r) * kSortThreads + threadIdx.x;
        if (i < n) atomicAdd(&h[(keys[i] >> shift) & (kRadixBins - 1)], 1);
    }
    __syncthreads();
    counts[int64_t(threadIdx.x) * nblocks + blockIdx.x] = h[threadIdx.x];
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
    radix_scatter_kernel(const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                         int64_t n, int shift, const int64_t* __restrict__ offsets, int64_t nblocks,
                         uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
                         IsectEpilogue ep) {
    __shared__ int64_t running[kRadixBins];
    __shared__ int32_t wc[kSortThreads / 32][kRadixBins];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    running[threadIdx.x] = offsets[int64_t(threadIdx.x) * nblocks + blockIdx.x];
    const int64_t base = int64_t(blockIdx.x) * kSortChunk;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int r = 0; r < kSortRounds; ++r) {
        const int64_t i = base + int64_t(r) * kSortThreads + threadIdx.x;
        if (base + int64_t(r) * kSortThreads >= n) break;  // uniform across the block
#pragma unroll
        for (int w = 0; w < kSortThreads / 32; ++w) wc[w][threadIdx.x] = 0;
        __syncthreads();
        const bool ok = i < n;
        uint32_t key = 0, val = 0;
        int digit = kRadixBins;  // sentinel for out-of-range lanes
        if (ok) {
            key = keys_in[i];
            val = vals_in[i];
            digit = (key >> shift) & (kRadixBins - 1);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, digit);
        const int rank = __popc(peers & lt_mask);
        if (ok && rank == 0) wc[wid][digit] = __popc(peers);
        __syncthreads();
        {
            int64_t s = running[threadIdx.x];
#pragma unroll
            for (int w = 0; w < kSortThreads / 32; ++w) {
                const int32_t c = wc[w][threadIdx.x];
                wc[w][threadIdx.x] = int32_t(s - running[threadIdx.x]);
                s += c;
            }
            // wc now holds offsets relative to running[]; store the new total
            __syncthreads();
            if (ok) {
                const int64_t pos = running[digit] + wc[wid][digit] + rank;
                if constexpr (kIsect) {
                    const int32_t bits = __float_as_int(ep.depths[val]);
                    // negative depths: the sign extension fills the tile bits
                    const uint64_t hi = bits < 0 ? 0xFFFFFFFF00000000ull : (uint64_t(key) << 32);
                    ep.isect_ids[pos] = int64_t(hi | uint64_t(uint32_t(bits)));
                    ep.flatten_ids[pos] = int32_t(val);
                } else {
                    keys_out[pos] = key;
                    vals_out[pos] = val;
                }
            }
            __syncthreads();
            running[threadIdx.x] = s;
        }
        __syncthreads();
    }
}

inline size_t radix_workspace_bytes(int64_t n) {
    const int64_t nb = sort_blocks(n);
    return Arena::round(size_t(nb) * kRadixBins * sizeof(int32_t)) +
           Arena::round(size_t(nb) * kRadixBins * sizeof(int64_t)) +
           scan_workspace_bytes(nb * kRadixBins);
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
    const int64_t nb = sort_blocks(n);
    Arena a(tmp, tmp_bytes);
    int32_t* counts = a.take<int32_t>(size_t(nb) * kRadixBins);
    int64_t* offs = a.take<int64_t>(size_t(nb) * kRadixBins);
    void* stmp = a.take<char>(scan_workspace_bytes(nb * kRadixBins));
    if (!counts || !offs || !stmp) return set_error(XSG_ERR_WORKSPACE, "radix sort: workspace too small");
    const int passes = (bits + kRadixBits - 1) / kRadixBits;
    IsectEpilogue none{};
    for (int p = 0; p < passes; ++p) {
        const int shift = p * kRadixBits;
        launch(radix_hist_kernel, unsigned(nb), kSortThreads, 0, st, keys, n, shift, counts, nb);
        int rc = exclusive_scan<int32_t>(counts, nb * kRadixBins, offs, nullptr, stmp, st);
        if (rc != XSG_OK) return rc;
        const bool last = (p == passes - 1);
        if (last && ep) {
            launch(radix_scatter_kernel<true>, unsigned(nb), kSortThreads, 0, st, 
                keys, vals, n, shift, offs, nb, nullptr, nullptr, *ep);
        } else {
            launch(radix_scatter_kernel<false>, unsigned(nb), kSortThreads, 0, st, 
                keys, vals, n, shift, offs, nb, keys_alt, vals_alt, none);
            uint32_t* t = keys; keys = keys_alt; keys_alt = t;
            t = vals; vals = vals_alt; vals_alt = t;
        }
    }
    if (keys_res) *keys_res = keys;
    if (vals_res) *vals_res = vals;
    return check_launch("radix_sort_pairs");
}

}  // namespace xsg
