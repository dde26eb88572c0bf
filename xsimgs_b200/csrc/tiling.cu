// Tile intersection for pinhole/fisheye images (regular 2D tiles) and for
// spherical/lidar range images (azimuth x elevation tiles), the sort of the
// intersections and the per-tile offsets.
//
// Order contract (the reference's cub::DeviceRadixSort::SortPairs on keys
// `tile << 32 | depth bits`, tiling_common.cu:102-162, is a stable sort of
// the emission order, which is Gaussian index then tile row-major):
//   sorted by (tile, depth bits as u32, Gaussian index, tile row-major).
// It is produced here without sorting 64-bit keys:
//   1. the visible Gaussians are compacted and sorted by depth bits with
//      three stable counting passes (so ties keep Gaussian order);
//   2. their intersections are emitted in that order, keyed by tile only;
//   3. stable counting passes on the tile bits move them into tile order,
//      and the last one writes the 64-bit ids and the flatten ids.
// The number of visible Gaussians stays on the device throughout.
// Negative depths (never produced by the projections) would make the
// reference's sign-extended key fill the tile bits; they are keyed with the
// all-ones tile value so the order still matches.
#include <algorithm>

#include "cameras.cuh"
#include "scan_sort.cuh"

namespace xsg {

constexpr int kTileThreads = 256;

__host__ __device__ inline int tile_bits_for(int64_t n_tiles) {
    // floor(log2(float(n))) + 1, as tiling_common.cu:236 computes it
    int b = 0;
    while ((int64_t(1) << (b + 1)) <= n_tiles) ++b;
    return b + 1;
}

// float -> int with the device's saturating conversion (as the reference's
// static_cast<int>(floorf(...)) compiles on sm_100a)
__device__ __forceinline__ int f2i(float v) { return __float2int_rz(v); }

struct Rect {
    int x0, y0, x1, y1;  // [x0, x1) x [y0, y1)
    __device__ __forceinline__ int count() const { return (y1 - y0) * (x1 - x0); }
};

// Tile rectangle of one Gaussian on a regular grid, regular_tiling.cu:34-56
__device__ __forceinline__ bool regular_rect(float2 m, float2 r, float2 ts, int ntx, int nty, Rect& rc) {
    rc = {0, 0, 0, 0};
    if (r.x <= 0 || r.y <= 0) return false;
    const float mx = m.x / ts.x, my = m.y / ts.y;
    const float rx = r.x / ts.x, ry = r.y / ts.y;
    rc.x0 = min(ntx, max(0, f2i(floorf(mx - rx))));
    rc.y0 = min(nty, max(0, f2i(floorf(my - ry))));
    rc.x1 = min(ntx, max(0, f2i(ceilf(mx + rx))));
    rc.y1 = min(nty, max(0, f2i(ceilf(my + ry))));
    return true;
}

// --------------------------------------------------------- regular grid --
// Adds the block's sum of `c` to *total with one atomic per block (a
// per-warp atomic on one address serialises ~n/32 atomics).
__device__ __forceinline__ void block_add_total(int c, unsigned long long* total) {
    __shared__ unsigned long long part[32];
    unsigned long long s = unsigned(c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) part[w] = s;
    __syncthreads();
    if (w == 0) {
        unsigned long long t = lane < int(blockDim.x >> 5) ? part[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0 && t) atomicAdd(total, t);
    }
}

__global__ void __launch_bounds__(kTileThreads)
    regular_count_kernel(const float2* __restrict__ means2d, const float2* __restrict__ radii, int64_t n,
                         float2 ts, int ntx, int nty, int32_t* __restrict__ counts,
                         unsigned long long* __restrict__ total) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    int c = 0;
    if (i < n) {
        Rect rc;
        if (regular_rect(means2d[i], radii[i], ts, ntx, nty, rc)) c = rc.count();
        counts[i] = c;
    }
    // warp-aggregated total
    block_add_total(c, total);
}

// Writes each Gaussian's intersections; with `order` (a permutation of the
// visible Gaussians) in that order and keyed by tile bucket, else in
// Gaussian order with the reference's 64-bit keys.
template <bool kSorted>
__global__ void __launch_bounds__(kTileThreads)
    regular_emit_kernel(const float2* __restrict__ means2d, const float2* __restrict__ radii,
                        const float* __restrict__ depths, int64_t n_items, float2 ts, int ntx, int nty,
                        int bucket_neg, const uint2* __restrict__ order, const int64_t* __restrict__ offsets,
                        uint2* __restrict__ buckets, int64_t* __restrict__ isect_ids,
                        int32_t* __restrict__ flatten_ids, const int64_t* __restrict__ n_dev, int64_t cap) {
    pdl_wait();
    pdl_trigger();
    const int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const bool in = p < (n_dev ? *n_dev : n_items);
    uint32_t g = 0;
    Rect rc{0, 0, 0, 0};
    bool has = false;
    if (in) {
        g = kSorted ? order[p].y : uint32_t(p);
        has = regular_rect(means2d[g], radii[g], ts, ntx, nty, rc);
    }
    const int cnt = has ? rc.count() : 0;
    const int64_t off0 = cnt > 0 ? offsets[p] : 0;
    const int32_t bits = has ? __float_as_int(depths[g]) : 0;
    auto put = [&](int64_t off, int x, int y, int32_t b, uint32_t gg) {
        if (off >= cap) return;  // capacity-bounded output: the rest is dropped, the count says so
        const uint32_t tile = uint32_t(y) * uint32_t(ntx) + uint32_t(x);
        if constexpr (kSorted) {
            buckets[off] = make_uint2(b < 0 ? uint32_t(bucket_neg) : tile, gg);
        } else {
            const uint64_t hi = b < 0 ? 0xFFFFFFFF00000000ull : (uint64_t(tile) << 32);
            isect_ids[off] = int64_t(hi | uint64_t(uint32_t(b)));
            flatten_ids[off] = int32_t(gg);
        }
    };
    // Gaussians with many tiles (close to the camera) are written by the
    // whole warp, one tile per lane, in the same row-major order; the rest by
    // their own lane
    constexpr int kCoop = 16;
    unsigned big = __ballot_sync(0xffffffffu, cnt > kCoop);
    while (big) {
        const int L = __ffs(big) - 1;
        big &= big - 1;
        const int lx0 = __shfl_sync(0xffffffffu, rc.x0, L), ly0 = __shfl_sync(0xffffffffu, rc.y0, L);
        const int lw = __shfl_sync(0xffffffffu, rc.x1 - rc.x0, L), lc = __shfl_sync(0xffffffffu, cnt, L);
        const int64_t lo = __shfl_sync(0xffffffffu, off0, L);
        const int32_t lb = __shfl_sync(0xffffffffu, bits, L);
        const uint32_t lg = __shfl_sync(0xffffffffu, g, L);
        for (int j = lane; j < lc; j += 32) {
            const int yy = j / lw;
            put(lo + j, lx0 + (j - yy * lw), ly0 + yy, lb, lg);
        }
    }
    if (cnt > 0 && cnt <= kCoop) {
        int64_t off = off0;
        for (int y = rc.y0; y < rc.y1; ++y)
            for (int x = rc.x0; x < rc.x1; ++x) put(off++, x, y, bits, g);
    }
}

// Visible (count > 0) Gaussians -> (depth bits, index) pairs, in index order.
__global__ void compact_visible_kernel(const int32_t* __restrict__ counts, const int64_t* __restrict__ pos,
                                       const float* __restrict__ depths, int64_t n, uint2* __restrict__ kv) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n || counts[i] <= 0) return;
    kv[pos[i]] = make_uint2(__float_as_uint(depths[i]), uint32_t(i));
}

__global__ void gather_counts_kernel(const int32_t* __restrict__ counts, const uint2* __restrict__ order,
                                     int64_t n, int32_t* __restrict__ out, const int64_t* __restrict__ n_dev) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < (n_dev ? *n_dev : n)) out[i] = counts[order[i].y];
}

// isect_offset_encode_kernel semantics (tiling_common.cu:25-71): offsets[t]
// is the first intersection index whose tile is >= t.
__global__ void offset_encode_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t n_tiles, int tb,
                                     int32_t* __restrict__ offsets) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    auto tile_of = [&](int64_t key) {
        const int64_t hi = key >> 32;
        return (hi >> tb) * n_tiles + (hi & ((int64_t(1) << tb) - 1));
    };
    const int64_t hc = ids[idx] >> 32;
    const int64_t cur = tile_of(ids[idx]);
    if (idx == 0)
        for (int64_t t = 0; t < cur + 1 && t < n_tiles; ++t) offsets[t] = 0;
    if (idx == n - 1)
        for (int64_t t = max(cur + 1, int64_t(0)); t < n_tiles; ++t) offsets[t] = int32_t(n);
    if (idx > 0) {
        const int64_t hp = ids[idx - 1] >> 32;
        if (hp == hc) return;
        const int64_t prev = tile_of(ids[idx - 1]);
        for (int64_t t = max(prev + 1, int64_t(0)); t < cur + 1 && t < n_tiles; ++t) offsets[t] = int32_t(idx);
    }
}

// The same with the intersection count on the device (`n_dev`, at most the
// capacity the grid is sized for); no intersections -> all offsets 0.
__global__ void offset_encode_dev_kernel(const int64_t* __restrict__ ids, const int64_t* __restrict__ n_dev,
                                         int64_t n_tiles, int tb, int32_t* __restrict__ offsets) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = *n_dev;
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (n == 0) {
        for (int64_t t = idx; t < n_tiles; t += int64_t(gridDim.x) * blockDim.x) offsets[t] = 0;
        return;
    }
    if (idx >= n) return;
    auto tile_of = [&](int64_t key) {
        const int64_t hi = key >> 32;
        return (hi >> tb) * n_tiles + (hi & ((int64_t(1) << tb) - 1));
    };
    const int64_t hc = ids[idx] >> 32;
    const int64_t cur = tile_of(ids[idx]);
    if (idx == 0)
        for (int64_t t = 0; t < cur + 1 && t < n_tiles; ++t) offsets[t] = 0;
    if (idx == n - 1)
        for (int64_t t = max(cur + 1, int64_t(0)); t < n_tiles; ++t) offsets[t] = int32_t(n);
    if (idx > 0) {
        const int64_t hp = ids[idx - 1] >> 32;
        if (hp == hc) return;
        const int64_t prev = tile_of(ids[idx - 1]);
        for (int64_t t = max(prev + 1, int64_t(0)); t < cur + 1 && t < n_tiles; ++t) offsets[t] = int32_t(idx);
    }
}

// counts[0] = the intersection total, counts[1] = min(total, cap): the
// number of intersections written and sorted
__global__ void clamp_count_kernel(const unsigned long long* __restrict__ total, int64_t cap,
                                   int64_t* __restrict__ counts) {
    pdl_wait();
    pdl_trigger();
    const int64_t t = int64_t(*total);
    counts[0] = t;
    counts[1] = t < cap ? t : cap;
}

// ------------------------------------------------ spherical / lidar grid --
struct SphTiling {
    int lidar;
    int n_az, n_el;
    float u_per_tile, v_per_tile;
    float2 img;
    const float* elev_bounds;
};

// tile_limits_irregular (phm_lidar_tiling.cu:52-91, increasing elevation
// boundaries) and tile_limits_regular (phm_spherical_tiling.cu:15-44) in
// exclusive [x0, x1) x [y0, y1) form.
__device__ __forceinline__ int sph_limits(const SphTiling& T, float2 m, float2 r, float umin, float umax,
                                          Rect& rc) {
    rc = {0, 0, 0, 0};
    const float lo = fmaxf(m.x - r.x, umin);
    const float hi = fminf(m.x + r.x, umax);
    if (hi <= lo) return 0;
    if (T.lidar) {
        const int tx0 = f2i(floorf(lo / T.u_per_tile));
        const int tx1 = f2i(ceilf(hi / T.u_per_tile)) - 1;
        const float vmin = m.y - r.y, vmax = m.y + r.y;
        const int N = T.n_el;
        int i = 0;
        while (i < N && T.elev_bounds[i] < vmin) ++i;
        const int ty0 = min(max(i - 1, 0), N - 1);
        while (i < N && T.elev_bounds[i] < vmax) ++i;
        const int ty1 = min(max(i - 1, 0), N - 1);
        rc = {tx0, ty0, tx1 + 1, ty1 + 1};
        return (ty1 - ty0 + 1) * (tx1 - tx0 + 1);
    }
    const int tx0 = f2i(floorf(lo / T.u_per_tile));
    const int ty0 = min(T.n_el, max(0, f2i(floorf((m.y - r.y) / T.v_per_tile))));
    const int tx1 = f2i(ceilf(hi / T.u_per_tile));
    const int ty1 = min(T.n_el, max(0, f2i(ceilf((m.y + r.y) / T.v_per_tile))));
    rc = {tx0, ty0, tx1, ty1};
    return (ty1 - ty0) * (tx1 - tx0);
}

}  // namespace xsg

// The UT projection pieces are shared with project.cu through this include.
#include "ut_device.cuh"

namespace xsg {

// Both rectangles of one Gaussian (the second only for flag 2, after a
// PositiveDelta re-projection): isect_lidar_tiles_kernel
// (phm_lidar_tiling.cu:96-234) / isect_spherical_tiles_kernel
// (phm_spherical_tiling.cu:47-174).
template <typename Cam>
__device__ __forceinline__ int sph_rects(const Cam& k, const SphTiling& T, const UTParams& up, int64_t i,
                                         const float* pts, const float* vel, const float* scales,
                                         const float4* quats, const float* opac, const uint8_t* flags,
                                         const float2* means2d, const float2* radii, Rect& r1, Rect& r2,
                                         bool& has2, float& depth2) {
    r1 = {0, 0, 0, 0};
    r2 = {0, 0, 0, 0};
    has2 = false;
    depth2 = 0.f;
    float2 rr = radii[i];
    const uint8_t fl = flags[i];
    if (rr.x <= 0 || rr.y <= 0 || fl == 0) return 0;
    float umin = 0.0f, umax = 1.0f;
    const float u_pose = fabsf(k.rolling.x) > 0.0f ? (k.pose - k.trigger) / k.rolling.x : 0.5f;
    if (fl == 2) {
        if (k.rolling.x > 0) umax = u_pose;
        else umin = u_pose;
    }
    const float2 m0 = means2d[i];
    const float2 m = make_float2(m0.x / T.img.x, m0.y / T.img.y);
    rr = make_float2(rr.x / T.img.x, rr.y / T.img.y);
    int cnt = sph_limits(T, m, rr, umin, umax, r1);
    if (fl == 2) {
        const v3 P = ld3(pts + 3 * i);
        const v3 V = vel ? ld3(vel + 3 * i) : mk3(0.f, 0.f, 0.f);
        const float o = opac ? opac[i] : 1.0f;
        v3 d[3];
        ut_deltas(up.sq, quats[i], ld3(scales + 3 * i), d);
        float2 m2, rad2;
        float dp2, tmp;
        if (ut_project(k, up, MODE_POS, P, V, o, d, m2, rad2, dp2, tmp)) {
            if (k.rolling.x > 0) {
                umin = ceilf(u_pose / T.u_per_tile) * T.u_per_tile + 1e-6f;
                umax = 1.0f;
            } else {
                umin = 0.0f;
                umax = floorf(u_pose / T.u_per_tile) * T.u_per_tile - 1e-6f;
            }
            cnt += sph_limits(T, make_float2(m2.x / T.img.x, m2.y / T.img.y),
                              make_float2(rad2.x / T.img.x, rad2.y / T.img.y), umin, umax, r2);
            has2 = true;
            depth2 = dp2;
        }
    }
    return cnt;
}

struct SphInputs {
    const float* pack;
    const float* pts;
    const float* vel;
    const float* scales;
    const float4* quats;
    const float* opac;
    const uint8_t* flags;
    const float2* means2d;
    const float2* radii;
    const float* depths;
};

template <typename Cam>
__global__ void __launch_bounds__(kTileThreads / 2)
    sph_count_kernel(SphInputs in, SphTiling T, UTParams up, int64_t n, int32_t* __restrict__ counts,
                     unsigned long long* __restrict__ total) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    int c = 0;
    if (i < n) {
        Cam k;
        k.load(in.pack);
        Rect r1, r2;
        bool has2;
        float d2;
        c = sph_rects(k, T, up, i, in.pts, in.vel, in.scales, in.quats, in.opac, in.flags, in.means2d,
                      in.radii, r1, r2, has2, d2);
        counts[i] = c;
    }
    block_add_total(c, total);
}

// Second-rectangle depths differ from depths[i]; the sorted path keys those
// intersections by a per-intersection depth kept in `isect_depth`.
template <typename Cam, bool kSorted>
__global__ void __launch_bounds__(kTileThreads / 2)
    sph_emit_kernel(SphInputs in, SphTiling T, UTParams up, int64_t n_items, const uint2* __restrict__ order,
                    const int64_t* __restrict__ offsets, uint2* __restrict__ buckets,
                    int64_t* __restrict__ isect_ids, int32_t* __restrict__ flatten_ids, int bucket_neg) {
    pdl_wait();
    pdl_trigger();
    const int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= n_items) return;
    const uint32_t g = kSorted ? order[p].y : uint32_t(p);
    Cam k;
    k.load(in.pack);
    Rect r1, r2;
    bool has2;
    float d2;
    const int c = sph_rects(k, T, up, g, in.pts, in.vel, in.scales, in.quats, in.opac, in.flags, in.means2d,
                            in.radii, r1, r2, has2, d2);
    if (c <= 0) return;
    int64_t off = offsets[p];
    auto fill = [&](const Rect& rc, float depth) {
        const int32_t bits = __float_as_int(depth);
        for (int y = rc.y0; y < rc.y1; ++y)
            for (int x = rc.x0; x < rc.x1; ++x) {
                const uint32_t tile = uint32_t(int64_t(y) * T.n_az + x);
                if constexpr (kSorted) {
                    buckets[off] = make_uint2(bits < 0 ? uint32_t(bucket_neg) : tile, g);
                } else {
                    const uint64_t hi = bits < 0 ? 0xFFFFFFFF00000000ull : (uint64_t(tile) << 32);
                    isect_ids[off] = int64_t(hi | uint64_t(uint32_t(bits)));
                    flatten_ids[off] = int32_t(g);
                }
                ++off;
            }
    };
    fill(r1, in.depths[g]);
    if (has2) fill(r2, d2);
}

// -------------------------------------------------------- host drivers --
// Workspace layout shared by the count and emit phases.
struct IsectWs {
    unsigned long long* total;
    int64_t* scan_out;      // n + 1
    void* scan_tmp;
    uint2 *g0, *g1;         // Gaussian presort (depth bits, index), n each
    int32_t* cnt_sorted;    // n
    uint2 *b0, *b1;         // tile sort (bucket, index or position), max_isects each
    void* sort_tmp;
    size_t sort_tmp_bytes;
    int64_t* kcopy;         // max_isects (generic 64-bit key sort)
    int32_t* fcopy;         // max_isects
};

// Scratch of the counting passes: 11-bit digits over n Gaussians or m
// intersections (depth words), up to 8-bit digits over m (tile bits).
static size_t sort_scratch_bytes(int64_t n, int64_t m) {
    const int64_t big = n > m ? n : m;
    return std::max(cs_workspace_bytes(big, 2048), cs_workspace_bytes(m, 256));
}

static size_t isect_ws_layout(int64_t n, int64_t m, void* base, size_t cap, IsectWs* ws) {
    Arena a(base, cap);
    const int64_t big = n > m ? n : m;
    IsectWs w{};
    w.total = a.take<unsigned long long>(1);
    w.scan_out = a.take<int64_t>(size_t(n + 1));
    w.scan_tmp = a.take<char>(scan_workspace_bytes(big + 1));
    w.g0 = a.take<uint2>(size_t(n));
    w.g1 = a.take<uint2>(size_t(n));
    w.cnt_sorted = a.take<int32_t>(size_t(n));
    w.b0 = a.take<uint2>(size_t(m));
    w.b1 = a.take<uint2>(size_t(m));
    w.sort_tmp_bytes = sort_scratch_bytes(n, m);
    w.sort_tmp = a.take<char>(w.sort_tmp_bytes);
    w.kcopy = a.take<int64_t>(size_t(m));
    w.fcopy = a.take<int32_t>(size_t(m));
    if (ws) *ws = w;
    // `used` is what the layout needs even when cap was too small
    size_t need = 0;
    need += Arena::round(8) + Arena::round(size_t(n + 1) * 8) + scan_workspace_bytes(big + 1);
    need += 2 * Arena::round(size_t(n) * 8) + Arena::round(size_t(n) * 4);
    need += 2 * Arena::round(size_t(m) * 8) + sort_scratch_bytes(n, m);
    need += Arena::round(size_t(m) * 8) + Arena::round(size_t(m) * 4);
    return need;
}

__global__ void split_key_kernel(const int64_t* __restrict__ ids, int64_t n, uint2* __restrict__ kv) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    kv[i] = make_uint2(uint32_t(uint64_t(ids[i])), uint32_t(i));
}

__global__ void gather_hi_kernel(const int64_t* __restrict__ ids, const uint2* __restrict__ perm, int64_t n,
                                 int tb, uint2* __restrict__ kv) {
    pdl_wait();
    pdl_trigger();
    const int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const uint32_t p = perm[j].y;
    kv[j] = make_uint2(uint32_t((uint64_t(ids[p]) >> 32) & ((uint64_t(1) << tb) - 1)), p);
}

__global__ void permute_isects_kernel(const int64_t* __restrict__ kin, const int32_t* __restrict__ fin,
                                      const uint2* __restrict__ perm, int64_t n, int64_t* __restrict__ kout,
                                      int32_t* __restrict__ fout) {
    pdl_wait();
    pdl_trigger();
    const int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const uint32_t p = perm[j].y;
    kout[j] = kin[p];
    fout[j] = fin[p];
}

// Stable LSD sort of interleaved (u32 key, u32 value) pairs on key bits
// [0, bits) with counting passes of up to `digit` bits, ping-ponging between
// kv0 and kv1; the result is returned in *res (one of the two).  With `ep` the
// last pass writes the 64-bit isect ids and flatten ids instead.
static int counting_sort(uint2* kv0, uint2* kv1, int64_t n, const int64_t* n_dev, int bits, int digit,
                         const IsectWs& w, cudaStream_t st, const IsectEpilogue* ep, uint2** res) {
    const int np = (bits + digit - 1) / digit;
    const int per = (bits + np - 1) / np;
    for (int p = 0; p < np; ++p) {
        const int lo = p * per, b = std::min(per, bits - lo);
        const bool last = p == np - 1;
        const int rc = counting_pass(kv0, kv1, n, n_dev, CsDigit{lo, uint32_t((uint64_t(1) << b) - 1)}, 1 << b,
                                     w.sort_tmp, w.sort_tmp_bytes, st, last ? ep : nullptr);
        if (rc != XSG_OK) return rc;
        std::swap(kv0, kv1);
    }
    if (res) *res = kv0;
    return XSG_OK;
}

// Stable sort of emitted (64-bit id, flatten id) pairs on id bits
// [0, 32 + tb), in place: by the depth word, then stably by the tile bits.
static int sort_isect_pairs_inplace(int64_t* ids, int32_t* flat, int64_t n, int tb, const struct IsectWs& w,
                                    cudaStream_t st) {
    launch_pdl(split_key_kernel, blocks_for(n, 256), 256, 0, st, ids, n, w.b0);
    uint2* res;
    int rc = counting_sort(w.b0, w.b1, n, nullptr, 32, 11, w, st, nullptr, &res);
    if (rc != XSG_OK) return rc;
    uint2* other = (res == w.b0) ? w.b1 : w.b0;
    launch_pdl(gather_hi_kernel, blocks_for(n, 256), 256, 0, st, ids, static_cast<const uint2*>(res), n, tb, other);
    rc = counting_sort(other, res, n, nullptr, tb, 8, w, st, nullptr, &res);
    if (rc != XSG_OK) return rc;
    XSG_CUDA(cudaMemcpyAsync(w.kcopy, ids, size_t(n) * 8, cudaMemcpyDeviceToDevice, st));
    XSG_CUDA(cudaMemcpyAsync(w.fcopy, flat, size_t(n) * 4, cudaMemcpyDeviceToDevice, st));
    launch_pdl(permute_isects_kernel, blocks_for(n, 256), 256, 0, st, w.kcopy, w.fcopy, static_cast<const uint2*>(res),
               n, ids, flat);
    return check_launch("sort_isect_pairs");
}

// Sorted emission shared by regular and spherical tilings: presort the
// visible Gaussians by depth, scan their counts in that order and let
// `emit(order, offsets, n_vis_upper, n_vis_dev)` write tile-keyed pairs, then
// bucket them stably by tile.  The number of visible Gaussians stays on the
// device (grids are sized for all n), so there is no host round trip here.
template <typename Emit>
static int sorted_isects(const int32_t* counts, const float* depths, int64_t n, int64_t n_isects,
                         int64_t n_tiles, const IsectWs& w, int64_t* isect_ids, int32_t* flatten_ids,
                         cudaStream_t st, Emit&& emit, const int64_t* n_isects_dev = nullptr) {
    // 1. compact visible Gaussians (count > 0); their number goes to scan_out[n]
    int rc = exclusive_scan<int32_t, true>(counts, n, w.scan_out, w.scan_out + n, w.scan_tmp, st);
    if (rc != XSG_OK) return rc;
    const int64_t* n_vis = w.scan_out + n;
    launch_pdl(compact_visible_kernel, blocks_for(n, 256), 256, 0, st, counts, static_cast<const int64_t*>(w.scan_out),
           depths, n, w.g0);
    // 2. stable sort by the 32 depth bits: three counting passes (11 + 11 + 10 bits)
    uint2* order = nullptr;
    rc = counting_sort(w.g0, w.g1, n, n_vis, 32, 11, w, st, nullptr, &order);
    if (rc != XSG_OK) return rc;
    // 3. counts in depth order -> emission offsets
    launch_pdl(gather_counts_kernel, blocks_for(n, 256), 256, 0, st, counts, static_cast<const uint2*>(order), n,
               w.cnt_sorted, n_vis);
    rc = exclusive_scan<int32_t>(w.cnt_sorted, n, w.scan_out, nullptr, w.scan_tmp, st, n_vis);
    if (rc != XSG_OK) return rc;
    emit(static_cast<const uint2*>(order), static_cast<const int64_t*>(w.scan_out), n, n_vis);
    // 4. stable counting passes on the tile bits (up to 8 bits each), the
    //    last of which writes the outputs
    IsectEpilogue ep{depths, isect_ids, flatten_ids};
    return counting_sort(w.b0, w.b1, n_isects, n_isects_dev, tile_bits_for(n_tiles), 8, w, st, &ep, nullptr);
}

}  // namespace xsg

using namespace xsg;

extern "C" {

size_t xsg_isect_workspace_size(int64_t n_gauss, int64_t max_isects) {
    return isect_ws_layout(n_gauss < 0 ? 0 : n_gauss, max_isects < 0 ? 0 : max_isects, nullptr, 0, nullptr);
}

int xsg_isect_regular_count(const float* means2d, const float* radii, int64_t n, int W, int H, int tsx,
                            int tsy, int32_t* counts, int64_t* n_isects_host, void* workspace,
                            size_t ws_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && W > 0 && H > 0 && tsx > 0 && tsy > 0 && n_isects_host, "isect_regular_tiles: bad arguments");
    XSG_REQUIRE(n == 0 || (means2d && radii && counts), "isect_regular_tiles: null input");
    cudaStream_t st = as_cuda(stream);
    IsectWs w;
    const size_t need = isect_ws_layout(n, 0, workspace, ws_bytes, &w);
    if (ws_bytes < need || !workspace) return set_error(XSG_ERR_WORKSPACE, "isect_regular_tiles: workspace too small");
    XSG_CUDA(cudaMemsetAsync(w.total, 0, sizeof(unsigned long long), st));
    const int ntx = (W + tsx - 1) / tsx, nty = (H + tsy - 1) / tsy;
    ScopedTimer tm("isect_count", st);
    if (n > 0)
        launch_pdl(regular_count_kernel, blocks_for(n, kTileThreads), kTileThreads, 0, st, 
            reinterpret_cast<const float2*>(means2d), reinterpret_cast<const float2*>(radii), n,
            make_float2(float(tsx), float(tsy)), ntx, nty, counts, w.total);
    unsigned long long tot = 0;
    XSG_CUDA(cudaMemcpyAsync(&tot, w.total, sizeof(tot), cudaMemcpyDeviceToHost, st));
    XSG_CUDA(cudaStreamSynchronize(st));
    *n_isects_host = int64_t(tot);
    if (tot >= (1ull << 31)) return set_error(XSG_ERR_UNSUPPORTED, "isect_regular_tiles: more than 2^31 intersections");
    return check_launch("isect_regular_count");
}

int xsg_isect_regular_emit(const float* means2d, const float* radii, const float* depths, int64_t n, int W,
                           int H, int tsx, int tsy, int sort, const int32_t* counts, int64_t n_isects,
                           int64_t* isect_ids, int32_t* flatten_ids, void* workspace, size_t ws_bytes,
                           xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && n_isects >= 0 && W > 0 && H > 0 && tsx > 0 && tsy > 0, "isect_regular_tiles: bad arguments");
    if (n_isects == 0) return XSG_OK;
    XSG_REQUIRE(means2d && radii && depths && counts && isect_ids && flatten_ids, "isect_regular_tiles: null input");
    cudaStream_t st = as_cuda(stream);
    IsectWs w;
    const size_t need = isect_ws_layout(n, sort ? n_isects : 0, workspace, ws_bytes, &w);
    if (ws_bytes < need || !workspace) return set_error(XSG_ERR_WORKSPACE, "isect_regular_tiles: workspace too small");
    const int ntx = (W + tsx - 1) / tsx, nty = (H + tsy - 1) / tsy;
    const float2 ts = make_float2(float(tsx), float(tsy));
    auto* m2 = reinterpret_cast<const float2*>(means2d);
    auto* r2 = reinterpret_cast<const float2*>(radii);
    if (!sort) {
        int rc = exclusive_scan<int32_t>(counts, n, w.scan_out, nullptr, w.scan_tmp, st);
        if (rc != XSG_OK) return rc;
        launch_pdl(regular_emit_kernel<false>, blocks_for(n, kTileThreads), kTileThreads, 0, st, 
            m2, r2, depths, n, ts, ntx, nty, 0, nullptr, w.scan_out, nullptr, isect_ids, flatten_ids,
            static_cast<const int64_t*>(nullptr), INT64_MAX);
        return check_launch("isect_regular_emit");
    }
    const int64_t n_tiles = int64_t(ntx) * nty;
    const int bucket_neg = int((int64_t(1) << tile_bits_for(n_tiles)) - 1);
    ScopedTimer tm("isect_emit_sort", st);
    return sorted_isects(counts, depths, n, n_isects, n_tiles, w, isect_ids, flatten_ids, st,
                         [&](const uint2* order, const int64_t* offs, int64_t n_up, const int64_t* n_vis) {
                             launch_pdl(regular_emit_kernel<true>, blocks_for(n_up, kTileThreads), kTileThreads, 0, st,
                                 m2, r2, depths, n_up, ts, ntx, nty, bucket_neg, order, offs, w.b0,
                                 nullptr, nullptr, n_vis, INT64_MAX);
                         });
}

int xsg_isect_regular_tiles_async(const float* means2d, const float* radii, const float* depths, int64_t n, int W,
                                  int H, int tsx, int tsy, int64_t capacity, int32_t* counts, int64_t* isect_ids,
                                  int32_t* flatten_ids, int32_t* offsets, int64_t* n_isects_dev, void* workspace,
                                  size_t ws_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && W > 0 && H > 0 && tsx > 0 && tsy > 0 && capacity > 0 && capacity < (int64_t(1) << 31),
                "isect_regular_tiles_async: bad arguments");
    XSG_REQUIRE(offsets && n_isects_dev && isect_ids && flatten_ids && (n == 0 || (means2d && radii && depths && counts)),
                "isect_regular_tiles_async: null argument");
    cudaStream_t st = as_cuda(stream);
    IsectWs w;
    const size_t need = isect_ws_layout(n, capacity, workspace, ws_bytes, &w);
    if (ws_bytes < need || !workspace) return set_error(XSG_ERR_WORKSPACE, "isect_regular_tiles_async: workspace too small");
    const int ntx = (W + tsx - 1) / tsx, nty = (H + tsy - 1) / tsy;
    const int64_t n_tiles = int64_t(ntx) * nty;
    const float2 ts = make_float2(float(tsx), float(tsy));
    auto* m2 = reinterpret_cast<const float2*>(means2d);
    auto* r2 = reinterpret_cast<const float2*>(radii);
    XSG_CUDA(cudaMemsetAsync(w.total, 0, sizeof(unsigned long long), st));
    {
        ScopedTimer tm("isect_count", st);
        if (n > 0)
            launch_pdl(regular_count_kernel, blocks_for(n, kTileThreads), kTileThreads, 0, st, m2, r2, n, ts, ntx, nty,
                   counts, w.total);
        launch_pdl(clamp_count_kernel, 1, 1, 0, st, static_cast<const unsigned long long*>(w.total), capacity,
               n_isects_dev);
    }
    const int64_t* n_written = n_isects_dev + 1;
    if (n > 0) {
        const int bucket_neg = int((int64_t(1) << tile_bits_for(n_tiles)) - 1);
        ScopedTimer tm("isect_emit_sort", st);
        const int rc = sorted_isects(
            counts, depths, n, capacity, n_tiles, w, isect_ids, flatten_ids, st,
            [&](const uint2* order, const int64_t* offs, int64_t n_up, const int64_t* n_vis) {
                launch_pdl(regular_emit_kernel<true>, blocks_for(n_up, kTileThreads), kTileThreads, 0, st, m2, r2,
                       depths, n_up, ts, ntx, nty, bucket_neg, order, offs, w.b0, nullptr, nullptr, n_vis,
                       capacity);
            },
            n_written);
        if (rc != XSG_OK) return rc;
    }
    launch_pdl(offset_encode_dev_kernel, blocks_for(capacity, 256), 256, 0, st, static_cast<const int64_t*>(isect_ids),
           n_written, n_tiles, tile_bits_for(n_tiles), offsets);
    return check_launch("isect_regular_tiles_async");
}

static SphTiling make_sph_tiling(int lidar, const float* elev_bounds, int n_elev, int tsx, int tsy, float W,
                                 float H) {
    SphTiling T;
    T.lidar = lidar;
    T.img = make_float2(W, H);
    T.elev_bounds = elev_bounds;
    T.u_per_tile = float(tsx) / W;
    if (lidar) {
        T.n_az = (int(W) + tsx - 1) / tsx;
        T.n_el = n_elev;
        T.v_per_tile = ceilf(H / float(n_elev)) / H;
    } else {
        T.n_az = int(ceilf(W / float(tsx)));
        T.n_el = int(ceilf(H / float(tsy)));
        T.v_per_tile = float(tsy) / H;
    }
    return T;
}

#define XSG_SPH_DISPATCH(lidar, BODY)                   \
    do {                                                \
        if (lidar) {                                    \
            using Cam = Spherical<true>;                \
            BODY;                                       \
        } else {                                        \
            using Cam = Spherical<false>;               \
            BODY;                                       \
        }                                               \
    } while (0)

int xsg_isect_spherical_count(int lidar, const float* pack, const float* pts, const float* vel,
                              const float* scales, const float* quats, const float* opac, const uint8_t* flags,
                              const float* means2d, const float* radii, const float* depths,
                              const float* elev_bounds, int n_elev, int64_t n, int tsx, int tsy, float W,
                              float H, float ua, float ub, float uk, int32_t* counts, int64_t* n_isects_host,
                              void* workspace, size_t ws_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && tsx > 0 && tsy > 0 && W > 0 && H > 0 && n_isects_host, "isect_spherical_tiles: bad arguments");
    XSG_REQUIRE(!lidar || (elev_bounds && n_elev > 0), "isect_lidar_tiles: elevation boundaries required");
    XSG_REQUIRE(n == 0 || (pack && pts && scales && quats && flags && means2d && radii && depths && counts),
                "isect_spherical_tiles: null input");
    XSG_REQUIRE(reinterpret_cast<uintptr_t>(quats) % 16 == 0, "isect_spherical_tiles: quats must be 16-byte aligned");
    cudaStream_t st = as_cuda(stream);
    IsectWs w;
    const size_t need = isect_ws_layout(n, 0, workspace, ws_bytes, &w);
    if (ws_bytes < need || !workspace) return set_error(XSG_ERR_WORKSPACE, "isect_spherical_tiles: workspace too small");
    XSG_CUDA(cudaMemsetAsync(w.total, 0, sizeof(unsigned long long), st));
    const SphTiling T = make_sph_tiling(lidar, elev_bounds, n_elev, tsx, tsy, W, H);
    const UTParams up = ut_params(ua, ub, uk, 1e-4f, 0.002f, 1.0f, W, H);
    SphInputs in{pack, pts, vel, scales, reinterpret_cast<const float4*>(quats), opac, flags,
                 reinterpret_cast<const float2*>(means2d), reinterpret_cast<const float2*>(radii), depths};
    if (n > 0)
        XSG_SPH_DISPATCH(lidar, (launch_pdl(sph_count_kernel<Cam>, blocks_for(n, kTileThreads / 2), kTileThreads / 2, 0, st, 
                                    in, T, up, n, counts, w.total)));
    unsigned long long tot = 0;
    XSG_CUDA(cudaMemcpyAsync(&tot, w.total, sizeof(tot), cudaMemcpyDeviceToHost, st));
    XSG_CUDA(cudaStreamSynchronize(st));
    *n_isects_host = int64_t(tot);
    if (tot >= (1ull << 31)) return set_error(XSG_ERR_UNSUPPORTED, "isect_spherical_tiles: more than 2^31 intersections");
    return check_launch("isect_spherical_count");
}

int xsg_isect_spherical_emit(int lidar, const float* pack, const float* pts, const float* vel,
                             const float* scales, const float* quats, const float* opac, const uint8_t* flags,
                             const float* means2d, const float* radii, const float* depths,
                             const float* elev_bounds, int n_elev, int64_t n, int tsx, int tsy, float W,
                             float H, float ua, float ub, float uk, int sort, const int32_t* counts,
                             int64_t n_isects, int64_t* isect_ids, int32_t* flatten_ids, void* workspace,
                             size_t ws_bytes, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && n_isects >= 0 && tsx > 0 && tsy > 0 && W > 0 && H > 0, "isect_spherical_tiles: bad arguments");
    if (n_isects == 0) return XSG_OK;
    XSG_REQUIRE(pack && pts && scales && quats && flags && means2d && radii && depths && counts && isect_ids &&
                    flatten_ids, "isect_spherical_tiles: null input");
    XSG_REQUIRE(reinterpret_cast<uintptr_t>(quats) % 16 == 0, "isect_spherical_tiles: quats must be 16-byte aligned");
    cudaStream_t st = as_cuda(stream);
    IsectWs w;
    const size_t need = isect_ws_layout(n, sort ? n_isects : 0, workspace, ws_bytes, &w);
    if (ws_bytes < need || !workspace) return set_error(XSG_ERR_WORKSPACE, "isect_spherical_tiles: workspace too small");
    const SphTiling T = make_sph_tiling(lidar, elev_bounds, n_elev, tsx, tsy, W, H);
    const UTParams up = ut_params(ua, ub, uk, 1e-4f, 0.002f, 1.0f, W, H);
    SphInputs in{pack, pts, vel, scales, reinterpret_cast<const float4*>(quats), opac, flags,
                 reinterpret_cast<const float2*>(means2d), reinterpret_cast<const float2*>(radii), depths};
    const int64_t n_tiles = int64_t(T.n_az) * T.n_el;
    const int bucket_neg = int((int64_t(1) << tile_bits_for(n_tiles)) - 1);
    if (!sort) {
        int rc = exclusive_scan<int32_t>(counts, n, w.scan_out, nullptr, w.scan_tmp, st);
        if (rc != XSG_OK) return rc;
        XSG_SPH_DISPATCH(lidar, (launch_pdl(sph_emit_kernel<Cam, false>, blocks_for(n, kTileThreads / 2), kTileThreads / 2, 0, st, 
                                    in, T, up, n, nullptr, w.scan_out, nullptr, isect_ids, flatten_ids,
                                    bucket_neg)));
        return check_launch("isect_spherical_emit");
    }
    // The second (wrap) rectangle of a flag-2 Gaussian carries its own depth,
    // so the presort by Gaussian depth does not order those intersections.
    // They are rare; the general path below sorts intersections by
    // (tile, depth bits) with two chained stable sorts instead.
    int rc = exclusive_scan<int32_t>(counts, n, w.scan_out, nullptr, w.scan_tmp, st);
    if (rc != XSG_OK) return rc;
    XSG_SPH_DISPATCH(lidar, (launch_pdl(sph_emit_kernel<Cam, false>, blocks_for(n, kTileThreads / 2), kTileThreads / 2, 0, st, 
                                in, T, up, n, nullptr, w.scan_out, nullptr, isect_ids, flatten_ids,
                                bucket_neg)));
    return sort_isect_pairs_inplace(isect_ids, flatten_ids, n_isects, tile_bits_for(n_tiles), w, st);
}

int xsg_isect_offset_encode(const int64_t* isect_ids, int64_t n_isects, int tw, int th, int32_t* offsets,
                            xsg_stream_t stream) {
    XSG_REQUIRE(tw > 0 && th > 0 && offsets && n_isects >= 0, "isect_offset_encode: bad arguments");
    cudaStream_t st = as_cuda(stream);
    const int64_t n_tiles = int64_t(tw) * th;
    if (n_isects == 0) {
        XSG_CUDA(cudaMemsetAsync(offsets, 0, size_t(n_tiles) * sizeof(int32_t), st));
        return XSG_OK;
    }
    XSG_REQUIRE(isect_ids, "isect_offset_encode: null isect_ids");
    launch_pdl(offset_encode_kernel, blocks_for(n_isects, 256), 256, 0, st, isect_ids, n_isects, n_tiles,
                                                                   tile_bits_for(n_tiles), offsets);
    return check_launch("isect_offset_encode");
}

}  // extern "C"
