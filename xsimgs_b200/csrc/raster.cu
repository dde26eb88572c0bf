// Per-tile 3D-evaluation alpha compositing, forward and backward, for
// sm_100a.  Semantics: rasterize_eval3d_fwd / _bwd and their dynamic
// variants in the reference (csrc/rasterization/eval3d_fwd.cu:34-166,
// eval3d_bwd.cu:38-294, eval3d_dynamic_fwd.cu:38-173,
// eval3d_dynamic_bwd.cu:68-310).
//
// Design (B200):
//  * A pack kernel turns each Gaussian into one 64-byte record
//      {M row 0, mu.x} {M row 1, mu.y} {M row 2, mu.z} {opacity, velocity}
//    with M = S^-1 R^T computed exactly as the reference does per load, and,
//    for static scenes, 48 bytes of view constants for the rays that start
//    at pixel 0's origin (M (o - mu), the quadric pre-test, the cone radius).
//  * One CTA per image tile, heaviest tiles first; each warp owns an 8 x 4
//    block of pixels and works on its own (no block barriers): it stages the
//    tile's records 32 at a time in its slice of shared memory, skips the
//    Gaussians no ray of its cone can see and, per lane, those whose quadric
//    test fails for every pixel, and stops when all its pixels saturate.
//  * The forward records per warp and batch of 32 list entries which ones
//    some pixel composited (contributor masks); a backward given the
//    forward's workspace visits exactly those, back to front.
//  * Backward: per (warp, Gaussian) event the 16 gradient values are reduced
//    with a transpose butterfly (16 shuffles) and added with four
//    red.global.add.v4.f32 into a per-Gaussian accumulator; dL/dM is summed
//    there and turned into quaternion / scale gradients once per Gaussian by
//    a finalize pass.
#include "common.cuh"

namespace xsg {

constexpr int kRecF4 = 4;  // float4 words per Gaussian record

struct RasterArgs {
    const float4* rec;        // [N][4]
    const float4* ext;        // [N][3] view constants for rays from ray_o[0] (static scenes; may be null)
    const float* means;       // [N,3] (bwd)
    const float* quats;       // [N,4] (bwd)
    const float* scales;      // [N,3] (bwd)
    const float* colors;      // [N,C]
    const float* ray_o;       // [H,W,3]
    const float* ray_d;       // [H,W,3]
    const float* ray_t;       // [H,W] (dynamic)
    const int32_t* offsets;   // [tiles]
    const int32_t* flatten;   // [n_isects]
    int64_t n_isects;
    const int64_t* n_isects_dev;  // the list length on the device (n_isects is then its capacity), or null
    int W, H, tsx, tsy, ntx, nty;
    // forward outputs
    float* out_rgb;
    float* out_depth;
    float* out_alpha;
    int32_t* out_last;
    // backward inputs/outputs
    const float* render_alpha;
    const int32_t* last_ids;
    const float* v_rgb;
    const float* v_depth;
    const float* v_alpha;
    float* G;                 // [N][NACC] gradient accumulator
    float* v_colors_direct;   // [N,C] when C > 4
    float* v_ray_o;
    float* v_ray_d;
    float* v_ray_t;
    unsigned long long* pair_counters;  // work counters (optional, xsg_set_pair_counters)
    const int32_t* tile_order;          // launch order of the tiles (optional)
    // contributor masks (optional): word ((start >> 5) + tile + k) * warps_per_tile + warp has
    // bit i set when list entry start + 32 k + i reached alpha >= 1/255 at one of the warp's
    // pixels before it saturated; the forward writes them, the backward visits only those entries
    uint32_t* masks;
    // after the masks: the union and the sum of the mask bits of each pair of
    // 8 x 4 blocks (2w, 2w + 1), over the image, counted by the forward; the
    // backward's choice between its two kernels (px2_chosen)
    unsigned long long* px2_stats;
};

// largest union of the block pairs' contributor masks, in percent of the
// pairs' two counts, for which the backward runs two pixels a lane
constexpr int kPx2UnionPct = 72;

// The two-pixels-a-lane backward pays a whole paired evaluation for an entry
// only one block of its pair composited, so it serves an image whose block
// pairs mostly composite the same Gaussians; the per-pixel backward serves
// the others (sparse angular sampling: lidar).  Both kernels are launched and
// read the forward's counts; the one not chosen returns at once.
__device__ __forceinline__ bool px2_chosen(const unsigned long long* stats) {
    return stats[0] * 100ull <= (unsigned long long)kPx2UnionPct * stats[1];
}

// Index of the contributor mask of batch k of a warp (tiles' batch ranges
// [(start >> 5) + tile, + ceil(len / 32)) never overlap).
__device__ __forceinline__ int64_t mask_index(int32_t start, int tile, int32_t k, int wpt, int wid) {
    return (int64_t(start >> 5) + tile + k) * wpt + wid;
}

static unsigned long long* g_pair_counters = nullptr;
// tile-order scratch is sized for images up to this many tiles (16k x 16k at 16x16)
constexpr int64_t kMaxTiles = int64_t(1) << 20;

// --------------------------------------------------------------- pack ----
__device__ __forceinline__ void view_consts(float4 r0, float4 r1, float4 r2, float4 r3, v3 o, float4* e);

// quat_to_rotmat (rasterization/utils.h:61-83) and S^-1 R^T
// (eval3d_fwd.cu:92-106): row i of M is (1 / s_i) * column i of R.  With
// `ext` (static scenes) also the view constants of the rays that start at
// o_ref[0..2], the origin of pixel 0.
__global__ void pack_records_kernel(const float* __restrict__ means, const float* __restrict__ vel,
                                    const float* __restrict__ quats, const float* __restrict__ scales,
                                    const float* __restrict__ opac, int64_t n, float4* __restrict__ rec,
                                    const float* __restrict__ o_ref, float4* __restrict__ ext,
                                    unsigned long long* __restrict__ px2_stats) {
    const int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (px2_stats && g < 2) px2_stats[g] = 0ull;  // the forward counts into them
    if (g >= n) return;
    float w = quats[4 * g], x = quats[4 * g + 1], y = quats[4 * g + 2], z = quats[4 * g + 3];
    const float inv_norm = rsqrtf(x * x + y * y + z * z + w * w);
    x *= inv_norm; y *= inv_norm; z *= inv_norm; w *= inv_norm;
    const float x2 = x * x, y2 = y * y, z2 = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    // columns of R
    const float c00 = 1.f - 2.f * (y2 + z2), c01 = 2.f * (xy + wz), c02 = 2.f * (xz - wy);
    const float c10 = 2.f * (xy - wz), c11 = 1.f - 2.f * (x2 + z2), c12 = 2.f * (yz + wx);
    const float c20 = 2.f * (xz + wy), c21 = 2.f * (yz - wx), c22 = 1.f - 2.f * (x2 + y2);
    const float sx = 1.0f / scales[3 * g], sy = 1.0f / scales[3 * g + 1], sz = 1.0f / scales[3 * g + 2];
    float4* r = rec + kRecF4 * g;
    const float4 q0 = make_float4(sx * c00, sx * c01, sx * c02, means[3 * g]);
    const float4 q1 = make_float4(sy * c10, sy * c11, sy * c12, means[3 * g + 1]);
    const float4 q2 = make_float4(sz * c20, sz * c21, sz * c22, means[3 * g + 2]);
    const float4 q3 = vel ? make_float4(opac[g], vel[3 * g], vel[3 * g + 1], vel[3 * g + 2])
                          : make_float4(opac[g], 0.f, 0.f, 0.f);
    r[0] = q0; r[1] = q1; r[2] = q2; r[3] = q3;
    if (ext) view_consts(q0, q1, q2, q3, mk3(o_ref[0], o_ref[1], o_ref[2]), ext + 3 * g);
}

// Heavy tiles first: tiles bucketed by floor(log2(intersection count)),
// buckets in descending order, tile order kept inside a bucket.  One CTA.
__global__ void __launch_bounds__(1024) tile_order_kernel(const int32_t* __restrict__ offsets, int n_tiles,
                                                          int32_t n_isects, const int64_t* __restrict__ n_isects_dev,
                                                          int32_t* __restrict__ order) {
    __shared__ int hist[33];
    __shared__ int base[33];
    if (n_isects_dev) n_isects = int32_t(*n_isects_dev);
    if (threadIdx.x < 33) hist[threadIdx.x] = 0;
    __syncthreads();
    auto bucket = [&](int t) {
        const int32_t e = (t == n_tiles - 1) ? n_isects : offsets[t + 1];
        const int32_t c = e - offsets[t];
        return c > 0 ? 32 - __clz(c) : 0;  // 0 for empty, 1 + floor(log2 c)
    };
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) atomicAdd(&hist[bucket(t)], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int b = 32; b >= 0; --b) {
            base[b] = run;
            run += hist[b];
        }
    }
    __syncthreads();
    // stable scatter: one pass per chunk of blockDim tiles, ranks by warp match
    for (int t0 = 0; t0 < n_tiles; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        const int b = t < n_tiles ? bucket(t) : -1;
        __shared__ int cnt[32][33];
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int k = lane; k < 33; k += 32) cnt[w][k] = 0;
        __syncthreads();
        const unsigned peers = __match_any_sync(0xffffffffu, b);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (b >= 0 && rank == 0) cnt[w][b] = __popc(peers);
        __syncthreads();
        if (b >= 0) {
            int before = 0;
            for (int ww = 0; ww < w; ++ww) before += cnt[ww][b];
            order[base[b] + before + rank] = t;
        }
        __syncthreads();
        if (threadIdx.x < 33) {
            int tot = 0;
            for (int ww = 0; ww < int(blockDim.x >> 5); ++ww) tot += cnt[ww][threadIdx.x];
            base[threadIdx.x] += tot;
        }
        __syncthreads();
    }
}

struct TileCtx {
    int tile, px, py;
    bool inside;
    int64_t pix;
    int32_t start, end;
};

__device__ __forceinline__ TileCtx tile_ctx(const RasterArgs& a) {
    TileCtx c;
    c.tile = a.tile_order ? a.tile_order[blockIdx.x] : int(blockIdx.x);
    const int ty = c.tile / a.ntx, tx = c.tile - ty * a.ntx;
    const int t = threadIdx.x;
    if ((a.tsx % 8 == 0) && (a.tsy % 4 == 0)) {
        // each warp covers an 8 x 4 block of the tile (lane 0 at its top-left)
        const int w = t >> 5, l = t & 31, wc = a.tsx >> 3;
        c.px = tx * a.tsx + (w % wc) * 8 + (l & 7);
        c.py = ty * a.tsy + (w / wc) * 4 + (l >> 3);
    } else {
        c.px = tx * a.tsx + t % a.tsx;
        c.py = ty * a.tsy + t / a.tsx;
    }
    c.inside = c.px < a.W && c.py < a.H;
    const int64_t lin = int64_t(c.py) * a.W + c.px;
    const int64_t last = int64_t(a.W) * a.H - 1;
    c.pix = lin < last ? lin : last;
    c.start = a.offsets[c.tile];
    c.end = (c.tile == a.ntx * a.nty - 1) ? int32_t(a.n_isects_dev ? *a.n_isects_dev : a.n_isects)
                                          : a.offsets[c.tile + 1];
    return c;
}

// ------------------------------------------------- evaluation arithmetic --
// The alpha of a (ray, Gaussian) pair (eval3d_fwd.cu:111-124: grd = M d,
// gn = grd / |grd|, gc = gn x gro with gro = M (o - mu), power = -|gc|^2 / 2)
// as a fixed sequence of explicitly rounded products and FMAs, nothing left
// to the compiler's contraction.  The sequence is the one the reference's
// own kernel gets from nvcc (-O3, FMA contraction on) for the same
// expressions, established by comparing bit patterns of alpha and t* over a
// million pairs: a 3-term sum of products x0 y0 + x1 y1 + x2 y2 (glm::dot,
// the rows of mat3 * vec3) is fma(x2, y2, fma(x0, y0, x1 y1)) and a cross
// component a b - c d is fma(a, b, -(c d)); t* = -(gro . grd) / (grd . grd)
// is the reference's correctly rounded division, computed as a
// Newton-corrected quotient (div_nr) that gave the same bits on every pair of
// the full-size test views.  So the compositing forward returns the
// reference's images bit for bit on the same tile lists.  The forward
// evaluates two list entries at a time with the paired FP32 instructions of
// sm_100 (fma / mul .f32x2, one entry per half) and the backward one entry at
// a time with the scalar form; both get bit-identical alpha and so take the
// same alpha >= 1/255 decisions.
__device__ __forceinline__ float fx_dot(v3 a, v3 b) {
    return __fmaf_rn(a.z, b.z, __fmaf_rn(a.x, b.x, __fmul_rn(a.y, b.y)));
}
// M v with M rows (r0,r1,r2).xyz (glm's mat3 * vec3, contracted as fx_dot)
__device__ __forceinline__ v3 fx_mrows(float4 r0, float4 r1, float4 r2, v3 v) {
    return mk3(fx_dot(mk3(r0.x, r0.y, r0.z), v), fx_dot(mk3(r1.x, r1.y, r1.z), v),
               fx_dot(mk3(r2.x, r2.y, r2.z), v));
}
// glm::cross component order
__device__ __forceinline__ v3 fx_cross(v3 a, v3 b) {
    return mk3(__fmaf_rn(a.y, b.z, -__fmul_rn(b.y, a.z)), __fmaf_rn(a.z, b.x, -__fmul_rn(b.z, a.x)),
               __fmaf_rn(a.x, b.y, -__fmul_rn(b.x, a.y)));
}
// (o - mu) of a moving Gaussian: mu + rt vel
__device__ __forceinline__ v3 fx_moved(v3 mu, v3 vel, float rt) {
    return mk3(__fmaf_rn(rt, vel.x, mu.x), __fmaf_rn(rt, vel.y, mu.y), __fmaf_rn(rt, vel.z, mu.z));
}
struct EvalTerms {
    v3 grd, gn, gc;
    float l, vis;  // |grd|^2, exp(power)
};
__device__ __forceinline__ EvalTerms fx_eval(float4 r0, float4 r1, float4 r2, v3 gro, v3 d) {
    EvalTerms e;
    e.grd = fx_mrows(r0, r1, r2, d);
    e.l = fx_dot(e.grd, e.grd);
    const float il = e.l > 0.0f ? rsqrtf(e.l) : 1.0f;
    e.gn = mk3(__fmul_rn(e.grd.x, il), __fmul_rn(e.grd.y, il), __fmul_rn(e.grd.z, il));
    e.gc = fx_cross(e.gn, gro);
    e.vis = __expf(__fmul_rn(-0.5f, fx_dot(e.gc, e.gc)));
    return e;
}

// a / b to within about half an ulp (nearly always the correctly rounded
// quotient): the approximate reciprocal, then one Newton correction of the
// quotient (Markstein).  The forward's t* and the backward's replay of T use
// it: it matches the reference's IEEE division where the approximate
// quotient does not, at two FMAs more and well below the cost of div.rn.
__device__ __forceinline__ float div_nr(float a, float b) {
    const float r = __fdividef(1.0f, b);
    const float q = __fmul_rn(a, r);
    return __fmaf_rn(__fmaf_rn(-b, q, a), r, q);
}

// The same operations on two entries at once: .x entry A, .y entry B.
struct p3 {
    float2 x, y, z;
};
__device__ __forceinline__ float2 pdup(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 pneg(float2 a) { return make_float2(-a.x, -a.y); }
__device__ __forceinline__ float2 pdot(p3 a, p3 b) {
    return __ffma2_rn(a.z, b.z, __ffma2_rn(a.x, b.x, __fmul2_rn(a.y, b.y)));
}
__device__ __forceinline__ p3 pcross(p3 a, p3 b) {
    return {__ffma2_rn(a.y, b.z, pneg(__fmul2_rn(b.y, a.z))), __ffma2_rn(a.z, b.x, pneg(__fmul2_rn(b.z, a.x))),
            __ffma2_rn(a.x, b.y, pneg(__fmul2_rn(b.x, a.y)))};
}

// ------------------------------------------------------- warp culling ----
// A warp's 32 pixel rays are bounded by one origin o_c (all origins within
// r_o of it) and a double cone of lines around the unit axis `ax` with
// half-angle theta (cos_t, sin_t).  A Gaussian can reach alpha >= 1/255 on a
// line only if the line meets the ellipsoid |M (x - mu)|^2 <= 2 ln(255 o),
// which lies inside the sphere of radius sqrt(2 ln(255 o)) * s_max around mu
// (s_max = 1 / min_i |row_i(M)|).  If every line of the cone misses that
// sphere, inflated by relative and absolute margins far larger than the
// rounding of either computation, no lane of the warp can accept the Gaussian:
// the forward and backward skip it without changing any result.
struct WarpCone {
    v3 oc, ax;
    float cos_t, sin_t, r_o, rt_max;
    bool on;
};

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_min_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ WarpCone warp_cone(bool inside, v3 o, v3 d, float rt) {
    WarpCone w;
    const float dl = dot3(d, d);
    const v3 dh = (inside && dl > 0.f) ? d * rsqrtf(dl) : mk3(0.f, 0.f, 0.f);
    v3 sum = dh;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        sum.x += __shfl_xor_sync(0xffffffffu, sum.x, off);
        sum.y += __shfl_xor_sync(0xffffffffu, sum.y, off);
        sum.z += __shfl_xor_sync(0xffffffffu, sum.z, off);
    }
    const float sl = dot3(sum, sum);
    w.ax = sl > 0.f ? sum * rsqrtf(sl) : mk3(0.f, 0.f, 1.f);
    w.cos_t = warp_min_f(inside ? dot3(dh, w.ax) : 1.0f) - 1e-5f;
    w.sin_t = sqrtf(fmaxf(0.f, 1.0f - w.cos_t * w.cos_t));
    w.oc = mk3(__shfl_sync(0xffffffffu, o.x, 0), __shfl_sync(0xffffffffu, o.y, 0),
               __shfl_sync(0xffffffffu, o.z, 0));
    const v3 dv = o - w.oc;
    w.r_o = warp_max_f(inside ? sqrtf(dot3(dv, dv)) : 0.f);
    w.rt_max = warp_max_f(inside ? fabsf(rt) : 0.f);
    // cull only narrow cones of directions (the pixels of one warp are a few
    // degrees apart); anything unusual keeps every Gaussian
    w.on = (w.cos_t > 0.5f) && __all_sync(0xffffffffu, !inside || (dl > 0.f && isfinite(dl)));
    return w;
}

// Radius of the sphere around mu that holds the Gaussian's alpha >= 1/255
// region: negative when the Gaussian is nowhere visible (opacity <= 1/255),
// infinite when no bound is known (keep it).
__device__ __forceinline__ float cone_radius(float4 r0, float4 r1, float4 r2, float4 r3) {
    const float op = r3.x;
    if (!(op * 255.0f > 1.0f)) return -1.0f;  // alpha <= opacity < 1/255 everywhere
    const float m0 = r0.x * r0.x + r0.y * r0.y + r0.z * r0.z;
    const float m1 = r1.x * r1.x + r1.y * r1.y + r1.z * r1.z;
    const float m2 = r2.x * r2.x + r2.y * r2.y + r2.z * r2.z;
    const float mmin = fminf(m0, fminf(m1, m2));  // 1 / s_max^2
    if (!(mmin > 0.f) || !isfinite(op)) return INFINITY;
    return sqrtf(2.0f * logf(op * 255.0f) / mmin);
}

// true: some line of the warp's cone may see alpha >= 1/255 of the Gaussian
// at mu (moving with vel when dyn) whose cone_radius is R0
__device__ __forceinline__ bool cone_may_hit_r(const WarpCone& w, float R0, v3 mu, v3 vel, bool dyn) {
    if (!w.on) return true;
    if (R0 < 0.0f) return false;
    float R = R0;
    if (dyn) R += w.rt_max * sqrtf(dot3(vel, vel));
    const v3 v = mu - w.oc;
    const float vn = sqrtf(dot3(v, v));
    R = (R + w.r_o) * 1.01f + 1e-4f * vn + 1e-6f;
    if (!isfinite(R) || !isfinite(vn) || vn <= R) return true;
    const float cp = fabsf(dot3(v, w.ax)) / vn;  // cos of the angle to the cone axis
    if (cp >= w.cos_t) return true;              // inside the cone
    const float sp = sqrtf(fmaxf(0.f, 1.0f - cp * cp));
    const float s_pt = sp * w.cos_t - cp * w.sin_t;  // sin(phi - theta) > 0
    return vn * s_pt <= R;
}

__device__ __forceinline__ bool cone_may_hit(const WarpCone& w, float4 r0, float4 r1, float4 r2, float4 r3,
                                             bool dyn) {
    if (!w.on) return true;
    return cone_may_hit_r(w, cone_radius(r0, r1, r2, r3), mk3(r0.w, r1.w, r2.w), mk3(r3.y, r3.z, r3.w), dyn);
}

// Exact per-pixel pre-test for warps whose pixels share one ray origin o
// (and, for moving Gaussians, one time offset).  With g = M (o - mu) and
// rho^2 = 2 ln(255 opacity), the line o + s d reaches alpha >= 1/255 iff its
// whitened distance to the centre is at most rho, i.e. iff
//   q(d) = d^T A d >= 0,  A = b b^T - k M^T M,  b = M^T g,  k = |g|^2 - rho^2
// (q(d) = |M d|^2 (rho^2 - dist^2)).  A is built once per Gaussian by the
// staging lane; every lane then evaluates q for its own direction with six
// FMAs and a Gaussian stays in the warp's list if any lane may see it.  The
// margin (in dist^2 units, scaled by max |M d|^2 / |d|^2) covers the float
// rounding of q and of the alpha computation with a wide safety factor.
struct Quad {
    float4 a;  // a00, a11, a22, 2 a01
    float4 b;  // 2 a02, 2 a12, margin * lambda_max, unused
};

__device__ __forceinline__ Quad quad_keep_all() {
    Quad q;
    q.a = make_float4(0.f, 0.f, 0.f, 0.f);
    q.b = make_float4(0.f, 0.f, 1.0f, 0.f);
    return q;
}

__device__ __forceinline__ Quad make_quad(float4 r0, float4 r1, float4 r2, float op, v3 mu, v3 o) {
    Quad q;
    if (!(op * 255.0f > 1.0f)) {  // alpha <= opacity < 1/255 on every line
        q.a = make_float4(0.f, 0.f, 0.f, 0.f);
        q.b = make_float4(0.f, 0.f, -1.0f, 0.f);
        return q;
    }
    const v3 m0 = mk3(r0.x, r0.y, r0.z), m1 = mk3(r1.x, r1.y, r1.z), m2 = mk3(r2.x, r2.y, r2.z);
    const v3 om = o - mu;
    const v3 g = mk3(dot3(m0, om), dot3(m1, om), dot3(m2, om));
    const float g2 = dot3(g, g);
    const float rho2 = 2.0f * logf(op * 255.0f);
    const float k = g2 - rho2;
    if (!(k > 0.0f) || !isfinite(g2)) return quad_keep_all();  // origin inside the ellipsoid
    const v3 b = g.x * m0 + g.y * m1 + g.z * m2;
    // M^T M = sum_i row_i row_i^T
    const float s00 = m0.x * m0.x + m1.x * m1.x + m2.x * m2.x;
    const float s11 = m0.y * m0.y + m1.y * m1.y + m2.y * m2.y;
    const float s22 = m0.z * m0.z + m1.z * m1.z + m2.z * m2.z;
    const float s01 = m0.x * m0.y + m1.x * m1.y + m2.x * m2.y;
    const float s02 = m0.x * m0.z + m1.x * m1.z + m2.x * m2.z;
    const float s12 = m0.y * m0.z + m1.y * m1.z + m2.y * m2.z;
    const float lmax = fmaxf(dot3(m0, m0), fmaxf(dot3(m1, m1), dot3(m2, m2)));
    const float marg = 1e-3f * rho2 + 1e-5f * sqrtf(g2) * (sqrtf(rho2) + 1.0f) + 1e-6f + 4e-6f * (g2 + fabsf(k));
    q.a = make_float4(b.x * b.x - k * s00, b.y * b.y - k * s11, b.z * b.z - k * s22, 2.0f * (b.x * b.y - k * s01));
    q.b = make_float4(2.0f * (b.x * b.z - k * s02), 2.0f * (b.y * b.z - k * s12), marg * lmax, 0.f);
    if (!isfinite(q.a.x) || !isfinite(q.a.y) || !isfinite(q.a.z) || !isfinite(q.a.w) || !isfinite(q.b.x) ||
        !isfinite(q.b.y) || !isfinite(q.b.z))
        return quad_keep_all();
    return q;
}

// The warp-independent work of staging a Gaussian for rays from origin o,
// done once per Gaussian by the pack pass: e[0] = quadric a, e[1] =
// (quadric b.xyz, cone_radius), e[2] = (M (o - mu), 0).
__device__ __forceinline__ void view_consts(float4 r0, float4 r1, float4 r2, float4 r3, v3 o, float4* e) {
    const v3 mu = mk3(r0.w, r1.w, r2.w);
    const Quad q = make_quad(r0, r1, r2, r3.x, mu, o);
    const v3 gro = fx_mrows(r0, r1, r2, o - mu);
    e[0] = q.a;
    e[1] = make_float4(q.b.x, q.b.y, q.b.z, cone_radius(r0, r1, r2, r3));
    e[2] = make_float4(gro.x, gro.y, gro.z, 0.f);
}

// per-lane direction products for the quadric pre-test
struct DirQ {
    float xx, yy, zz, xy, xz, yz, dd;
};
__device__ __forceinline__ DirQ dir_q(v3 d) {
    DirQ r{d.x * d.x, d.y * d.y, d.z * d.z, d.x * d.y, d.x * d.z, d.y * d.z, 0.f};
    r.dd = r.xx + r.yy + r.zz;
    return r;
}
__device__ __forceinline__ float eval_quad(const float4& A, const float4& B, const DirQ& q) {
    return A.x * q.xx + A.y * q.yy + A.z * q.zz + A.w * q.xy + B.x * q.xz + B.y * q.yz + B.z * q.dd;
}

// ------------------------------------------------------------ forward ----
// Warp-independent: each warp owns 32 pixels (an 8 x 4 block of a tile),
// takes the tile's list 32 entries at a time and stops as soon as all its
// pixels are saturated.  There is no block-wide barrier; the CTA only groups
// a tile's warps on one SM so they share L1.
//
// Per batch, lane i stages entry i: it loads the record, runs the warp-cone
// test and leaves the quadric terms in shared memory, and the quadric loop
// keeps the entries some lane may see.  The staging lanes of those then write
// their records, in list order, as pairs: kept entry 2j in the low and 2j+1
// in the high half of pair j's float2 components.  The evaluation loop reads
// one pair at a time, computes both alphas with the paired FP32 instructions
// and composites the two entries in order.
constexpr int kWarpSlot = 32;
constexpr int kPairs = kWarpSlot / 2;
constexpr uint16_t kNoSlot = 0xffffu;

// float2 components of a staged pair: 0-8 M row-major, 9-11 M (o - mu) when
// the warp has one ray origin and -mu otherwise, 12 opacity, then -velocity
// (dynamic) and the colour channels (CDIM <= 4)
template <int CDIM, bool kDyn>
struct PairLayout {
    static constexpr bool kColor = CDIM > 0 && CDIM <= 4;
    static constexpr int kVel = 13;
    static constexpr int kCol = kDyn ? 16 : 13;
    static constexpr int kComps = kCol + (kColor ? CDIM : 0);
    static constexpr int kWords = (kComps + 1) / 2;  // float4 words a pair uses
    static constexpr int kStride = kWords + 1;       // padded: pairs start in different banks
    // float4 per warp: quadric terms (2 per entry), pairs, Gaussian ids and pair slots
    static constexpr int kWarpF4 = 2 * kWarpSlot + kPairs * kStride + (kWarpSlot * 6) / 16;
};

// component C of a pair (float2: entry A, entry B) out of its float4 words
template <int C>
__device__ __forceinline__ float2 pc(const float4* w) {
    return (C & 1) ? make_float2(w[C >> 1].z, w[C >> 1].w) : make_float2(w[C >> 1].x, w[C >> 1].y);
}

template <int CDIM, bool kDyn>
__global__ void __launch_bounds__(256, 4) raster_fwd_kernel(RasterArgs a) {
    using PL = PairLayout<CDIM, kDyn>;
    constexpr bool kStageColor = PL::kColor;
    constexpr int CSZ = CDIM > 0 ? CDIM : 1;
    extern __shared__ float4 smem4[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float4* sqa = smem4 + wid * PL::kWarpF4;
    float4* sqb = sqa + kWarpSlot;
    float4* sp = sqb + kWarpSlot;  // [kPairs][kStride]
    int32_t* sid = reinterpret_cast<int32_t*>(sp + kPairs * PL::kStride);
    uint16_t* sslot = reinterpret_cast<uint16_t*>(sid + kWarpSlot);

    const TileCtx c = tile_ctx(a);
    const v3 o = c.inside ? ld3(a.ray_o + 3 * c.pix) : mk3(0.f, 0.f, 0.f);
    const v3 d = c.inside ? ld3(a.ray_d + 3 * c.pix) : mk3(0.f, 0.f, 0.f);
    const float rt = (kDyn && c.inside && a.ray_t) ? a.ray_t[c.pix] : 0.0f;
    // lane 0 has the warp's left-most, top-most pixel: if it is outside the
    // image every lane is
    const v3 o0 = mk3(__shfl_sync(0xffffffffu, o.x, 0), __shfl_sync(0xffffffffu, o.y, 0),
                      __shfl_sync(0xffffffffu, o.z, 0));
    const bool same = !c.inside || (__float_as_uint(o.x) == __float_as_uint(o0.x) &&
                                    __float_as_uint(o.y) == __float_as_uint(o0.y) &&
                                    __float_as_uint(o.z) == __float_as_uint(o0.z));
    // static scene and one ray origin for the warp: M (o - mu) once per Gaussian
    const bool uni = !kDyn && __all_sync(0xffffffffu, same);
    const WarpCone cone = warp_cone(c.inside, o, d, rt);
    // the quadric pre-test needs one origin (and one time offset) per warp
    const float rt0 = __shfl_sync(0xffffffffu, rt, 0);
    const bool qcull = __all_sync(0xffffffffu, same && (!kDyn || !c.inside || rt == rt0));
    // rays from pixel 0's origin: the pack pass has the view constants
    const bool gref = !kDyn && a.ext && uni && __float_as_uint(o0.x) == __float_as_uint(a.ray_o[0]) &&
                      __float_as_uint(o0.y) == __float_as_uint(a.ray_o[1]) &&
                      __float_as_uint(o0.z) == __float_as_uint(a.ray_o[2]);
    const DirQ dq = dir_q(d);
    const p3 d2 = {pdup(d.x), pdup(d.y), pdup(d.z)};

    bool done = !c.inside;
    float T = 1.0f, depth = 0.0f;
    float acc[CSZ];
#pragma unroll
    for (int k = 0; k < CSZ; ++k) acc[k] = 0.f;
    int32_t cur = 0;
    int32_t stop = c.end;  // index of the terminating pair, for the pair counters
    unsigned n_contrib = 0;
    // warp-level work counters (staged, cone-passed, quadric-passed, evaluated)
    unsigned long long w_staged = 0, w_cone = 0, w_quad = 0, w_eval = 0;
    const bool counting = a.pair_counters != nullptr;
    int32_t n_batches = 0;  // batches this warp took (and wrote masks for)
    for (int32_t base = c.start; base < c.end; base += kWarpSlot) {
        if (__all_sync(0xffffffffu, done)) break;
        ++n_batches;
        const int32_t idx = base + lane;
        bool keep = false;
        float4 r0 = make_float4(0.f, 0.f, 0.f, 0.f), r1 = r0, r2 = r0, r3 = r0, cc = r0;
        if (idx < c.end) {
            const int32_t g = a.flatten[idx];
            const float4* r = a.rec + int64_t(kRecF4) * g;
            r0 = r[0]; r1 = r[1]; r2 = r[2]; r3 = r[3];
            Quad qd = quad_keep_all();
            if (gref) {
                const float4* e = a.ext + 3 * int64_t(g);
                const float4 e0 = e[0], e1 = e[1], e2 = e[2];
                keep = cone_may_hit_r(cone, e1.w, mk3(r0.w, r1.w, r2.w), mk3(0.f, 0.f, 0.f), false);
                if (keep) {
                    qd.a = e0;
                    qd.b = make_float4(e1.x, e1.y, e1.z, 0.f);
                }
                r0.w = e2.x; r1.w = e2.y; r2.w = e2.z;  // M (o - mu)
            } else {
                keep = cone_may_hit(cone, r0, r1, r2, r3, kDyn);
                if (qcull && keep) {
                    v3 mu = mk3(r0.w, r1.w, r2.w);
                    if (kDyn) mu = mu + rt0 * mk3(r3.y, r3.z, r3.w);
                    qd = make_quad(r0, r1, r2, r3.x, mu, o0);
                }
                if (uni) {
                    const v3 gro = fx_mrows(r0, r1, r2, o0 - mk3(r0.w, r1.w, r2.w));
                    r0.w = gro.x; r1.w = gro.y; r2.w = gro.z;
                } else {
                    r0.w = -r0.w; r1.w = -r1.w; r2.w = -r2.w;  // -mu
                }
            }
            sqa[lane] = qd.a;
            sqb[lane] = qd.b;
            if constexpr (kStageColor) {
                const float* cp = a.colors + int64_t(g) * CDIM;
                cc.x = cp[0];
                if (CDIM > 1) cc.y = cp[1];
                if (CDIM > 2) cc.z = cp[2];
                if (CDIM > 3) cc.w = cp[3];
            } else {
                sid[lane] = g;
            }
        }
        unsigned live = __ballot_sync(0xffffffffu, keep);
        __syncwarp();
        if (counting) {
            w_staged += unsigned(min(kWarpSlot, c.end - base));
            w_cone += unsigned(__popc(live));
        }
        if (qcull) {
            unsigned m = live;
            live = 0u;
            while (m) {
                const int t = __ffs(m) - 1;
                m &= m - 1;
                const float q = eval_quad(sqa[t], sqb[t], dq);
                if (__any_sync(0xffffffffu, !done && q >= 0.0f)) live |= 1u << t;
            }
        }
        const int n_live = __popc(live);
        if (counting) w_quad += unsigned(n_live);
        // kept entries, ranked in list order, into the pair layout
        if ((live >> lane) & 1u) {
            const int rank = __popc(live & ((1u << lane) - 1u));
            float* p = reinterpret_cast<float*>(sp + (rank >> 1) * PL::kStride) + (rank & 1);
            auto put = [&](int comp, float v) { p[(comp >> 1) * 4 + (comp & 1) * 2] = v; };
            put(0, r0.x); put(1, r0.y); put(2, r0.z);
            put(3, r1.x); put(4, r1.y); put(5, r1.z);
            put(6, r2.x); put(7, r2.y); put(8, r2.z);
            put(9, r0.w); put(10, r1.w); put(11, r2.w);
            put(12, r3.x);
            if (kDyn) {
                put(PL::kVel, -r3.y); put(PL::kVel + 1, -r3.z); put(PL::kVel + 2, -r3.w);
            }
            if constexpr (kStageColor) {
                put(PL::kCol, cc.x);
                if (CDIM > 1) put(PL::kCol + 1, cc.y);
                if (CDIM > 2) put(PL::kCol + 2, cc.z);
                if (CDIM > 3) put(PL::kCol + 3, cc.w);
            }
            sslot[rank] = uint16_t(lane);
            if (rank == n_live - 1 && !(rank & 1)) sslot[rank + 1] = kNoSlot;  // odd count: B is empty
        }
        __syncwarp();
        unsigned lmask = 0u;  // entries this lane composited (for the contributor mask)
        // one entry of the current pair; true when the pixel saturated on it
        auto composite = [&](float ov, float od, float l, int t, const float (&col)[4]) -> bool {
            const float alpha = fminf(0.999f, ov);
            if (alpha < 1.f / 255.f) return false;
            const float hit_t = div_nr(-od, l);
            const float nT = T * (1.0f - alpha);
            if (nT <= 1e-4f) {
                done = true;
                stop = base + t;
                return true;
            }
            const float vis = alpha * T;
            depth += vis * hit_t;
            if constexpr (kStageColor) {
#pragma unroll
                for (int k = 0; k < CDIM; ++k) acc[k] += col[k] * vis;
            } else if constexpr (CDIM > 0) {
                const float* cp = a.colors + int64_t(sid[t]) * CDIM;
#pragma unroll 4
                for (int k = 0; k < CDIM; ++k) acc[k] += cp[k] * vis;
            }
            cur = base + t;
            T = nT;
            ++n_contrib;
            lmask |= 1u << t;
            return false;
        };
        const int n_pairs = (n_live + 1) >> 1;
        for (int j = 0; j < n_pairs && !done; ++j) {
            float4 w[PL::kWords];
#pragma unroll
            for (int k = 0; k < PL::kWords; ++k) w[k] = sp[j * PL::kStride + k];
            const uint32_t slots = reinterpret_cast<const uint32_t*>(sslot)[j];
            const int tA = int(slots & 0xffffu), tB = int(slots >> 16);
            if (counting) w_eval += (tB == kNoSlot) ? 1 : 2;
            p3 gro = {pc<9>(w), pc<10>(w), pc<11>(w)};
            if (!uni) {
                // the pair holds -mu: gro = M (o - mu) for this lane's origin
                p3 nmu = gro;
                if (kDyn) {
                    const float2 r2 = pdup(rt);
                    nmu = {__ffma2_rn(r2, pc<PL::kVel>(w), nmu.x), __ffma2_rn(r2, pc<PL::kVel + 1>(w), nmu.y),
                           __ffma2_rn(r2, pc<PL::kVel + 2>(w), nmu.z)};
                }
                const p3 omm = {__fadd2_rn(pdup(o.x), nmu.x), __fadd2_rn(pdup(o.y), nmu.y),
                                __fadd2_rn(pdup(o.z), nmu.z)};
                gro = {pdot({pc<0>(w), pc<1>(w), pc<2>(w)}, omm), pdot({pc<3>(w), pc<4>(w), pc<5>(w)}, omm),
                       pdot({pc<6>(w), pc<7>(w), pc<8>(w)}, omm)};
            }
            const p3 grd = {pdot({pc<0>(w), pc<1>(w), pc<2>(w)}, d2), pdot({pc<3>(w), pc<4>(w), pc<5>(w)}, d2),
                            pdot({pc<6>(w), pc<7>(w), pc<8>(w)}, d2)};
            const float2 l = pdot(grd, grd);
            const float2 il = make_float2(l.x > 0.0f ? rsqrtf(l.x) : 1.0f, l.y > 0.0f ? rsqrtf(l.y) : 1.0f);
            const p3 gn = {__fmul2_rn(grd.x, il), __fmul2_rn(grd.y, il), __fmul2_rn(grd.z, il)};
            const p3 gc = pcross(gn, gro);
            const float2 pw = __fmul2_rn(pdup(-0.5f), pdot(gc, gc));
            const float2 ov = __fmul2_rn(pc<12>(w), make_float2(__expf(pw.x), __expf(pw.y)));
            const float2 od = pdot(gro, grd);
            float colA[4] = {0.f, 0.f, 0.f, 0.f}, colB[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (kStageColor) {
                colA[0] = pc<PL::kCol>(w).x; colB[0] = pc<PL::kCol>(w).y;
                if constexpr (CDIM > 1) { colA[1] = pc<PL::kCol + 1>(w).x; colB[1] = pc<PL::kCol + 1>(w).y; }
                if constexpr (CDIM > 2) { colA[2] = pc<PL::kCol + 2>(w).x; colB[2] = pc<PL::kCol + 2>(w).y; }
                if constexpr (CDIM > 3) { colA[3] = pc<PL::kCol + 3>(w).x; colB[3] = pc<PL::kCol + 3>(w).y; }
            }
            if (composite(ov.x, od.x, l.x, tA, colA)) break;
            if (tB != kNoSlot && composite(ov.y, od.y, l.y, tB, colB)) break;
        }
        const unsigned cmask = a.masks ? __reduce_or_sync(0xffffffffu, lmask) : 0u;
        if (a.masks && lane == 0)
            a.masks[mask_index(c.start, c.tile, (base - c.start) >> 5, int(blockDim.x >> 5), wid)] = cmask;
        __syncwarp();
    }
    if (a.pair_counters) {
        // evaluated pairs as the reference counts them: every pair of the
        // tile's list up to and including the terminating one
        unsigned long long e = c.inside ? (unsigned long long)(min(stop + 1, c.end) - c.start) : 0ull;
        unsigned long long k = n_contrib;
#pragma unroll
        for (int o_ = 16; o_ > 0; o_ >>= 1) {
            e += __shfl_xor_sync(0xffffffffu, e, o_);
            k += __shfl_xor_sync(0xffffffffu, k, o_);
        }
        // lanes leave the evaluation loop when they saturate: the warp's count is the longest
        w_eval = __reduce_max_sync(0xffffffffu, unsigned(w_eval));
        if (lane == 0) {
            atomicAdd(a.pair_counters, e);
            atomicAdd(a.pair_counters + 1, k);
            atomicAdd(a.pair_counters + 2, w_staged);
            atomicAdd(a.pair_counters + 3, w_cone);
            atomicAdd(a.pair_counters + 4, w_quad);
            atomicAdd(a.pair_counters + 5, w_eval);
        }
    }
    if (a.px2_stats && (c.tile & 3) == 0) {
        // union and sum of the mask bits of this tile's block pairs, for the
        // backward's choice of kernel (every fourth tile is a large enough sample)
        __shared__ int32_t s_nb[32];
        __shared__ unsigned long long s_cnt[2];
        if (threadIdx.x < 2) s_cnt[threadIdx.x] = 0ull;
        if (lane == 0) s_nb[wid] = n_batches;
        __syncthreads();
        if (!(wid & 1)) {
            const int wpt = int(blockDim.x >> 5);
            const int32_t kA = s_nb[wid] - 1, kB = s_nb[wid + 1] - 1;
            unsigned u = 0u, both = 0u;
            for (int32_t k = lane; k <= max(kA, kB); k += 32) {
                const uint32_t mA = k <= kA ? a.masks[mask_index(c.start, c.tile, k, wpt, wid)] : 0u;
                const uint32_t mB = k <= kB ? a.masks[mask_index(c.start, c.tile, k, wpt, wid + 1)] : 0u;
                u += unsigned(__popc(mA | mB));
                both += unsigned(__popc(mA) + __popc(mB));
            }
            u = __reduce_add_sync(0xffffffffu, u);
            both = __reduce_add_sync(0xffffffffu, both);
            if (lane == 0) {
                atomicAdd(&s_cnt[0], (unsigned long long)u);
                atomicAdd(&s_cnt[1], (unsigned long long)both);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && (s_cnt[0] | s_cnt[1])) {
            atomicAdd(a.px2_stats, s_cnt[0]);
            atomicAdd(a.px2_stats + 1, s_cnt[1]);
            if (a.pair_counters) {
                atomicAdd(a.pair_counters + 6, s_cnt[0]);
                atomicAdd(a.pair_counters + 7, s_cnt[1]);
            }
        }
    }
    if (c.inside) {
        a.out_alpha[c.pix] = 1.0f - T;
        a.out_depth[c.pix] = depth;
#pragma unroll
        for (int k = 0; k < CDIM; ++k) a.out_rgb[c.pix * CDIM + k] = acc[k];
        a.out_last[c.pix] = cur;
    }
}

// ----------------------------------------------------------- backward ----
// Per-Gaussian gradient accumulator (floats):
//   0-2 v_mean   3 v_opacity   4-12 dL/dM (3x3, row-major)   13-15 v_colour
//   16 v_colour[3] (C == 4)   then v_velocity (dynamic).
// The quaternion/scale gradients are linear in dL/dM for a fixed Gaussian, so
// dL/dM is summed over all pixels and the reference's per-pair
// quat_scale_to_preci_half_vjp (rasterization/utils.h:232-263) is applied
// once per Gaussian in the finalize pass.
//   factored warps (static scene, no ray gradients, see raster_bwd_kernel):
//   kFactSlot + 0-2 sum of v_gro, + 3 v_opacity.
template <int CDIM, bool kDyn, bool kRayGrad>
struct Acc {
    static constexpr int kExtraColor = (CDIM == 4) ? 1 : 0;
    static constexpr int kVel = 16 + kExtraColor;
    static constexpr bool kFact = !kDyn && !kRayGrad;
    static constexpr int kFactSlot = (CDIM == 4) ? 20 : 16;
    static constexpr int N = kFact ? kFactSlot + 4 : ((kDyn || CDIM == 4) ? 20 : 16);
};
// largest accumulator width of any variant (floats per Gaussian)
constexpr int kMaxAcc = 24;

// Transpose butterfly: on entry every lane holds v[0..15]; on exit lane L
// holds in v[0] the warp-wide sum of value index (L >> 1) & 15.
__device__ __forceinline__ void butterfly16(float (&v)[16], int lane) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const bool up = lane & 16;
        const float send = up ? v[i] : v[i + 8];
        const float keep = up ? v[i + 8] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = lane & 8;
        const float send = up ? v[i] : v[i + 4];
        const float keep = up ? v[i + 4] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = lane & 4;
        const float send = up ? v[i] : v[i + 2];
        const float keep = up ? v[i + 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
        const bool up = lane & 2;
        const float send = up ? v[0] : v[1];
        const float keep = up ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Warp-independent like the forward: each warp walks the tile's list back to
// front from its own last contributor, and every (warp, Gaussian) event with a
// contributing lane is reduced in registers (butterfly) and added to the
// Gaussian's accumulator with four vector reductions.
//
// kRayGrad = false skips the per-pixel ray gradients (v_ray_o, v_ray_d,
// v_ray_time_delta), which callers whose rays need no gradient do not use.
// Then, in a warp whose pixels all share the ray origin of pixel 0 (static
// scenes, global shutter), the terms linear in (o - mu) are factored out of
// the per-pixel sums: each lane contributes v_gro instead of
// v_mean = -M^T v_gro and only the v_grd (x) d part of dL/dM, the warp sums go
// to the accumulator's factored slots, and the finalize pass adds
// sum(v_gro) (x) (o - mu) to dL/dM and -M^T sum(v_gro) to v_mean once per
// Gaussian.
template <int CDIM, bool kDyn, bool kRayGrad>
__global__ void __launch_bounds__(256, 3) raster_bwd_kernel(RasterArgs a) {
    constexpr bool kStageColor = CDIM > 0 && CDIM <= 4;
    constexpr int CSZ = CDIM > 0 ? CDIM : 1;
    using AC = Acc<CDIM, kDyn, kRayGrad>;
    constexpr int NA = AC::N;
    extern __shared__ float4 smem4[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float4* s0 = smem4 + wid * (8 * kWarpSlot);
    float4* s1 = s0 + kWarpSlot;
    float4* s2 = s1 + kWarpSlot;
    float4* s3 = s2 + kWarpSlot;
    float4* sc = s3 + kWarpSlot;
    float4* sqa = sc + kWarpSlot;
    float4* sqb = sqa + kWarpSlot;
    float4* sgro = sqb + kWarpSlot;
    int32_t* sid = reinterpret_cast<int32_t*>(smem4 + (blockDim.x >> 5) * 8 * kWarpSlot) + wid * kWarpSlot;

    if (a.px2_stats && px2_chosen(a.px2_stats)) return;  // the two-pixels-a-lane kernel has the image
    const TileCtx c = tile_ctx(a);
    const bool inside = c.inside;
    const v3 o = inside ? ld3(a.ray_o + 3 * c.pix) : mk3(0.f, 0.f, 0.f);
    const v3 d = inside ? ld3(a.ray_d + 3 * c.pix) : mk3(0.f, 0.f, 0.f);
    const float rt = (kDyn && inside) ? a.ray_t[c.pix] : 0.0f;
    const float T_final = 1.0f - a.render_alpha[c.pix];
    float T = T_final;
    float buf[CSZ];
    float vc[CSZ];
#pragma unroll
    for (int k = 0; k < CSZ; ++k) {
        buf[k] = 0.f;
        vc[k] = 0.f;
    }
    const int32_t bin_final = inside ? a.last_ids[c.pix] : -1;
    if (a.v_rgb) {
#pragma unroll
        for (int k = 0; k < CDIM; ++k) vc[k] = inside ? a.v_rgb[c.pix * CDIM + k] : 0.f;
    }
    const float vd = inside ? a.v_depth[c.pix] : 0.f;
    const float va = inside ? a.v_alpha[c.pix] : 0.f;
    v3 vro = mk3(0.f, 0.f, 0.f), vrd = mk3(0.f, 0.f, 0.f);
    float vtime = 0.f, dbuf = 0.f;

    const WarpCone cone = warp_cone(inside, o, d, rt);
    const v3 o0 = mk3(__shfl_sync(0xffffffffu, o.x, 0), __shfl_sync(0xffffffffu, o.y, 0),
                      __shfl_sync(0xffffffffu, o.z, 0));
    const float rt0 = __shfl_sync(0xffffffffu, rt, 0);
    const bool qcull = __all_sync(0xffffffffu, !inside || (__float_as_uint(o.x) == __float_as_uint(o0.x) &&
                                                          __float_as_uint(o.y) == __float_as_uint(o0.y) &&
                                                          __float_as_uint(o.z) == __float_as_uint(o0.z) &&
                                                          (!kDyn || rt == rt0)));
    const DirQ dq = dir_q(d);
    // warp-uniform: every pixel of the warp has pixel 0's ray origin
    const bool oref = qcull && __float_as_uint(o0.x) == __float_as_uint(a.ray_o[0]) &&
                      __float_as_uint(o0.y) == __float_as_uint(a.ray_o[1]) &&
                      __float_as_uint(o0.z) == __float_as_uint(a.ray_o[2]);
    const bool fact = AC::kFact && oref;
    // rays from pixel 0's origin: the pack pass has the view constants
    const bool gref = !kDyn && a.ext && oref;
    // this warp's last contributor bounds where it starts
    int32_t wmax = bin_final;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, off));
    // one entry of the staged batch (slot t, list index gidx) for all lanes of the warp
    auto process = [&](int t, int32_t gidx) {
        bool valid = inside && (gidx <= bin_final);
        const float4 r0 = s0[t], r1 = s1[t], r2 = s2[t], r3 = s3[t];
        v3 mu = mk3(r0.w, r1.w, r2.w);
        const v3 vel = mk3(r3.y, r3.z, r3.w);
        if (kDyn) mu = fx_moved(mu, vel, rt);
        const v3 omm = o - mu;
        v3 gro;
        if (gref) {
            const float4 ge = sgro[t];
            gro = mk3(ge.x, ge.y, ge.z);
        } else {
            gro = fx_mrows(r0, r1, r2, omm);
        }
        // the forward's arithmetic: same alpha, same decisions
        const EvalTerms ev = fx_eval(r0, r1, r2, gro, d);
        const v3 grd = ev.grd, gn = ev.gn, gc = ev.gc;
        const float l = ev.l, vis = ev.vis;
        const float op = r3.x;
        const float alpha = fminf(0.99f, op * vis);
        if (alpha < 1.f / 255.f) valid = false;
        if (!__any_sync(0xffffffffu, valid)) return;

        float gv[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) gv[k] = 0.f;
        float gvel[3] = {0.f, 0.f, 0.f};
        float gcol[CSZ];
#pragma unroll
        for (int k = 0; k < CSZ; ++k) gcol[k] = 0.f;
        if (valid) {
            const float od = fx_dot(gro, grd);
            const float hit_t = div_nr(-od, l);
            const float ra = div_nr(1.0f, fmaxf(1e-6f, 1.0f - alpha));
            T *= ra;
            const float fac = alpha * T;
            float rgb[CSZ];
            if constexpr (kStageColor) {
                const float4 cc = sc[t];
                rgb[0] = cc.x;
                if (CDIM > 1) rgb[1] = cc.y;
                if (CDIM > 2) rgb[2] = cc.z;
                if (CDIM > 3) rgb[3] = cc.w;
            } else if constexpr (CDIM > 0) {
                const float* cp = a.colors + int64_t(sid[t]) * CDIM;
#pragma unroll 4
                for (int k = 0; k < CDIM; ++k) rgb[k] = cp[k];
            }
            float v_alpha = 0.f;
#pragma unroll
            for (int k = 0; k < CDIM; ++k) {
                gcol[k] = vc[k] * fac;
                v_alpha += (rgb[k] * T - buf[k] * ra) * vc[k];
            }
            v_alpha += (hit_t * T - dbuf * ra) * vd;
            v_alpha += T_final * ra * va;
            // hit distance t* = -(gro . grd) / (grd . grd)
            const float dLdt = vd * fac;
            const float il2 = __fdividef(1.0f, l);
            v3 v_gro = (-dLdt * il2) * grd;
            v3 v_grd = (dLdt * il2 * il2) * (2.0f * od * grd - l * gro);
            if (op * vis <= 0.99f) {
                const float v_vis = op * v_alpha;
                const float v_dist = -0.5f * vis * v_vis;
                const v3 v_gc = 2.0f * v_dist * gc;
                const v3 v_gn = -1.0f * cross3(v_gc, gro);
                v_gro = v_gro + cross3(v_gc, gn);
                if (l > 0.0f) {
                    const float il = rsqrtf(l);
                    const float il3 = il * il * il;
                    v_grd = v_grd + (il * v_gn - il3 * dot3(v_gn, grd) * grd);
                } else {
                    v_grd = v_grd + v_gn;
                }
                if (kRayGrad || kDyn || !fact) {
                    // v_(o - mu) = M^T v_gro
                    const v3 v_omm = mk3(r0.x * v_gro.x + r1.x * v_gro.y + r2.x * v_gro.z,
                                         r0.y * v_gro.x + r1.y * v_gro.y + r2.y * v_gro.z,
                                         r0.z * v_gro.x + r1.z * v_gro.y + r2.z * v_gro.z);
                    gv[0] = -v_omm.x; gv[1] = -v_omm.y; gv[2] = -v_omm.z;
                    if constexpr (kRayGrad) {
                        // v_ray_d = M^T v_grd
                        const v3 v_d = mk3(r0.x * v_grd.x + r1.x * v_grd.y + r2.x * v_grd.z,
                                           r0.y * v_grd.x + r1.y * v_grd.y + r2.y * v_grd.z,
                                           r0.z * v_grd.x + r1.z * v_grd.y + r2.z * v_grd.z);
                        vro = vro + v_omm;
                        vrd = vrd + v_d;
                        if (kDyn) vtime += -dot3(v_omm, vel);
                    }
                    if (kDyn) {
                        gvel[0] = -v_omm.x * rt; gvel[1] = -v_omm.y * rt; gvel[2] = -v_omm.z * rt;
                    }
                } else {
                    gv[0] = v_gro.x; gv[1] = v_gro.y; gv[2] = v_gro.z;
                }
                gv[3] = vis * v_alpha;
                // dL/dM row i = v_grd[i] d + v_gro[i] (o - mu); in factored
                // warps the finalize pass adds the second term
                v3 vM0 = v_grd.x * d, vM1 = v_grd.y * d, vM2 = v_grd.z * d;
                if (!fact) {
                    vM0 = vM0 + v_gro.x * omm;
                    vM1 = vM1 + v_gro.y * omm;
                    vM2 = vM2 + v_gro.z * omm;
                }
                gv[4] = vM0.x; gv[5] = vM0.y; gv[6] = vM0.z;
                gv[7] = vM1.x; gv[8] = vM1.y; gv[9] = vM1.z;
                gv[10] = vM2.x; gv[11] = vM2.y; gv[12] = vM2.z;
            }
#pragma unroll
            for (int k = 0; k < CDIM; ++k) buf[k] += rgb[k] * fac;
            dbuf += fac * hit_t;
        }
        if constexpr (kStageColor) {
#pragma unroll
            for (int k = 0; k < (CDIM < 3 ? CDIM : 3); ++k) gv[13 + k] = gcol[k];
        }
        butterfly16(gv, lane);
        // lanes 8k+0/2/4/6 hold values 4k..4k+3: gather them into lane 8k
        const float g1 = __shfl_down_sync(0xffffffffu, gv[0], 2);
        const float g2 = __shfl_down_sync(0xffffffffu, gv[0], 4);
        const float g3 = __shfl_down_sync(0xffffffffu, gv[0], 6);
        float* dst = a.G + int64_t(sid[t]) * NA;
        // a factored warp's first group (sum of v_gro, v_opacity) goes to its own slots
        const int slot = (fact && lane == 0) ? AC::kFactSlot : (lane >> 1);
        if ((lane & 7) == 0) red_add_v4(dst + slot, gv[0], g1, g2, g3);
        if constexpr (CDIM == 4 || kDyn) {
            float e0 = 0.f, e1 = 0.f, e2 = 0.f, e3 = 0.f;
            if constexpr (CDIM == 4) e0 = warp_sum(gcol[3]);
            if constexpr (kDyn) {
                const float x0 = warp_sum(gvel[0]), x1 = warp_sum(gvel[1]), x2 = warp_sum(gvel[2]);
                if (AC::kVel == 16) { e0 = x0; e1 = x1; e2 = x2; }
                else { e1 = x0; e2 = x1; e3 = x2; }
            }
            if (lane == 0) red_add_v4(dst + 16, e0, e1, e2, e3);
        }
        if constexpr (!kStageColor && CDIM > 0) {
            // wide colours: warp-reduced straight into the output
            for (int k = 0; k < CDIM; ++k) {
                const float sv = warp_sum(gcol[k]);
                if (lane == 0 && sv != 0.f) atomicAdd(a.v_colors_direct + int64_t(sid[t]) * CDIM + k, sv);
            }
        }
    };
    if (a.masks) {
        // the forward's contributor masks: visit only entries some lane of
        // this warp composited, without the cone and quadric pre-tests
        const int wpt = int(blockDim.x >> 5);
        // a pixel without contributors has last id 0: stay inside the tile's list
        const int32_t wlast = min(wmax, c.end - 1);
        for (int32_t k = wlast >= c.start ? (wlast - c.start) >> 5 : -1; k >= 0; --k) {
            const uint32_t cm = a.masks[mask_index(c.start, c.tile, k, wpt, wid)];
            if (!cm) continue;
            const int32_t base = c.start + (k << 5);
            if ((cm >> lane) & 1u) {
                const int32_t g = a.flatten[base + lane];
                const float4* r = a.rec + int64_t(kRecF4) * g;
                s0[lane] = r[0]; s1[lane] = r[1]; s2[lane] = r[2]; s3[lane] = r[3];
                if (gref) sgro[lane] = a.ext[3 * int64_t(g) + 2];  // M (o - mu)
                if constexpr (kStageColor) {
                    float4 cc = make_float4(0.f, 0.f, 0.f, 0.f);
                    const float* cp = a.colors + int64_t(g) * CDIM;
                    cc.x = cp[0];
                    if (CDIM > 1) cc.y = cp[1];
                    if (CDIM > 2) cc.z = cp[2];
                    if (CDIM > 3) cc.w = cp[3];
                    sc[lane] = cc;
                }
                sid[lane] = g;
            }
            __syncwarp();
            unsigned live = cm;
            while (live) {
                const int t = 31 - __clz(live);
                live &= ~(1u << t);
                process(t, base + t);
            }
            __syncwarp();
        }
    } else {
        for (int32_t top = min(c.end - 1, wmax); top >= c.start; top -= kWarpSlot) {
            const int32_t idx = top - lane;
            bool keep = false;
            if (idx >= c.start) {
                const int32_t g = a.flatten[idx];
                const float4* r = a.rec + int64_t(kRecF4) * g;
                const float4 r0 = r[0], r1 = r[1], r2 = r[2], r3 = r[3];
                Quad qd = quad_keep_all();
                if (gref) {
                    const float4* e = a.ext + 3 * int64_t(g);
                    const float4 e0 = e[0], e1 = e[1];
                    sgro[lane] = e[2];  // M (o - mu)
                    keep = cone_may_hit_r(cone, e1.w, mk3(r0.w, r1.w, r2.w), mk3(0.f, 0.f, 0.f), false);
                    if (keep) {
                        qd.a = e0;
                        qd.b = make_float4(e1.x, e1.y, e1.z, 0.f);
                    }
                } else {
                    keep = cone_may_hit(cone, r0, r1, r2, r3, kDyn);
                    if (qcull && keep) {
                        v3 mu = mk3(r0.w, r1.w, r2.w);
                        if (kDyn) mu = mu + rt0 * mk3(r3.y, r3.z, r3.w);
                        qd = make_quad(r0, r1, r2, r3.x, mu, o0);
                    }
                }
                sqa[lane] = qd.a;
                sqb[lane] = qd.b;
                s0[lane] = r0; s1[lane] = r1; s2[lane] = r2; s3[lane] = r3;
                if constexpr (kStageColor) {
                    float4 cc = make_float4(0.f, 0.f, 0.f, 0.f);
                    const float* cp = a.colors + int64_t(g) * CDIM;
                    cc.x = cp[0];
                    if (CDIM > 1) cc.y = cp[1];
                    if (CDIM > 2) cc.z = cp[2];
                    if (CDIM > 3) cc.w = cp[3];
                    sc[lane] = cc;
                }
                sid[lane] = g;
            }
            unsigned live = __ballot_sync(0xffffffffu, keep);
            __syncwarp();
            if (qcull) {
                unsigned m = live;
                live = 0u;
                while (m) {
                    const int t = __ffs(m) - 1;
                    m &= m - 1;
                    const float q = eval_quad(sqa[t], sqb[t], dq);
                    if (__any_sync(0xffffffffu, inside && (top - t <= bin_final) && q >= 0.0f)) live |= 1u << t;
                }
            }
            while (live) {
                const int t = __ffs(live) - 1;
                live &= live - 1;
                process(t, top - t);
            }
            __syncwarp();
        }
    }
    if (kRayGrad && inside) {
        st3(a.v_ray_o + 3 * c.pix, vro);
        st3(a.v_ray_d + 3 * c.pix, vrd);
        if (kDyn) a.v_ray_t[c.pix] = vtime;
    }
}

// ------------------------------------------ backward, two pixels a lane --
// The static-scene backward without ray gradients (the training call), when
// the forward's contributor masks are at hand, with two pixels per lane: a
// warp owns two of the forward's 8 x 4 pixel blocks (pixel A of lane l is
// lane l of the forward's warp 2w, pixel B lane l of warp 2w + 1), visits the
// union of their masks back to front, evaluates every entry for both pixels
// at once with the paired FP32 instructions (.x pixel A, .y pixel B; the
// Gaussian's values are staged duplicated, so each is a ready pair) and adds
// the two pixels' gradient values before the butterfly, which so runs once
// per 64 pixels.  The alpha arithmetic is the forward's (fx_eval, per half).
//
// The colour and depth terms of v_alpha are carried as one running sum per
// pixel: with X = sum_k rgb_k vc_k + hit_t vd, the reference's
//   v_alpha = sum_k (rgb_k T - buf_k ra) vc_k + (hit_t T - dbuf ra) vd + T_final ra va
// equals T X - ra Z with Z = sum_k buf_k vc_k + dbuf vd - T_final va, and
// every contributing entry adds fac X to Z.
template <int CDIM>
struct Px2 {
    // duplicated float2 components of a staged entry: 0-8 M row-major,
    // 9-11 -mu, 12 opacity, 13-15 M (o - mu) for rays from pixel 0's origin,
    // then the colour channels
    static constexpr int kNmu = 9, kOp = 12, kGro = 13, kCol = 16;
    static constexpr int kWords = (kCol + CDIM + 1) / 2;  // float4 per entry
    static constexpr size_t warp_bytes() { return size_t(kWarpSlot) * (kWords * sizeof(float4) + sizeof(int32_t)); }
};

__device__ __forceinline__ p3 pscale(p3 a, float2 s) {
    return {__fmul2_rn(a.x, s), __fmul2_rn(a.y, s), __fmul2_rn(a.z, s)};
}
__device__ __forceinline__ float hsum(float2 a) { return a.x + a.y; }

template <int CDIM>
__global__ void __launch_bounds__(128, 4) raster_bwd_px2_kernel(RasterArgs a) {
    using L = Px2<CDIM>;
    using AC = Acc<CDIM, false, false>;
    constexpr int NA = AC::N;
    constexpr int CSZ = CDIM > 0 ? CDIM : 1;
    extern __shared__ float4 smem4[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float4* sw = smem4 + wid * (L::kWords * kWarpSlot);  // [kWords][32]
    int32_t* sid = reinterpret_cast<int32_t*>(smem4 + (blockDim.x >> 5) * L::kWords * kWarpSlot) + wid * kWarpSlot;

    if (!px2_chosen(a.px2_stats)) return;  // the per-pixel kernel has the image
    const int tile = a.tile_order ? a.tile_order[blockIdx.x] : int(blockIdx.x);
    const int ty = tile / a.ntx, tx = tile - ty * a.ntx;
    const int wc = a.tsx >> 3;
    const int fA = 2 * wid, fB = 2 * wid + 1;  // the forward's warps
    const int pxA = tx * a.tsx + (fA % wc) * 8 + (lane & 7), pyA = ty * a.tsy + (fA / wc) * 4 + (lane >> 3);
    const int pxB = tx * a.tsx + (fB % wc) * 8 + (lane & 7), pyB = ty * a.tsy + (fB / wc) * 4 + (lane >> 3);
    const bool inA = pxA < a.W && pyA < a.H, inB = pxB < a.W && pyB < a.H;
    const int64_t pixA = int64_t(pyA) * a.W + pxA, pixB = int64_t(pyB) * a.W + pxB;
    const int32_t start = a.offsets[tile];
    const int32_t end = (tile == a.ntx * a.nty - 1) ? int32_t(a.n_isects_dev ? *a.n_isects_dev : a.n_isects)
                                                    : a.offsets[tile + 1];

    // pixels outside the image get a harmless ray and never contribute
    const v3 o_ref = ld3(a.ray_o);
    const v3 oA = inA ? ld3(a.ray_o + 3 * pixA) : o_ref, oB = inB ? ld3(a.ray_o + 3 * pixB) : o_ref;
    const v3 dA = inA ? ld3(a.ray_d + 3 * pixA) : mk3(0.f, 0.f, 1.f);
    const v3 dB = inB ? ld3(a.ray_d + 3 * pixB) : mk3(0.f, 0.f, 1.f);
    auto same = [](v3 u, v3 v) {
        return __float_as_uint(u.x) == __float_as_uint(v.x) && __float_as_uint(u.y) == __float_as_uint(v.y) &&
               __float_as_uint(u.z) == __float_as_uint(v.z);
    };
    // every pixel has pixel 0's ray origin: factored accumulation, view constants
    const bool fact = __all_sync(0xffffffffu, same(oA, o_ref) && same(oB, o_ref));
    const bool gref = fact && a.ext;
    const p3 o2 = {make_float2(oA.x, oB.x), make_float2(oA.y, oB.y), make_float2(oA.z, oB.z)};
    const p3 d2 = {make_float2(dA.x, dB.x), make_float2(dA.y, dB.y), make_float2(dA.z, dB.z)};
    const int32_t binA = inA ? a.last_ids[pixA] : -1, binB = inB ? a.last_ids[pixB] : -1;
    float2 T = make_float2(inA ? 1.0f - a.render_alpha[pixA] : 1.0f, inB ? 1.0f - a.render_alpha[pixB] : 1.0f);
    float2 vc[CSZ];
#pragma unroll
    for (int k = 0; k < CSZ; ++k) vc[k] = make_float2(0.f, 0.f);
    if (a.v_rgb) {
#pragma unroll
        for (int k = 0; k < CDIM; ++k)
            vc[k] = make_float2(inA ? a.v_rgb[pixA * CDIM + k] : 0.f, inB ? a.v_rgb[pixB * CDIM + k] : 0.f);
    }
    const float2 vd = make_float2(inA ? a.v_depth[pixA] : 0.f, inB ? a.v_depth[pixB] : 0.f);
    const float2 va = make_float2(inA ? a.v_alpha[pixA] : 0.f, inB ? a.v_alpha[pixB] : 0.f);
    float2 nZ = __fmul2_rn(T, va);  // -Z = T_final va before any entry
    // each forward warp's last contributor, inside the tile's list: the
    // forward wrote that warp's masks for every batch up to it, and no others
    int32_t wA = binA, wB = binB;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        wA = max(wA, __shfl_xor_sync(0xffffffffu, wA, off));
        wB = max(wB, __shfl_xor_sync(0xffffffffu, wB, off));
    }
    wA = min(wA, end - 1);
    wB = min(wB, end - 1);
    const int32_t kA = wA >= start ? (wA - start) >> 5 : -1, kB = wB >= start ? (wB - start) >> 5 : -1;
    const int wpt = (a.tsx * a.tsy) >> 5;  // the forward's warps per tile


    auto process = [&](int t, int32_t gidx) {
        float4 w[L::kWords];
#pragma unroll
        for (int k = 0; k < L::kWords; ++k) w[k] = sw[k * kWarpSlot + t];
        const p3 M0 = {pc<0>(w), pc<1>(w), pc<2>(w)}, M1 = {pc<3>(w), pc<4>(w), pc<5>(w)},
                 M2 = {pc<6>(w), pc<7>(w), pc<8>(w)};
        p3 omm = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)}, gro;
        if (gref) {
            gro = {pc<L::kGro>(w), pc<L::kGro + 1>(w), pc<L::kGro + 2>(w)};
        } else {
            omm = {__fadd2_rn(o2.x, pc<L::kNmu>(w)), __fadd2_rn(o2.y, pc<L::kNmu + 1>(w)),
                   __fadd2_rn(o2.z, pc<L::kNmu + 2>(w))};
            gro = {pdot(M0, omm), pdot(M1, omm), pdot(M2, omm)};
        }
        const p3 grd = {pdot(M0, d2), pdot(M1, d2), pdot(M2, d2)};
        const float2 l = pdot(grd, grd);
        const float2 il = make_float2(l.x > 0.0f ? rsqrtf(l.x) : 1.0f, l.y > 0.0f ? rsqrtf(l.y) : 1.0f);
        const p3 gn = pscale(grd, il);
        const p3 gc = pcross(gn, gro);
        const float2 pw = __fmul2_rn(pdup(-0.5f), pdot(gc, gc));
        const float2 vis = make_float2(__expf(pw.x), __expf(pw.y));
        const float2 op = pc<L::kOp>(w);
        const float2 ov = __fmul2_rn(op, vis);
        const float alA = fminf(0.99f, ov.x), alB = fminf(0.99f, ov.y);
        const bool vA = inA && gidx <= binA && !(alA < 1.f / 255.f);
        const bool vB = inB && gidx <= binB && !(alB < 1.f / 255.f);
        const unsigned vmask = __ballot_sync(0xffffffffu, vA || vB);
        if (!vmask) return;
        if (a.pair_counters && lane == 0) {
            // work counters 8-10: entries processed, lanes with a contributing
            // pixel over them, entries with at most two such lanes
            atomicAdd(a.pair_counters + 8, 1ull);
            atomicAdd(a.pair_counters + 9, (unsigned long long)__popc(vmask));
            if (__popc(vmask) <= 2) atomicAdd(a.pair_counters + 10, 1ull);
        }

        const float2 od = pdot(gro, grd);
        const float hA = div_nr(-od.x, l.x), hB = div_nr(-od.y, l.y);
        const float2 ra = make_float2(div_nr(1.0f, fmaxf(1e-6f, 1.0f - alA)),
                                      div_nr(1.0f, fmaxf(1e-6f, 1.0f - alB)));
        T = make_float2(vA ? T.x * ra.x : T.x, vB ? T.y * ra.y : T.y);
        const float2 nfac = make_float2(vA ? -(alA * T.x) : 0.f, vB ? -(alB * T.y) : 0.f);
        // X = sum_k rgb_k vc_k + hit_t vd
        float2 X = __fmul2_rn(make_float2(hA, hB), vd);
        if constexpr (CDIM > 0) X = __ffma2_rn(pc<L::kCol>(w), vc[0], X);
        if constexpr (CDIM > 1) X = __ffma2_rn(pc<L::kCol + 1>(w), vc[1], X);
        if constexpr (CDIM > 2) X = __ffma2_rn(pc<L::kCol + 2>(w), vc[2], X);
        if constexpr (CDIM > 3) X = __ffma2_rn(pc<L::kCol + 3>(w), vc[3], X);
        const float2 v_alpha = __ffma2_rn(T, X, __fmul2_rn(ra, nZ));  // T X - ra Z
        nZ = __ffma2_rn(nfac, X, nZ);                                 // Z += fac X

        // the alpha-dependent gradients: zero where the pixel does not
        // contribute or its alpha was clamped
        const bool kA = vA && ov.x <= 0.99f, kB = vB && ov.y <= 0.99f;
        const float2 il2 = make_float2(__fdividef(1.0f, l.x), __fdividef(1.0f, l.y));
        const float2 ndl = __fmul2_rn(vd, nfac);  // -dL/dt* = -vd fac
        const float2 c1 = make_float2(kA ? ndl.x * il2.x : 0.f, kB ? ndl.y * il2.y : 0.f);
        const float2 vae = make_float2(kA ? v_alpha.x : 0.f, kB ? v_alpha.y : 0.f);
        // hit distance t* = -(gro . grd) / l: v_gro = -dLdt / l grd,
        // v_grd = dLdt / l^2 (2 od grd - l gro) = (c1 / l) (l gro - 2 od grd)
        p3 v_gro = pscale(grd, c1);
        const float2 c2 = __fmul2_rn(c1, il2);
        const float2 ntod = __fmul2_rn(od, pdup(-2.0f));
        p3 v_grd = {__fmul2_rn(c2, __ffma2_rn(ntod, grd.x, __fmul2_rn(l, gro.x))),
                    __fmul2_rn(c2, __ffma2_rn(ntod, grd.y, __fmul2_rn(l, gro.y))),
                    __fmul2_rn(c2, __ffma2_rn(ntod, grd.z, __fmul2_rn(l, gro.z)))};
        // power = -|gc|^2 / 2: v_gc = -(vis op v_alpha) gc
        const float2 q = pneg(__fmul2_rn(vis, __fmul2_rn(op, vae)));
        const p3 v_gc = pscale(gc, q);
        const p3 v_gn = pcross(gro, v_gc);
        const p3 xg = pcross(v_gc, gn);
        v_gro = {__fadd2_rn(v_gro.x, xg.x), __fadd2_rn(v_gro.y, xg.y), __fadd2_rn(v_gro.z, xg.z)};
        // normalisation: v_grd += il v_gn - il^3 (v_gn . grd) grd
        const float2 s = pneg(__fmul2_rn(__fmul2_rn(__fmul2_rn(il, il), il), pdot(v_gn, grd)));
        v_grd = {__ffma2_rn(s, grd.x, __ffma2_rn(il, v_gn.x, v_grd.x)),
                 __ffma2_rn(s, grd.y, __ffma2_rn(il, v_gn.y, v_grd.y)),
                 __ffma2_rn(s, grd.z, __ffma2_rn(il, v_gn.z, v_grd.z))};

        float gv[16];
        if (fact) {
            gv[0] = hsum(v_gro.x); gv[1] = hsum(v_gro.y); gv[2] = hsum(v_gro.z);
        } else {
            // v_mean = -M^T v_gro
            gv[0] = -hsum(__ffma2_rn(M2.x, v_gro.z, __ffma2_rn(M1.x, v_gro.y, __fmul2_rn(M0.x, v_gro.x))));
            gv[1] = -hsum(__ffma2_rn(M2.y, v_gro.z, __ffma2_rn(M1.y, v_gro.y, __fmul2_rn(M0.y, v_gro.x))));
            gv[2] = -hsum(__ffma2_rn(M2.z, v_gro.z, __ffma2_rn(M1.z, v_gro.y, __fmul2_rn(M0.z, v_gro.x))));
        }
        gv[3] = hsum(__fmul2_rn(vis, vae));
        // dL/dM row i = v_grd[i] d (+ v_gro[i] (o - mu) when not factored)
        const float2 vg[3] = {v_grd.x, v_grd.y, v_grd.z};
        const float2 vo[3] = {v_gro.x, v_gro.y, v_gro.z};
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            float2 m0 = __fmul2_rn(vg[i], d2.x), m1 = __fmul2_rn(vg[i], d2.y), m2 = __fmul2_rn(vg[i], d2.z);
            if (!fact) {
                m0 = __ffma2_rn(vo[i], omm.x, m0);
                m1 = __ffma2_rn(vo[i], omm.y, m1);
                m2 = __ffma2_rn(vo[i], omm.z, m2);
            }
            gv[4 + 3 * i] = hsum(m0);
            gv[5 + 3 * i] = hsum(m1);
            gv[6 + 3 * i] = hsum(m2);
        }
        float gc3 = 0.f;
#pragma unroll
        for (int k = 0; k < 3; ++k) gv[13 + k] = k < CDIM ? -hsum(__fmul2_rn(vc[k < CSZ ? k : 0], nfac)) : 0.f;
        if constexpr (CDIM == 4) gc3 = -hsum(__fmul2_rn(vc[3], nfac));

        float* dst = a.G + int64_t(sid[t]) * NA;
        butterfly16(gv, lane);
        // lanes 8k+0/2/4/6 hold values 4k..4k+3: gather them into lane 8k
        const float g1 = __shfl_down_sync(0xffffffffu, gv[0], 2);
        const float g2 = __shfl_down_sync(0xffffffffu, gv[0], 4);
        const float g3 = __shfl_down_sync(0xffffffffu, gv[0], 6);
        // a factored warp's first group (sum of v_gro, v_opacity) goes to its own slots
        const int slot = (fact && lane == 0) ? AC::kFactSlot : (lane >> 1);
        if ((lane & 7) == 0) red_add_v4(dst + slot, gv[0], g1, g2, g3);
        if constexpr (CDIM == 4) {
            const float e0 = warp_sum(gc3);
            if (lane == 0) red_add_v4(dst + 16, e0, 0.f, 0.f, 0.f);
        }
    };

    for (int32_t k = max(kA, kB); k >= 0; --k) {
        const uint32_t cm = (k <= kA ? a.masks[mask_index(start, tile, k, wpt, fA)] : 0u) |
                            (k <= kB ? a.masks[mask_index(start, tile, k, wpt, fB)] : 0u);
        if (!cm) continue;
        const int32_t base = start + (k << 5);
        if ((cm >> lane) & 1u) {
            const int32_t g = a.flatten[base + lane];
            const float4* r = a.rec + int64_t(kRecF4) * g;
            const float4 r0 = r[0], r1 = r[1], r2 = r[2], r3 = r[3];
            const float4 e2 = gref ? a.ext[3 * int64_t(g) + 2] : make_float4(0.f, 0.f, 0.f, 0.f);  // M (o - mu)
            float4* s = sw + lane;
            s[0 * kWarpSlot] = make_float4(r0.x, r0.x, r0.y, r0.y);
            s[1 * kWarpSlot] = make_float4(r0.z, r0.z, r1.x, r1.x);
            s[2 * kWarpSlot] = make_float4(r1.y, r1.y, r1.z, r1.z);
            s[3 * kWarpSlot] = make_float4(r2.x, r2.x, r2.y, r2.y);
            s[4 * kWarpSlot] = make_float4(r2.z, r2.z, -r0.w, -r0.w);
            s[5 * kWarpSlot] = make_float4(-r1.w, -r1.w, -r2.w, -r2.w);
            s[6 * kWarpSlot] = make_float4(r3.x, r3.x, e2.x, e2.x);
            s[7 * kWarpSlot] = make_float4(e2.y, e2.y, e2.z, e2.z);
            if constexpr (CDIM > 0) {
                const float* cp = a.colors + int64_t(g) * CDIM;
                const float c0 = cp[0], c1 = CDIM > 1 ? cp[1] : 0.f;
                s[8 * kWarpSlot] = make_float4(c0, c0, c1, c1);
                if constexpr (CDIM > 2) {
                    const float c2 = cp[2], c3 = CDIM > 3 ? cp[3] : 0.f;
                    s[9 * kWarpSlot] = make_float4(c2, c2, c3, c3);
                }
            }
            sid[lane] = g;
        }
        __syncwarp();
        unsigned live = cm;
        while (live) {
            const int t = 31 - __clz(live);
            live &= ~(1u << t);
            process(t, base + t);
        }
        __syncwarp();
    }
}

// Accumulator -> output layout, with the quaternion / scale VJP of the summed
// dL/dM (quat_scale_to_preci_half_vjp, rasterization/utils.h:208-263).
template <int CDIM, bool kDyn, bool kRayGrad>
__global__ void grads_finalize_kernel(const float* __restrict__ G, const float* __restrict__ quats,
                                      const float* __restrict__ scales, const float* __restrict__ means,
                                      const float* __restrict__ ray_o, int64_t n, float* __restrict__ v_means,
                                      float* __restrict__ v_vel, float* __restrict__ v_quats,
                                      float* __restrict__ v_scales, float* __restrict__ v_opac,
                                      float* __restrict__ v_colors) {
    using AC = Acc<CDIM, kDyn, kRayGrad>;
    constexpr int NA = AC::N;
    const int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (g >= n) return;
    float A[NA];
    const float4* s = reinterpret_cast<const float4*>(G + g * NA);
#pragma unroll
    for (int k = 0; k < NA / 4; ++k) {
        const float4 v = s[k];
        A[4 * k] = v.x; A[4 * k + 1] = v.y; A[4 * k + 2] = v.z; A[4 * k + 3] = v.w;
    }
    v3 vM0 = mk3(A[4], A[5], A[6]), vM1 = mk3(A[7], A[8], A[9]), vM2 = mk3(A[10], A[11], A[12]);
    float w = quats[4 * g], x = quats[4 * g + 1], y = quats[4 * g + 2], z = quats[4 * g + 3];
    const float inv = rsqrtf(x * x + y * y + z * z + w * w);
    x *= inv; y *= inv; z *= inv; w *= inv;
    const float x2 = x * x, y2 = y * y, z2 = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float wx = w * x, wy = w * y, wz = w * z;
    // columns of R
    const v3 C0 = mk3(1.f - 2.f * (y2 + z2), 2.f * (xy + wz), 2.f * (xz - wy));
    const v3 C1 = mk3(2.f * (xy - wz), 1.f - 2.f * (x2 + z2), 2.f * (yz + wx));
    const v3 C2 = mk3(2.f * (xz + wy), 2.f * (yz - wx), 1.f - 2.f * (x2 + y2));
    const float isx = 1.0f / scales[3 * g], isy = 1.0f / scales[3 * g + 1], isz = 1.0f / scales[3 * g + 2];
    v3 vmean = mk3(A[0], A[1], A[2]);
    float vop = A[3];
    if constexpr (AC::kFact) {
        // factored warps: s = sum(v_gro) over pixels with the origin o of pixel 0
        constexpr int F = AC::kFactSlot;
        const v3 sg = mk3(A[F], A[F + 1], A[F + 2]);
        vop += A[F + 3];
        const v3 om = mk3(ray_o[0], ray_o[1], ray_o[2]) - ld3(means + 3 * g);
        vM0 = vM0 + sg.x * om;
        vM1 = vM1 + sg.y * om;
        vM2 = vM2 + sg.z * om;
        // row i of M = C_i / s_i:  v_mean -= M^T s
        vmean = vmean - ((sg.x * isx) * C0 + (sg.y * isy) * C1 + (sg.z * isz) * C2);
    }
    v_means[3 * g] = vmean.x; v_means[3 * g + 1] = vmean.y; v_means[3 * g + 2] = vmean.z;
    v_opac[g] = vop;
    v_scales[3 * g] = -isx * isx * dot3(C0, vM0);
    v_scales[3 * g + 1] = -isy * isy * dot3(C1, vM1);
    v_scales[3 * g + 2] = -isz * isz * dot3(C2, vM2);
    // V(c, r) = dL/dR[row r][col c] = dL/dM[c][r] / s_c
    const v3 V0 = isx * vM0, V1 = isy * vM1, V2 = isz * vM2;
    const float gw = 2.f * (x * (V1.z - V2.y) + y * (V2.x - V0.z) + z * (V0.y - V1.x));
    const float gx = 2.f * (-2.f * x * (V1.y + V2.z) + y * (V0.y + V1.x) + z * (V0.z + V2.x) + w * (V1.z - V2.y));
    const float gy = 2.f * (x * (V0.y + V1.x) - 2.f * y * (V0.x + V2.z) + z * (V1.z + V2.y) + w * (V2.x - V0.z));
    const float gz = 2.f * (x * (V0.z + V2.x) + y * (V1.z + V2.y) - 2.f * z * (V0.x + V1.y) + w * (V0.y - V1.x));
    const float dq = gw * w + gx * x + gy * y + gz * z;
    v_quats[4 * g] = (gw - dq * w) * inv;
    v_quats[4 * g + 1] = (gx - dq * x) * inv;
    v_quats[4 * g + 2] = (gy - dq * y) * inv;
    v_quats[4 * g + 3] = (gz - dq * z) * inv;
    if constexpr (CDIM > 0 && CDIM <= 4) {
#pragma unroll
        for (int k = 0; k < CDIM; ++k) v_colors[g * CDIM + k] = (k < 3) ? A[13 + k] : A[16];
    }
    if constexpr (kDyn) {
        v_vel[3 * g] = A[AC::kVel]; v_vel[3 * g + 1] = A[AC::kVel + 1]; v_vel[3 * g + 2] = A[AC::kVel + 2];
    }
}

// ------------------------------------------------------------ dispatch ---
#define XSG_CDIM_CASES(X) \
    X(0) X(1) X(2) X(3) X(4) X(5) X(8) X(9) X(16) X(17) X(32) X(33) X(64) X(65) X(128) X(129) X(256) X(257) X(512) X(513)

static const int kSupported[] = {0, 1, 2, 3, 4, 5, 8, 9, 16, 17, 32, 33, 64, 65, 128, 129, 256, 257, 512, 513};

template <int CDIM, bool kDyn>
static size_t fwd_smem(int bs) { return size_t(bs / 32) * PairLayout<CDIM, kDyn>::kWarpF4 * sizeof(float4); }
// the backward stages per slot 4 record words, the colour, the quadric terms
// and M (o - mu) of view-constant warps (8 float4), and the Gaussian id
static size_t bwd_smem(int bs) { return size_t(bs / 32) * kWarpSlot * (8 * sizeof(float4) + sizeof(int32_t)); }

template <int CDIM, bool kDyn>
static int launch_fwd(const RasterArgs& a, int bs, cudaStream_t st) {
    const size_t sm = fwd_smem<CDIM, kDyn>(bs);
    auto fn = raster_fwd_kernel<CDIM, kDyn>;
    if (sm > 48 * 1024) XSG_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
    {
        ScopedTimer tm("rasterize_fwd", st);
        launch(fn, unsigned(a.ntx * a.nty), bs, sm, st, a);
    }
    return check_launch("rasterize_fwd");
}

struct FinalizeOut {
    float *v_means, *v_vel, *v_quats, *v_scales, *v_opac, *v_colors;
};

template <int CDIM, bool kDyn, bool kRayGrad>
static int launch_bwd(const RasterArgs& a, int bs, cudaStream_t st, int64_t n_gauss, FinalizeOut fin) {
    bool done = false;
    if constexpr (!kDyn && !kRayGrad && CDIM <= 4) {
        // two pixels a lane: needs the masks and an even count of 8 x 4 warp blocks per tile
        if (a.px2_stats) {
            const size_t sm = size_t(bs / 64) * Px2<CDIM>::warp_bytes();
            auto fn = raster_bwd_px2_kernel<CDIM>;
            if (sm > 48 * 1024)
                XSG_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
            // and the per-pixel one: the forward's mask counts choose which works
            RasterArgs b = a;
            const size_t sm1 = bwd_smem(bs);
            auto fn1 = raster_bwd_kernel<CDIM, kDyn, kRayGrad>;
            if (sm1 > 48 * 1024)
                XSG_CUDA(cudaFuncSetAttribute(fn1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm1)));
            ScopedTimer tm("rasterize_bwd", st);
            launch(fn, unsigned(a.ntx * a.nty), bs / 2, sm, st, b);
            launch(fn1, unsigned(a.ntx * a.nty), bs, sm1, st, b);
            done = true;
        }
    }
    if (!done) {
        const size_t sm = bwd_smem(bs);
        auto fn = raster_bwd_kernel<CDIM, kDyn, kRayGrad>;
        if (sm > 48 * 1024) XSG_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
        ScopedTimer tm("rasterize_bwd", st);
        RasterArgs b = a;
        b.px2_stats = nullptr;
        launch(fn, unsigned(a.ntx * a.nty), bs, sm, st, b);
    }
    if (a.G && n_gauss > 0)
        launch(grads_finalize_kernel<CDIM, kDyn, kRayGrad>, blocks_for(n_gauss, 256), 256, 0, st, a.G, a.quats,
               a.scales, a.means, a.ray_o, n_gauss, fin.v_means, fin.v_vel, fin.v_quats, fin.v_scales, fin.v_opac,
               fin.v_colors);
    return check_launch("rasterize_bwd");
}

static bool cdim_supported(int c) {
    for (int v : kSupported)
        if (v == c) return true;
    return false;
}

static int check_common(int64_t n_gauss, int W, int H, int tsx, int tsy, int tiles_w, int tiles_h,
                        int64_t n_isects, int cdim) {
    XSG_REQUIRE(n_gauss >= 0 && n_isects >= 0 && W > 0 && H > 0, "rasterize: bad sizes");
    XSG_REQUIRE(tsx > 0 && tsy > 0 && tsx * tsy <= 1024 && (tsx * tsy) % 32 == 0,
                "rasterize: tile_size_x * tile_size_y must be a multiple of 32 and at most 1024");
    XSG_REQUIRE(tiles_w > 0 && tiles_h > 0, "rasterize: bad tile grid");
    XSG_REQUIRE(n_isects < (int64_t(1) << 31), "rasterize: too many intersections");
    if (!cdim_supported(cdim))
        return set_error(XSG_ERR_UNSUPPORTED, "Unsupported number of channels: " + std::to_string(cdim));
    return XSG_OK;
}

// words of the contributor masks: one per (batch of 32 list entries, warp),
// tile batch ranges start at (start >> 5) + tile (see mask_index)
static int64_t mask_batch_words(int64_t n_isects, int64_t n_tiles, int tile_pixels) {
    if (n_isects <= 0 || n_tiles <= 0 || tile_pixels < 32) return 0;
    return (n_isects / 32 + n_tiles + 2) * (tile_pixels / 32);
}
// ... followed by the two 64-bit block-pair counts (px2_stats)
static int64_t px2_stats_word(int64_t n_isects, int64_t n_tiles, int tile_pixels) {
    return (mask_batch_words(n_isects, n_tiles, tile_pixels) + 1) & ~int64_t(1);
}
static int64_t mask_words(int64_t n_isects, int64_t n_tiles, int tile_pixels) {
    return mask_batch_words(n_isects, n_tiles, tile_pixels) ? px2_stats_word(n_isects, n_tiles, tile_pixels) + 4 : 0;
}
// the block-pair counts exist (and the backward may run two pixels a lane)
// for static scenes with staged colours, 8 x 4 warp blocks and an even count
// of them per tile
static bool px2_layout(int cdim, bool dyn, int tsx, int tsy) {
    return !dyn && cdim <= 4 && tsx % 8 == 0 && tsy % 4 == 0 && ((tsx * tsy) / 32) % 2 == 0;
}

}  // namespace xsg

using namespace xsg;

extern "C" {

void xsg_set_pair_counters(unsigned long long* counters) { g_pair_counters = counters; }

int xsg_raster_supported_channels(int* out, int cap) {
    const int n = int(sizeof(kSupported) / sizeof(int));
    for (int i = 0; i < n && i < cap; ++i) out[i] = kSupported[i];
    return n;
}

size_t xsg_rasterize_workspace_size(int64_t n_gauss, int cdim, int64_t n_isects, int64_t n_tiles,
                                    int tile_pixels) {
    (void)cdim;
    if (n_gauss < 0) n_gauss = 0;
    // packed records, view constants, tile order, contributor masks (when the
    // intersection and tile counts are given) and the gradient accumulator
    return Arena::round(size_t(n_gauss) * kRecF4 * sizeof(float4)) +
           Arena::round(size_t(n_gauss) * 3 * sizeof(float4)) +
           Arena::round(size_t(kMaxTiles) * sizeof(int32_t)) +
           Arena::round(size_t(mask_words(n_isects, n_tiles, tile_pixels)) * sizeof(uint32_t)) +
           Arena::round(size_t(n_gauss) * kMaxAcc * sizeof(float));
}

int xsg_rasterize_fwd(const float* means, const float* velocity, const float* quats, const float* scales,
                      const float* colors, int cdim, const float* opacities, int64_t n_gauss, int W, int H,
                      int tsx, int tsy, const float* ray_o, const float* ray_d, const float* ray_time_delta,
                      const int32_t* tile_offsets, int tiles_w, int tiles_h, const int32_t* flatten_ids,
                      int64_t n_isects, float* renders, float* depths, float* alphas, int32_t* last_ids,
                      void* workspace, size_t ws_bytes, xsg_stream_t stream, const int64_t* n_isects_dev) {
    int rc = check_common(n_gauss, W, H, tsx, tsy, tiles_w, tiles_h, n_isects, cdim);
    if (rc != XSG_OK) return rc;
    XSG_REQUIRE(means && quats && scales && opacities && ray_o && ray_d && tile_offsets && depths && alphas &&
                    last_ids, "rasterize_fwd: null argument");
    XSG_REQUIRE(cdim == 0 || (colors && renders), "rasterize_fwd: colors required");
    XSG_REQUIRE(n_isects == 0 || flatten_ids, "rasterize_fwd: null flatten_ids");
    cudaStream_t st = as_cuda(stream);
    Arena ar(workspace, ws_bytes);
    float4* rec = ar.take<float4>(size_t(n_gauss) * kRecF4);
    float4* ext = ar.take<float4>(size_t(n_gauss) * 3);
    const int64_t n_tiles = int64_t(tiles_w) * tiles_h;
    int32_t* order = n_tiles <= kMaxTiles ? ar.take<int32_t>(size_t(kMaxTiles)) : nullptr;
    // contributor masks for the backward, when the workspace was sized for them
    const int64_t nmw = mask_words(n_isects, n_tiles, tsx * tsy);
    const bool with_masks =
        nmw > 0 && ws_bytes >= xsg_rasterize_workspace_size(n_gauss, cdim, n_isects, n_tiles, tsx * tsy);
    uint32_t* masks = with_masks ? ar.take<uint32_t>(size_t(nmw)) : nullptr;
    if ((n_gauss > 0 && (!rec || !ext)) || (n_gauss > 0 && !workspace))
        return set_error(XSG_ERR_WORKSPACE, "rasterize_fwd: workspace too small");
    const bool dyn = velocity != nullptr;
    if (dyn) ext = nullptr;  // moving Gaussians: no per-view constants
    unsigned long long* px2_stats =
        (masks && px2_layout(cdim, dyn, tsx, tsy))
            ? reinterpret_cast<unsigned long long*>(masks + px2_stats_word(n_isects, n_tiles, tsx * tsy))
            : nullptr;
    if (order)
        launch(tile_order_kernel, 1, 1024, 0, st, tile_offsets, int(n_tiles), int32_t(n_isects), n_isects_dev, order);
    if (n_gauss > 0)
        launch(pack_records_kernel, blocks_for(n_gauss, 256), 256, 0, st, means, velocity, quats, scales, opacities,
               n_gauss, rec, ray_o, ext, px2_stats);
    RasterArgs a{};
    a.rec = rec; a.ext = n_gauss > 0 ? ext : nullptr; a.means = means; a.quats = quats; a.scales = scales; a.colors = colors;
    a.ray_o = ray_o; a.ray_d = ray_d; a.ray_t = ray_time_delta;
    a.offsets = tile_offsets; a.flatten = flatten_ids; a.n_isects = n_isects; a.n_isects_dev = n_isects_dev;
    a.W = W; a.H = H; a.tsx = tsx; a.tsy = tsy; a.ntx = tiles_w; a.nty = tiles_h;
    a.out_rgb = renders; a.out_depth = depths; a.out_alpha = alphas; a.out_last = last_ids;
    a.pair_counters = g_pair_counters;
    a.tile_order = order;
    a.masks = masks;
    a.px2_stats = px2_stats;
    const int bs = tsx * tsy;
#define XSG_FWD_CASE(C)                                                             \
    case C:                                                                         \
        return dyn ? launch_fwd<C, true>(a, bs, st) : launch_fwd<C, false>(a, bs, st);
    switch (cdim) {
        XSG_CDIM_CASES(XSG_FWD_CASE)
        default: break;
    }
#undef XSG_FWD_CASE
    return set_error(XSG_ERR_UNSUPPORTED, "Unsupported number of channels: " + std::to_string(cdim));
}

int xsg_rasterize_bwd(const float* means, const float* velocity, const float* quats, const float* scales,
                      const float* colors, int cdim, const float* opacities, int64_t n_gauss, int W, int H,
                      int tsx, int tsy, const float* ray_o, const float* ray_d, const float* ray_time_delta,
                      const int32_t* tile_offsets, int tiles_w, int tiles_h, const int32_t* flatten_ids,
                      int64_t n_isects, const float* render_alphas, const int32_t* last_ids,
                      const float* v_renders, const float* v_depths, const float* v_alphas, float* v_means,
                      float* v_velocity, float* v_quats, float* v_scales, float* v_colors, float* v_opacities,
                      float* v_ray_o, float* v_ray_d, float* v_ray_time_delta, void* workspace, size_t ws_bytes,
                      int workspace_from_forward, xsg_stream_t stream, const int64_t* n_isects_dev) {
    int rc = check_common(n_gauss, W, H, tsx, tsy, tiles_w, tiles_h, n_isects, cdim);
    if (rc != XSG_OK) return rc;
    const bool dyn = velocity != nullptr;
    XSG_REQUIRE(means && quats && scales && opacities && ray_o && ray_d && tile_offsets && render_alphas &&
                    last_ids && v_depths && v_alphas && v_means && v_quats && v_scales && v_opacities,
                "rasterize_bwd: null argument");
    // the ray gradients are all requested or all skipped
    const bool ray_grads = v_ray_o != nullptr;
    XSG_REQUIRE((v_ray_d != nullptr) == ray_grads && (!dyn || (v_ray_time_delta != nullptr) == ray_grads),
                "rasterize_bwd: pass all of v_ray_o / v_ray_d (/ v_ray_time_delta) or none");
    XSG_REQUIRE(cdim == 0 || (colors && v_colors), "rasterize_bwd: colors required");
    XSG_REQUIRE(!dyn || (ray_time_delta && v_velocity), "rasterize_dynamic_bwd: ray_time_delta is required");
    XSG_REQUIRE(n_isects == 0 || flatten_ids, "rasterize_bwd: null flatten_ids");
    cudaStream_t st = as_cuda(stream);
    Arena ar(workspace, ws_bytes);
    float4* rec = ar.take<float4>(size_t(n_gauss) * kRecF4);
    float4* ext = ar.take<float4>(size_t(n_gauss) * 3);
    const int64_t n_tiles = int64_t(tiles_w) * tiles_h;
    // same layout as the forward's (records, view constants, tile order), then the accumulator
    int32_t* order = n_tiles <= kMaxTiles ? ar.take<int32_t>(size_t(kMaxTiles)) : nullptr;
    // the forward's contributor masks (same layout and condition as there)
    const bool reuse = workspace_from_forward != 0;
    const int64_t nmw = mask_words(n_isects, n_tiles, tsx * tsy);
    const bool with_masks = reuse && nmw > 0 &&
                            ws_bytes >= xsg_rasterize_workspace_size(n_gauss, cdim, n_isects, n_tiles, tsx * tsy);
    uint32_t* masks = with_masks ? ar.take<uint32_t>(size_t(nmw)) : nullptr;
    // Acc<CDIM, kDyn, kRayGrad>::N
    const int na = (!dyn && !ray_grads) ? (cdim == 4 ? 24 : 20) : ((dyn || cdim == 4) ? 20 : 16);
    float* G = ar.take<float>(size_t(n_gauss) * na);
    if (n_gauss > 0 && (!rec || !ext || !G)) return set_error(XSG_ERR_WORKSPACE, "rasterize_bwd: workspace too small");
    if (dyn) ext = nullptr;  // moving Gaussians: no per-view constants
    // every pixel of the image belongs to exactly one tile thread, which
    // writes its v_ray_o / v_ray_d (/ v_ray_time_delta): no pre-zeroing
    // the forward's workspace already holds the tile order, records and view constants
    if (order && !reuse)
        launch(tile_order_kernel, 1, 1024, 0, st, tile_offsets, int(n_tiles), int32_t(n_isects), n_isects_dev,
               order);
    if (n_gauss > 0) {
        XSG_CUDA(cudaMemsetAsync(G, 0, size_t(n_gauss) * na * sizeof(float), st));
        if (cdim > 4) XSG_CUDA(cudaMemsetAsync(v_colors, 0, size_t(n_gauss) * cdim * sizeof(float), st));
        if (!reuse)
            launch(pack_records_kernel, blocks_for(n_gauss, 256), 256, 0, st, means, velocity, quats, scales,
                   opacities, n_gauss, rec, ray_o, ext, nullptr);
    }
    RasterArgs a{};
    a.rec = rec; a.ext = n_gauss > 0 ? ext : nullptr; a.means = means; a.quats = quats; a.scales = scales; a.colors = colors;
    a.ray_o = ray_o; a.ray_d = ray_d; a.ray_t = ray_time_delta;
    a.offsets = tile_offsets; a.flatten = flatten_ids; a.n_isects = n_isects; a.n_isects_dev = n_isects_dev;
    a.W = W; a.H = H; a.tsx = tsx; a.tsy = tsy; a.ntx = tiles_w; a.nty = tiles_h;
    a.render_alpha = render_alphas; a.last_ids = last_ids;
    a.v_rgb = v_renders; a.v_depth = v_depths; a.v_alpha = v_alphas;
    a.G = G; a.v_colors_direct = v_colors;
    a.tile_order = order;
    a.pair_counters = g_pair_counters;
    a.masks = masks;  // written by the forward into the same workspace
    a.px2_stats = (masks && px2_layout(cdim, dyn, tsx, tsy))
                      ? reinterpret_cast<unsigned long long*>(masks + px2_stats_word(n_isects, n_tiles, tsx * tsy))
                      : nullptr;
    a.v_ray_o = v_ray_o; a.v_ray_d = v_ray_d; a.v_ray_t = v_ray_time_delta;
    const int bs = tsx * tsy;
    FinalizeOut fin{v_means, v_velocity, v_quats, v_scales, v_opacities, v_colors};
    int lrc = XSG_OK;
#define XSG_BWD_CASE(C)                                                                          \
    case C:                                                                                      \
        lrc = dyn ? (ray_grads ? launch_bwd<C, true, true>(a, bs, st, n_gauss, fin)                \
                               : launch_bwd<C, true, false>(a, bs, st, n_gauss, fin))              \
                  : (ray_grads ? launch_bwd<C, false, true>(a, bs, st, n_gauss, fin)               \
                               : launch_bwd<C, false, false>(a, bs, st, n_gauss, fin));            \
        break;
    switch (cdim) {
        XSG_CDIM_CASES(XSG_BWD_CASE)
        default: return set_error(XSG_ERR_UNSUPPORTED, "unsupported feature dimension: " + std::to_string(cdim));
    }
#undef XSG_BWD_CASE
    if (lrc != XSG_OK) return lrc;
    return XSG_OK;
}

}  // extern "C"
