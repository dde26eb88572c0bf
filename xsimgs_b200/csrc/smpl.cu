// SMPL skinning on sm_100a: joint-chain composition (local -> global joint
// transforms) and linear-blend skinning of Gaussians into a scene container,
// forward and backward.  Semantics: smpl_local_to_global_fwd/bwd
// (csrc/nodes/smpl_local_to_global.cu:29-338), smpl_lbs_skinning(_bwd)
// (csrc/nodes/smpl_lbs_skinning.cu:11-353), smpl_ids_compaction
// (csrc/nodes/smpl.cu:15-74) of the reference.
//
// Quaternions are (w, x, y, z) in memory; products are Hamilton products;
// R(q) is the quaternion polynomial; std() is unit length with w >= 0;
// matrix -> quaternion is Shepperd's method (trace branch when the trace is
// positive, else the largest diagonal element).
//
// Layout of the work:
//   local -> global   one warp per body, lane j = joint j (24 of 32 lanes);
//                     the chain is composed level by level (depth <= 8) with
//                     shuffles; the backward accumulates the children's
//                     gradients into their parents level by level, deepest
//                     first (reverse-mode over the kinematic tree), through
//                     a per-warp shared-memory slot per joint.
//   skinning          one CTA per (vertex block, body): the body's 24 joint
//                     matrices are built once into shared memory; one thread
//                     per vertex blends them (24 x 12 FMAs) and reads its
//                     weights coalesced from [N, 24, V].  The backward
//                     reduces the joint gradients over the CTA (warp
//                     butterflies, then shared memory) and applies the
//                     matrix -> quaternion VJP once per joint and CTA, so it
//                     issues 7 global atomics per joint per CTA instead of
//                     per vertex.
#include "quat.cuh"

namespace xsg {
namespace {

constexpr int kJ = 24;
__constant__ int8_t c_parent[kJ] = {-1, 0, 0, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 9, 9, 12, 13, 14, 16, 17, 18, 19, 20, 21};
__constant__ int8_t c_depth[kJ] = {0, 1, 1, 1, 2, 2, 2, 3, 3, 3, 4, 4, 4, 4, 4, 5, 5, 5, 6, 6, 7, 7, 8, 8};
// children of each joint (-1 padded; joint 0 and joint 9 have three)
__constant__ int8_t c_children[kJ][3] = {
    {1, 2, 3},    {4, -1, -1},  {5, -1, -1},  {6, -1, -1},   {7, -1, -1},   {8, -1, -1},
    {9, -1, -1},  {10, -1, -1}, {11, -1, -1}, {12, 13, 14},  {-1, -1, -1},  {-1, -1, -1},
    {15, -1, -1}, {16, -1, -1}, {17, -1, -1}, {-1, -1, -1},  {18, -1, -1},  {19, -1, -1},
    {20, -1, -1}, {21, -1, -1}, {22, -1, -1}, {23, -1, -1},  {-1, -1, -1},  {-1, -1, -1}};
constexpr int kMaxDepth = 8;

struct Tf {
    Q q;
    v3 t;
};

__device__ __forceinline__ Tf compose(const Tf& a, const Tf& b) { return {qmul(a.q, b.q), rot(a.q, b.t) + a.t}; }
__device__ __forceinline__ void compose_bwd(const Tf& a, const Tf& b, Q dq, v3 dt, Q& da_q, v3& da_t, Q& db_q,
                                            v3& db_t) {
    da_q = qadd(qmul(dq, conj(b.q)), rot_bwd_q(a.q, b.t, dt));
    da_t = dt;
    db_q = qmul(conj(a.q), dq);
    db_t = rot(conj(a.q), dt);
}

__device__ __forceinline__ Q shfl_q(Q q, int src) {
    return {__shfl_sync(0xffffffffu, q.w, src), __shfl_sync(0xffffffffu, q.x, src),
            __shfl_sync(0xffffffffu, q.y, src), __shfl_sync(0xffffffffu, q.z, src)};
}
__device__ __forceinline__ v3 shfl_v(v3 v, int src) {
    return {__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src),
            __shfl_sync(0xffffffffu, v.z, src)};
}

// One body's joint data in lane j (lanes >= 24 mirror joint 23 and are ignored).
struct Chain {
    int j, parent, depth;
    Q raw;
    v3 J;
    Tf L, G;
};

__device__ __forceinline__ Chain build_chain(int lane, int64_t obj, const float* local_q, const float* joints) {
    Chain c;
    c.j = min(lane, kJ - 1);
    c.parent = c_parent[c.j];
    c.depth = c_depth[c.j];
    const int64_t o = obj * kJ + c.j;
    c.raw = ldq(local_q + 4 * o);
    c.J = ld3(joints + 3 * o);
    const v3 Jp = shfl_v(c.J, max(c.parent, 0));
    c.L = {qstd(c.raw), c.parent < 0 ? c.J : c.J - Jp};
    c.G = c.L;
#pragma unroll
    for (int d = 1; d <= kMaxDepth; ++d) {
        const Tf Gp{shfl_q(c.G.q, max(c.parent, 0)), shfl_v(c.G.t, max(c.parent, 0))};
        if (c.depth == d) c.G = compose(Gp, c.L);
    }
    return c;
}

constexpr int kBodiesPerBlock = 8;

__global__ void __launch_bounds__(32 * kBodiesPerBlock)
    l2g_fwd_kernel(const uint32_t* __restrict__ ids, int64_t batch, int64_t n_objects, const float* __restrict__ local_q,
                   const float* __restrict__ joints, const float* __restrict__ a0q, const float* __restrict__ a0t,
                   float* __restrict__ out_q, float* __restrict__ out_t) {
    const int64_t b = int64_t(blockIdx.x) * kBodiesPerBlock + threadIdx.y;
    const int lane = threadIdx.x;
    if (b >= batch) return;  // warp-uniform
    const int64_t obj = ids[b];
    if (obj >= n_objects) return;  // warp-uniform; documented: out-of-range ids are skipped
    const Chain c = build_chain(lane, obj, local_q, joints);
    if (lane >= kJ) return;
    const int64_t o = obj * kJ + c.j;
    Tf T{c.G.q, c.G.t - rot(c.G.q, c.J)};
    const Tf out = compose(T, Tf{ldq(a0q + 4 * o), ld3(a0t + 3 * o)});
    stq(out_q + 4 * (b * kJ + c.j), out.q);
    st3(out_t + 3 * (b * kJ + c.j), out.t);
}

__global__ void __launch_bounds__(32 * kBodiesPerBlock)
    l2g_bwd_kernel(const uint32_t* __restrict__ ids, int64_t batch, int64_t n_objects, const float* __restrict__ local_q,
                   const float* __restrict__ joints, const float* __restrict__ a0q, const float* __restrict__ a0t,
                   const float* __restrict__ g_q, const float* __restrict__ g_t, float* __restrict__ d_local_q,
                   float* __restrict__ d_a0q, float* __restrict__ d_a0t) {
    __shared__ float s_da[kBodiesPerBlock][kJ][4];
    const int64_t b = int64_t(blockIdx.x) * kBodiesPerBlock + threadIdx.y;
    const int lane = threadIdx.x;
    if (b >= batch) return;
    const int64_t obj = ids[b];
    if (obj >= n_objects) return;
    const Chain c = build_chain(lane, obj, local_q, joints);
    const int64_t o = obj * kJ + c.j, ob = b * kJ + c.j;
    // output = T o A with T = (G.q, G.t - R(G.q) J)
    const Tf T{c.G.q, c.G.t - rot(c.G.q, c.J)};
    const Tf A{ldq(a0q + 4 * o), ld3(a0t + 3 * o)};
    Q dT_q, dA_q;
    v3 dT_t, dA_t;
    compose_bwd(T, A, ldq(g_q + 4 * ob), ld3(g_t + 3 * ob), dT_q, dT_t, dA_q, dA_t);
    if (lane < kJ) {
        stq(d_a0q + 4 * o, dA_q);
        st3(d_a0t + 3 * o, dA_t);
    }
    // through the -R(G.q) J translation
    Q dG_q = qadd(dT_q, rot_bwd_q(c.G.q, c.J, -1.0f * dT_t));
    v3 dG_t = dT_t;
    // reverse over the tree: G_j = G_parent o L_j, deepest level first
    Q dL_q = dG_q;  // the root's L is its G
    const int w = threadIdx.y;
#pragma unroll 1
    for (int d = kMaxDepth; d >= 1; --d) {
        const Tf Gp{shfl_q(c.G.q, max(c.parent, 0)), shfl_v(c.G.t, max(c.parent, 0))};
        if (lane < kJ && c.depth == d) {
            Q da_q;
            v3 da_t, db_t;
            compose_bwd(Gp, c.L, dG_q, dG_t, da_q, da_t, dL_q, db_t);
            s_da[w][c.j][0] = da_q.w; s_da[w][c.j][1] = da_q.x; s_da[w][c.j][2] = da_q.y; s_da[w][c.j][3] = da_q.z;
            // the parent's translation gradient is da_t, summed below
        }
        __syncwarp();
        // the parents at depth d - 1 add their children's (q, t) gradients;
        // the translation part is the children's dG_t itself (da_t = dt)
        if (lane < kJ && c.depth == d - 1) {
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const int ch = c_children[c.j][k];
                if (ch >= 0) {
                    dG_q.w += s_da[w][ch][0]; dG_q.x += s_da[w][ch][1];
                    dG_q.y += s_da[w][ch][2]; dG_q.z += s_da[w][ch][3];
                }
            }
        }
        // translation gradients: parent += sum of children's dG_t
        const v3 child_t = dG_t;
        v3 add_t = mk3(0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int ch = c_children[c.j][k];
            const v3 tv = shfl_v(child_t, max(ch, 0));
            if (lane < kJ && c.depth == d - 1 && ch >= 0) add_t = add_t + tv;
        }
        dG_t = dG_t + add_t;
        if (c.depth == d - 1 && c.parent < 0) dL_q = dG_q;  // the root
        __syncwarp();
    }
    if (lane < kJ) stq(d_local_q + 4 * o, qstd_bwd(c.raw, dL_q));
}

// ------------------------------------------------------------ skinning --
// rows [R(q) | t]
__device__ __forceinline__ void to_mat34(Q q, v3 t, float4 m[3]) {
    const float w = q.w, x = q.x, y = q.y, z = q.z;
    m[0] = make_float4(1.f - 2.f * (y * y + z * z), 2.f * (x * y - w * z), 2.f * (x * z + w * y), t.x);
    m[1] = make_float4(2.f * (x * y + w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - w * x), t.y);
    m[2] = make_float4(2.f * (x * z - w * y), 2.f * (y * z + w * x), 1.f - 2.f * (x * x + y * y), t.z);
}
// (dq, dt) of sum_rc G[r][c] * mat34(q, t)[r][c]
__device__ __forceinline__ void to_mat34_bwd(Q q, const float G[3][4], Q& dq, v3& dt) {
    const float w = q.w, x = q.x, y = q.y, z = q.z;
    dq.w = 2.f * (-z * G[0][1] + y * G[0][2] + z * G[1][0] - x * G[1][2] - y * G[2][0] + x * G[2][1]);
    dq.x = 2.f * (y * G[0][1] + z * G[0][2] + y * G[1][0] - 2.f * x * G[1][1] - w * G[1][2] + z * G[2][0] +
                  w * G[2][1] - 2.f * x * G[2][2]);
    dq.y = 2.f * (-2.f * y * G[0][0] + x * G[0][1] + w * G[0][2] + x * G[1][0] + z * G[1][2] - w * G[2][0] +
                  z * G[2][1] - 2.f * y * G[2][2]);
    dq.z = 2.f * (-2.f * z * G[0][0] - w * G[0][1] + x * G[0][2] + w * G[1][0] - 2.f * z * G[1][1] + y * G[1][2] +
                  x * G[2][0] + y * G[2][1]);
    dt = mk3(G[0][3], G[1][3], G[2][3]);
}

__device__ __forceinline__ int shepperd_branch(const float m[3][4]) {
    const float tr = m[0][0] + m[1][1] + m[2][2];
    if (tr > 0.f) return 0;
    if (m[0][0] > m[1][1] && m[0][0] > m[2][2]) return 1;
    if (m[1][1] > m[2][2]) return 2;
    return 3;
}
// Shepperd: the selected component is s / 4, the other three are
// (m_ij -+ m_ji) / s, with s = 2 sqrt(1 +- diagonal terms).
__device__ __forceinline__ float shepperd_s(const float m[3][4], int br) {
    const float a = m[0][0], b = m[1][1], c = m[2][2];
    const float rad = br == 0 ? a + b + c + 1.f : br == 1 ? 1.f + a - b - c : br == 2 ? 1.f + b - a - c : 1.f + c - a - b;
    return sqrtf(rad) * 2.f;
}
__device__ __forceinline__ Q from_matrix(const float m[3][4], int br, float s) {
    const float is = 1.0f / s;
    switch (br) {
        case 0: return {0.25f * s, (m[2][1] - m[1][2]) * is, (m[0][2] - m[2][0]) * is, (m[1][0] - m[0][1]) * is};
        case 1: return {(m[2][1] - m[1][2]) * is, 0.25f * s, (m[0][1] + m[1][0]) * is, (m[0][2] + m[2][0]) * is};
        case 2: return {(m[0][2] - m[2][0]) * is, (m[0][1] + m[1][0]) * is, 0.25f * s, (m[1][2] + m[2][1]) * is};
        default: return {(m[1][0] - m[0][1]) * is, (m[0][2] + m[2][0]) * is, (m[1][2] + m[2][1]) * is, 0.25f * s};
    }
}
// gradient of from_matrix w.r.t. the 3x3 part, added into dm
__device__ __forceinline__ void from_matrix_bwd(int br, float s, Q q, Q g, float dm[3][4]) {
    const float is = 1.0f / s;
    float ds = 0.f;
    // numerator entries (r0,c0,+1) and (r1,c1,sign) of each non-s/4 component
    auto term = [&](float val, float gv, int r0, int c0, int r1, int c1, float s1) {
        dm[r0][c0] += gv * is;
        dm[r1][c1] += s1 * gv * is;
        ds -= gv * val * is;
    };
    if (br == 0) {
        ds += 0.25f * g.w;
        term(q.x, g.x, 2, 1, 1, 2, -1.f);
        term(q.y, g.y, 0, 2, 2, 0, -1.f);
        term(q.z, g.z, 1, 0, 0, 1, -1.f);
    } else if (br == 1) {
        ds += 0.25f * g.x;
        term(q.w, g.w, 2, 1, 1, 2, -1.f);
        term(q.y, g.y, 0, 1, 1, 0, 1.f);
        term(q.z, g.z, 0, 2, 2, 0, 1.f);
    } else if (br == 2) {
        ds += 0.25f * g.y;
        term(q.w, g.w, 0, 2, 2, 0, -1.f);
        term(q.x, g.x, 0, 1, 1, 0, 1.f);
        term(q.z, g.z, 1, 2, 2, 1, 1.f);
    } else {
        ds += 0.25f * g.z;
        term(q.w, g.w, 1, 0, 0, 1, -1.f);
        term(q.x, g.x, 0, 2, 2, 0, 1.f);
        term(q.y, g.y, 1, 2, 2, 1, 1.f);
    }
    const float k = ds * 2.f * is;  // d s / d radicand = 2 / s
    dm[0][0] += (br == 0 || br == 1) ? k : -k;
    dm[1][1] += (br == 0 || br == 2) ? k : -k;
    dm[2][2] += (br == 0 || br == 3) ? k : -k;
}

constexpr int kSkinThreads = 256;

struct SkinIn {
    const uint32_t* valid_ids;
    const float* gq;
    const float* gt;
    const float* vertices;
    const float* quats;
    const float* weights;
    const uint32_t* inst_ids;
    int64_t n_objects, V, n_instances, global_offset;
};

// blended 3x4 matrix of vertex v of body object `obj`
__device__ __forceinline__ void blend(const float4 (*sM)[3], const float* __restrict__ weights, int64_t obj,
                                      int64_t V, int64_t v, float W[3][4]) {
    float4 r0 = make_float4(0.f, 0.f, 0.f, 0.f), r1 = r0, r2 = r0;
    const float* wp = weights + obj * kJ * V + v;
#pragma unroll 8
    for (int j = 0; j < kJ; ++j) {
        const float w = __ldg(wp + int64_t(j) * V);
        const float4 a = sM[j][0], b = sM[j][1], c = sM[j][2];
        r0.x += w * a.x; r0.y += w * a.y; r0.z += w * a.z; r0.w += w * a.w;
        r1.x += w * b.x; r1.y += w * b.y; r1.z += w * b.z; r1.w += w * b.w;
        r2.x += w * c.x; r2.y += w * c.y; r2.z += w * c.z; r2.w += w * c.w;
    }
    W[0][0] = r0.x; W[0][1] = r0.y; W[0][2] = r0.z; W[0][3] = r0.w;
    W[1][0] = r1.x; W[1][1] = r1.y; W[1][2] = r1.z; W[1][3] = r1.w;
    W[2][0] = r2.x; W[2][1] = r2.y; W[2][2] = r2.z; W[2][3] = r2.w;
}

__global__ void __launch_bounds__(kSkinThreads)
    lbs_fwd_kernel(SkinIn in, const float* __restrict__ inst_t, const float* __restrict__ inst_v,
                   float* __restrict__ out_pos, float* __restrict__ out_rot, float* __restrict__ out_vel,
                   uint8_t* __restrict__ out_mask) {
    __shared__ float4 sM[kJ][3];
    const int64_t b = blockIdx.y;
    const int64_t obj = in.valid_ids[b];
    if (obj >= in.n_objects) return;  // block-uniform
    const int64_t inst = in.inst_ids[obj];
    if (inst >= in.n_instances) return;
    if (threadIdx.x < kJ) {
        const int64_t o = b * kJ + threadIdx.x;
        to_mat34(ldq(in.gq + 4 * o), ld3(in.gt + 3 * o), sM[threadIdx.x]);
    }
    __syncthreads();
    const int64_t v = int64_t(blockIdx.x) * kSkinThreads + threadIdx.x;
    if (v >= in.V) return;
    float W[3][4];
    blend(sM, in.weights, obj, in.V, v, W);
    const int64_t fv = obj * in.V + v, out = in.global_offset + fv;
    const v3 p = ld3(in.vertices + 3 * fv);
    const v3 T = ld3(inst_t + 3 * inst);
    st3(out_pos + 3 * out, mk3(W[0][0] * p.x + W[0][1] * p.y + W[0][2] * p.z + W[0][3] + T.x,
                               W[1][0] * p.x + W[1][1] * p.y + W[1][2] * p.z + W[1][3] + T.y,
                               W[2][0] * p.x + W[2][1] * p.y + W[2][2] * p.z + W[2][3] + T.z));
    const int br = shepperd_branch(W);
    const Q lbs = qstd(from_matrix(W, br, shepperd_s(W, br)));
    stq(out_rot + 4 * out, qmul(lbs, ldq(in.quats + 4 * fv)));
    if (out_vel) st3(out_vel + 3 * out, ld3(inst_v + 3 * inst));
    if (out_mask) out_mask[out] = 1;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(kSkinThreads)
    lbs_bwd_kernel(SkinIn in, const float* __restrict__ g_pos, const float* __restrict__ g_rot,
                   const float* __restrict__ g_vel, float* __restrict__ d_gq, float* __restrict__ d_gt,
                   float* __restrict__ d_vertices, float* __restrict__ d_quats, float* __restrict__ d_weights,
                   float* __restrict__ d_inst_v, float* __restrict__ d_inst_t) {
    __shared__ float4 sM[kJ][3];
    __shared__ float sAcc[kJ][12];
    __shared__ float sInst[6];
    const int64_t b = blockIdx.y;
    const int64_t obj = in.valid_ids[b];
    if (obj >= in.n_objects) return;  // block-uniform
    const int64_t inst = in.inst_ids[obj];
    if (inst >= in.n_instances) return;
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < kJ) {
        const int64_t o = b * kJ + tid;
        to_mat34(ldq(in.gq + 4 * o), ld3(in.gt + 3 * o), sM[tid]);
    }
    for (int i = tid; i < kJ * 12; i += kSkinThreads) (&sAcc[0][0])[i] = 0.f;
    if (tid < 6) sInst[tid] = 0.f;
    __syncthreads();

    const int64_t v = int64_t(blockIdx.x) * kSkinThreads + tid;
    const bool live = v < in.V;
    float dW[3][4] = {};
    v3 gv = mk3(0.f, 0.f, 0.f), gvel = mk3(0.f, 0.f, 0.f);
    if (live) {
        float W[3][4];
        blend(sM, in.weights, obj, in.V, v, W);
        const int64_t fv = obj * in.V + v, out = in.global_offset + fv;
        const v3 p = ld3(in.vertices + 3 * fv);
        const int br = shepperd_branch(W);
        const float s = shepperd_s(W, br);
        const Q fm = from_matrix(W, br, s);
        const Q lbs = qstd(fm);
        const Q vq = ldq(in.quats + 4 * fv);
        gv = ld3(g_pos + 3 * out);
        const Q gr = ldq(g_rot + 4 * out);
        if (g_vel) gvel = ld3(g_vel + 3 * out);
        // out_rot = lbs (x) vq
        const Q d_fm = qstd_bwd(fm, qmul(gr, conj(vq)));
        stq(d_quats + 4 * fv, qmul(conj(lbs), gr));
        from_matrix_bwd(br, s, fm, d_fm, dW);
        const float pv[4] = {p.x, p.y, p.z, 1.f};
        const float g3[3] = {gv.x, gv.y, gv.z};
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) dW[r][c] += g3[r] * pv[c];
        st3(d_vertices + 3 * fv, mk3(gv.x * W[0][0] + gv.y * W[1][0] + gv.z * W[2][0],
                                     gv.x * W[0][1] + gv.y * W[1][1] + gv.z * W[2][1],
                                     gv.x * W[0][2] + gv.y * W[1][2] + gv.z * W[2][2]));
    }
    // per joint: d_weights and the CTA sum of w * dW (the joint matrix gradient)
    const float* wp = in.weights + obj * kJ * in.V + v;
    float* dwp = d_weights + obj * kJ * in.V + v;
#pragma unroll 1
    for (int j = 0; j < kJ; ++j) {
        const float w = live ? __ldg(wp + int64_t(j) * in.V) : 0.f;
        if (live) {
            const float4 a = sM[j][0], bb = sM[j][1], c = sM[j][2];
            dwp[int64_t(j) * in.V] = a.x * dW[0][0] + a.y * dW[0][1] + a.z * dW[0][2] + a.w * dW[0][3] +
                                     bb.x * dW[1][0] + bb.y * dW[1][1] + bb.z * dW[1][2] + bb.w * dW[1][3] +
                                     c.x * dW[2][0] + c.y * dW[2][1] + c.z * dW[2][2] + c.w * dW[2][3];
        }
        if (!__any_sync(0xffffffffu, w != 0.f)) continue;  // warp-uniform
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float t = warp_sum(w * dW[r][c]);
                if (lane == 0) atomicAdd(&sAcc[j][r * 4 + c], t);
            }
    }
    {
        const float t0 = warp_sum(gv.x), t1 = warp_sum(gv.y), t2 = warp_sum(gv.z);
        const float t3 = warp_sum(gvel.x), t4 = warp_sum(gvel.y), t5 = warp_sum(gvel.z);
        if (lane == 0) {
            atomicAdd(&sInst[0], t0); atomicAdd(&sInst[1], t1); atomicAdd(&sInst[2], t2);
            atomicAdd(&sInst[3], t3); atomicAdd(&sInst[4], t4); atomicAdd(&sInst[5], t5);
        }
    }
    __syncthreads();
    if (tid < kJ) {
        float G[3][4];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) G[r][c] = sAcc[tid][r * 4 + c];
        const int64_t o = b * kJ + tid;
        Q dq;
        v3 dt;
        to_mat34_bwd(ldq(in.gq + 4 * o), G, dq, dt);
        atomicAdd(d_gq + 4 * o, dq.w); atomicAdd(d_gq + 4 * o + 1, dq.x);
        atomicAdd(d_gq + 4 * o + 2, dq.y); atomicAdd(d_gq + 4 * o + 3, dq.z);
        atomicAdd(d_gt + 3 * o, dt.x); atomicAdd(d_gt + 3 * o + 1, dt.y); atomicAdd(d_gt + 3 * o + 2, dt.z);
    } else if (tid == kJ) {
        atomicAdd(d_inst_t + 3 * inst, sInst[0]);
        atomicAdd(d_inst_t + 3 * inst + 1, sInst[1]);
        atomicAdd(d_inst_t + 3 * inst + 2, sInst[2]);
        if (g_vel && d_inst_v) {
            atomicAdd(d_inst_v + 3 * inst, sInst[3]);
            atomicAdd(d_inst_v + 3 * inst + 1, sInst[4]);
            atomicAdd(d_inst_v + 3 * inst + 2, sInst[5]);
        }
    }
}

// ----------------------------------------------------------- compaction --
constexpr int kCompactThreads = 1024;

// One CTA walks the ids in chunks of 1024, so the output keeps the input
// order (ascending indices), like the reference's single-block scan.
__global__ void __launch_bounds__(kCompactThreads)
    compaction_kernel(const uint32_t* __restrict__ ids, int64_t n, const uint8_t* __restrict__ mask,
                      int64_t n_instances, uint32_t* __restrict__ out, int64_t* __restrict__ count) {
    __shared__ int warp_tot[kCompactThreads / 32];
    __shared__ int64_t base;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int64_t start = 0; start < n; start += kCompactThreads) {
        const int64_t i = start + tid;
        bool keep = false;
        if (i < n) {
            const uint32_t id = ids[i];
            keep = id < n_instances && mask[id] != 0;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) warp_tot[wid] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int k = 0; k < kCompactThreads / 32; ++k) {
            const int t = warp_tot[k];
            before += k < wid ? t : 0;
            total += t;
        }
        if (keep) out[base + before + __popc(bal & ((1u << lane) - 1u))] = uint32_t(i);
        __syncthreads();
        if (tid == 0) base += total;
        __syncthreads();
    }
    if (tid == 0) *count = base;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace xsg

using namespace xsg;

extern "C" int xsg_smpl_local_to_global_fwd(const uint32_t* local_q_ids, int64_t batch, const float* local_q,
                                            const float* joints, const float* a0_inv_q, const float* a0_inv_t,
                                            int64_t n_objects, float* out_q, float* out_t, xsg_stream_t stream) {
    XSG_REQUIRE(batch >= 0 && n_objects >= 0, "smpl_local_to_global_fwd: negative size");
    if (batch == 0) return XSG_OK;
    XSG_REQUIRE(local_q_ids && local_q && joints && a0_inv_q && a0_inv_t && out_q && out_t,
                "smpl_local_to_global_fwd: null pointer");
    XSG_REQUIRE(aligned16(local_q) && aligned16(a0_inv_q) && aligned16(out_q),
                "smpl_local_to_global_fwd: quaternion arrays must be 16-byte aligned");
    const cudaStream_t st = as_cuda(stream);
    launch(l2g_fwd_kernel, dim3(blocks_for(batch, kBodiesPerBlock)), dim3(32, kBodiesPerBlock), 0, st,
           local_q_ids, batch, n_objects, local_q, joints, a0_inv_q, a0_inv_t, out_q, out_t);
    return check_launch("smpl_local_to_global_fwd");
}

extern "C" int xsg_smpl_local_to_global_bwd(const uint32_t* local_q_ids, int64_t batch, const float* local_q,
                                            const float* joints, const float* a0_inv_q, const float* a0_inv_t,
                                            int64_t n_objects, const float* grad_out_q, const float* grad_out_t,
                                            float* d_local_q, float* d_a0_inv_q, float* d_a0_inv_t,
                                            xsg_stream_t stream) {
    XSG_REQUIRE(batch >= 0 && n_objects >= 0, "smpl_local_to_global_bwd: negative size");
    if (batch == 0) return XSG_OK;
    XSG_REQUIRE(local_q_ids && local_q && joints && a0_inv_q && a0_inv_t && grad_out_q && grad_out_t && d_local_q &&
                    d_a0_inv_q && d_a0_inv_t,
                "smpl_local_to_global_bwd: null pointer");
    XSG_REQUIRE(aligned16(local_q) && aligned16(a0_inv_q) && aligned16(grad_out_q) && aligned16(d_local_q) &&
                    aligned16(d_a0_inv_q),
                "smpl_local_to_global_bwd: quaternion arrays must be 16-byte aligned");
    const cudaStream_t st = as_cuda(stream);
    launch(l2g_bwd_kernel, dim3(blocks_for(batch, kBodiesPerBlock)), dim3(32, kBodiesPerBlock), 0, st,
           local_q_ids, batch, n_objects, local_q, joints, a0_inv_q, a0_inv_t, grad_out_q, grad_out_t, d_local_q,
           d_a0_inv_q, d_a0_inv_t);
    return check_launch("smpl_local_to_global_bwd");
}

static int skin_check(const char* what, int64_t n_valid, int64_t n_objects, int64_t V, int64_t n_instances,
                      int64_t global_offset, int64_t container_size) {
    if (n_valid < 0 || n_objects < 0 || V < 0 || n_instances < 0 || global_offset < 0 || container_size < 0)
        return set_error(XSG_ERR_INVALID_ARGUMENT, std::string(what) + ": negative size");
    if (n_valid > 65535) return set_error(XSG_ERR_UNSUPPORTED, std::string(what) + ": more than 65535 bodies");
    if (global_offset + n_objects * V > container_size)
        return set_error(XSG_ERR_INVALID_ARGUMENT,
                         std::string(what) + ": global_offset + objects x vertices exceeds the container size");
    return XSG_OK;
}

extern "C" int xsg_smpl_lbs_skinning_fwd(const uint32_t* valid_ids, int64_t n_valid, const float* global_q,
                                         const float* global_t, const float* vertices, const float* quats,
                                         const float* weights, int64_t n_objects, int64_t n_vertices,
                                         const uint32_t* instance_ids, const float* instance_t,
                                         const float* instance_v, int64_t n_instances, int64_t global_offset,
                                         int64_t container_size, float* out_positions, float* out_rotations,
                                         float* out_velocities, uint8_t* out_mask, xsg_stream_t stream) {
    int rc = skin_check("smpl_lbs_skinning", n_valid, n_objects, n_vertices, n_instances, global_offset,
                        container_size);
    if (rc) return rc;
    if (n_valid == 0 || n_vertices == 0) return XSG_OK;
    XSG_REQUIRE(valid_ids && global_q && global_t && vertices && quats && weights && instance_ids && instance_t &&
                    out_positions && out_rotations && (!out_velocities || instance_v),
                "smpl_lbs_skinning: null pointer");
    XSG_REQUIRE(aligned16(global_q) && aligned16(quats) && aligned16(out_rotations),
                "smpl_lbs_skinning: quaternion arrays must be 16-byte aligned");
    SkinIn in{valid_ids, global_q, global_t, vertices, quats, weights, instance_ids,
              n_objects, n_vertices, n_instances, global_offset};
    ScopedTimer tm("lbs_fwd", as_cuda(stream));
    launch(lbs_fwd_kernel, dim3(blocks_for(n_vertices, kSkinThreads), unsigned(n_valid)), dim3(kSkinThreads), 0,
           as_cuda(stream), in, instance_t, instance_v, out_positions, out_rotations, out_velocities, out_mask);
    return check_launch("smpl_lbs_skinning");
}

extern "C" int xsg_smpl_lbs_skinning_bwd(const uint32_t* valid_ids, int64_t n_valid, const uint32_t* instance_ids,
                                         const float* global_q, const float* global_t, const float* vertices,
                                         const float* quats, const float* weights, int64_t n_objects,
                                         int64_t n_vertices, int64_t n_instances, int64_t global_offset,
                                         int64_t container_size, const float* grad_positions,
                                         const float* grad_rotations, const float* grad_velocities,
                                         float* d_global_q, float* d_global_t, float* d_vertices, float* d_quats,
                                         float* d_weights, float* d_instance_v, float* d_instance_t,
                                         xsg_stream_t stream) {
    int rc = skin_check("smpl_lbs_skinning_bwd", n_valid, n_objects, n_vertices, n_instances, global_offset,
                        container_size);
    if (rc) return rc;
    if (n_valid == 0 || n_vertices == 0) return XSG_OK;
    XSG_REQUIRE(valid_ids && instance_ids && global_q && global_t && vertices && quats && weights && grad_positions &&
                    grad_rotations && d_global_q && d_global_t && d_vertices && d_quats && d_weights && d_instance_t,
                "smpl_lbs_skinning_bwd: null pointer");
    XSG_REQUIRE(aligned16(global_q) && aligned16(quats) && aligned16(grad_rotations) && aligned16(d_quats),
                "smpl_lbs_skinning_bwd: quaternion arrays must be 16-byte aligned");
    SkinIn in{valid_ids, global_q, global_t, vertices, quats, weights, instance_ids,
              n_objects, n_vertices, n_instances, global_offset};
    ScopedTimer tm("lbs_bwd", as_cuda(stream));
    launch(lbs_bwd_kernel, dim3(blocks_for(n_vertices, kSkinThreads), unsigned(n_valid)), dim3(kSkinThreads), 0,
           as_cuda(stream), in, grad_positions, grad_rotations, grad_velocities, d_global_q, d_global_t, d_vertices,
           d_quats, d_weights, d_instance_v, d_instance_t);
    return check_launch("smpl_lbs_skinning_bwd");
}

extern "C" int xsg_smpl_ids_compaction(const uint32_t* instance_ids, int64_t n, const uint8_t* instance_mask,
                                       int64_t n_instances, uint32_t* out_ids, int64_t* count, int64_t* n_out_host,
                                       xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && n_instances >= 0 && n_out_host, "smpl_ids_compaction: bad arguments");
    if (n == 0) {
        *n_out_host = 0;
        return XSG_OK;
    }
    XSG_REQUIRE(instance_ids && instance_mask && out_ids && count, "smpl_ids_compaction: null pointer");
    const cudaStream_t st = as_cuda(stream);
    launch(compaction_kernel, dim3(1), dim3(kCompactThreads), 0, st, instance_ids, n, instance_mask, n_instances,
           out_ids, count);
    int rc = check_launch("smpl_ids_compaction");
    if (rc) return rc;
    XSG_CUDA(cudaMemcpyAsync(n_out_host, count, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    XSG_CUDA(cudaStreamSynchronize(st));
    return XSG_OK;
}
