// xsimgs-b200 CPU ORACLE, SMPL part — test infrastructure only, never a
// product path.  Scalar C++17 restatement of the reference's SMPL kernels:
//   smpl_local_to_global_fwd/bwd   csrc/nodes/smpl_local_to_global.cu:29-279
//   smpl_lbs_skinning(_bwd)        csrc/nodes/smpl_lbs_skinning.cu:11-268
//   smpl_ids_compaction            csrc/nodes/smpl.cu:15-74
// following the reference's own order of operations (the backward of
// local-to-global walks each joint's root path with inverse compositions,
// as smpl_local_to_global.cu:203-257 does).
//
// PARITY STATUS: unpinned (the reference needs the absent pytoast library).
// The pieces the reference takes from pytoast are restated from the
// mathematics and marked "toast:" — quaternions are (w, x, y, z) in memory
// like every other quaternion of the reference (rasterization/utils.h:61-62);
// products are Hamilton products; rotation of a vector is the polynomial
// R(q) v; std() is unit length with w >= 0; from_matrix() is Shepperd's
// method (trace branch when the trace is positive, else the largest
// diagonal element).
//
// Built together with xsg_oracle.cpp by oracle/build.py.

#include <cmath>
#include <cstdint>
#include <vector>

namespace {

constexpr int kJoints = 24;
// smpl_local_to_global.cu:42-46
constexpr int kParents[kJoints] = {-1, 0, 0, 0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 9, 9, 12, 13, 14, 16, 17, 18, 19, 20, 21};

struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };
struct SE3 { Q4 q; V3 t; };

inline V3 add(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline V3 sub(V3 a, V3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline V3 scl(float s, V3 a) { return {s * a.x, s * a.y, s * a.z}; }
inline float dot3(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline V3 crs(V3 a, V3 b) { return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }
inline Q4 qadd(Q4 a, Q4 b) { return {a.w + b.w, a.x + b.x, a.y + b.y, a.z + b.z}; }
inline Q4 conj(Q4 q) { return {q.w, -q.x, -q.y, -q.z}; }
inline V3 vec(Q4 q) { return {q.x, q.y, q.z}; }

// toast: Hamilton product
inline Q4 qmul(Q4 a, Q4 b) {
    const V3 av = vec(a), bv = vec(b);
    const V3 v = add(add(scl(a.w, bv), scl(b.w, av)), crs(av, bv));
    return {a.w * b.w - dot3(av, bv), v.x, v.y, v.z};
}
// toast: rotation R(q) p = p + 2 (w (u x p) + u x (u x p)), u = vec(q)
inline V3 rot(Q4 q, V3 p) {
    const V3 u = vec(q);
    const V3 uv = crs(u, p);
    return add(p, scl(2.f, add(scl(q.w, uv), crs(u, uv))));
}
// d/dq of g . R(q) p (R(q) as the polynomial above)
inline Q4 rot_bwd_q(Q4 q, V3 p, V3 g) {
    const V3 u = vec(q);
    const float up = dot3(u, p), ug = dot3(u, g), pg = dot3(p, g);
    const V3 pxg = crs(p, g);
    const V3 du = add(add(scl(2.f * q.w, pxg), scl(2.f * up, g)), sub(scl(2.f * ug, p), scl(4.f * pg, u)));
    return {2.f * dot3(g, crs(u, p)), du.x, du.y, du.z};
}
// toast: std() — unit length, w >= 0
inline Q4 qstd(Q4 q) {
    float n = 1.0f / std::sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    if (q.w < 0.f) n = -n;
    return {q.w * n, q.x * n, q.y * n, q.z * n};
}
inline Q4 qstd_bwd(Q4 raw, Q4 g) {
    const float l = std::sqrt(raw.w * raw.w + raw.x * raw.x + raw.y * raw.y + raw.z * raw.z);
    const float s = raw.w < 0.f ? -1.f : 1.f;
    const Q4 n{raw.w / l, raw.x / l, raw.y / l, raw.z / l};
    const float ng = n.w * g.w + n.x * g.x + n.y * g.y + n.z * g.z;
    const float k = s / l;
    return {k * (g.w - n.w * ng), k * (g.x - n.x * ng), k * (g.y - n.y * ng), k * (g.z - n.z * ng)};
}

inline SE3 compose(const SE3& a, const SE3& b) { return {qmul(a.q, b.q), add(rot(a.q, b.t), a.t)}; }
inline SE3 inverse(const SE3& a) {
    const Q4 qi = conj(a.q);
    return {qi, scl(-1.f, rot(qi, a.t))};
}
// gradients of c = a o b
inline void compose_bwd(const SE3& a, const SE3& b, Q4 dq, V3 dt, Q4& da_q, V3& da_t, Q4& db_q, V3& db_t) {
    da_q = qadd(qmul(dq, conj(b.q)), rot_bwd_q(a.q, b.t, dt));
    da_t = dt;
    db_q = qmul(conj(a.q), dq);
    db_t = rot(conj(a.q), dt);
}

// toast: se3 to_matrix_3x4 — rows [R(q) | t]
inline void to_mat34(Q4 q, V3 t, float m[3][4]) {
    const float w = q.w, x = q.x, y = q.y, z = q.z;
    m[0][0] = 1.f - 2.f * (y * y + z * z); m[0][1] = 2.f * (x * y - w * z); m[0][2] = 2.f * (x * z + w * y);
    m[1][0] = 2.f * (x * y + w * z); m[1][1] = 1.f - 2.f * (x * x + z * z); m[1][2] = 2.f * (y * z - w * x);
    m[2][0] = 2.f * (x * z - w * y); m[2][1] = 2.f * (y * z + w * x); m[2][2] = 1.f - 2.f * (x * x + y * y);
    m[0][3] = t.x; m[1][3] = t.y; m[2][3] = t.z;
}
inline void to_mat34_bwd(Q4 q, const double G[3][4], double dq[4], double dt[3]) {
    const double w = q.w, x = q.x, y = q.y, z = q.z;
    dq[0] = 2 * (-z * G[0][1] + y * G[0][2] + z * G[1][0] - x * G[1][2] - y * G[2][0] + x * G[2][1]);
    dq[1] = 2 * (y * G[0][1] + z * G[0][2] + y * G[1][0] - 2 * x * G[1][1] - w * G[1][2] + z * G[2][0] +
                 w * G[2][1] - 2 * x * G[2][2]);
    dq[2] = 2 * (-2 * y * G[0][0] + x * G[0][1] + w * G[0][2] + x * G[1][0] + z * G[1][2] - w * G[2][0] +
                 z * G[2][1] - 2 * y * G[2][2]);
    dq[3] = 2 * (-2 * z * G[0][0] - w * G[0][1] + x * G[0][2] + w * G[1][0] - 2 * z * G[1][1] + y * G[1][2] +
                 x * G[2][0] + y * G[2][1]);
    dt[0] = G[0][3]; dt[1] = G[1][3]; dt[2] = G[2][3];
}

// toast: from_matrix — Shepperd's method on the 3x3 part
inline int shepperd_branch(const float m[3][4]) {
    const float tr = m[0][0] + m[1][1] + m[2][2];
    if (tr > 0.f) return 0;
    if (m[0][0] > m[1][1] && m[0][0] > m[2][2]) return 1;
    if (m[1][1] > m[2][2]) return 2;
    return 3;
}
inline Q4 from_matrix(const float m[3][4]) {
    switch (shepperd_branch(m)) {
        case 0: {
            const float s = std::sqrt(m[0][0] + m[1][1] + m[2][2] + 1.f) * 2.f;
            return {0.25f * s, (m[2][1] - m[1][2]) / s, (m[0][2] - m[2][0]) / s, (m[1][0] - m[0][1]) / s};
        }
        case 1: {
            const float s = std::sqrt(1.f + m[0][0] - m[1][1] - m[2][2]) * 2.f;
            return {(m[2][1] - m[1][2]) / s, 0.25f * s, (m[0][1] + m[1][0]) / s, (m[0][2] + m[2][0]) / s};
        }
        case 2: {
            const float s = std::sqrt(1.f + m[1][1] - m[0][0] - m[2][2]) * 2.f;
            return {(m[0][2] - m[2][0]) / s, (m[0][1] + m[1][0]) / s, 0.25f * s, (m[1][2] + m[2][1]) / s};
        }
        default: {
            const float s = std::sqrt(1.f + m[2][2] - m[0][0] - m[1][1]) * 2.f;
            return {(m[1][0] - m[0][1]) / s, (m[0][2] + m[2][0]) / s, (m[1][2] + m[2][1]) / s, 0.25f * s};
        }
    }
}
// gradient of from_matrix w.r.t. the 3x3 part (the translation column gets none)
inline void from_matrix_bwd(const float m[3][4], Q4 q, Q4 g, float dm[3][4]) {
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 4; ++c) dm[r][c] = 0.f;
    const int b = shepperd_branch(m);
    // every branch: one component is s / 4, the other three are (+-m_ij +- m_ji) / s
    float s;
    int diag_sign[3];
    if (b == 0) { s = std::sqrt(m[0][0] + m[1][1] + m[2][2] + 1.f) * 2.f; diag_sign[0] = diag_sign[1] = diag_sign[2] = 1; }
    else if (b == 1) { s = std::sqrt(1.f + m[0][0] - m[1][1] - m[2][2]) * 2.f; diag_sign[0] = 1; diag_sign[1] = diag_sign[2] = -1; }
    else if (b == 2) { s = std::sqrt(1.f + m[1][1] - m[0][0] - m[2][2]) * 2.f; diag_sign[1] = 1; diag_sign[0] = diag_sign[2] = -1; }
    else { s = std::sqrt(1.f + m[2][2] - m[0][0] - m[1][1]) * 2.f; diag_sign[2] = 1; diag_sign[0] = diag_sign[1] = -1; }
    const float is = 1.f / s;
    float ds = 0.f;
    // (component value, gradient, entries (r, c, sign) of the numerator)
    auto term = [&](float val, float gv, int r0, int c0, float s0, int r1, int c1, float s1) {
        dm[r0][c0] += s0 * gv * is;
        dm[r1][c1] += s1 * gv * is;
        ds -= gv * val * is;
    };
    if (b == 0) {
        ds += 0.25f * g.w;
        term(q.x, g.x, 2, 1, 1.f, 1, 2, -1.f);
        term(q.y, g.y, 0, 2, 1.f, 2, 0, -1.f);
        term(q.z, g.z, 1, 0, 1.f, 0, 1, -1.f);
    } else if (b == 1) {
        ds += 0.25f * g.x;
        term(q.w, g.w, 2, 1, 1.f, 1, 2, -1.f);
        term(q.y, g.y, 0, 1, 1.f, 1, 0, 1.f);
        term(q.z, g.z, 0, 2, 1.f, 2, 0, 1.f);
    } else if (b == 2) {
        ds += 0.25f * g.y;
        term(q.w, g.w, 0, 2, 1.f, 2, 0, -1.f);
        term(q.x, g.x, 0, 1, 1.f, 1, 0, 1.f);
        term(q.z, g.z, 1, 2, 1.f, 2, 1, 1.f);
    } else {
        ds += 0.25f * g.z;
        term(q.w, g.w, 1, 0, 1.f, 0, 1, -1.f);
        term(q.x, g.x, 0, 2, 1.f, 2, 0, 1.f);
        term(q.y, g.y, 1, 2, 1.f, 2, 1, 1.f);
    }
    // s = 2 sqrt(radicand): d s / d radicand = 2 / s
    for (int i = 0; i < 3; ++i) dm[i][i] += ds * 2.f * is * float(diag_sign[i]);
}

inline Q4 ldq(const float* p) { return {p[0], p[1], p[2], p[3]}; }
inline V3 ld3(const float* p) { return {p[0], p[1], p[2]}; }
inline void stq(float* p, Q4 q) { p[0] = q.w; p[1] = q.x; p[2] = q.y; p[3] = q.z; }
inline void st3(float* p, V3 v) { p[0] = v.x; p[1] = v.y; p[2] = v.z; }

// local transforms of one object (smpl_local_to_global.cu:60-69)
void local_transforms(const float* local_q, const float* joints, int64_t obj, SE3 L[kJoints], V3 J[kJoints],
                      Q4 raw[kJoints]) {
    for (int j = 0; j < kJoints; ++j) J[j] = ld3(joints + (obj * kJoints + j) * 3);
    for (int j = 0; j < kJoints; ++j) {
        raw[j] = ldq(local_q + (obj * kJoints + j) * 4);
        const V3 rel = j == 0 ? J[j] : sub(J[j], J[kParents[j]]);
        L[j] = {qstd(raw[j]), rel};
    }
}

}  // namespace

extern "C" {

// smpl_local_to_global_fwd_kernel, smpl_local_to_global.cu:29-88: global
// transform of joint j of object ids[b] = L_root o ... o L_j, translated by
// -R J_j and composed with a0_inv.
void xsgo_smpl_local_to_global_fwd(int64_t batch, const uint32_t* ids, const float* local_q, const float* joints,
                                   const float* a0q, const float* a0t, float* out_q, float* out_t) {
    for (int64_t b = 0; b < batch; ++b) {
        const int64_t obj = ids[b];
        SE3 L[kJoints]; V3 J[kJoints]; Q4 raw[kJoints];
        local_transforms(local_q, joints, obj, L, J, raw);
        for (int j = 0; j < kJoints; ++j) {
            SE3 r = L[j];
            for (int p = kParents[j]; p != -1; p = kParents[p]) r = compose(L[p], r);
            r.t = sub(r.t, rot(r.q, J[j]));
            const int64_t o = obj * kJoints + j;
            r = compose(r, SE3{ldq(a0q + 4 * o), ld3(a0t + 3 * o)});
            stq(out_q + (b * kJoints + j) * 4, r.q);
            st3(out_t + (b * kJoints + j) * 3, r.t);
        }
    }
}

// smpl_local_to_global_bwd_kernel, smpl_local_to_global.cu:123-279.  The
// gradients of the local translations and of the joints are not propagated,
// as in the reference (:243-257).  d_* are [N, 24, .], written for the
// objects named in ids (callers zero them).
void xsgo_smpl_local_to_global_bwd(int64_t batch, const uint32_t* ids, const float* local_q, const float* joints,
                                   const float* a0q, const float* a0t, const float* out_q, const float* out_t,
                                   const float* gq, const float* gt, float* d_local_q, float* d_a0q, float* d_a0t) {
    // the root paths (joint_path_indices / root_to_leaf_paths, :143-170) as parent chains
    for (int64_t b = 0; b < batch; ++b) {
        const int64_t obj = ids[b];
        SE3 L[kJoints]; V3 J[kJoints]; Q4 raw[kJoints];
        local_transforms(local_q, joints, obj, L, J, raw);
        Q4 acc[kJoints];
        for (int j = 0; j < kJoints; ++j) acc[j] = {0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < kJoints; ++j) {
            const int64_t o = obj * kJoints + j, ob = b * kJoints + j;
            const SE3 a0{ldq(a0q + 4 * o), ld3(a0t + 3 * o)};
            const SE3 out{ldq(out_q + 4 * ob), ld3(out_t + 3 * ob)};
            SE3 result = compose(out, inverse(a0));
            Q4 g_q, da0_q; V3 g_t, da0_t;
            compose_bwd(result, a0, ldq(gq + 4 * ob), ld3(gt + 3 * ob), g_q, g_t, da0_q, da0_t);
            stq(d_a0q + 4 * o, da0_q);
            st3(d_a0t + 3 * o, da0_t);
            // result.t -= R(result.q) J
            g_q = qadd(g_q, rot_bwd_q(result.q, J[j], scl(-1.f, g_t)));
            result.t = add(result.t, rot(result.q, J[j]));
            // walk root -> j
            int path[kJoints], len = 0;
            for (int p = j; p != -1; p = kParents[p]) path[len++] = p;
            for (int k = len - 1; k >= 1; --k) {
                const SE3& a = L[path[k]];
                const SE3 bb = compose(inverse(a), result);
                Q4 da_q, db_q; V3 da_t, db_t;
                compose_bwd(a, bb, g_q, g_t, da_q, da_t, db_q, db_t);
                acc[path[k]] = qadd(acc[path[k]], da_q);
                result = bb;
                g_q = db_q;
                g_t = db_t;
            }
            acc[j] = qadd(acc[j], g_q);
        }
        for (int j = 0; j < kJoints; ++j) stq(d_local_q + (obj * kJoints + j) * 4, qstd_bwd(raw[j], acc[j]));
    }
}

// smpl_lbs_skinning_kernel, smpl_lbs_skinning.cu:11-91
void xsgo_smpl_lbs_fwd(int64_t B, int64_t V, const uint32_t* valid_ids, const float* gq, const float* gt,
                       const float* vertices, const float* quats, const float* weights, const uint32_t* inst_ids,
                       const float* inst_t, const float* inst_v, int64_t global_offset, float* out_pos,
                       float* out_rot, float* out_vel, uint8_t* out_mask) {
    for (int64_t b = 0; b < B; ++b) {
        const int64_t obj = valid_ids[b];
        float M[kJoints][3][4];
        for (int j = 0; j < kJoints; ++j)
            to_mat34(ldq(gq + (b * kJoints + j) * 4), ld3(gt + (b * kJoints + j) * 3), M[j]);
        const int64_t inst = inst_ids[obj];
        for (int64_t v = 0; v < V; ++v) {
            float W[3][4] = {};
            for (int j = 0; j < kJoints; ++j) {
                const float w = weights[(obj * kJoints + j) * V + v];
                for (int r = 0; r < 3; ++r)
                    for (int c = 0; c < 4; ++c) W[r][c] += w * M[j][r][c];
            }
            const int64_t fv = obj * V + v, out = global_offset + fv;
            const V3 p = ld3(vertices + 3 * fv);
            V3 P;
            P.x = W[0][0] * p.x + W[0][1] * p.y + W[0][2] * p.z + W[0][3];
            P.y = W[1][0] * p.x + W[1][1] * p.y + W[1][2] * p.z + W[1][3];
            P.z = W[2][0] * p.x + W[2][1] * p.y + W[2][2] * p.z + W[2][3];
            st3(out_pos + 3 * out, add(P, ld3(inst_t + 3 * inst)));
            stq(out_rot + 4 * out, qmul(qstd(from_matrix(W)), ldq(quats + 4 * fv)));
            if (out_vel) st3(out_vel + 3 * out, ld3(inst_v + 3 * inst));
            if (out_mask) out_mask[out] = 1;
        }
    }
}

// smpl_lbs_skinning_bwd_kernel, smpl_lbs_skinning.cu:137-268.  d_global_q /
// d_global_t / d_inst_* are accumulated (callers zero them); d_vertices,
// d_quats and d_weights are written for the valid objects.
void xsgo_smpl_lbs_bwd(int64_t B, int64_t V, const uint32_t* valid_ids, const uint32_t* inst_ids, const float* gq,
                       const float* gt, const float* vertices, const float* quats, const float* weights,
                       int64_t global_offset, const float* g_pos, const float* g_rot, const float* g_vel,
                       float* d_gq, float* d_gt, float* d_vertices, float* d_quats, float* d_weights, float* d_inst_v,
                       float* d_inst_t) {
    for (int64_t b = 0; b < B; ++b) {
        const int64_t obj = valid_ids[b];
        Q4 Q[kJoints];
        float M[kJoints][3][4];
        for (int j = 0; j < kJoints; ++j) {
            Q[j] = ldq(gq + (b * kJoints + j) * 4);
            to_mat34(Q[j], ld3(gt + (b * kJoints + j) * 3), M[j]);
        }
        std::vector<double> dq(kJoints * 4, 0.0), dt(kJoints * 3, 0.0);
        double dit[3] = {0, 0, 0}, div[3] = {0, 0, 0};
        const int64_t inst = inst_ids[obj];
        for (int64_t v = 0; v < V; ++v) {
            float W[3][4] = {};
            for (int j = 0; j < kJoints; ++j) {
                const float w = weights[(obj * kJoints + j) * V + v];
                for (int r = 0; r < 3; ++r)
                    for (int c = 0; c < 4; ++c) W[r][c] += w * M[j][r][c];
            }
            const int64_t fv = obj * V + v, out = global_offset + fv;
            const V3 p = ld3(vertices + 3 * fv);
            const Q4 fm = from_matrix(W);
            const Q4 lbs = qstd(fm);
            const Q4 vq = ldq(quats + 4 * fv);
            const V3 gv = ld3(g_pos + 3 * out);
            const Q4 gr = ldq(g_rot + 4 * out);
            // out_rot = lbs (x) vq
            const Q4 d_lbs = qmul(gr, conj(vq));
            const Q4 d_vq = qmul(conj(lbs), gr);
            const Q4 d_fm = qstd_bwd(fm, d_lbs);
            float dW[3][4];
            from_matrix_bwd(W, fm, d_fm, dW);
            const float pv[4] = {p.x, p.y, p.z, 1.f};
            const float g3[3] = {gv.x, gv.y, gv.z};
            for (int r = 0; r < 3; ++r)
                for (int c = 0; c < 4; ++c) dW[r][c] += g3[r] * pv[c];
            V3 dp;
            dp.x = gv.x * W[0][0] + gv.y * W[1][0] + gv.z * W[2][0];
            dp.y = gv.x * W[0][1] + gv.y * W[1][1] + gv.z * W[2][1];
            dp.z = gv.x * W[0][2] + gv.y * W[1][2] + gv.z * W[2][2];
            for (int j = 0; j < kJoints; ++j) {
                const int64_t wo = (obj * kJoints + j) * V + v;
                const float w = weights[wo];
                float s = 0.f;
                double G[3][4];
                for (int r = 0; r < 3; ++r)
                    for (int c = 0; c < 4; ++c) {
                        s += M[j][r][c] * dW[r][c];
                        G[r][c] = double(w) * dW[r][c];
                    }
                d_weights[wo] = s;
                double gqj[4], gtj[3];
                to_mat34_bwd(Q[j], G, gqj, gtj);
                for (int k = 0; k < 4; ++k) dq[j * 4 + k] += gqj[k];
                for (int k = 0; k < 3; ++k) dt[j * 3 + k] += gtj[k];
            }
            st3(d_vertices + 3 * fv, dp);
            stq(d_quats + 4 * fv, d_vq);
            dit[0] += gv.x; dit[1] += gv.y; dit[2] += gv.z;
            if (g_vel && d_inst_v) {
                const V3 gvel = ld3(g_vel + 3 * out);
                div[0] += gvel.x; div[1] += gvel.y; div[2] += gvel.z;
            }
        }
        for (int j = 0; j < kJoints; ++j) {
            for (int k = 0; k < 4; ++k) d_gq[(b * kJoints + j) * 4 + k] += float(dq[j * 4 + k]);
            for (int k = 0; k < 3; ++k) d_gt[(b * kJoints + j) * 3 + k] += float(dt[j * 3 + k]);
        }
        for (int k = 0; k < 3; ++k) d_inst_t[3 * inst + k] += float(dit[k]);
        if (g_vel && d_inst_v)
            for (int k = 0; k < 3; ++k) d_inst_v[3 * inst + k] += float(div[k]);
    }
}

// smpl_ids_compaction_kernel, smpl.cu:15-49: indices i (ascending) with
// instance_mask[instance_ids[i]] != 0.  Returns the count.
int64_t xsgo_smpl_ids_compaction(const uint32_t* instance_ids, int64_t n, const uint8_t* mask, uint32_t* out) {
    int64_t c = 0;
    for (int64_t i = 0; i < n; ++i)
        if (mask[instance_ids[i]]) out[c++] = uint32_t(i);
    return c;
}

}  // extern "C"
