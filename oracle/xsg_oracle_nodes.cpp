// xsimgs-b200 CPU ORACLE, scene-assembly nodes — test infrastructure only,
// never a product path.  Scalar C++17 restatement of the reference's
//   copy_gs_rigid_transform_fwd/bwd   csrc/nodes/container.cu:12-159
//   packed_mask_from_instances        csrc/nodes/gs_masking.cu:8-43
//   interpolate_smpl_poses_fwd/bwd    csrc/nodes/smpl_interpolate.cu:13-226
//
// PARITY STATUS: unpinned (the reference needs the absent pytoast library).
// toast conventions assumed as in xsg_oracle_smpl.cpp (w-first Hamilton
// quaternions, R(q) as the quaternion polynomial, std() = unit with w >= 0),
// and toast: slerp(a, b, t) = shortest-arc spherical interpolation (b negated
// when a . b < 0) with a normalised linear interpolation when a . b > 0.9995.
//
// Built together with xsg_oracle.cpp by oracle/build.py.

#include <cmath>
#include <cstdint>

namespace {

struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };

inline V3 add(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline V3 sub(V3 a, V3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline V3 scl(float s, V3 a) { return {s * a.x, s * a.y, s * a.z}; }
inline float dot3(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline V3 crs(V3 a, V3 b) { return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }
inline Q4 qadd(Q4 a, Q4 b) { return {a.w + b.w, a.x + b.x, a.y + b.y, a.z + b.z}; }
inline Q4 qscl(float s, Q4 a) { return {s * a.w, s * a.x, s * a.y, s * a.z}; }
inline float qdot(Q4 a, Q4 b) { return a.w * b.w + a.x * b.x + a.y * b.y + a.z * b.z; }
inline Q4 conj(Q4 q) { return {q.w, -q.x, -q.y, -q.z}; }
inline V3 vec(Q4 q) { return {q.x, q.y, q.z}; }
inline Q4 qmul(Q4 a, Q4 b) {
    const V3 av = vec(a), bv = vec(b);
    const V3 v = add(add(scl(a.w, bv), scl(b.w, av)), crs(av, bv));
    return {a.w * b.w - dot3(av, bv), v.x, v.y, v.z};
}
inline V3 rot(Q4 q, V3 p) {
    const V3 u = vec(q);
    const V3 uv = crs(u, p);
    return add(p, scl(2.f, add(scl(q.w, uv), crs(u, uv))));
}
inline Q4 rot_bwd_q(Q4 q, V3 p, V3 g) {
    const V3 u = vec(q);
    const float up = dot3(u, p), ug = dot3(u, g), pg = dot3(p, g);
    const V3 du = add(add(scl(2.f * q.w, crs(p, g)), scl(2.f * up, g)), sub(scl(2.f * ug, p), scl(4.f * pg, u)));
    return {2.f * dot3(g, crs(u, p)), du.x, du.y, du.z};
}
inline Q4 qstd(Q4 q) {
    float n = 1.0f / std::sqrt(qdot(q, q));
    if (q.w < 0.f) n = -n;
    return qscl(n, q);
}
inline Q4 qstd_bwd(Q4 raw, Q4 g) {
    const float l = std::sqrt(qdot(raw, raw));
    const float s = raw.w < 0.f ? -1.f : 1.f;
    const Q4 n = qscl(1.0f / l, raw);
    const float ng = qdot(n, g);
    return qscl(s / l, qadd(g, qscl(-ng, n)));
}

constexpr float kSlerpLinear = 0.9995f;

// toast: slerp
inline Q4 slerp(Q4 a, Q4 b, float t) {
    float d = qdot(a, b);
    if (d < 0.f) { b = qscl(-1.f, b); d = -d; }
    if (d > kSlerpLinear) {
        const Q4 r = qadd(a, qscl(t, qadd(b, qscl(-1.f, a))));
        return qscl(1.0f / std::sqrt(qdot(r, r)), r);
    }
    const float th = std::acos(d), s = std::sin(th);
    return qadd(qscl(std::sin((1.f - t) * th) / s, a), qscl(std::sin(t * th) / s, b));
}

// gradients of slerp w.r.t. a, b and t
inline void slerp_bwd(Q4 a, Q4 b, float t, Q4 g, Q4& da, Q4& db, float& dt) {
    float d = qdot(a, b);
    const float sg = d < 0.f ? -1.f : 1.f;
    Q4 bb = qscl(sg, b);
    d = sg * d;
    Q4 dbb;
    if (d > kSlerpLinear) {
        const Q4 diff = qadd(bb, qscl(-1.f, a));
        const Q4 r = qadd(a, qscl(t, diff));
        const float il = 1.0f / std::sqrt(qdot(r, r));
        const Q4 q = qscl(il, r);
        const Q4 dr = qscl(il, qadd(g, qscl(-qdot(q, g), q)));
        da = qscl(1.f - t, dr);
        dbb = qscl(t, dr);
        dt = qdot(dr, diff);
    } else {
        const float th = std::acos(d), s = std::sin(th), c = d;
        const float sa = std::sin((1.f - t) * th), sb = std::sin(t * th);
        const float ca = sa / s, cb = sb / s;
        const float ga = qdot(g, a), gb = qdot(g, bb);
        // d ca / d th, d cb / d th; d th / d d = -1 / s
        const float dca = ((1.f - t) * std::cos((1.f - t) * th) * s - sa * c) / (s * s);
        const float dcb = (t * std::cos(t * th) * s - sb * c) / (s * s);
        const float dd = -(dca * ga + dcb * gb) / s;
        da = qadd(qscl(ca, g), qscl(dd, bb));
        dbb = qadd(qscl(cb, g), qscl(dd, a));
        dt = (-th * std::cos((1.f - t) * th) / s) * ga + (th * std::cos(t * th) / s) * gb;
    }
    db = qscl(sg, dbb);
}

inline Q4 ldq(const float* p) { return {p[0], p[1], p[2], p[3]}; }
inline V3 ld3(const float* p) { return {p[0], p[1], p[2]}; }
inline void stq(float* p, Q4 q) { p[0] = q.w; p[1] = q.x; p[2] = q.y; p[3] = q.z; }
inline void st3(float* p, V3 v) { p[0] = v.x; p[1] = v.y; p[2] = v.z; }

inline int64_t out_row(int64_t p, uint32_t inst, int64_t offset, const uint32_t* per_inst, const uint32_t* gs_off) {
    return gs_off ? offset + int64_t(per_inst[inst]) + int64_t(gs_off[p]) : offset + p;
}

// interpolation frame bracket (smpl_interpolate.cu:34-52)
inline void bracket(const float* times, int frames, float q, int& l, int& r) {
    int f = frames;
    for (int i = 0; i < frames; ++i)
        if (times[i] >= q) { f = i; break; }
    l = f == 0 ? 0 : f - 1;
    r = f < frames - 1 ? f : frames - 1;
}

}  // namespace

extern "C" {

// copy_gs_rigid_transform_fwd_kernel, container.cu:12-71
void xsgo_rigid_transform_fwd(int64_t n, const float* pos, const float* rotq, const uint32_t* inst_id,
                              const float* iq, const float* it, const float* iv, const float* iw, const uint8_t* imask,
                              int64_t offset, const uint32_t* per_inst, const uint32_t* gs_off, float* out_pos,
                              float* out_rot, float* out_vel, uint8_t* out_mask) {
    for (int64_t p = 0; p < n; ++p) {
        const uint32_t k = inst_id[p];
        if (!imask[k]) continue;
        const Q4 q = ldq(iq + 4 * k);
        const int64_t o = out_row(p, k, offset, per_inst, gs_off);
        const V3 pr = rot(q, ld3(pos + 3 * p));
        st3(out_pos + 3 * o, add(pr, ld3(it + 3 * k)));
        stq(out_rot + 4 * o, qmul(q, ldq(rotq + 4 * p)));
        if (out_vel) st3(out_vel + 3 * o, add(ld3(iv + 3 * k), crs(ld3(iw + 3 * k), pr)));
        if (out_mask) out_mask[o] = 1;
    }
}

// copy_gs_rigid_transform_bwd_kernel, container.cu:74-154; grad_* are
// accumulated for the instances (callers zero them) and written for the
// particles whose instance is enabled.
void xsgo_rigid_transform_bwd(int64_t n, const float* pos, const float* rotq, const uint32_t* inst_id,
                              const float* iq, const float* iw, const uint8_t* imask, int64_t offset,
                              const uint32_t* per_inst, const uint32_t* gs_off, const float* v_pos,
                              const float* v_rot, const float* v_vel, float* g_pos, float* g_rot, float* g_q,
                              float* g_t, float* g_v, float* g_w) {
    for (int64_t p = 0; p < n; ++p) {
        const uint32_t k = inst_id[p];
        if (!imask[k]) continue;
        const Q4 q = ldq(iq + 4 * k);
        const V3 w = ld3(iw + 3 * k);
        const V3 pp = ld3(pos + 3 * p);
        const int64_t o = out_row(p, k, offset, per_inst, gs_off);
        const V3 gp = ld3(v_pos + 3 * o);
        g_t[3 * k] += gp.x; g_t[3 * k + 1] += gp.y; g_t[3 * k + 2] += gp.z;
        V3 gpr = gp;
        if (v_vel) {
            const V3 gv = ld3(v_vel + 3 * o);
            g_v[3 * k] += gv.x; g_v[3 * k + 1] += gv.y; g_v[3 * k + 2] += gv.z;
            const V3 gw = crs(rot(q, pp), gv);
            g_w[3 * k] += gw.x; g_w[3 * k + 1] += gw.y; g_w[3 * k + 2] += gw.z;
            gpr = add(gpr, crs(gv, w));
        }
        const Q4 dq1 = rot_bwd_q(q, pp, gpr);
        st3(g_pos + 3 * p, rot(conj(q), gpr));
        const Q4 gr = ldq(v_rot + 4 * o);
        const Q4 dq2 = qmul(gr, conj(ldq(rotq + 4 * p)));
        stq(g_rot + 4 * p, qmul(conj(q), gr));
        const Q4 dq = qadd(dq1, dq2);
        g_q[4 * k] += dq.w; g_q[4 * k + 1] += dq.x; g_q[4 * k + 2] += dq.y; g_q[4 * k + 3] += dq.z;
    }
}

// mask_from_instances_kernel, gs_masking.cu:8-24: bit i = (id < 0 ? 1 : mask[id])
void xsgo_packed_mask_from_instances(int64_t n, const int32_t* ids, const uint8_t* mask, uint32_t* out) {
    for (int64_t w = 0; w < (n + 31) / 32; ++w) out[w] = 0u;
    for (int64_t i = 0; i < n; ++i) {
        const bool on = ids[i] < 0 ? true : mask[ids[i]] != 0;
        if (on) out[i / 32] |= 1u << (i % 32);
    }
}

// interpolate_smpl_poses_fwd_kernel, smpl_interpolate.cu:13-57
void xsgo_interpolate_smpl_fwd(int64_t n_obj, int frames, int joints, float query, const float* poses,
                               const float* times, const float* root_q, const uint32_t* inst_ids, float* out) {
    for (int64_t o = 0; o < n_obj; ++o) {
        int l, r;
        bracket(times + o * frames, frames, query, l, r);
        const float lt = times[o * frames + l], rt = times[o * frames + r];
        float wgt = (query - lt) / (rt - lt);
        wgt = std::isnan(wgt) ? 0.f : std::fmin(1.f, std::fmax(0.f, wgt));  // __saturatef
        for (int j = 0; j < joints; ++j) {
            float* dst = out + (o * joints + j) * 4;
            if (j == 0) {
                stq(dst, ldq(root_q + 4 * inst_ids[o]));
                continue;
            }
            const int64_t base = o * joints * frames + j;
            const Q4 a = qstd(ldq(poses + 4 * (base + int64_t(l) * joints)));
            const Q4 b = qstd(ldq(poses + 4 * (base + int64_t(r) * joints)));
            stq(dst, slerp(a, b, wgt));
        }
    }
}

// interpolate_smpl_poses_bwd_kernel, smpl_interpolate.cu:101-195; d_poses is
// written at the two bracketing frames, d_root_q accumulated (callers zero
// both), *d_query overwritten.
void xsgo_interpolate_smpl_bwd(int64_t n_obj, int frames, int joints, float query, const float* poses,
                               const float* times, const uint32_t* inst_ids, const float* g_out, float* d_poses,
                               float* d_root_q, float* d_query) {
    double dqt = 0.0;
    for (int64_t o = 0; o < n_obj; ++o) {
        int l, r;
        bracket(times + o * frames, frames, query, l, r);
        const float lt = times[o * frames + l], rt = times[o * frames + r];
        const float dt = rt - lt;
        const float raw = dt > 0.f ? (query - lt) / dt : 0.5f;
        const float wgt = std::fmin(1.f, std::fmax(0.f, raw));
        for (int j = 0; j < joints; ++j) {
            const Q4 g = ldq(g_out + (o * joints + j) * 4);
            if (j == 0) {
                const uint32_t k = inst_ids[o];
                d_root_q[4 * k] += g.w; d_root_q[4 * k + 1] += g.x;
                d_root_q[4 * k + 2] += g.y; d_root_q[4 * k + 3] += g.z;
                continue;
            }
            const int64_t base = o * joints * frames + j;
            const int64_t li = base + int64_t(l) * joints, ri = base + int64_t(r) * joints;
            const Q4 ra = ldq(poses + 4 * li), rb = ldq(poses + 4 * ri);
            Q4 da, db;
            float dw;
            slerp_bwd(qstd(ra), qstd(rb), wgt, g, da, db, dw);
            const Q4 gl = qstd_bwd(ra, da), gr = qstd_bwd(rb, db);
            if (li == ri) {
                stq(d_poses + 4 * li, qadd(gl, gr));
            } else {
                stq(d_poses + 4 * li, gl);
                stq(d_poses + 4 * ri, gr);
            }
            if (raw > 0.f && raw < 1.f && dt > 0.f) dqt += dw / dt;
        }
    }
    *d_query = float(dqt);
}

// image_to_{hwc_rgb,hwc_rgba,chw_rgb}_byte, csrc/nodes/img_layout.cu:9-54:
// (uint8)(saturate(x) * 255) per channel, saturate(NaN) = 0; layout 0 = HWC
// RGB, 1 = HWC RGBA (alpha 255), 2 = planar CHW RGB.
void xsgo_image_to_bytes(int layout, int64_t n, const float* in, uint8_t* out) {
    auto byte = [](float x) {
        const float s = x > 0.0f ? (x < 1.0f ? x : 1.0f) : 0.0f;
        return static_cast<uint8_t>(s * 255.0f);
    };
    for (int64_t i = 0; i < n; ++i) {
        const uint8_t r = byte(in[3 * i]), g = byte(in[3 * i + 1]), b = byte(in[3 * i + 2]);
        if (layout == 0) {
            out[3 * i] = r; out[3 * i + 1] = g; out[3 * i + 2] = b;
        } else if (layout == 1) {
            out[4 * i] = r; out[4 * i + 1] = g; out[4 * i + 2] = b; out[4 * i + 3] = 255;
        } else {
            out[i] = r; out[n + i] = g; out[2 * n + i] = b;
        }
    }
}

}  // extern "C"
