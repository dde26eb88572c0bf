// Scene assembly around the render path on sm_100a: rigid per-instance
// transforms of Gaussians into the scene container (forward / backward),
// packed visibility masks from instance ids, and SMPL keyframe-pose
// interpolation (forward / backward).  Semantics: copy_gs_rigid_transform_*
// (csrc/nodes/container.cu:12-159), packed_mask_from_instances
// (csrc/nodes/gs_masking.cu:8-43) and interpolate_smpl_poses_*
// (csrc/nodes/smpl_interpolate.cu:13-226) of the reference.
//
// Quaternion conventions as in quat.cuh; slerp(a, b, t) is the shortest-arc
// spherical interpolation (b negated when a . b < 0) with a normalised
// linear interpolation when a . b > 0.9995.
#include "quat.cuh"

namespace xsg {
namespace {

constexpr int kNodeThreads = 256;

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------- rigid transform --
struct RigidIn {
    const float* pos;
    const float* rot;
    const uint32_t* inst;
    const float* iq;
    const float* it;
    const float* iv;
    const float* iw;
    const uint8_t* imask;
    const uint32_t* per_inst;
    const uint32_t* gs_off;
    int64_t n, n_inst, offset, size;
};

// container row of particle p (instance k), or -1 outside the container
__device__ __forceinline__ int64_t rigid_row(const RigidIn& in, int64_t p, uint32_t k) {
    const int64_t r = in.gs_off ? in.offset + int64_t(in.per_inst[k]) + int64_t(in.gs_off[p]) : in.offset + p;
    return (r >= 0 && r < in.size) ? r : -1;
}

__global__ void __launch_bounds__(kNodeThreads)
    rigid_fwd_kernel(RigidIn in, float* __restrict__ out_pos, float* __restrict__ out_rot,
                     float* __restrict__ out_vel, uint8_t* __restrict__ out_mask) {
    const int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= in.n) return;
    const uint32_t k = in.inst[p];
    if (k >= in.n_inst || !in.imask[k]) return;
    const int64_t r = rigid_row(in, p, k);
    if (r < 0) return;
    const Q q = ldq(in.iq + 4 * k);
    const v3 pr = rot(q, ld3(in.pos + 3 * p));
    st3(out_pos + 3 * r, pr + ld3(in.it + 3 * k));
    stq(out_rot + 4 * r, qmul(q, ldq(in.rot + 4 * p)));
    if (out_vel) st3(out_vel + 3 * r, ld3(in.iv + 3 * k) + cross3(ld3(in.iw + 3 * k), pr));
    if (out_mask) out_mask[r] = 1;
}

__global__ void __launch_bounds__(kNodeThreads)
    rigid_bwd_kernel(RigidIn in, const float* __restrict__ v_pos, const float* __restrict__ v_rot,
                     const float* __restrict__ v_vel, float* __restrict__ g_pos, float* __restrict__ g_rot,
                     float* __restrict__ g_q, float* __restrict__ g_t, float* __restrict__ g_v,
                     float* __restrict__ g_w) {
    const int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    // 13 instance-gradient values of this particle: q (4), t (3), v (3), w (3)
    float acc[13];
#pragma unroll
    for (int i = 0; i < 13; ++i) acc[i] = 0.f;
    uint32_t k = 0xffffffffu;
    if (p < in.n) {
        const uint32_t kk = in.inst[p];
        if (kk < in.n_inst && in.imask[kk]) {
            const int64_t r = rigid_row(in, p, kk);
            if (r >= 0) {
                k = kk;
                const Q q = ldq(in.iq + 4 * k);
                const v3 w = ld3(in.iw + 3 * k);
                const v3 pp = ld3(in.pos + 3 * p);
                const v3 gp = ld3(v_pos + 3 * r);
                v3 gpr = gp;
                acc[4] = gp.x; acc[5] = gp.y; acc[6] = gp.z;
                if (v_vel) {
                    const v3 gv = ld3(v_vel + 3 * r);
                    const v3 gw = cross3(rot(q, pp), gv);
                    acc[7] = gv.x; acc[8] = gv.y; acc[9] = gv.z;
                    acc[10] = gw.x; acc[11] = gw.y; acc[12] = gw.z;
                    gpr = gpr + cross3(gv, w);
                }
                const Q dq1 = rot_bwd_q(q, pp, gpr);
                st3(g_pos + 3 * p, rot(conj(q), gpr));
                const Q gr = ldq(v_rot + 4 * r);
                const Q dq2 = qmul(gr, conj(ldq(in.rot + 4 * p)));
                stq(g_rot + 4 * p, qmul(conj(q), gr));
                acc[0] = dq1.w + dq2.w; acc[1] = dq1.x + dq2.x; acc[2] = dq1.y + dq2.y; acc[3] = dq1.z + dq2.z;
            }
        }
    }
    // a warp of one instance reduces before its atomics (the usual case:
    // particles of an instance are stored together)
    const uint32_t k0 = __shfl_sync(0xffffffffu, k, 0);
    const bool uniform = __all_sync(0xffffffffu, k == k0 || k == 0xffffffffu);
    float* dst[13];
    if (uniform) {
        if (k0 == 0xffffffffu) return;
#pragma unroll
        for (int i = 0; i < 13; ++i) acc[i] = warp_sum_f(acc[i]);
        if (lane != 0) return;
        k = k0;
    } else if (k == 0xffffffffu) {
        return;
    }
    dst[0] = g_q + 4 * k; dst[1] = dst[0] + 1; dst[2] = dst[0] + 2; dst[3] = dst[0] + 3;
    dst[4] = g_t + 3 * k; dst[5] = dst[4] + 1; dst[6] = dst[4] + 2;
    dst[7] = g_v + 3 * k; dst[8] = dst[7] + 1; dst[9] = dst[7] + 2;
    dst[10] = g_w + 3 * k; dst[11] = dst[10] + 1; dst[12] = dst[10] + 2;
#pragma unroll
    for (int i = 0; i < 13; ++i)
        if ((i < 7 || v_vel) && acc[i] != 0.f) atomicAdd(dst[i], acc[i]);
}

// ----------------------------------------------------------- packed mask --
__global__ void __launch_bounds__(kNodeThreads)
    packed_mask_kernel(const int32_t* __restrict__ ids, int64_t n, const uint8_t* __restrict__ mask, int64_t n_inst,
                       uint32_t* __restrict__ out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    bool on = false;
    if (i < n) {
        const int32_t id = ids[i];
        on = id < 0 ? true : (id < n_inst && mask[id] != 0);
    }
    const unsigned bits = __ballot_sync(0xffffffffu, on);  // every lane takes part; lanes past n vote 0
    if ((threadIdx.x & 31) == 0 && i < n) out[i >> 5] = bits;
}

// --------------------------------------------------------- interpolation --
constexpr float kSlerpLinear = 0.9995f;

__device__ __forceinline__ float qdot(Q a, Q b) { return a.w * b.w + a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ Q qscl(float s, Q a) { return {s * a.w, s * a.x, s * a.y, s * a.z}; }

__device__ __forceinline__ Q slerp(Q a, Q b, float t) {
    float d = qdot(a, b);
    if (d < 0.f) { b = qscl(-1.f, b); d = -d; }
    if (d > kSlerpLinear) {
        const Q r = qadd(a, qscl(t, qadd(b, qscl(-1.f, a))));
        return qscl(rsqrtf(qdot(r, r)), r);
    }
    const float th = acosf(d), s = sinf(th);
    return qadd(qscl(sinf((1.f - t) * th) / s, a), qscl(sinf(t * th) / s, b));
}

__device__ __forceinline__ void slerp_bwd(Q a, Q b, float t, Q g, Q& da, Q& db, float& dt) {
    float d = qdot(a, b);
    const float sg = d < 0.f ? -1.f : 1.f;
    const Q bb = qscl(sg, b);
    d = sg * d;
    Q dbb;
    if (d > kSlerpLinear) {
        const Q diff = qadd(bb, qscl(-1.f, a));
        const Q r = qadd(a, qscl(t, diff));
        const float il = rsqrtf(qdot(r, r));
        const Q q = qscl(il, r);
        const Q dr = qscl(il, qadd(g, qscl(-qdot(q, g), q)));
        da = qscl(1.f - t, dr);
        dbb = qscl(t, dr);
        dt = qdot(dr, diff);
    } else {
        const float th = acosf(d), s = sinf(th);
        const float sa = sinf((1.f - t) * th), sb = sinf(t * th);
        const float ca = sa / s, cb = sb / s;
        const float ga = qdot(g, a), gb = qdot(g, bb);
        const float dca = ((1.f - t) * cosf((1.f - t) * th) * s - sa * d) / (s * s);
        const float dcb = (t * cosf(t * th) * s - sb * d) / (s * s);
        const float dd = -(dca * ga + dcb * gb) / s;
        da = qadd(qscl(ca, g), qscl(dd, bb));
        dbb = qadd(qscl(cb, g), qscl(dd, a));
        dt = (-th * cosf((1.f - t) * th) / s) * ga + (th * cosf(t * th) / s) * gb;
    }
    db = qscl(sg, dbb);
}

// first keyframe at or after the query, as smpl_interpolate.cu:34-52
__device__ __forceinline__ void bracket(const float* times, int frames, float q, int& l, int& r) {
    int f = frames;
    for (int i = 0; i < frames; ++i)
        if (times[i] >= q) { f = i; break; }
    l = f == 0 ? 0 : f - 1;
    r = f < frames - 1 ? f : frames - 1;
}

// one thread per (body, joint)
__global__ void __launch_bounds__(kNodeThreads)
    interp_fwd_kernel(int64_t n_obj, int frames, int joints, const float* __restrict__ query,
                      const float* __restrict__ poses, const float* __restrict__ times,
                      const float* __restrict__ root_q, const uint32_t* __restrict__ inst, int64_t n_inst,
                      float* __restrict__ out) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n_obj * joints) return;
    const int64_t o = t / joints;
    const int j = int(t - o * joints);
    const float qt = query[0];
    int l, r;
    bracket(times + o * frames, frames, qt, l, r);
    const float lt = times[o * frames + l], rt = times[o * frames + r];
    const float w = __saturatef((qt - lt) / (rt - lt));
    if (j == 0) {
        const uint32_t k = inst[o];
        stq(out + 4 * t, k < n_inst ? ldq(root_q + 4 * k) : Q{0.f, 0.f, 0.f, 0.f});
        return;
    }
    const int64_t base = o * int64_t(joints) * frames + j;
    const Q a = qstd(ldq(poses + 4 * (base + int64_t(l) * joints)));
    const Q b = qstd(ldq(poses + 4 * (base + int64_t(r) * joints)));
    stq(out + 4 * t, slerp(a, b, w));
}

__global__ void __launch_bounds__(kNodeThreads)
    interp_bwd_kernel(int64_t n_obj, int frames, int joints, const float* __restrict__ query,
                      const float* __restrict__ poses, const float* __restrict__ times,
                      const uint32_t* __restrict__ inst, int64_t n_inst, const float* __restrict__ g_out,
                      float* __restrict__ d_poses, float* __restrict__ d_root, float* __restrict__ d_query) {
    __shared__ float part[kNodeThreads / 32];
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    float dq_local = 0.f;
    if (t < n_obj * joints) {
        const int64_t o = t / joints;
        const int j = int(t - o * joints);
        const float qt = query[0];
        int l, r;
        bracket(times + o * frames, frames, qt, l, r);
        const float lt = times[o * frames + l], rt = times[o * frames + r];
        const float dt = rt - lt;
        const float raw = dt > 0.f ? (qt - lt) / dt : 0.5f;
        const float w = __saturatef(raw);
        const Q g = ldq(g_out + 4 * t);
        if (j == 0) {
            const uint32_t k = inst[o];
            if (k < n_inst) {
                atomicAdd(d_root + 4 * k, g.w); atomicAdd(d_root + 4 * k + 1, g.x);
                atomicAdd(d_root + 4 * k + 2, g.y); atomicAdd(d_root + 4 * k + 3, g.z);
            }
        } else {
            const int64_t base = o * int64_t(joints) * frames + j;
            const int64_t li = base + int64_t(l) * joints, ri = base + int64_t(r) * joints;
            const Q ra = ldq(poses + 4 * li), rb = ldq(poses + 4 * ri);
            Q da, db;
            float dw;
            slerp_bwd(qstd(ra), qstd(rb), w, g, da, db, dw);
            const Q gl = qstd_bwd(ra, da), gr = qstd_bwd(rb, db);
            if (li == ri) {
                stq(d_poses + 4 * li, qadd(gl, gr));
            } else {
                stq(d_poses + 4 * li, gl);
                stq(d_poses + 4 * ri, gr);
            }
            if (raw > 0.f && raw < 1.f && dt > 0.f) dq_local = dw / dt;
        }
    }
    dq_local = warp_sum_f(dq_local);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = dq_local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int i = 0; i < kNodeThreads / 32; ++i) s += part[i];
        if (s != 0.f) atomicAdd(d_query, s);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace xsg

using namespace xsg;

extern "C" int xsg_rigid_transform_fwd(int64_t n, const float* positions, const float* rotations,
                                       const uint32_t* instance_ids, const float* inst_q, const float* inst_t,
                                       const float* inst_v, const float* inst_w, const uint8_t* inst_mask,
                                       int64_t n_instances, int64_t buffer_offset,
                                       const uint32_t* per_instance_offsets, const uint32_t* gs_inst_offsets,
                                       int64_t container_size, float* out_positions, float* out_rotations,
                                       float* out_velocities, uint8_t* out_mask, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && n_instances >= 0 && buffer_offset >= 0 && container_size >= 0,
                "copy_gs_rigid_transform_fwd: negative size");
    XSG_REQUIRE((per_instance_offsets == nullptr) == (gs_inst_offsets == nullptr),
                "copy_gs_rigid_transform_fwd: pass both per_instance_offsets and gs_inst_offsets or neither");
    XSG_REQUIRE(gs_inst_offsets || buffer_offset + n <= container_size,
                "copy_gs_rigid_transform_fwd: buffer_offset + N exceeds the output buffer");
    if (n == 0) return XSG_OK;
    XSG_REQUIRE(positions && rotations && instance_ids && inst_q && inst_t && inst_mask && out_positions &&
                    out_rotations && (!out_velocities || (inst_v && inst_w)),
                "copy_gs_rigid_transform_fwd: null pointer");
    XSG_REQUIRE(aligned16(rotations) && aligned16(inst_q) && aligned16(out_rotations),
                "copy_gs_rigid_transform_fwd: quaternion arrays must be 16-byte aligned");
    RigidIn in{positions, rotations, instance_ids, inst_q, inst_t, inst_v, inst_w, inst_mask,
               per_instance_offsets, gs_inst_offsets, n, n_instances, buffer_offset, container_size};
    launch(rigid_fwd_kernel, blocks_for(n, kNodeThreads), kNodeThreads, 0, as_cuda(stream), in, out_positions,
           out_rotations, out_velocities, out_mask);
    return check_launch("copy_gs_rigid_transform_fwd");
}

extern "C" int xsg_rigid_transform_bwd(int64_t n, const float* positions, const float* rotations,
                                       const uint32_t* instance_ids, const float* inst_q, const float* inst_w,
                                       const uint8_t* inst_mask, int64_t n_instances, int64_t buffer_offset,
                                       const uint32_t* per_instance_offsets, const uint32_t* gs_inst_offsets,
                                       int64_t container_size, const float* v_positions, const float* v_rotations,
                                       const float* v_velocities, float* grad_positions, float* grad_rotations,
                                       float* grad_q, float* grad_t, float* grad_v, float* grad_w,
                                       xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && n_instances >= 0 && buffer_offset >= 0 && container_size >= 0,
                "copy_gs_rigid_transform_bwd: negative size");
    XSG_REQUIRE((per_instance_offsets == nullptr) == (gs_inst_offsets == nullptr),
                "copy_gs_rigid_transform_bwd: pass both per_instance_offsets and gs_inst_offsets or neither");
    XSG_REQUIRE(gs_inst_offsets || buffer_offset + n <= container_size,
                "copy_gs_rigid_transform_bwd: buffer_offset + N exceeds the gradient buffer");
    if (n == 0) return XSG_OK;
    XSG_REQUIRE(positions && rotations && instance_ids && inst_q && inst_mask && v_positions && v_rotations &&
                    grad_positions && grad_rotations && grad_q && grad_t && (!v_velocities || (inst_w && grad_v && grad_w)),
                "copy_gs_rigid_transform_bwd: null pointer");
    XSG_REQUIRE(aligned16(rotations) && aligned16(inst_q) && aligned16(v_rotations) && aligned16(grad_rotations),
                "copy_gs_rigid_transform_bwd: quaternion arrays must be 16-byte aligned");
    RigidIn in{positions, rotations, instance_ids, inst_q, nullptr, nullptr, inst_w, inst_mask,
               per_instance_offsets, gs_inst_offsets, n, n_instances, buffer_offset, container_size};
    launch(rigid_bwd_kernel, blocks_for(n, kNodeThreads), kNodeThreads, 0, as_cuda(stream), in, v_positions,
           v_rotations, v_velocities, grad_positions, grad_rotations, grad_q, grad_t, grad_v, grad_w);
    return check_launch("copy_gs_rigid_transform_bwd");
}

extern "C" int xsg_packed_mask_from_instances(const int32_t* instance_ids, int64_t n, const uint8_t* instance_mask,
                                              int64_t n_instances, uint32_t* out, xsg_stream_t stream) {
    XSG_REQUIRE(n >= 0 && n_instances >= 0, "packed_mask_from_instances: negative size");
    if (n == 0) return XSG_OK;
    XSG_REQUIRE(instance_ids && out && (instance_mask || n_instances == 0),
                "packed_mask_from_instances: null pointer");
    launch(packed_mask_kernel, blocks_for(n, kNodeThreads), kNodeThreads, 0, as_cuda(stream), instance_ids, n,
           instance_mask, n_instances, out);
    return check_launch("packed_mask_from_instances");
}

extern "C" int xsg_interpolate_smpl_poses_fwd(int64_t n_objects, int frames, int joints, const float* query_time,
                                              const float* poses, const float* pose_times, const float* root_q,
                                              const uint32_t* instance_ids, int64_t n_instances, float* out,
                                              xsg_stream_t stream) {
    XSG_REQUIRE(n_objects >= 0 && frames > 0 && joints > 0, "interpolate_smpl_poses_fwd: bad sizes");
    if (n_objects == 0) return XSG_OK;
    XSG_REQUIRE(query_time && poses && pose_times && root_q && instance_ids && out,
                "interpolate_smpl_poses_fwd: null pointer");
    XSG_REQUIRE(aligned16(poses) && aligned16(root_q) && aligned16(out),
                "interpolate_smpl_poses_fwd: quaternion arrays must be 16-byte aligned");
    launch(interp_fwd_kernel, blocks_for(n_objects * joints, kNodeThreads), kNodeThreads, 0, as_cuda(stream),
           n_objects, frames, joints, query_time, poses, pose_times, root_q, instance_ids, n_instances, out);
    return check_launch("interpolate_smpl_poses_fwd");
}

extern "C" int xsg_interpolate_smpl_poses_bwd(int64_t n_objects, int frames, int joints, const float* query_time,
                                              const float* poses, const float* pose_times,
                                              const uint32_t* instance_ids, int64_t n_instances,
                                              const float* grad_out, float* d_poses, float* d_root_q,
                                              float* d_query_time, xsg_stream_t stream) {
    XSG_REQUIRE(n_objects >= 0 && frames > 0 && joints > 0, "interpolate_smpl_poses_bwd: bad sizes");
    if (n_objects == 0) return XSG_OK;
    XSG_REQUIRE(query_time && poses && pose_times && instance_ids && grad_out && d_poses && d_root_q && d_query_time,
                "interpolate_smpl_poses_bwd: null pointer");
    XSG_REQUIRE(aligned16(poses) && aligned16(grad_out) && aligned16(d_poses),
                "interpolate_smpl_poses_bwd: quaternion arrays must be 16-byte aligned");
    launch(interp_bwd_kernel, blocks_for(n_objects * joints, kNodeThreads), kNodeThreads, 0, as_cuda(stream),
           n_objects, frames, joints, query_time, poses, pose_times, instance_ids, n_instances, grad_out, d_poses,
           d_root_q, d_query_time);
    return check_launch("interpolate_smpl_poses_bwd");
}
