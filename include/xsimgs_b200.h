/*
 * xsimgs-b200 C ABI — the boundary between host code (the PyTorch extension
 * xsimgs_b200._C, or any C/ctypes/cffi caller) and the sm_100a kernels in
 * libxsimgs_b200.so.
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless its name ends in
 *     `_host`.  Arrays are dense, row-major, float32 unless stated.
 *   - Every entry point enqueues work on `stream` and returns without
 *     synchronising, except where a count must come back to the host (the
 *     `*_count` tiling calls), which synchronise `stream` once.
 *   - Return value: XSG_OK (0) or an XSG_ERR_* code; xsg_last_error() gives a
 *     message (thread-local, valid until the next call on that thread).
 *   - Scratch memory is never allocated inside the library: entry points that
 *     need it take `workspace` + `workspace_bytes`, and a matching
 *     *_workspace_size() call says how much.
 *
 * Each declaration cites the reference (whesense/xsimgs) function it replaces,
 * as path:line within that project.
 */
#ifndef XSIMGS_B200_H
#define XSIMGS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* xsg_stream_t; /* == cudaStream_t */

enum xsg_status {
    XSG_OK = 0,
    XSG_ERR_INVALID_ARGUMENT = 1,
    XSG_ERR_UNSUPPORTED = 2,
    XSG_ERR_CUDA = 3,
    XSG_ERR_WORKSPACE = 4,
};

/* Camera models; the pack layout (float32 words) is the reference's
 * Camera<Impl> struct (include/cameras/camera.h:67-183) viewed as floats:
 *   [0:4) q0 (w,x,y,z) camera->world rotation   [4:7) t0   [7:10) v   [10:13) w
 *   [13] padding   [14:16) rolling_time   [16] trigger_time   [17] pose_time
 *   then the camera impl, aligned as its struct is (16 bytes when it holds a
 *   float4, so from word 20 with words 18..19 padding):
 *     PINHOLE   [18:22) f.x f.y c.x c.y (normalised by image size) -> 22 words
 *     FISHEYE   [20:28) f.x f.y c.x c.y k1 k2 k3 k4                 -> 28 words
 *     SPHERICAL [18:22) phi_min phi_range theta_min theta_range     -> 22 words
 *     LIDAR     [18:22) the same 4 limits, [22:24) the 64-bit device
 *               address of the per-row elevation table (beam_v)      -> 24 words
 *     DISTORTED [20:32) f.x f.y c.x c.y, k1 k2 p1 p2, k3 k4 k5 k6 (OpenCV
 *               rational + tangential model), [32] max_radius^2,
 *               [33:36) padding                                      -> 36 words
 * Padding words are zero.  The impls are in csrc/cameras/perspective.cu:7-71,
 * fisheye_opencv.cu:5-188, spherical.h:34-100 and
 * distorted_perspective.cu:6-230; the lidar address words follow
 * src/xsimgs/cameras/ext/lidar.py:14-19.  (The layout takes the reference's
 * pytoast quaternion as four floats without extra alignment, which nothing
 * in the reference pins.) */
enum xsg_camera_type {
    XSG_CAM_PINHOLE = 0,
    XSG_CAM_FISHEYE = 1,
    XSG_CAM_SPHERICAL = 2,
    XSG_CAM_LIDAR = 3,
    XSG_CAM_DISTORTED = 4,
};
int xsg_camera_pack_words(int camera_type);
/* First word of the camera impl (intrinsics) in the pack: 18 or 20. */
int xsg_camera_intrinsics_word(int camera_type);

const char* xsg_last_error(void);
const char* xsg_version(void);

/* Instrumentation (no counterpart in the reference; used by the benchmark):
 * the number of kernels this library has launched in the process, and
 * optional CUDA-event timing of the main kernels by name ("rasterize_fwd",
 * "rasterize_bwd", ...).  xsg_timing_query synchronises the recorded events
 * and returns their summed duration and count. */
long long xsg_launch_count(void);
void xsg_timing_enable(int on);
void xsg_timing_reset(void);
int xsg_timing_query(const char* name, double* total_ms, long long* launches);
/* FP32 FMA peak probe: launches `blocks` x 512 threads of iters x 128
 * independent FMAs, writes the FLOP count to *flops (time it with events). */
int xsg_fp32_probe(float* scratch, int iters, int blocks, xsg_stream_t stream, double* flops);
/* Work counters of the compositing kernels: when `counters` (12 x u64,
 * device, zeroed by the caller) is set, every xsg_rasterize_fwd adds to it
 * [0] the evaluated and [1] the contributing (pixel, Gaussian) pairs as the
 * reference counts them, and, per (warp of 32 pixels, Gaussian), [2] the
 * entries staged from the tile lists, [3] those passing the warp's cone
 * test, [4] those passing the per-lane quadric test and [5] those evaluated.
 * With a workspace sized for contributor masks (static scene, colour channels
 * <= 4, tile sides multiples of 8 and 4, an even count of 8 x 4 blocks per
 * tile) it also adds, over the pairs of 8 x 4 pixel blocks (2w, 2w + 1) of
 * every fourth tile, [6] the union and [7] the sum of the two blocks'
 * contributor counts per list entry: the backward runs two pixels a lane when
 * [6] is at most 72 % of [7] for the image.  The two-pixels-a-lane backward
 * adds [8] the list entries its warps process, [9] the lanes holding a
 * contributing pixel summed over them and [10] the entries with at most two
 * such lanes.  NULL (the default) turns counting off. */
void xsg_set_pair_counters(unsigned long long* counters);

/* Camera rays: ray_o/ray_d [H, W, 3] (ray_o and valid may be NULL).
 * Replaces launch_camera_ray_fwd, include/cameras/ray_kernels.h:8-59. */
int xsg_camera_rays(int camera_type, const float* pack, int width, int height,
                    int world_space, int normalized, float* ray_o, float* ray_d,
                    uint8_t* valid, xsg_stream_t stream);

/* Per-pixel capture time (delta=0) or time relative to pose_time (delta=1),
 * out [H, W].  Replaces pixel_time_fwd / pixel_time_delta_fwd,
 * include/cameras/time_kernels.h:5-82. */
int xsg_pixel_time(int camera_type, const float* pack, int width, int height, int delta,
                   float* out, xsg_stream_t stream);
/* The same from normalised uv [n, 2]; time_kernels.h:30-112. */
int xsg_pixel_time_from_uv(int camera_type, const float* pack, const float* uv, int64_t n,
                           int delta, float* out, xsg_stream_t stream);

/* Distortion lookup of the DISTORTED camera: out [H, W, 2] = the distorted
 * normalised uv of each pixel centre, mapped to [-1, 1] (grid_sample's
 * range) unless normalized_range != 0.  Other camera types:
 * XSG_ERR_UNSUPPORTED.  Replaces undistort_map,
 * include/cameras/distortion.h:33-56. */
int xsg_undistort_map(int camera_type, const float* pack, int width, int height,
                      int normalized_range, float* out, xsg_stream_t stream);

/* Camera-parameter gradients.  Each call writes d_pack (one float per pack
 * word, xsg_camera_pack_words(camera_type) of them) in full: the gradient of
 * sum(d_out * out) with respect to the pack, zero for the padding word, the
 * lidar table address and the spherical/lidar angle limits (the reference
 * gives the limits no gradient).  Deterministic: per-CTA partial sums go to
 * `workspace` and are added in a fixed order.
 * Workspace: xsg_camera_grad_workspace_size() bytes (a constant). */
size_t xsg_camera_grad_workspace_size(void);
/* Backward of xsg_camera_rays; d_ray_o may be NULL (no origin gradient), and
 * is ignored when world_space == 0.  Replaces launch_camera_ray_bwd /
 * camera_ray_backward_kernel_cuda, include/cameras/ray_kernels.h:61-155, with
 * the impl backward of perspective.cu:18-34 and fisheye_opencv.cu:77-141. */
int xsg_camera_rays_bwd(int camera_type, const float* pack, int width, int height,
                        int world_space, int normalized, const float* d_ray_o,
                        const float* d_ray_d, float* d_pack, void* workspace,
                        size_t workspace_bytes, xsg_stream_t stream);
/* Backward of xsg_pixel_time (grad [H, W]).  Replaces pixel_time_bwd /
 * pixel_time_delta_bwd, include/cameras/time_kernels.h:115-145, 177-204, 239-267, 299-327. */
int xsg_pixel_time_bwd(int camera_type, const float* pack, int width, int height, int delta,
                       const float* grad, float* d_pack, void* workspace,
                       size_t workspace_bytes, xsg_stream_t stream);
/* Backward of xsg_pixel_time_from_uv (grad [n]); also writes d_uv [n, 2]
 * (may be NULL) = grad * rolling_time.  uv and d_uv 8-byte aligned.
 * Replaces pixel_time_from_uv_bwd / pixel_time_delta_from_uv_bwd,
 * include/cameras/time_kernels.h:147-175, 206-237, 269-297, 329-361. */
int xsg_pixel_time_from_uv_bwd(int camera_type, const float* pack, const float* uv, int64_t n,
                               int delta, const float* grad, float* d_pack, float* d_uv,
                               void* workspace, size_t workspace_bytes, xsg_stream_t stream);

/* Rolling-shutter point projection, out uvdt [n, 4] and mask [n] (u8).
 * force_no_jacobian selects the fixed-point iteration (projection_nojac).
 * Replaces camera_projection_fwd, include/cameras/projection_kernels.h:259-309. */
int xsg_projection(int camera_type, const float* pack, const float* points,
                   const float* points_velocity, int64_t n, float residual_thr,
                   float max_residual, float max_margin, int projection_mode,
                   int force_no_jacobian, float* uvdt, uint8_t* mask, xsg_stream_t stream);

/* Unscented-transform Gaussian projection.  Outputs flags u8[n], radii [n,2],
 * means2d [n,2], depths [n] are fully written (zero where not visible).
 * phm != 0 selects the phase-modelling variant (spherical / lidar only).
 * Replaces launch_unscented_transform, include/cameras/ut_kernels.h:255-305,
 * and launch_unscented_transform_phm, include/cameras/ut_phm_kernels.h:123-173. */
int xsg_projection_utgs(int camera_type, const float* pack, const float* points,
                        const float* points_velocity, const float* scales,
                        const float* quats, const float* opacity, int64_t n, float width,
                        float height, float ut_alpha, float ut_beta, float ut_kappa,
                        float residual_thr, float max_residual, float max_margin, int phm,
                        uint8_t* flags, float* radii, float* means2d, float* depths,
                        xsg_stream_t stream);

/* Zero radii of masked-out Gaussians, in place.  mask u8[n] (bool) or
 * packed_mask u32[ceil(n/32)]; exactly one must be non-NULL.
 * Replaces mask_radii / mask_radii_packed, csrc/tiling/mask_radii.cu:10-88. */
int xsg_mask_radii(const uint8_t* mask, const uint32_t* packed_mask, int64_t n, float* radii,
                   xsg_stream_t stream);

/* Tile intersection, two phases.
 *   1. *_count fills tiles_per_gauss i32[n] and returns the intersection
 *      total in *n_isects_host (synchronises `stream`).
 *   2. *_emit writes isect_ids i64[n_isects] (tile << 32 | depth bits) and
 *      flatten_ids i32[n_isects], sorted by (tile, depth, Gaussian index) when
 *      sort != 0, else in emission order.
 * Workspace: xsg_isect_workspace_size(n, 0) bytes for *_count, and
 * xsg_isect_workspace_size(n, sort ? n_isects : 0) for *_emit.
 * Regular tiles replace isect_regular_tiles, csrc/tiling/regular_tiling.cu:72-135,
 * with sort_intersections, tiling_common.cu:102-162. */
size_t xsg_isect_workspace_size(int64_t n_gauss, int64_t max_isects);
int xsg_isect_regular_count(const float* means2d, const float* radii, int64_t n, int width,
                            int height, int tile_size_x, int tile_size_y,
                            int32_t* tiles_per_gauss, int64_t* n_isects_host, void* workspace,
                            size_t workspace_bytes, xsg_stream_t stream);
int xsg_isect_regular_emit(const float* means2d, const float* radii, const float* depths,
                           int64_t n, int width, int height, int tile_size_x, int tile_size_y,
                           int sort, const int32_t* tiles_per_gauss, int64_t n_isects,
                           int64_t* isect_ids, int32_t* flatten_ids, void* workspace,
                           size_t workspace_bytes, xsg_stream_t stream);

/* Regular tiling with no host round trip: count, emit, sort and offset
 * encoding in one call that never synchronises `stream`.  Output buffers are
 * sized for `capacity` intersections (isect_ids i64[capacity], flatten_ids
 * i32[capacity], offsets i32[tiles_h * tiles_w]); on the device,
 * n_isects_dev[0] receives the intersection total and n_isects_dev[1] =
 * min(total, capacity), the number written.  The lists are the ones
 * *_count + *_emit(sort = 1) + xsg_isect_offset_encode produce whenever
 * total <= capacity; when it is larger they hold the first `capacity`
 * intersections in depth order only, and the caller, reading
 * n_isects_dev[0] later, must redo the view with a larger capacity.
 * Pass n_isects_dev + 1 and n_isects = capacity to xsg_rasterize_fwd /
 * xsg_rasterize_bwd.  Workspace: xsg_isect_workspace_size(n, capacity).
 * Same reference interface as *_count + *_emit. */
int xsg_isect_regular_tiles_async(const float* means2d, const float* radii, const float* depths,
                                  int64_t n, int width, int height, int tile_size_x,
                                  int tile_size_y, int64_t capacity, int32_t* tiles_per_gauss,
                                  int64_t* isect_ids, int32_t* flatten_ids, int32_t* offsets,
                                  int64_t* n_isects_dev, void* workspace, size_t workspace_bytes,
                                  xsg_stream_t stream);

/* Azimuth/elevation tiling for range images.  lidar != 0: irregular
 * elevation tiles bounded by elev_bounds[n_elev] (every tile_size_y-th beam
 * value); else regular tiles of tile_size_x x tile_size_y.  Gaussians with
 * flag 2 (wrap-around) are projected a second time.
 * Replaces isect_lidar_tiles, csrc/tiling/phm_lidar_tiling.cu:239-351, and
 * isect_spherical_tiles, csrc/tiling/phm_spherical_tiling.cu:179-291. */
int xsg_isect_spherical_count(int lidar, const float* pack, const float* points,
                              const float* points_velocity, const float* scales,
                              const float* quats, const float* opacity, const uint8_t* flags,
                              const float* means2d, const float* radii, const float* depths,
                              const float* elev_bounds, int n_elev, int64_t n, int tile_size_x,
                              int tile_size_y, float width, float height, float ut_alpha,
                              float ut_beta, float ut_kappa, int32_t* tiles_per_gauss,
                              int64_t* n_isects_host, void* workspace, size_t workspace_bytes,
                              xsg_stream_t stream);
int xsg_isect_spherical_emit(int lidar, const float* pack, const float* points,
                             const float* points_velocity, const float* scales,
                             const float* quats, const float* opacity, const uint8_t* flags,
                             const float* means2d, const float* radii, const float* depths,
                             const float* elev_bounds, int n_elev, int64_t n, int tile_size_x,
                             int tile_size_y, float width, float height, float ut_alpha,
                             float ut_beta, float ut_kappa, int sort,
                             const int32_t* tiles_per_gauss, int64_t n_isects,
                             int64_t* isect_ids, int32_t* flatten_ids, void* workspace,
                             size_t workspace_bytes, xsg_stream_t stream);

/* Per-tile start offsets i32[tile_height, tile_width] from sorted isect_ids.
 * Replaces isect_offset_encode, csrc/tiling/tiling_common.cu:25-99. */
int xsg_isect_offset_encode(const int64_t* isect_ids, int64_t n_isects, int tile_width,
                            int tile_height, int32_t* offsets, xsg_stream_t stream);

/* Channel counts the compositing kernels are built for (the reference's
 * ndim_cases, csrc/rasterization/common.h:5-25).  Writes up to `cap` values
 * and returns how many there are. */
int xsg_raster_supported_channels(int* out, int cap);

/* Forward compositing.  velocity/ray_time_delta non-NULL selects the dynamic
 * variant.  colors [N, cdim] may be NULL with cdim = 0.  Outputs renders
 * [H, W, cdim], depths/alphas [H, W], last_ids i32[H, W].
 * Workspace: xsg_rasterize_workspace_size(n_gauss, cdim, n_isects, n_tiles,
 * tile_size_x * tile_size_y) bytes, or with n_isects = n_tiles = 0 the
 * minimum.  n_isects_dev (device, may be NULL) holds the list length when
 * it is only known on the device; n_isects is then its upper bound (the
 * capacity the lists were allocated for) and sizes the workspace.  The larger
 * size also holds per-warp contributor masks that the
 * forward writes and that a backward given the same workspace
 * (workspace_from_forward) uses to visit only the list entries some pixel
 * of the warp composited.
 * Replaces rasterize_eval3d_fwd, csrc/rasterization/eval3d_fwd.cu:248-308,
 * and rasterize_eval3d_dynamic_fwd, eval3d_dynamic_fwd.cu:259-323. */
size_t xsg_rasterize_workspace_size(int64_t n_gauss, int cdim, int64_t n_isects, int64_t n_tiles,
                                    int tile_pixels);
int xsg_rasterize_fwd(const float* means, const float* velocity, const float* quats,
                      const float* scales, const float* colors, int cdim,
                      const float* opacities, int64_t n_gauss, int width, int height,
                      int tile_size_x, int tile_size_y, const float* ray_o,
                      const float* ray_d, const float* ray_time_delta,
                      const int32_t* tile_offsets, int tiles_w, int tiles_h,
                      const int32_t* flatten_ids, int64_t n_isects, float* renders,
                      float* depths, float* alphas, int32_t* last_ids, void* workspace,
                      size_t workspace_bytes, xsg_stream_t stream, const int64_t* n_isects_dev);

/* Backward compositing.  Gradient outputs are overwritten (zeroed first):
 * v_means/v_velocity [N,3], v_quats [N,4], v_scales [N,3], v_opacities [N],
 * v_colors [N, cdim] (NULL when cdim = 0), v_ray_o/v_ray_d [H, W, 3],
 * v_ray_time_delta [H, W] (dynamic only).  v_renders may be NULL.  Passing
 * NULL for all of v_ray_o, v_ray_d (and v_ray_time_delta) skips the per-pixel
 * ray gradients, which is cheaper when the rays need none.  With
 * workspace_from_forward != 0, `workspace` must be the one the matching
 * xsg_rasterize_fwd call (same inputs) used, unchanged since: its packed
 * Gaussian records and tile order are reused instead of rebuilt.
 * Replaces rasterize_eval3d_bwd, csrc/rasterization/eval3d_bwd.cu:297-403,
 * and rasterize_eval3d_dynamic_bwd, eval3d_dynamic_bwd.cu:312-429. */
int xsg_rasterize_bwd(const float* means, const float* velocity, const float* quats,
                      const float* scales, const float* colors, int cdim,
                      const float* opacities, int64_t n_gauss, int width, int height,
                      int tile_size_x, int tile_size_y, const float* ray_o,
                      const float* ray_d, const float* ray_time_delta,
                      const int32_t* tile_offsets, int tiles_w, int tiles_h,
                      const int32_t* flatten_ids, int64_t n_isects,
                      const float* render_alphas, const int32_t* last_ids,
                      const float* v_renders, const float* v_depths, const float* v_alphas,
                      float* v_means, float* v_velocity, float* v_quats, float* v_scales,
                      float* v_colors, float* v_opacities, float* v_ray_o, float* v_ray_d,
                      float* v_ray_time_delta, void* workspace, size_t workspace_bytes,
                      int workspace_from_forward, xsg_stream_t stream,
                      const int64_t* n_isects_dev);

/* Spherical-harmonics colour, degree 0..4; layout_3kn selects [3, K, N]
 * coefficients (else [N, K, 3]); coeffs_dc optionally holds band 0 apart;
 * mask is a packed u32 bitmask or NULL.  out [N, 3] (masked rows untouched).
 * Replaces spherical_harmonics_fused_fwd, csrc/color/sh_fwd.cu:162-245. */
int xsg_sh_fwd(int degree, const float* origin, const float* positions, const float* coeffs,
               const float* coeffs_dc, const uint32_t* mask, int layout_3kn, int64_t n,
               int dim, float* out, xsg_stream_t stream);
/* Backward: d_coeffs (shape of coeffs), d_coeffs_dc (shape of coeffs_dc or
 * NULL), d_positions [N, 3], d_origin [3] — all overwritten.
 * Replaces spherical_harmonics_fused_bwd, csrc/color/sh_bwd.cu:317-376. */
size_t xsg_sh_bwd_workspace_size(int64_t n);
int xsg_sh_bwd(int degree, const float* origin, const float* positions, const float* coeffs,
               const float* coeffs_dc, const uint32_t* mask, int layout_3kn, int64_t n,
               int dim, const float* d_out, float* d_coeffs, float* d_coeffs_dc,
               float* d_positions, float* d_origin, void* workspace, size_t workspace_bytes,
               xsg_stream_t stream);

/* Allocation-free spherical-harmonics backward.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory (a host
 * runtime that only lends the library the buffers it owns, or code that must
 * not call cudaMalloc).  Same arguments and results as xsg_sh_bwd without the
 * workspace; its scratch (per-block partial sums of d_origin) is a fixed
 * 768 KiB device array that each GPU loading the library keeps until exit.
 *   - n may be at most xsg_sh_bwd_noalloc_max_gaussians() (2^23); larger n
 *     returns XSG_ERR_INVALID_ARGUMENT.
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *     `stream` must belong to the current device (else
 *     XSG_ERR_INVALID_ARGUMENT).  The looked-up address is cached per device
 *     ordinal for the life of the process and does not survive a
 *     cudaDeviceReset.
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams, other threads) race and must be serialised by the caller.
 *     Each call writes every partial it reads, so no clearing is needed.
 *   - Nothing is allocated or freed. */
int64_t xsg_sh_bwd_noalloc_max_gaussians(void);
int xsg_sh_bwd_noalloc(int degree, const float* origin, const float* positions, const float* coeffs,
                       const float* coeffs_dc, const uint32_t* mask, int layout_3kn, int64_t n, int dim,
                       const float* d_out, float* d_coeffs, float* d_coeffs_dc, float* d_positions,
                       float* d_origin, xsg_stream_t stream);

/* Spherical-harmonics backward split for multi-view training (no
 * counterpart in the reference, which renders one view per call).  The
 * coefficient gradient summed over views j is sum_j Y(dir_j) (x) d_out_j, so a
 * multi-GPU step can exchange the per-view colour gradients d_out [n, 3] and
 * origins instead of the [n, K, 3] coefficient gradients.  Layout [n, K, 3]
 * with band 0 in `coeffs`, no mask, degree 0..4, K <= 64.
 *   xsg_sh_positions_bwd:    d_positions [n, 3] = position gradient summed
 *                            over the n_views views (origins [n_views, 3],
 *                            d_out [n_views, n, 3]); overwrites.
 *   xsg_sh_coeffs_bwd_multi: d_coeffs [n, K, 3] = coefficient gradient summed
 *                            over the n_views views; overwrites; bands past
 *                            the degree get zero. */
int xsg_sh_positions_bwd(int degree, int n_views, const float* origins, const float* positions,
                         const float* coeffs, int64_t n, int dim, const float* d_out, float* d_positions,
                         xsg_stream_t stream);
int xsg_sh_coeffs_bwd_multi(int degree, int n_views, const float* origins, const float* positions, int64_t n,
                            int dim, const float* d_out, float* d_coeffs, xsg_stream_t stream);

/* ------------------------------------------------------------- SMPL ---- *
 * 24-joint SMPL kinematic chain (parents as csrc/nodes/smpl_local_to_global
 * .cu:42-46).  Quaternions (w, x, y, z), 16-byte aligned arrays.  Bodies are
 * addressed by uint32 ids into the N "object" arrays; ids >= n_objects are
 * skipped (their outputs are left untouched). */

/* Replaces smpl_local_to_global_fwd (csrc/nodes/smpl_local_to_global.cu:91-122).
 * For b < batch and obj = local_q_ids[b]: global transform of each joint
 * (local transforms std(local_q[obj, j]) with translations joints[obj, j] -
 * joints[obj, parent], composed root to leaf, translated by -R J_j, then
 * composed with (a0_inv_q, a0_inv_t)[obj, j]) -> out_q [batch, 24, 4],
 * out_t [batch, 24, 3].  local_q, joints, a0_inv_*: [n_objects, 24, .]. */
int xsg_smpl_local_to_global_fwd(const uint32_t* local_q_ids, int64_t batch, const float* local_q,
                                 const float* joints, const float* a0_inv_q, const float* a0_inv_t,
                                 int64_t n_objects, float* out_q, float* out_t, xsg_stream_t stream);

/* Replaces smpl_local_to_global_bwd (csrc/nodes/smpl_local_to_global.cu:282-325).
 * Gradients w.r.t. local_q (through std()) and a0_inv_q / a0_inv_t, written
 * at the rows of the objects named in local_q_ids (callers zero the rest);
 * the local translations (joints) get none, as in the reference.  The
 * forward outputs the reference also passes are not needed: the chain is
 * recomputed. */
int xsg_smpl_local_to_global_bwd(const uint32_t* local_q_ids, int64_t batch, const float* local_q,
                                 const float* joints, const float* a0_inv_q, const float* a0_inv_t,
                                 int64_t n_objects, const float* grad_out_q, const float* grad_out_t,
                                 float* d_local_q, float* d_a0_inv_q, float* d_a0_inv_t, xsg_stream_t stream);

/* Replaces smpl_lbs_skinning (csrc/nodes/smpl_lbs_skinning.cu:94-134).  For
 * b < n_valid, obj = valid_ids[b], v < n_vertices: W = sum_j weights[obj, j,
 * v] [R(global_q[b, j]) | global_t[b, j]]; written at row r = global_offset +
 * obj * n_vertices + v of the container: out_positions[r] = W [x; 1] +
 * instance_t[instance_ids[obj]], out_rotations[r] = std(from_matrix(W)) (x)
 * quats[obj, v], out_velocities[r] = instance_v[instance_ids[obj]] (if given),
 * out_mask[r] = 1 (if given).  vertices [N, V, 3], quats [N, V, 4], weights
 * [N, 24, V]; global_offset + N * V <= container_size. */
int xsg_smpl_lbs_skinning_fwd(const uint32_t* valid_ids, int64_t n_valid, const float* global_q,
                              const float* global_t, const float* vertices, const float* quats,
                              const float* weights, int64_t n_objects, int64_t n_vertices,
                              const uint32_t* instance_ids, const float* instance_t, const float* instance_v,
                              int64_t n_instances, int64_t global_offset, int64_t container_size,
                              float* out_positions, float* out_rotations, float* out_velocities,
                              uint8_t* out_mask, xsg_stream_t stream);

/* Replaces smpl_lbs_skinning_bwd (csrc/nodes/smpl_lbs_skinning.cu:271-341).
 * d_global_q / d_global_t [n_valid, 24, .] and d_instance_t / d_instance_v
 * [n_instances, 3] are ACCUMULATED (zero them first); d_vertices, d_quats,
 * d_weights are written at the valid objects' rows.  grad_velocities and
 * d_instance_v may be null (no velocity gradient). */
int xsg_smpl_lbs_skinning_bwd(const uint32_t* valid_ids, int64_t n_valid, const uint32_t* instance_ids,
                              const float* global_q, const float* global_t, const float* vertices,
                              const float* quats, const float* weights, int64_t n_objects, int64_t n_vertices,
                              int64_t n_instances, int64_t global_offset, int64_t container_size,
                              const float* grad_positions, const float* grad_rotations,
                              const float* grad_velocities, float* d_global_q, float* d_global_t,
                              float* d_vertices, float* d_quats, float* d_weights, float* d_instance_v,
                              float* d_instance_t, xsg_stream_t stream);

/* Replaces smpl_ids_compaction (csrc/nodes/smpl.cu:52-86): the indices i <
 * n, ascending, with instance_mask[instance_ids[i]] != 0 (ids >=
 * n_instances count as masked out) -> out_ids [n], their number in *count
 * (device) and *n_out_host.  Synchronises `stream` once for the count; any
 * n (the reference's kernel stops at 1024). */
int xsg_smpl_ids_compaction(const uint32_t* instance_ids, int64_t n, const uint8_t* instance_mask,
                            int64_t n_instances, uint32_t* out_ids, int64_t* count, int64_t* n_out_host,
                            xsg_stream_t stream);

/* ------------------------------------------------- scene assembly ---- *
 * Replaces copy_gs_rigid_transform_fwd (csrc/nodes/container.cu:157-199).
 * For each particle p whose instance k = instance_ids[p] is enabled
 * (inst_mask[k] != 0), at container row r = buffer_offset + p, or
 * buffer_offset + per_instance_offsets[k] + gs_inst_offsets[p] when both
 * offset arrays are given: out_positions[r] = R(inst_q[k]) positions[p] +
 * inst_t[k], out_rotations[r] = inst_q[k] (x) rotations[p],
 * out_velocities[r] = inst_v[k] + inst_w[k] x R(inst_q[k]) positions[p] (if
 * given), out_mask[r] = 1 (if given).  Rows outside [0, container_size) and
 * ids >= n_instances are skipped. */
int xsg_rigid_transform_fwd(int64_t n, const float* positions, const float* rotations,
                            const uint32_t* instance_ids, const float* inst_q, const float* inst_t,
                            const float* inst_v, const float* inst_w, const uint8_t* inst_mask,
                            int64_t n_instances, int64_t buffer_offset, const uint32_t* per_instance_offsets,
                            const uint32_t* gs_inst_offsets, int64_t container_size, float* out_positions,
                            float* out_rotations, float* out_velocities, uint8_t* out_mask, xsg_stream_t stream);
/* Replaces copy_gs_rigid_transform_bwd (container.cu:202-250).  grad_q,
 * grad_t [K, .] (and grad_v, grad_w when v_velocities is given) are
 * ACCUMULATED; grad_positions / grad_rotations are written for the enabled
 * particles (zero the rest first). */
int xsg_rigid_transform_bwd(int64_t n, const float* positions, const float* rotations,
                            const uint32_t* instance_ids, const float* inst_q, const float* inst_w,
                            const uint8_t* inst_mask, int64_t n_instances, int64_t buffer_offset,
                            const uint32_t* per_instance_offsets, const uint32_t* gs_inst_offsets,
                            int64_t container_size, const float* v_positions, const float* v_rotations,
                            const float* v_velocities, float* grad_positions, float* grad_rotations,
                            float* grad_q, float* grad_t, float* grad_v, float* grad_w, xsg_stream_t stream);

/* Float RGB image [n_pixels, 3] -> bytes, each channel
 * (uint8)(saturate(x) * 255) (NaN -> 0):
 *   XSG_IMG_HWC_RGB  out [n_pixels, 3]
 *   XSG_IMG_HWC_RGBA out [n_pixels, 4], alpha 255
 *   XSG_IMG_CHW_RGB  out [3, n_pixels] (planar)
 * image 4-byte aligned; 16-byte aligned image and output take the vector
 * path.  Replaces image_to_hwc_rgb_byte / image_to_hwc_rgba_byte /
 * image_to_chw_rgb_byte, csrc/nodes/img_layout.cu:9-115. */
enum xsg_image_layout {
    XSG_IMG_HWC_RGB = 0,
    XSG_IMG_HWC_RGBA = 1,
    XSG_IMG_CHW_RGB = 2,
};
int xsg_image_to_bytes(int layout, const float* image, int64_t n_pixels, uint8_t* out,
                       xsg_stream_t stream);

/* Replaces packed_mask_from_instances (csrc/nodes/gs_masking.cu:27-43):
 * out u32[ceil(n/32)], bit i = 1 when instance_ids[i] < 0 (not an
 * instance) or instance_mask[instance_ids[i]] != 0; bits past n are 0. */
int xsg_packed_mask_from_instances(const int32_t* instance_ids, int64_t n, const uint8_t* instance_mask,
                                   int64_t n_instances, uint32_t* out, xsg_stream_t stream);

/* Replaces interpolate_smpl_poses_fwd (csrc/nodes/smpl_interpolate.cu:60-98):
 * poses [N, frames, joints, 4], pose_times [N, frames] (ascending),
 * query_time [1] (device) -> out [N, joints, 4]: joint 0 = root_q[instance_ids[n]],
 * the others slerp(std(pose at the last key before the query),
 * std(pose at the first key at or after it), saturated weight). */
int xsg_interpolate_smpl_poses_fwd(int64_t n_objects, int frames, int joints, const float* query_time,
                                   const float* poses, const float* pose_times, const float* root_q,
                                   const uint32_t* instance_ids, int64_t n_instances, float* out,
                                   xsg_stream_t stream);
/* Replaces interpolate_smpl_poses_bwd (smpl_interpolate.cu:198-226): d_poses
 * written at the two bracketing keys (zero it first), d_root_q and
 * d_query_time [1] ACCUMULATED.  As in the reference, a zero key interval
 * uses weight 0.5 in the backward. */
int xsg_interpolate_smpl_poses_bwd(int64_t n_objects, int frames, int joints, const float* query_time,
                                   const float* poses, const float* pose_times, const uint32_t* instance_ids,
                                   int64_t n_instances, const float* grad_out, float* d_poses, float* d_root_q,
                                   float* d_query_time, xsg_stream_t stream);

/* ---- multi-GPU gradient exchange (no reference counterpart) ----
 * Kernels for the sensor-sharded render step on NVSwitch systems.  Buffers
 * are symmetric (same size on every rank, one multicast address for all
 * copies, e.g. from torch's symmetric memory); `mc_addr` / `mc_dst` are
 * multicast virtual addresses.
 * xsg_exchange_barrier: peer_flags is a device array of `world` pointers, one
 * per rank, to that rank's `world` uint32 flag words (zeroed once before the
 * first barrier); every rank passes the same, strictly increasing `epoch` per
 * barrier.  A rank that does not arrive within timeout_s sets *err (device
 * int) to 1 + its rank and the barrier returns.
 * xsg_nvls_allreduce_sum_f32: in-place sum over ranks of n floats (n a
 * multiple of 4) at mc_addr; call between two barriers.
 * xsg_nvls_broadcast_f32: writes the n local floats at src into every rank's
 * copy at mc_dst (an all-gather when each rank writes its own slice); call
 * between two barriers. */
int xsg_exchange_barrier(uint32_t* const* peer_flags, int rank, int world, uint32_t epoch,
                         double timeout_s, int* err, xsg_stream_t stream);
int xsg_nvls_allreduce_sum_f32(uint64_t mc_addr, int64_t n, int rank, int world,
                               xsg_stream_t stream);
int xsg_nvls_broadcast_f32(const float* src, uint64_t mc_dst, int64_t n, xsg_stream_t stream);
/* At most n CTAs per exchange kernel (0: four per SM, the default). */
void xsg_exchange_set_max_ctas(int n);

#ifdef __cplusplus
}
#endif

#endif /* XSIMGS_B200_H */
