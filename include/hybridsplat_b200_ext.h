/* Extensions of the B200 HybridSplat library beyond the reference C ABI.
 *
 * These entry points have no counterpart in the reference library
 * (rasterizer/include/hybridsplat_rasterizer_c_api.h declares none of them);
 * a caller that binds only the reference ABI never sees them. Status codes
 * and the error-text convention are those of hybridsplat_rasterizer_c_api.h.
 */
#ifndef HYBRIDSPLAT_B200_EXT_H_
#define HYBRIDSPLAT_B200_EXT_H_

#include "hybridsplat_rasterizer_c_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Test hook for the bounded device waits. Every wait of the sorts and scans
 * behind the raster calls (a decoupled look-back on a predecessor block's
 * status, the bulk copy of a sort tile) gives up after about one second of
 * device time; the call then returns HS_STATUS_CUDA_ERROR naming the wait,
 * its outputs are invalid, and the next call on the handle starts clean.
 * This makes the next raster call on `handle` (either backend, v1 or many_v2)
 * run its depth sort with the block of tile `tile` of the first pass never
 * publishing its status, so the waits of the following blocks run out. One
 * call only; tile = 0xffffffff cancels. A call with at most `tile` sort
 * tiles is unaffected. No counterpart in the reference library. */
HS_API int32_t hs_b200_test_stall_lookback_v1(
    HsRasterizerHandle handle, uint32_t tile, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Turns per-stage device timing of the raster calls (hs_flashgs_forward_f32_v1
 * and hs_rasterizer_forward_f32_v1) on or off for this handle. While on, each
 * raster call records four CUDA events on its stream: start, end of
 * preprocess, start of blending, end of blending. Off by default. */
HS_API int32_t hs_b200_stage_timing_enable_v1(
    HsRasterizerHandle handle, int32_t enable, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Waits for the recorded events, writes the summed milliseconds of the three
 * stages (preprocess, binning, blending) since the previous read to
 * stage_ms3[0..2] and the number of timed raster calls to *raster_calls
 * (may be null), then resets the sums. */
HS_API int32_t hs_b200_stage_timing_read_v1(
    HsRasterizerHandle handle, double* stage_ms3, uint64_t* raster_calls,
    char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* Tile-strip variants of the two raster entry points, for sharding one frame
 * across GPUs by rows of 16x16 tiles. Arguments are those of
 * hs_flashgs_forward_f32_v1 / hs_rasterizer_forward_f32_v1 with the strip
 * [tile_row_begin, tile_row_end) inserted after the handle (0 <= begin < end
 * <= ceil(height / 16), else HS_STATUS_RANGE_ERROR). Every Gaussian is
 * preprocessed, but pairs are emitted, sorted and rendered only for tiles of
 * the strip: each tile's list is the full-frame list, so the strip's pixels are
 * identical to those of a full-frame call. Only the strip's output rows are
 * written; *num_rendered / *rendered count the strip's pairs. No counterpart
 * in the reference library. */
HS_API int32_t hs_b200_flashgs_forward_rows_f32_v1(
    HsRasterizerHandle handle, uint32_t tile_row_begin, uint32_t tile_row_end,
    uint64_t point_count, int32_t width, int32_t height, const float* positions3,
    const float* shs48, const float* colors3, int32_t use_sh, const float* opacities1,
    const float* covariance6, const float* scales2, float scale_modifier, const float* rotations4,
    const float* specular1, const float* roughness1, const float* camera_position3,
    const float* camera_rotation9, float focal_x, float focal_y, float z_far, float z_near,
    const float* background3, uint64_t initial_pair_capacity, float* output_color3,
    float* output_other2, float* output_depth1, float* output_alpha1, float* output_normal3,
    float* output_median_depth1, float* output_distortion1, int32_t* output_num_rendered,
    char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_b200_rasterizer_forward_rows_f32_v1(
    HsRasterizerHandle handle, uint32_t tile_row_begin, uint32_t tile_row_end,
    uint64_t point_count, const float* background5, int32_t width, int32_t height,
    const float* means3d, const float* colors5, const float* opacities, const float* scales2,
    float scale_modifier, const float* rotations4, const float* viewmatrix4x4,
    const float* projmatrix4x4, const float* camera_position3, float tan_fovx, float tan_fovy,
    int32_t prefiltered, float* output_color5, float* output_aux7, float* output_weight,
    int32_t* output_radii, int32_t* output_rendered, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* The standard five-channel forward of hs_rasterizer_forward_f32_v1 without
 * any allocation: no context, no cudaMalloc/cudaFree/cudaHostAlloc. Every
 * scratch buffer comes from one 8 MiB device array inside the library (its
 * address is looked up with cudaGetSymbolAddress on the first call on each
 * device, so make that first call before any stream capture and before any
 * phase where the runtime must not load modules). No counterpart in the reference library. Same arguments as
 * hs_rasterizer_forward_f32_v1 with a device ordinal in place of the handle,
 * same outputs. Limits: point_count <= 16384, ceil(W/16)*ceil(H/16) <= 4096
 * tiles, <= 262144 emitted (tile, Gaussian) pairs; beyond them the call
 * returns HS_STATUS_RANGE_ERROR naming the limit (the pair limit is known only
 * after preprocessing, so outputs are then incomplete). All calls on a device
 * share the array: they are serialised by a process-wide lock and run on the
 * legacy default stream, so calls that overlap on the GPU (for example the
 * same work issued on other streams) would race; the call clears the words
 * that must start at zero itself. Inputs must be complete before the call: a
 * caller that produced them on a non-blocking stream synchronises that stream
 * first (the legacy default stream does not wait for non-blocking streams).
 * The call reads the pair count and, after queuing the renderer, its
 * wait-status word back with blocking copies into host stack memory, so it
 * returns once the frame is rendered; a bounded wait that gave up fails this
 * call (HS_STATUS_CUDA_ERROR) and not the next. The caller's current device is
 * restored on return. The scratch address is cached per device ordinal for
 * the life of the process: do not use this entry point across
 * cudaDeviceReset. */
HS_API int32_t hs_b200_rasterizer_forward_noalloc_f32_v1(
    int32_t device, uint64_t point_count, const float* background5, int32_t width,
    int32_t height, const float* means3d, const float* colors5, const float* opacities,
    const float* scales2, float scale_modifier, const float* rotations4,
    const float* viewmatrix4x4, const float* projmatrix4x4, const float* camera_position3,
    float tan_fovx, float tan_fovy, int32_t prefiltered, float* output_color5, float* output_aux7,
    float* output_weight, int32_t* output_radii, int32_t* output_rendered, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Arguments of one hs_flashgs_forward_f32_v1 call (same names, meaning and
 * checks) plus a strip of 16x16 tile rows as in
 * hs_b200_flashgs_forward_rows_f32_v1 (tile_row_end = UINT32_MAX: the whole
 * frame). camera_position3, camera_rotation9 and background3 are host
 * pointers, read before the call returns. */
typedef struct HsB200FlashgsCallV2 {
    HsRasterizerHandle handle;
    uint64_t point_count;
    int32_t width;
    int32_t height;
    const float* positions3;
    const float* shs48;
    const float* colors3;
    int32_t use_sh;
    float scale_modifier;
    const float* opacities1;
    const float* covariance6;
    const float* scales2;
    const float* rotations4;
    const float* specular1;
    const float* roughness1;
    const float* camera_position3;
    const float* camera_rotation9;
    float focal_x;
    float focal_y;
    float z_far;
    float z_near;
    const float* background3;
    uint64_t initial_pair_capacity;
    float* output_color3;
    float* output_other2;
    float* output_depth1;
    float* output_alpha1;
    float* output_normal3;
    float* output_median_depth1;
    float* output_distortion1;
    int32_t* output_num_rendered;
    uint32_t tile_row_begin;
    uint32_t tile_row_end;
} HsB200FlashgsCallV2;

/* Arguments of one hs_rasterizer_forward_f32_v1 call plus a tile-row strip,
 * as above. */
typedef struct HsB200RasterizerCallV2 {
    HsRasterizerHandle handle;
    uint64_t point_count;
    const float* background5;
    int32_t width;
    int32_t height;
    const float* means3d;
    const float* colors5;
    const float* opacities;
    const float* scales2;
    float scale_modifier;
    int32_t prefiltered;
    const float* rotations4;
    const float* viewmatrix4x4;
    const float* projmatrix4x4;
    const float* camera_position3;
    float tan_fovx;
    float tan_fovy;
    float* output_color5;
    float* output_aux7;
    float* output_weight;
    int32_t* output_radii;
    int32_t* output_rendered;
    uint32_t tile_row_begin;
    uint32_t tile_row_end;
} HsB200RasterizerCallV2;

/* Runs call_count independent raster calls concurrently, for example the
 * base and reflection branches of one view. Each call needs its own handle
 * (distinct handles, all on one device); each handle's workspaces, counters
 * and stage timing are used as by a single call. The calls run on per-handle
 * streams ordered after the work queued on `stream` (a cudaStream_t; NULL is
 * the legacy default stream the v1 entry points use), and `stream` is ordered
 * after all of them, so outputs are ready for work queued there next. Every
 * preprocess and binning stage is queued before any tile renderer, so the
 * latency-bound stages of the calls overlap. Outputs are identical to those
 * of the calls made one by one. As in the v1 calls, the host waits once per
 * call for its pair count. All arguments are checked before any work is
 * queued; after an error during execution the outputs are unspecified. No
 * counterpart in the reference library. */
HS_API int32_t hs_b200_flashgs_forward_many_v2(
    const HsB200FlashgsCallV2* calls, uint32_t call_count, void* stream, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;
HS_API int32_t hs_b200_rasterizer_forward_many_v2(
    const HsB200RasterizerCallV2* calls, uint32_t call_count, void* stream, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* ---- one whole standard view in one call ----
 *
 * The session's per-view sequence of the standard backend
 * (render_hybridsplat_view, renderer.py:232-341, with postprocess_raster,
 * math.py:426-463) as one entry point, on `stream` (NULL = the legacy default
 * stream): base colours (direction + SH + concatenation), reflection prefix
 * and suffix, the reflection trace (optional: on reflection_handle's built
 * scene) or given reflection colours, the base and reflection raster calls
 * run concurrently (as hs_b200_rasterizer_forward_many_v2), the fusion from
 * the raster calls' colour planes, and (optional) the raw-map postprocess
 * whose camera terms and pixel rays run on a side stream beside the rasters.
 * Every output equals that of the same steps called one by one. The host
 * waits once per raster call for its pair count, as the v1 calls do (the pair
 * capacity is grown on the host), so a view cannot be captured in a CUDA
 * graph. All buffers are device memory. No counterpart in the reference
 * library. */
typedef struct HsB200StandardGroupV2 {
    uint64_t count;
    const float* means3d;       /* [P,3] */
    const float* opacities;     /* [P,1] activated */
    const float* scales2;       /* [P,2] activated */
    const float* rotations4;    /* [P,4] activated (normalised) */
    const float* specular;      /* [P,1] activated */
    const float* roughness;     /* [P,1] activated */
    const float* background5;
    float* colors5;             /* [P,5] written: the raster call's colours */
    float* output_color5;       /* raster call outputs, as hs_rasterizer_forward_f32_v1 */
    float* output_aux7;
    float* output_weight;
    int32_t* output_radii;
    int32_t* output_rendered;
} HsB200StandardGroupV2;

typedef struct HsB200StandardViewV2 {
    uint32_t struct_size;                 /* sizeof(HsB200StandardViewV2) */
    HsRasterizerHandle base_handle;       /* base raster and the postprocess's camera terms */
    HsRasterizerHandle reflection_handle; /* reflection raster and the trace scene (distinct handle) */
    int32_t width;
    int32_t height;
    float tan_fovx;
    float tan_fovy;
    double fov_x;                          /* FoVx, FoVy of the camera (postprocess intrinsics) */
    double fov_y;
    const float* viewmatrix4x4;            /* world_view_transform as the session stores it */
    const float* projmatrix4x4;            /* full_proj_transform */
    const float* camera_position3;         /* camera centre */
    HsB200StandardGroupV2 base;
    HsB200StandardGroupV2 reflection;
    /* base colours: sh[P,3,sh_coefficients] channel-major, active degree */
    const float* base_sh;
    uint32_t sh_coefficients;
    uint32_t sh_degree;
    /* reflection preparation (written): prefix [R,9], normal column [R,3],
     * suffix [R,36]; with trace == 1 also the trace's ray origins and
     * directions [R,3] (suffix columns 12..14 and 9..11; unused otherwise) */
    const float* reflection_rotation_raw4;
    float* reflection_rotation9;
    float* reflection_normal3;
    float* reflection_rays36;
    float* reflection_ray_origins3;
    float* reflection_ray_directions3;
    /* reflection colours: trace == 0 takes reflection_rgb3 [R,3]; trace == 1
     * traces (hs_optix_trace_f32_v1 arguments below, rays from the suffix,
     * scale modifier 1, start_from_first 0) and writes its outputs */
    const float* reflection_rgb3;
    int32_t trace;
    const float* trace_background3;
    const float* reflection_shs;          /* [R,coefficients,3] */
    uint32_t trace_coefficients;
    uint32_t trace_degree;
    const float* reflection_others2;      /* [R,2]; read when use_others */
    int32_t use_others;
    int32_t max_trace_depth;
    float specular_threshold;
    float* trace_rgb3;
    float* trace_depth1;
    float* trace_acc1;
    float* trace_normal3;
    float* trace_dist1;
    float* trace_aux2;
    float* trace_mid32;
    float* trace_wet1;
    /* fusion: [H*W,3] each */
    float* fused_rgb3;
    float* diffuse_rgb3;
    float* reflection_rgb_map3;
    /* postprocess (when camera30 is not NULL): hs_b200_postprocess_camera_f32_v1
     * and hs_b200_standard_postprocess_f32_v1 */
    double depth_ratio;
    float* camera30;
    float* pixel_rays3;
    float* rgb_map3;
    float* acc_map;
    float* dpt_map;
    float* norm_map3;
    float* surf_norm_map3;
    float* dist_map;
    float* spec_map;
    float* rough_map;
    void* raster_begin_event;              /* optional cudaEvent_t, recorded when both calls' binning
                                            * is done and the tile renderers may start */
    void* stream;
} HsB200StandardViewV2;

HS_API int32_t hs_b200_standard_view_v2(
    const HsB200StandardViewV2* view, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* ---- one whole FlashGS view in one call ----
 *
 * The session's per-view sequence of the FlashGS backend
 * (render_hybridsplat_flashgs_view, renderer.py:344-446, with
 * _flashgs_postprocess, renderer.py:176-202) as one entry point, on `stream`
 * (NULL = the legacy default stream): the reflection preparation from the
 * trace group (the standard-activated reflection Gaussians the session traces),
 * the reflection trace (optional: on reflection.handle's built scene; its
 * colours then feed the reflection raster) or given reflection colours, the
 * base (use_sh = 1) and reflection (use_sh = 0) FlashGS calls run
 * concurrently (as hs_b200_flashgs_forward_many_v2), the fusion from the
 * raster calls' colour planes and (optional) the FlashGS raw-map
 * postprocess. Every output equals that of the same steps called one by one.
 * The host waits once per raster call for its pair count, as the v1 calls do.
 * Device buffers, except the FlashGS calls' host camera values. No
 * counterpart in the reference library. */
typedef struct HsB200FlashgsViewV2 {
    uint32_t struct_size;                  /* sizeof(HsB200FlashgsViewV2) */
    HsB200FlashgsCallV2 base;              /* use_sh = 1; tile rows must be the whole frame */
    HsB200FlashgsCallV2 reflection;        /* use_sh = 0; colors3 is ignored when trace == 1 */
    const float* world_view4x4;            /* device world_view_transform (trace, postprocess) */
    const float* full_proj4x4;             /* device full_proj_transform (trace) */
    const float* camera_center3;           /* device camera centre (reflection rays, trace) */
    /* the trace group, reflection.point_count Gaussians: xyz [R,3], raw
     * quaternions [R,4]; the preparation writes prefix [R,9], normal column
     * [R,3], suffix [R,36] and, with trace == 1, the ray origins and
     * directions [R,3] */
    const float* trace_means3d;
    const float* trace_rotation_raw4;
    float* reflection_rotation9;
    float* reflection_normal3;
    float* reflection_rays36;
    float* reflection_ray_origins3;
    float* reflection_ray_directions3;
    /* trace == 1: hs_optix_trace_f32_v1 of the trace group (scale modifier 1,
     * start_from_first 0); trace_rgb3 becomes the reflection call's colours */
    int32_t trace;
    const float* trace_background3;
    const float* trace_shs;                /* [R,coefficients,3] */
    uint32_t trace_coefficients;
    uint32_t trace_degree;
    const float* trace_others2;            /* [R,2]; read when use_others */
    const float* trace_opacities;          /* [R,1] activated */
    const float* trace_scales2;            /* [R,2] activated */
    const float* trace_rotations4;         /* [R,4] normalised */
    int32_t use_others;
    int32_t max_trace_depth;
    float specular_threshold;
    float* trace_rgb3;
    float* trace_depth1;
    float* trace_acc1;
    float* trace_normal3;
    float* trace_dist1;
    float* trace_aux2;
    float* trace_mid32;
    float* trace_wet1;
    /* fusion: [H*W,3] each */
    float* fused_rgb3;
    float* diffuse_rgb3;
    float* reflection_rgb_map3;
    /* postprocess == 1: hs_b200_flashgs_postprocess_f32_v1 of the base call
     * with the normal rotation world_view[:3,:3]^T; maps [H*W,C] */
    int32_t postprocess;
    float* rgb_map3;
    float* acc_map;
    float* dpt_map;
    float* norm_map3;
    float* surf_norm_map3;
    float* dist_map;
    float* spec_map;
    void* raster_begin_event;              /* optional cudaEvent_t, as in HsB200StandardViewV2 */
    void* stream;
} HsB200FlashgsViewV2;

HS_API int32_t hs_b200_flashgs_view_v2(
    const HsB200FlashgsViewV2* view, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* Graph replays of hs_b200_standard_view_v2, counted on its base handle.
 * An untraced view on a non-default stream, without raster_begin_event,
 * whose argument block and buffers repeat those of one of the last eight
 * such calls on the same base handle is captured as one CUDA graph (captures;
 * at most four are kept, the least recently used dropped); later calls with
 * that argument block replay it (replays: one graph launch, no host wait
 * before the renderers, the call returning after both raster calls' binning
 * as the direct path does). A replay whose pair count exceeds the capacity
 * it was captured for (an eighth plus 16384 above the largest of the last 16 counts), or that breaks a
 * limit the direct path checks, is rendered again directly (reruns), with
 * the direct path's outputs and status. The environment variable
 * HS_B200_VIEW_GRAPHS=0 turns the replays off. No counterpart in the
 * reference library. */
HS_API int32_t hs_b200_view_graph_stats_v1(
    HsRasterizerHandle base_handle, uint64_t* captures, uint64_t* replays, uint64_t* reruns, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Self-check of the packed FP32x2 arithmetic the rasterisers use (each lane
 * evaluates two pixels with sm_100 pair instructions whose components must
 * round exactly as the scalar instructions): for the count / 2 input pairs
 * (a, b, c, d at 2i and 2i + 1), every packed helper variant is compared bit
 * for bit, per component, with the scalar helper; mismatches16[k] receives
 * the number of differing pairs of operation k (mul, add, sub, fma, the two
 * mad, the two msub and the two nmad forms, the three dot2 and the three
 * diff2 forms). Device pointers; legacy default stream. A test entry; no
 * counterpart in the reference library. */
HS_API int32_t hs_b200_test_pair_ops_v1(
    const float* a, const float* b, const float* c, const float* d, uint64_t count,
    uint32_t* mismatches16, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* The standard branch's colours in one pass: hs_rasterizer_precise_direction_f32_v1
 * of points[count,3] from center3, hs_rasterizer_precise_sh_to_rgb_f32_v1 of
 * sh[count,3,coefficient_count] (channel-major, as the reference passes its
 * transposed features) at that direction, and the concatenation
 * [rgb, specular, roughness] into colors5[count,5] that the reference session
 * performs in Jittor (renderer.py:260-266). Bit-identical to the three steps;
 * same argument checks as the SH entry point. All pointers are device
 * pointers; legacy default stream. No counterpart in the reference library. */
HS_API int32_t hs_b200_precise_sh_colors5_f32_v1(
    const float* sh, uint32_t coefficient_count, uint32_t degree, const float* points,
    const float* center3, const float* specular, const float* roughness, uint64_t count,
    float* colors5, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* hs_rasterizer_precise_fuse_maps_f32_v1 with channel-first inputs: base_rgb and
 * reflection_rgb are three planes of pixel_count values each (the first three
 * planes of a raster call's colour output), specular one plane. Outputs are
 * the interleaved [pixel_count, 3] maps of the v1 entry point, bit-identical
 * to transposing the inputs and calling it. No counterpart in the reference
 * library. */
HS_API int32_t hs_b200_precise_fuse_maps_planar_f32_v1(
    const float* base_rgb, const float* reflection_rgb, const float* specular, float* diffuse,
    float* final_rgb, float* stored_reflection, uint64_t pixel_count, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Synchronous copy of the last standard forward's per-Gaussian blend state
 * into HOST buffers: image-space centre points_xy2[P,2], the ray-splat
 * transform rows transmats9[P,9] (Tu, Tv, Tw, the layout of the reference's
 * transMats, forward.cu:194-198) and normal_opacity4[P,4] (the flipped normal
 * and the opacity, forward.cu:248). Entries of Gaussians whose radius is 0
 * are unspecified. point_capacity must hold the last call's point count.
 * Diagnostic only; the standard counterpart of hs_flashgs_debug_copy_v1,
 * which the reference library has no equivalent of. */
HS_API int32_t hs_b200_standard_debug_copy_v1(
    HsRasterizerHandle handle, uint64_t point_capacity, float* points_xy2, float* transmats9,
    float* normal_opacity4, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* World-space pixel rays of one view, the first half of the standard
 * session's depth_to_normal (math.py:351-401): rays_n3[H*W,3] =
 * ((x, y, 1) @ inverse_intrinsics3x3^T) @ rotation3x3^T for every pixel in
 * row-major order, each product rounded as the TF32 tensor-op GEMM of
 * hs_rasterizer_precise_matmul_nt_n3k3_f32_v2 rounds it, so the rays equal the
 * reference session's; both products run in one tensor-core kernel.
 * inverse_intrinsics3x3 is the inverse intrinsic matrix and rotation3x3 the
 * camera-to-world rotation c2w[:3,:3], both row-major device matrices (the
 * outputs of hs_rasterizer_precise_general_inverse_f32_v2). scratch_n3 (H*W*3
 * floats, distinct from rays_n3) is written only for images of fewer than 8
 * pixels, which take the two cuBLAS calls themselves (cuBLAS rounds those
 * differently). Legacy default stream. */
HS_API int32_t hs_b200_pixel_rays_f32_v1(
    HsRasterizerHandle handle, int32_t width, int32_t height, const float* inverse_intrinsics3x3,
    const float* rotation3x3, float* scratch_n3, float* rays_n3, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* The per-view camera terms of the standard postprocess in one call on
 * `stream` (a cudaStream_t; NULL = legacy default stream), so that a session
 * can compute them beside the raster calls: the intrinsics built as
 * depth_to_normal builds them from width, height and the fields of view
 * (math.py:338-389), their inverse and the inverse of world_view_transform^T
 * through the two precise_general_inverse computations, and the world-space
 * pixel rays of hs_b200_pixel_rays_f32_v1. Writes camera30 (device, 30 floats,
 * row-major): [0..8] the inverse intrinsics, [9..17] the camera-to-world
 * rotation c2w[:3,:3], [18..20] the origin c2w[:3,3], [21..29] the normal
 * rotation world_view_transform[:3,:3]^T; and rays_n3 (device, H*W*3). All
 * bit-identical to ops of the same names on the legacy stream. world_view4x4
 * is the [4,4] device matrix as the session stores it. Calls on one handle
 * are ordered among themselves (they share a workspace region); they do not
 * share it with the other helpers. */
HS_API int32_t hs_b200_postprocess_camera_f32_v1(
    HsRasterizerHandle handle, int32_t width, int32_t height, double fov_x, double fov_y,
    const float* world_view4x4, float* camera30, float* rays_n3, void* stream, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* The standard session's raw-map postprocess of one view in one pass
 * (postprocess_raster, math.py:426-463, with depth_to_normal): from the raster
 * call's color5[5,H,W] and aux7[7,H,W], the pixel rays of
 * hs_b200_pixel_rays_f32_v1, origin3 = c2w[:3,3] and normal_rotation3x3 =
 * world_view_transform[:3,:3]^T (row-major), it writes the flattened HWC maps
 * rgb_map3[H*W,3], acc_map, dpt_map (precise depth divide blended with the
 * median by depth_ratio), norm_map3 (normal @ normal_rotation3x3),
 * surf_norm_map3 (normalised cross product of the central differences of the
 * depth-scaled rays, times alpha, zero on the border), dist_map, spec_map and
 * rough_map ([H*W] each). All pointers are device pointers; legacy default
 * stream. No counterpart in the reference library (the session runs these
 * steps as separate framework kernels). */
HS_API int32_t hs_b200_standard_postprocess_f32_v1(
    int32_t width, int32_t height, const float* color5, const float* aux7, const float* rays_n3,
    const float* origin3, const float* normal_rotation3x3, double depth_ratio, float* rgb_map3,
    float* acc_map, float* dpt_map, float* norm_map3, float* surf_norm_map3, float* dist_map,
    float* spec_map, float* rough_map, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* The FlashGS session's raw-map postprocess (_flashgs_postprocess,
 * renderer.py:176-202) in one pass: from a FlashGS forward's color3, other2,
 * depth1, alpha1 and normal3 planes it writes rgb_map3[H*W,3], acc_map,
 * dpt_map (precise depth divide with the session's non-finite mapping),
 * norm_map3 (normal @ normal_rotation3x3) and spec_map (other[0]);
 * surf_norm_map3 and dist_map, when not null, are zero-filled. All pointers
 * are device pointers; legacy default stream. */
HS_API int32_t hs_b200_flashgs_postprocess_f32_v1(
    int32_t width, int32_t height, const float* color3, const float* other2, const float* depth1,
    const float* alpha1, const float* normal3, const float* normal_rotation3x3, float* rgb_map3,
    float* acc_map, float* dpt_map, float* norm_map3, float* surf_norm_map3, float* dist_map,
    float* spec_map, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* ---- multi-GPU replicas: an NCCL communicator behind the C ABI ----
 *
 * One process per GPU. The forward renderer has no per-frame exchange (every
 * GPU holds a replica of the Gaussians and renders its own views or its own
 * strip of tile rows), so the only collectives are a broadcast of the scene
 * arrays at session start, straight into each rank's device buffers, and a
 * few host values (per-rank timings, a barrier). libnccl.so.2 is loaded with
 * dlopen on first use. Communicators are created non-blocking and every
 * operation is polled against timeout_s: a rank that never joins or leaves
 * mid-operation makes the others return HS_STATUS_CUDA_ERROR (the
 * communicator is then aborted and only hs_b200_comm_destroy_v1 remains
 * valid) instead of hanging. Every call restores the caller's current
 * device. No counterpart in the reference library (it has no multi-GPU
 * path). */
typedef struct HsB200Comm* HsB200CommHandle;

/* A new 128-byte NCCL unique id (rank 0 creates it and hands it to the other
 * ranks out of band). */
HS_API int32_t hs_b200_comm_unique_id_v1(
    uint8_t* id128, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* Joins rank `rank` of `rank_count` on CUDA device `device`; returns once
 * every rank has joined, or fails after timeout_s seconds. */
HS_API int32_t hs_b200_comm_create_v1(
    int32_t device, int32_t rank_count, int32_t rank, const uint8_t* id128, double timeout_s,
    HsB200CommHandle* out_comm, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* In-place broadcast of `bytes` bytes of device memory from rank `root`.
 * Ordered after the work queued on `stream` (a cudaStream_t, NULL = legacy
 * default stream) and returns when the data has arrived; `stream` is then
 * ordered after the broadcast. */
HS_API int32_t hs_b200_comm_broadcast_v1(
    HsB200CommHandle comm, void* buffer, uint64_t bytes, int32_t root, void* stream,
    char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* out[i] = max over ranks of values[i] (host doubles, count <= 512). */
HS_API int32_t hs_b200_comm_allreduce_max_f64_v1(
    HsB200CommHandle comm, const double* values, double* out, uint32_t count, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Returns once every rank has entered the barrier. */
HS_API int32_t hs_b200_comm_barrier_v1(
    HsB200CommHandle comm, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

/* Finalizes and frees the communicator (null is accepted). */
HS_API int32_t hs_b200_comm_destroy_v1(
    HsB200CommHandle comm, char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

#ifdef __cplusplus
}
#endif

#endif /* HYBRIDSPLAT_B200_EXT_H_ */
