/*
 * Stable C ABI of the HybridSplat forward renderer, B200 (sm_100a) build.
 *
 * Every declaration below is binary-compatible with the reference library
 * `libhybridsplat_rasterizer.so`, ABI version 2
 * (jittor_hybridsplat/ops/native/include/hybridsplat_rasterizer_c_api.h).
 * The Jittor custom ops and the ctypes runtime of the reference
 * (jittor_hybridsplat/ops/native_runtime.py:164-423) bind these names,
 * argument orders and struct layouts unchanged, so this library is a
 * drop-in replacement for the reference `.so`.
 *
 * Conventions shared by every entry point:
 *  - The return value is an HsStatus. On failure a NUL-terminated message is
 *    written to error_text (truncated to error_capacity); on success the
 *    buffer is cleared. error_capacity != 0 with error_text == NULL is
 *    rejected with HS_STATUS_INVALID_ARGUMENT.
 *  - Tensor pointers are device pointers on the context's device unless a
 *    comment says "host". Work is queued on the legacy default stream (0),
 *    like the reference; calls return before the GPU finishes unless stated.
 *  - Exceptions never cross this boundary.
 */
#ifndef HYBRIDSPLAT_RASTERIZER_C_API_H_
#define HYBRIDSPLAT_RASTERIZER_C_API_H_

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#if defined(HS_RASTERIZER_BUILDING_LIBRARY)
#define HS_API __declspec(dllexport)
#else
#define HS_API __declspec(dllimport)
#endif
#else
#define HS_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
#define HS_NOEXCEPT noexcept
extern "C" {
#else
#define HS_NOEXCEPT
#endif

/* Reference: hybridsplat_rasterizer_c_api.h:24 */
#define HS_RASTERIZER_ABI_VERSION 2u

typedef struct HsRasterizerContext* HsRasterizerHandle;

/* Status codes, values fixed by the reference (c_api.h:28-37). */
typedef enum HsStatus {
    HS_STATUS_OK = 0,
    HS_STATUS_INVALID_ARGUMENT = 1,
    HS_STATUS_ABI_MISMATCH = 2,
    HS_STATUS_RANGE_ERROR = 3,
    HS_STATUS_CUDA_ERROR = 4,
    HS_STATUS_OUT_OF_MEMORY = 5,
    HS_STATUS_BUSY = 6,
    HS_STATUS_INTERNAL_ERROR = 7
} HsStatus;

/* Versioned stats structs; callers fill struct_size and abi_version
 * (reference c_api.h:39-107, checked as in c_api.cpp:625-632). */
typedef struct HsRasterizerWorkspaceStatsV1 {
    uint32_t struct_size;
    uint32_t abi_version;
    int32_t device;
    uint32_t reserved;
    uint64_t geometry_bytes;
    uint64_t binning_bytes;
    uint64_t image_bytes;
    uint64_t current_bytes;
    uint64_t peak_bytes;
    uint64_t growth_count;
} HsRasterizerWorkspaceStatsV1;

typedef struct HsOptixWorkspaceStatsV1 {
    uint32_t struct_size;
    uint32_t abi_version;
    int32_t device;
    uint32_t scene_ready;
    uint64_t params_bytes;
    uint64_t gas_output_bytes;
    uint64_t gas_scratch_bytes;
    uint64_t dist3_bytes;
    uint64_t current_bytes;
    uint64_t peak_bytes;
    uint64_t growth_count;
    uint64_t scene_signature;
    uint64_t gas_build_count;
    uint64_t pipeline_create_count;
} HsOptixWorkspaceStatsV1;

typedef struct HsMathWorkspaceStatsV2 {
    uint32_t struct_size;
    uint32_t abi_version;
    int32_t device;
    uint32_t handles_ready;
    uint64_t workspace_bytes;
    uint64_t current_bytes;
    uint64_t peak_bytes;
    uint64_t growth_count;
    uint64_t handle_create_count;
    uint64_t camera_center_calls;
    uint64_t general_inverse_calls;
    uint64_t matmul_calls;
    uint64_t pixel_world_calls;
} HsMathWorkspaceStatsV2;

typedef struct HsFlashgsWorkspaceStatsV1 {
    uint32_t struct_size;
    uint32_t abi_version;
    int32_t device;
    uint32_t initialized;
    uint64_t gaussian_capacity;
    uint64_t pair_capacity;
    uint64_t range_capacity;
    uint64_t output_pixel_capacity;
    uint64_t gaussian_bytes;
    uint64_t pair_bytes;
    uint64_t cub_bytes;
    uint64_t ranges_bytes;
    uint64_t output_bytes;
    uint64_t current_bytes;
    uint64_t peak_bytes;
    uint64_t growth_count;
    uint64_t overflow_retry_count;
    uint64_t forward_calls;
    uint64_t last_point_count;
    uint64_t last_num_rendered;
    uint64_t last_tile_count;
} HsFlashgsWorkspaceStatsV1;

/* Lifetime and diagnostics (reference c_api.h:109-146, c_api.cpp:503-790). */
HS_API uint32_t hs_rasterizer_abi_version(void) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_build_info(
    char* output_text,
    uint64_t output_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_create(
    int32_t device,
    HsRasterizerHandle* handle,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_synchronize(
    HsRasterizerHandle handle,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_workspace_stats(
    HsRasterizerHandle handle,
    HsRasterizerWorkspaceStatsV1* stats,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_release_workspace(
    HsRasterizerHandle handle,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_math_workspace_stats_v2(
    HsRasterizerHandle handle,
    HsMathWorkspaceStatsV2* stats,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_destroy(
    HsRasterizerHandle handle,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Deterministic FlashGS 16x16 forward (reference c_api.h:148-188,
 * c_api.cpp:792-928, flashgs_backend.cu:339-607). Gaussian inputs and all
 * outputs are contiguous device FP32 buffers. camera_position3,
 * camera_rotation9 (row-major, world-to-camera rows) and background3 are
 * host arrays read before return. use_sh selects shs48 ([P,16,3]) or
 * colors3 ([P,3]). Outputs are channel-first: color[3,H,W], other[2,H,W],
 * depth[1,H,W], alpha[1,H,W], normal[3,H,W], median_depth[1,H,W],
 * distortion[1,H,W]; output_num_rendered is a device int32 holding the
 * number of (tile, Gaussian) pairs. Results are bit-identical to the
 * reference FlashGS backend on the same inputs. */
HS_API int32_t hs_flashgs_forward_f32_v1(
    HsRasterizerHandle handle,
    uint64_t point_count,
    int32_t width,
    int32_t height,
    const float* positions3,
    const float* shs48,
    const float* colors3,
    int32_t use_sh,
    const float* opacities1,
    const float* covariance6,
    const float* scales2,
    float scale_modifier,
    const float* rotations4,
    const float* specular1,
    const float* roughness1,
    const float* camera_position3,
    const float* camera_rotation9,
    float focal_x,
    float focal_y,
    float z_far,
    float z_near,
    const float* background3,
    uint64_t initial_pair_capacity,
    float* output_color3,
    float* output_other2,
    float* output_depth1,
    float* output_alpha1,
    float* output_normal3,
    float* output_median_depth1,
    float* output_distortion1,
    int32_t* output_num_rendered,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_flashgs_workspace_stats_v1(
    HsRasterizerHandle handle,
    HsFlashgsWorkspaceStatsV1* stats,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Host-side load-time activation of FlashGS parameters (reference
 * c_api.h:196-214, flashgs_prepare.cpp:30-84): sigmoid of opacity,
 * specular and roughness, exp of the two scales, quaternion normalisation
 * and the 3D covariance with a 1e-6 third scale. All buffers are host FP32. */
HS_API int32_t hs_flashgs_prepare_npz_host_f32_v1(
    uint64_t point_count,
    const float* opacity_raw1,
    const float* scaling_raw2,
    const float* rotation_raw4,
    const float* specular_raw1,
    const float* roughness_raw1,
    float* opacity1,
    float* scaling2,
    float* rotation4,
    float* covariance6,
    float* specular1,
    float* roughness1,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Synchronous copy of the last FlashGS forward's per-Gaussian preprocess
 * state, sorted (tile|depth, index) pairs and tile ranges into HOST buffers
 * (reference c_api.h:216-238, flashgs_backend.cu:645-709). Diagnostic only. */
HS_API int32_t hs_flashgs_debug_copy_v1(
    HsRasterizerHandle handle,
    uint64_t point_capacity,
    uint64_t pair_capacity,
    uint64_t tile_capacity,
    float* points_xy2,
    float* rgb3,
    float* other2,
    float* conic_opacity4,
    float* normal_opacity4,
    float* tu3,
    float* tv3,
    float* tw3,
    uint64_t* sorted_keys,
    uint32_t* sorted_values,
    int32_t* tile_ranges2,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Five-channel 2DGS rasteriser, "standard" backend (reference
 * c_api.h:240-271, c_api.cpp:1037-1134, full_rasterizer.cu:203-394).
 * All pointers are device buffers, including background5, the two
 * column-major 4x4 matrices and camera_position3. Outputs: color[5,H,W]
 * (+T*background), aux[7,H,W] = depth, alpha, normal[3], median depth,
 * distortion; weight[P] accumulated blend weights; radii[P]; rendered[1]. */
HS_API int32_t hs_rasterizer_forward_f32_v1(
    HsRasterizerHandle handle,
    uint64_t point_count,
    const float* background5,
    int32_t width,
    int32_t height,
    const float* means3d,
    const float* colors5,
    const float* opacities,
    const float* scales2,
    float scale_modifier,
    const float* rotations4,
    const float* viewmatrix4x4,
    const float* projmatrix4x4,
    const float* camera_position3,
    float tan_fovx,
    float tan_fovy,
    int32_t prefiltered,
    float* output_color5,
    float* output_aux7,
    float* output_weight,
    int32_t* output_radii,
    int32_t* output_rendered,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* OptiX reflection tracing (reference c_api.h:273-333). The OptiX SDK is not
 * part of this build; these entry points exist so that callers link, and
 * return HS_STATUS_INTERNAL_ERROR with an explanatory message. */
HS_API int32_t hs_optix_build_scene_v1(
    HsRasterizerHandle handle,
    const float* vertices3,
    uint64_t vertex_count,
    const int32_t* triangles3,
    uint64_t triangle_count,
    uint64_t scene_signature,
    int32_t rebuild,
    int32_t* output_status,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_optix_trace_f32_v1(
    HsRasterizerHandle handle,
    uint64_t ray_count,
    const float* ray_origins3,
    const float* ray_directions3,
    const float* background3,
    const float* means3d,
    const float* shs_m3,
    uint32_t coefficient_count,
    uint32_t degree,
    const float* others2,
    const float* opacities,
    const float* scales2,
    float scale_modifier,
    const float* rotations4,
    const float* viewmatrix4x4,
    const float* projmatrix4x4,
    const float* camera_position3,
    int32_t start_from_first,
    int32_t max_trace_depth,
    float specular_threshold,
    int32_t use_others,
    float* output_rgb3,
    float* output_depth1,
    float* output_acc1,
    float* output_normal3,
    float* output_dist1,
    float* output_aux2,
    float* output_mid32,
    float* output_wet1,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_optix_workspace_stats_v1(
    HsRasterizerHandle handle,
    HsOptixWorkspaceStatsV1* stats,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_optix_release_scene_v1(
    HsRasterizerHandle handle,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Elementwise activations with fixed FP32 rounding (reference
 * c_api.h:335-369; precise_exp.cu:11-20, precise_activation.cu:11-55).
 * count == 0 accepts NULL buffers. Bit-identical to the reference. */
HS_API int32_t hs_rasterizer_precise_exp_f32_v1(
    const float* input,
    float* output,
    uint64_t count,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_precise_sigmoid_f32_v1(
    const float* input,
    float* output,
    uint64_t count,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_precise_normalize4_f32_v1(
    const float* input4,
    float* output4,
    uint64_t count,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Two-branch fusion: diffuse = base*(1-s), reflection = (refl*s)*2,
 * final = diffuse + 0.5*reflection, all [pixel_count,3] with s [pixel_count]. */
HS_API int32_t hs_rasterizer_precise_fuse_maps_f32_v1(
    const float* base_rgb,
    const float* reflection_rgb,
    const float* specular,
    float* diffuse,
    float* final_rgb,
    float* stored_reflection,
    uint64_t pixel_count,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* SH to RGB, sh [count,3,coefficient_count], directions [count,3]
 * (reference c_api.h:371-383, precise_sh.cu:11-138). */
HS_API int32_t hs_rasterizer_precise_sh_to_rgb_f32_v1(
    const float* sh,
    const float* directions,
    uint64_t count,
    uint32_t coefficient_count,
    uint32_t degree,
    float* output,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* normalize(points - center) (reference c_api.h:385-395,
 * precise_direction.cu:11-35). */
HS_API int32_t hs_rasterizer_precise_direction_f32_v1(
    const float* points,
    const float* center,
    uint64_t count,
    float* output,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Camera and matrix helpers (reference c_api.h:397-450). They are per-view
 * O(1) or post-processing work; this build keeps them as cuBLAS/cuSOLVER
 * library calls issued the same way as the reference. */
HS_API int32_t hs_rasterizer_precise_camera_center_f32_v2(
    HsRasterizerHandle handle,
    const float* rotation3x3,
    const float* translation3x1,
    float* output3,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_precise_general_inverse_f32_v2(
    HsRasterizerHandle handle,
    const float* input,
    uint32_t dimension,
    float* output,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_precise_matmul_nt_n3k3_f32_v2(
    HsRasterizerHandle handle,
    const float* left_n3,
    const float* right3x3,
    uint64_t count,
    float* output_n3,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_precise_pixel_world_f32_v2(
    HsRasterizerHandle handle,
    const float* rotation3x3,
    const float* vectors_n3,
    uint64_t count,
    float* output_n3,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Quaternion to rotation matrix for the OptiX disk geometry (reference
 * c_api.h:452-464, precise_disk_rotation.cu:58-125). */
HS_API int32_t hs_rasterizer_precise_disk_rotation_f32_v1(
    const float* rotation_wxyz,
    uint64_t count,
    float* rotation_matrix9,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Reflection-ray generation, prefix and suffix stages (reference
 * c_api.h:466-491, precise_reflection_trace.cu:119-330). */
HS_API int32_t hs_rasterizer_precise_reflection_prefix_f32_v1(
    const float* rotation_wxyz,
    uint64_t count,
    float* rotation_matrix9,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

HS_API int32_t hs_rasterizer_precise_reflection_suffix_f32_v1(
    const float* xyz,
    const float* camera_center,
    const float* normal_raw3,
    uint64_t count,
    float* output36,
    char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

#ifdef __cplusplus
}
#endif

#endif
