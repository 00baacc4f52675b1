// Test-only harness linked into oracle/_ref/libref_hybridsplat.so together
// with the reference's own native sources (see oracle/build_ref.py). It is
// never part of the product library.
//
// 1. c_api.cpp calls hs_optix_release_context (declared in the reference's
//    optix/optix_backend.h:5, defined in optix_backend.cpp, which needs the
//    OptiX SDK and cannot be built here). The context never owns OptiX state
//    in the oracle, so the release is a no-op.
// 2. ref_flashgs_render_direct / ref_standard_render_direct run the reference
//    render kernels (vendor/flashgs/cuda_rasterizer/render.cu:777-791 and
//    vendor/standard_rasterizer/forward.cu:447-481) on caller-supplied
//    per-Gaussian state, so the blend arithmetic can be checked on inputs
//    chosen by the tests instead of only through the preprocess.
#include <cuda_runtime.h>

#include <cstdint>

#include "ops.h"      // reference flashgs entry points (namespace flashgs)
#include "forward.h"  // reference standard rasteriser (namespace FORWARD)

struct HsRasterizerContext;

void hs_optix_release_context(HsRasterizerContext*) noexcept {}

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

REF_EXPORT int ref_flashgs_render_direct(
    int num_rendered,
    int width,
    int height,
    float2* points_xy,
    float3* rgb,
    float2* other,
    float4* conic_opacity,
    float4* normal_opacity,
    float3* tu,
    float3* tv,
    float3* tw,
    uint64_t* keys_sorted,
    uint32_t* values_sorted,
    int2* ranges,
    float bg_r,
    float bg_g,
    float bg_b,
    float3* out_color_hwc,
    float2* out_other_hwc,
    float* out_depth,
    float* out_alpha,
    float3* out_normal_hwc,
    float* out_median_depth,
    float* out_distortion) {
    flashgs::render_16x16(num_rendered, width, height, points_xy, rgb, other,
                          conic_opacity, normal_opacity, tu, tv, tw, keys_sorted,
                          values_sorted, ranges, make_float3(bg_r, bg_g, bg_b),
                          out_color_hwc, out_other_hwc, out_depth, out_alpha,
                          out_normal_hwc, out_median_depth, out_distortion, nullptr);
    const cudaError_t status = cudaDeviceSynchronize();
    return static_cast<int>(status);
}

REF_EXPORT int ref_standard_render_direct(
    int width,
    int height,
    const uint2* ranges,
    const uint32_t* point_list,
    const float2* means2d,
    const float* colors5,
    const float* transmats9,
    const float* depths,
    const float4* normal_opacity,
    float* final_t3,
    uint32_t* n_contrib2,
    const float* background5,
    float* out_color5,
    float* out_aux7,
    float* out_weight) {
    const dim3 grid((width + 15) / 16, (height + 15) / 16, 1);
    const dim3 block(16, 16, 1);
    FORWARD::render(grid, block, ranges, point_list, width, height, 0.0f, 0.0f,
                    means2d, colors5, transmats9, depths, normal_opacity, final_t3,
                    n_contrib2, background5, out_color5, out_aux7, out_weight);
    const cudaError_t status = cudaDeviceSynchronize();
    return static_cast<int>(status);
}

// 3. ref_standard_preprocess_direct runs the reference preprocess kernel
//    (vendor/standard_rasterizer/forward.cu:148-251 via FORWARD::preprocess,
//    forward.cu:483-537) with precomputed colours and no SH, and returns its
//    per-Gaussian state: radii, image-space centres, view depths, the 3x3
//    ray-splat transforms (Tu, Tv, Tw rows) and normal|opacity. The caller
//    zero-fills the outputs; entries of culled Gaussians are left as they are.
REF_EXPORT int ref_standard_preprocess_direct(
    int count,
    const float* means3d,
    const float* scales2,
    float scale_modifier,
    const float* rotations4,
    const float* opacities,
    const float* colors5,
    const float* viewmatrix,
    const float* projmatrix,
    int width,
    int height,
    float tan_fovx,
    float tan_fovy,
    int32_t* radii,
    float2* means2d,
    float* depths,
    float* transmats9,
    float* rgb5,
    float4* normal_opacity,
    uint32_t* tiles_touched) {
    const dim3 grid((width + 15) / 16, (height + 15) / 16, 1);
    const float focal_y = static_cast<float>(height) / (2.0f * tan_fovy);
    const float focal_x = static_cast<float>(width) / (2.0f * tan_fovx);
    FORWARD::preprocess(count, 0, 0, means3d, reinterpret_cast<const glm::vec2*>(scales2), scale_modifier,
                        reinterpret_cast<const glm::vec4*>(rotations4), opacities, nullptr, nullptr, nullptr,
                        colors5, viewmatrix, projmatrix, nullptr, width, height, focal_x, focal_y, tan_fovx,
                        tan_fovy, radii, means2d, depths, transmats9, rgb5, normal_opacity, grid,
                        tiles_touched, false);
    const cudaError_t status = cudaDeviceSynchronize();
    return static_cast<int>(status);
}
