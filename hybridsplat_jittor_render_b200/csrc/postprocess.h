// Launchers of the raw-map postprocess (postprocess.cu). All pointers are
// device pointers; an empty image is a no-op.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hs {
namespace post {

// The session's flattened HWC maps of one standard view.
struct StandardMaps {
    float* rgb3;
    float* acc;
    float* dpt;
    float* norm3;
    float* surf_norm3;
    float* dist;
    float* spec;
    float* rough;
};

// The session's maps of one FlashGS view; surf_norm3 and dist may be null
// (they are zero for this backend).
struct FlashgsMaps {
    float* rgb3;
    float* acc;
    float* dpt;
    float* norm3;
    float* surf_norm3;
    float* dist;
    float* spec;
};

// pixels[H*W,3] = (x, y, 1), the input of depth_to_normal's first GEMM.
cudaError_t pixel_grid(int width, int height, float* out3, cudaStream_t s);

// Row counts from which the reference's TF32 cuBLAS GEMM takes its tensor-op
// path, which pixel_rays and matmul_nt_n3k3 reproduce (below it, callers use
// cuBLAS itself).
constexpr uint64_t kMmaMinRows = 8;

// rays[H*W,3] = ((x, y, 1) @ K^-T) @ R^T for every pixel, each product the
// TF32 tensor-op GEMM of the reference (one MMA kernel, no scratch).
cudaError_t pixel_rays(int width, int height, const float* inverse_intrinsics3x3,
                       const float* rotation3x3, float* rays3, cudaStream_t s);

// out[N,3] = left[N,3] @ right[3,3]^T, the reference's TF32 tensor-op GEMM.
cudaError_t matmul_nt_n3k3(const float* left_n3, const float* right3x3, uint64_t rows,
                           float* out_n3, cudaStream_t s);

// The inputs of a view's two camera inverses: K = [[fx, 0, cx], [0, fy, cy],
// [0, 0, 1]] into k9 and world_view4x4 transposed into wt16 (row-major).
cudaError_t camera_inputs(float fx, float cx, float fy, float cy, const float* world_view4x4, float* k9,
                          float* wt16, cudaStream_t s);

// From the camera-to-world matrix c2w16 (row-major 4x4) and world_view4x4:
// out[9..17] = c2w[:3,:3], out[18..20] = c2w[:3,3], out[21..29] =
// world_view[:3,:3]^T (out[0..8], the inverse intrinsics, are not touched).
cudaError_t camera_pack(const float* c2w16, const float* world_view4x4, float* out30, cudaStream_t s);

// keep = float(1 - ratio) and ratio as the caller rounded them.
cudaError_t standard(int width, int height, const float* color5, const float* aux7,
                     const float* rays3, const float* origin3, const float* rotation9, float keep,
                     float ratio, const StandardMaps& maps, cudaStream_t s);

// standard() and, in the same pass, the colour fusion of the view
// (fuse_maps_planar of color5 planes 0..2, reflection_color5 planes 0..2 and
// color5 plane 3); bit-identical to the two launches.
cudaError_t standard_with_fusion(int width, int height, const float* color5, const float* aux7, const float* rays3,
                                 const float* origin3, const float* rotation9, float keep, float ratio,
                                 const StandardMaps& maps, const float* reflection_color5, float* diffuse3,
                                 float* final_rgb3, float* stored3, cudaStream_t s);

cudaError_t flashgs(int width, int height, const float* color3, const float* other2,
                    const float* depth1, const float* alpha1, const float* normal3,
                    const float* rotation9, const FlashgsMaps& maps, cudaStream_t s);
// flashgs() with the normal rotation world_view[:3,:3]^T read from the
// row-major world_view_transform (_flashgs_postprocess, renderer.py:188)
// and, when reflection_color3 is not null, the colour fusion of the view
// (fuse_maps_planar of color3, reflection_color3 and other2 plane 0) in the
// same pass.
cudaError_t flashgs_from_view(int width, int height, const float* color3, const float* other2,
                              const float* depth1, const float* alpha1, const float* normal3,
                              const float* world_view4x4, const FlashgsMaps& maps, const float* reflection_color3,
                              float* diffuse3, float* final_rgb3, float* stored3, cudaStream_t s);

}  // namespace post
}  // namespace hs
