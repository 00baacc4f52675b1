// Launchers for the fixed-rounding elementwise kernels (precise.cu,
// precise_exp.cu). All pointers are device pointers; count == 0 is a no-op.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hs {
namespace precise {

cudaError_t exp(const float* in, float* out, uint64_t count, cudaStream_t s);
cudaError_t sigmoid(const float* in, float* out, uint64_t count, cudaStream_t s);
cudaError_t normalize4(const float* in, float* out, uint64_t count, cudaStream_t s);
cudaError_t fuse_maps(const float* base, const float* refl, const float* specular, float* diffuse,
                      float* final_rgb, float* stored, uint64_t pixels, cudaStream_t s);
cudaError_t direction(const float* points, const float* center, uint64_t count, float* out,
                      cudaStream_t s);
cudaError_t sh_to_rgb(const float* sh, const float* dirs, uint64_t count, uint32_t coefficients,
                      uint32_t degree, float* out, cudaStream_t s);
// direction + sh_to_rgb + [rgb, specular, roughness] concatenation in one pass.
cudaError_t sh_colors5(const float* sh, uint32_t coefficients, uint32_t degree,
                      const float* points, const float* center, const float* specular,
                      const float* roughness, uint64_t count, float* out5, cudaStream_t s);
// fuse_maps reading channel-first colour planes.
cudaError_t fuse_maps_planar(const float* base, const float* refl, const float* specular,
                             float* diffuse, float* final_rgb, float* stored, uint64_t pixels,
                             cudaStream_t s);
cudaError_t reflection_prefix(const float* rot, uint64_t count, float* out, cudaStream_t s);
cudaError_t reflection_suffix(const float* xyz, const float* center, const float* normal_raw,
                              uint64_t count, float* out36, cudaStream_t s);
cudaError_t disk_rotation(const float* rot, uint64_t count, float* out, cudaStream_t s);
// reflection_prefix, its third column (normal3), reflection_suffix and, when
// origins3 / colors5 are not null, the suffix rows' ray origins and
// directions and [rgb3, specular, roughness], in one pass; bit-identical to
// the separate kernels.
cudaError_t reflection_view(const float* rot_raw, const float* xyz, const float* center, uint64_t count,
                            float* rot9, float* normal3, float* out36, float* origins3, float* directions3,
                            const float* rgb3, const float* specular, const float* roughness, float* colors5,
                            cudaStream_t s);
// sh_colors5 of the base group and reflection_view of the reflection group in
// one launch (side by side in one grid when the SH rows are 16 aligned
// coefficients and both groups are non-empty, else the two launches);
// bit-identical to them.
cudaError_t view_prologue(const float* sh, uint32_t coefficients, uint32_t degree, const float* points,
                          const float* center, const float* specular, const float* roughness, uint64_t count,
                          float* out5, const float* rot_raw, const float* xyz, uint64_t reflection_count,
                          float* rot9, float* normal3, float* out36, float* origins3, float* directions3,
                          const float* rgb3, const float* reflection_specular, const float* reflection_roughness,
                          float* colors5, cudaStream_t s);

// Tiny kernels used around the cuBLAS / cuSOLVER camera helpers.
cudaError_t negate9(const float* in, float* out, cudaStream_t s);
cudaError_t column_to_row_major(const float* in, uint32_t dimension, float* out, cudaStream_t s);

}  // namespace precise
}  // namespace hs
