// Glue kernels of the per-view entry (view.cu). Device pointers; count == 0
// is a no-op.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hs {
namespace view {

// out3[i] = rot9[i] column 2 (row-major 3 x 3): the reflective normal the
// reflection suffix takes.
cudaError_t normal_column(const float* rot9, uint64_t count, float* out3, cudaStream_t s);

// The trace's contiguous ray origins and directions from the reflection
// suffix's packed [count, 36] rows (columns 12..14 and 9..11).
cudaError_t split_rays(const float* packed36, uint64_t count, float* origins3, float* directions3,
                       cudaStream_t s);

// out5[i] = [rgb3[i], specular[i], roughness[i]].
cudaError_t colors5(const float* rgb3, const float* specular, const float* roughness, uint64_t count,
                    float* out5, cudaStream_t s);

}  // namespace view
}  // namespace hs
