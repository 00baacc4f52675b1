// Glue kernel of the per-view entry (view.cu). Device pointers; count == 0
// is a no-op.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hs {
namespace view {

// out5[i] = [rgb3[i], specular[i], roughness[i]].
cudaError_t colors5(const float* rgb3, const float* specular, const float* roughness, uint64_t count,
                    float* out5, cudaStream_t s);

}  // namespace view
}  // namespace hs
