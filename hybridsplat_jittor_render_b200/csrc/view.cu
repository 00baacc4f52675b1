// Glue kernel of the per-view entry (hs_b200_standard_view_v2, c_api.cpp):
// the concatenation of the traced reflection colours with the reflection
// group's specular and roughness that the session does in Jittor
// (renderer.py:306-308); no arithmetic. The untraced view concatenates in the
// fused reflection preparation (precise.cu reflection_view_kernel).
#include <cuda_runtime.h>

#include <cstdint>

#include "view.h"

namespace hs {
namespace view {
namespace {

constexpr int kThreads = 256;

unsigned grid_for(uint64_t items) {
    const uint64_t blocks = (items + kThreads - 1) / kThreads;
    return static_cast<unsigned>(blocks < 148u * 16u ? (blocks > 0 ? blocks : 1) : 148u * 16u);
}

// out5[i] = [rgb3[i], specular[i], roughness[i]].
__global__ void __launch_bounds__(kThreads) colors5_kernel(const float* __restrict__ rgb3,
                                                           const float* __restrict__ specular,
                                                           const float* __restrict__ roughness, uint64_t count,
                                                           float* __restrict__ out5) {
    for (uint64_t i = blockIdx.x * uint64_t(kThreads) + threadIdx.x; i < count; i += uint64_t(gridDim.x) * kThreads) {
        out5[5 * i] = rgb3[3 * i];
        out5[5 * i + 1] = rgb3[3 * i + 1];
        out5[5 * i + 2] = rgb3[3 * i + 2];
        out5[5 * i + 3] = specular[i];
        out5[5 * i + 4] = roughness[i];
    }
}

}  // namespace

cudaError_t colors5(const float* rgb3, const float* specular, const float* roughness, uint64_t count,
                    float* out5, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    colors5_kernel<<<grid_for(count), kThreads, 0, s>>>(rgb3, specular, roughness, count, out5);
    return cudaGetLastError();
}

}  // namespace view
}  // namespace hs
