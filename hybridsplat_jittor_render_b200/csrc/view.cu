// Glue kernels of the per-view entry (hs_b200_standard_view_v2, c_api.cpp):
// the copies between the session's steps that Jittor does with slicing and
// concatenation (renderer.py:260-311). Each is a gather or a concatenation;
// no arithmetic.
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

// normal_raw[i] = rotation[i][:, 2] (the third column of a row-major 3 x 3).
__global__ void __launch_bounds__(kThreads) normal_column_kernel(const float* __restrict__ rot9, uint64_t count,
                                                                  float* __restrict__ out3) {
    for (uint64_t i = blockIdx.x * uint64_t(kThreads) + threadIdx.x; i < count; i += uint64_t(gridDim.x) * kThreads) {
        const float* r = rot9 + 9 * i;
        out3[3 * i] = r[2];
        out3[3 * i + 1] = r[5];
        out3[3 * i + 2] = r[8];
    }
}

// The trace's ray origins (columns 12..14) and directions (9..11) of the
// reflection suffix's [count, 36] output.
__global__ void __launch_bounds__(kThreads) split_rays_kernel(const float* __restrict__ packed36, uint64_t count,
                                                               float* __restrict__ origins3,
                                                               float* __restrict__ directions3) {
    for (uint64_t i = blockIdx.x * uint64_t(kThreads) + threadIdx.x; i < count; i += uint64_t(gridDim.x) * kThreads) {
        const float* p = packed36 + 36 * i;
        for (int c = 0; c < 3; ++c) {
            origins3[3 * i + c] = p[12 + c];
            directions3[3 * i + c] = p[9 + c];
        }
    }
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

cudaError_t normal_column(const float* rot9, uint64_t count, float* out3, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    normal_column_kernel<<<grid_for(count), kThreads, 0, s>>>(rot9, count, out3);
    return cudaGetLastError();
}

cudaError_t split_rays(const float* packed36, uint64_t count, float* origins3, float* directions3,
                       cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    split_rays_kernel<<<grid_for(count), kThreads, 0, s>>>(packed36, count, origins3, directions3);
    return cudaGetLastError();
}

cudaError_t colors5(const float* rgb3, const float* specular, const float* roughness, uint64_t count,
                    float* out5, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    colors5_kernel<<<grid_for(count), kThreads, 0, s>>>(rgb3, specular, roughness, count, out5);
    return cudaGetLastError();
}

}  // namespace view
}  // namespace hs
