// expf over a buffer (reference rasterizer/precise_exp.cu:11-20). Kept in its
// own translation unit with nvcc's default --fmad=true, matching how the
// reference compiles that file, since expf is the only operation.
#include <cuda_runtime.h>

#include <cstdint>

#include "precise.h"

namespace hs {
namespace precise {
namespace {

__global__ void exp_kernel(const float* __restrict__ in, float* __restrict__ out,
                           uint64_t count) {
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        out[i] = expf(in[i]);
    }
}

__global__ void negate9_kernel(const float* __restrict__ in, float* __restrict__ out) {
    // precise_camera_center.cu:9-18: -R in physical row-major order.
    if (threadIdx.x < 9) out[threadIdx.x] = -in[threadIdx.x];
}

__global__ void column_to_row_major_kernel(const float* __restrict__ in, uint32_t dimension,
                                           float* __restrict__ out) {
    // precise_matrix.cu:7-19
    const uint32_t index = threadIdx.x;
    if (index >= dimension * dimension) return;
    const uint32_t row = index / dimension;
    const uint32_t column = index - row * dimension;
    out[index] = in[row + column * dimension];
}

}  // namespace

cudaError_t exp(const float* in, float* out, uint64_t count, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    const uint64_t needed = (count + 255) / 256;
    const uint64_t cap = static_cast<uint64_t>(sms) * 8;
    exp_kernel<<<static_cast<unsigned>(needed < cap ? needed : cap), 256, 0, s>>>(in, out, count);
    return cudaGetLastError();
}

cudaError_t negate9(const float* in, float* out, cudaStream_t s) {
    negate9_kernel<<<1, 32, 0, s>>>(in, out);
    return cudaGetLastError();
}

cudaError_t column_to_row_major(const float* in, uint32_t dimension, float* out, cudaStream_t s) {
    column_to_row_major_kernel<<<1, 16, 0, s>>>(in, dimension, out);
    return cudaGetLastError();
}

}  // namespace precise
}  // namespace hs
