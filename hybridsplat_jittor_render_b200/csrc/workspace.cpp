// Grow-only device buffers owned by a context (context.h).
#include <algorithm>

#include "context.h"

namespace hs {

namespace {
constexpr uint64_t kGranule = 2ull * 1024ull * 1024ull;
}

cudaError_t ensure_buffer(DeviceBuffer& buffer, uint64_t required, uint64_t* growth_count) {
    const uint64_t target = (std::max<uint64_t>(required, 1) + kGranule - 1) & ~(kGranule - 1);
    if (buffer.ptr != nullptr && buffer.bytes >= target) return cudaSuccess;
    void* replacement = nullptr;
    cudaError_t status = cudaMalloc(&replacement, target);
    if (status != cudaSuccess) return status;
    if (buffer.ptr != nullptr) {
        // Work queued earlier may still read the old allocation.
        status = cudaDeviceSynchronize();
        if (status == cudaSuccess) status = cudaFree(buffer.ptr);
        if (status != cudaSuccess) {
            cudaFree(replacement);
            return status;
        }
    }
    buffer.ptr = replacement;
    buffer.bytes = target;
    if (growth_count != nullptr) ++*growth_count;
    return cudaSuccess;
}

cudaError_t release_buffer(DeviceBuffer& buffer) {
    cudaError_t status = cudaSuccess;
    if (buffer.ptr != nullptr) status = cudaFree(buffer.ptr);
    buffer.ptr = nullptr;
    buffer.bytes = 0;
    return status;
}

}  // namespace hs
