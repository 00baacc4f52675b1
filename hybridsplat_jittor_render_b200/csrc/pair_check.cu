// Self-check of the packed FP32x2 helpers (fp.cuh) against the scalar
// helpers they mirror: every variant of every helper evaluated on pairs of
// inputs, each component compared bit for bit with the scalar result (NaNs
// included).
// Backs hs_b200_test_pair_ops_v1; the rasterisers' exactness rests on these
// identities.
#include <cuda_runtime.h>

#include <cstdint>

#include "fp.cuh"
#include "pair_check.h"

namespace hs {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ bool same_bits(float x, float y) { return __float_as_uint(x) == __float_as_uint(y); }

__device__ __forceinline__ void check(uint32_t* mismatches, int op, float2 packed, float s0, float s1) {
    if (!same_bits(packed.x, s0) || !same_bits(packed.y, s1)) atomicAdd(&mismatches[op], 1u);
}

__global__ void __launch_bounds__(kThreads) pair_check_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                              const float* __restrict__ c, const float* __restrict__ d,
                                                              uint64_t pairs, uint32_t* __restrict__ mismatches) {
    for (uint64_t i = blockIdx.x * uint64_t(kThreads) + threadIdx.x; i < pairs; i += uint64_t(gridDim.x) * kThreads) {
        const float2 A = make_float2(a[2 * i], a[2 * i + 1]), B = make_float2(b[2 * i], b[2 * i + 1]);
        const float2 C = make_float2(c[2 * i], c[2 * i + 1]), D = make_float2(d[2 * i], d[2 * i + 1]);
        check(mismatches, 0, mul2(A, B), mul(A.x, B.x), mul(A.y, B.y));
        check(mismatches, 1, add2(A, B), add(A.x, B.x), add(A.y, B.y));
        check(mismatches, 2, sub2(A, B), sub(A.x, B.x), sub(A.y, B.y));
        check(mismatches, 3, fma2(A, B, C), fma(A.x, B.x, C.x), fma(A.y, B.y, C.y));
        for (int v = 0; v < 2; ++v) {
            check(mismatches, 4 + v, mad_x2(v, A, B, C), mad(v, A.x, B.x, C.x), mad(v, A.y, B.y, C.y));
            check(mismatches, 6 + v, msub_x2(v, A, B, C), msub(v, A.x, B.x, C.x), msub(v, A.y, B.y, C.y));
            check(mismatches, 8 + v, nmad_x2(v, A, B, C), nmad(v, A.x, B.x, C.x), nmad(v, A.y, B.y, C.y));
        }
        for (int v = 0; v < 3; ++v) {
            check(mismatches, 10 + v, dot2_x2(v, A, B, C, D), dot2(v, A.x, B.x, C.x, D.x),
                  dot2(v, A.y, B.y, C.y, D.y));
            check(mismatches, 13 + v, diff2_x2(v, A, B, C, D), diff2(v, A.x, B.x, C.x, D.x),
                  diff2(v, A.y, B.y, C.y, D.y));
        }
    }
}

}  // namespace

cudaError_t pair_check(const float* a, const float* b, const float* c, const float* d, uint64_t count,
                       uint32_t* mismatches16, cudaStream_t s) {
    const uint64_t pairs = count / 2;
    cudaError_t e = cudaMemsetAsync(mismatches16, 0, kPairCheckOps * sizeof(uint32_t), s);
    if (e != cudaSuccess || pairs == 0) return e;
    const uint64_t blocks = (pairs + kThreads - 1) / kThreads;
    pair_check_kernel<<<static_cast<unsigned>(blocks < 148u * 8u ? blocks : 148u * 8u), kThreads, 0, s>>>(
        a, b, c, d, pairs, mismatches16);
    return cudaGetLastError();
}

}  // namespace hs
