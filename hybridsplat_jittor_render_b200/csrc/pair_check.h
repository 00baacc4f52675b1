// Self-check of the packed FP32x2 helpers (pair_check.cu). Device pointers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hs {

// Operations checked, in the order of the mismatch counters: mul2, add2,
// sub2, fma2, mad_x2 v0..1, msub_x2 v0..1, nmad_x2 v0..1, dot2_x2 v0..2,
// diff2_x2 v0..2.
constexpr int kPairCheckOps = 16;

// mismatches16[op] = number of input pairs (a, b, c, d at 2i and 2i + 1, for
// i < count / 2) where the packed helper differs from the scalar helper in
// either component.
cudaError_t pair_check(const float* a, const float* b, const float* c, const float* d, uint64_t count,
                       uint32_t* mismatches16, cudaStream_t s);

}  // namespace hs
