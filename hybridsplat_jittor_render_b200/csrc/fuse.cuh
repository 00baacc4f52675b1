// The session's colour fusion of one pixel (precise_activation.cu:36-55,
// math.py:301-311) from channel-first planes, shared by the fusion kernel
// (precise.cu) and the per-view epilogue (postprocess.cu), so the two write
// the same bits.
#pragma once

#include <cstdint>

#include "fp.cuh"

namespace hs {

// base and refl: three planes of `pixels` values; s: the pixel's specular.
// diffuse = base (1 - s), stored = 2 (refl s), final = diffuse + stored / 2,
// each an [pixels, 3] map.
__device__ __forceinline__ void fuse_planar_pixel(const float* __restrict__ base, const float* __restrict__ refl,
                                                  float s, uint64_t pixels, uint64_t p,
                                                  float* __restrict__ diffuse, float* __restrict__ final_rgb,
                                                  float* __restrict__ stored) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float dv = mul(base[c * pixels + p], sub(1.0f, s));
        const float rv = mul(mul(refl[c * pixels + p], s), 2.0f);
        diffuse[3 * p + c] = dv;
        stored[3 * p + c] = rv;
        final_rgb[3 * p + c] = add(dv, mul(0.5f, rv));
    }
}

}  // namespace hs
