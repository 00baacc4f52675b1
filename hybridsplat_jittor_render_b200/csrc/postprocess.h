// Launchers of the raw-map postprocess (postprocess.cu). All pointers are
// device pointers; an empty image is a no-op.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hs {
namespace post {

// The session's flattened HWC maps of one standard view.
struct StandardMaps {
    float* rgb3;
    float* acc;
    float* dpt;
    float* norm3;
    float* surf_norm3;
    float* dist;
    float* spec;
    float* rough;
};

// The session's maps of one FlashGS view; surf_norm3 and dist may be null
// (they are zero for this backend).
struct FlashgsMaps {
    float* rgb3;
    float* acc;
    float* dpt;
    float* norm3;
    float* surf_norm3;
    float* dist;
    float* spec;
};

// pixels[H*W,3] = (x, y, 1), the input of depth_to_normal's first GEMM.
cudaError_t pixel_grid(int width, int height, float* out3, cudaStream_t s);

// keep = float(1 - ratio) and ratio as the caller rounded them.
cudaError_t standard(int width, int height, const float* color5, const float* aux7,
                     const float* rays3, const float* origin3, const float* rotation9, float keep,
                     float ratio, const StandardMaps& maps, cudaStream_t s);

cudaError_t flashgs(int width, int height, const float* color3, const float* other2,
                    const float* depth1, const float* alpha1, const float* normal3,
                    const float* rotation9, const FlashgsMaps& maps, cudaStream_t s);

}  // namespace post
}  // namespace hs
