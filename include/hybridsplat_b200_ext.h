/* Extensions of the B200 HybridSplat library beyond the reference C ABI.
 *
 * These entry points have no counterpart in the reference library
 * (rasterizer/include/hybridsplat_rasterizer_c_api.h declares none of them);
 * a caller that binds only the reference ABI never sees them. Status codes
 * and the error-text convention are those of hybridsplat_rasterizer_c_api.h.
 */
#ifndef HYBRIDSPLAT_B200_EXT_H_
#define HYBRIDSPLAT_B200_EXT_H_

#include "hybridsplat_rasterizer_c_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Turns per-stage device timing of the raster calls (hs_flashgs_forward_f32_v1
 * and hs_rasterizer_forward_f32_v1) on or off for this handle. While on, each
 * raster call records four CUDA events on its stream: start, end of
 * preprocess, start of blending, end of blending. Off by default. */
HS_API int32_t hs_b200_stage_timing_enable_v1(
    HsRasterizerHandle handle, int32_t enable, char* error_text,
    uint64_t error_capacity) HS_NOEXCEPT;

/* Waits for the recorded events, writes the summed milliseconds of the three
 * stages (preprocess, binning, blending) since the previous read to
 * stage_ms3[0..2] and the number of timed raster calls to *raster_calls
 * (may be null), then resets the sums. */
HS_API int32_t hs_b200_stage_timing_read_v1(
    HsRasterizerHandle handle, double* stage_ms3, uint64_t* raster_calls,
    char* error_text, uint64_t error_capacity) HS_NOEXCEPT;

#ifdef __cplusplus
}
#endif

#endif /* HYBRIDSPLAT_B200_EXT_H_ */
