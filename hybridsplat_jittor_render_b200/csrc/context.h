// Per-handle state behind HsRasterizerHandle.
//
// Mirrors the ownership rules of the reference context
// (rasterizer/context_internal.h:10-72, c_api.cpp:85-127): every scratch
// buffer is owned by the context, grows only, is rounded to 2 MiB, and is
// replaced only after the device has drained the work that may still read
// the old allocation. Callers' tensors are never retained across calls.
#pragma once

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusolverDn.h>

#include <array>
#include <cstdint>
#include <mutex>
#include <vector>

struct HsRasterizerContext;

namespace hs {

struct DeviceBuffer {
    void* ptr = nullptr;
    uint64_t bytes = 0;
};

// Grow-only device allocation with 2 MiB granularity; `geometric` grows to at
// least 1.25x the previous size. The old buffer is freed after
// cudaDeviceSynchronize (reference c_api.cpp:85-127, flashgs_backend.cu:56-86).
cudaError_t ensure_buffer(DeviceBuffer& buffer, uint64_t required, uint64_t* growth_count,
                          bool geometric = false);
cudaError_t release_buffer(DeviceBuffer& buffer);

// Carves aligned sub-ranges out of one workspace allocation.
struct Carver {
    unsigned char* base;
    uint64_t offset = 0;
    explicit Carver(void* b) : base(static_cast<unsigned char*>(b)) {}
    template <class T>
    T* take(uint64_t count) {
        offset = (offset + 255u) & ~uint64_t(255u);
        T* p = reinterpret_cast<T*>(base == nullptr ? nullptr : base + offset);
        offset += count * sizeof(T);
        return p;
    }
};

// Optional device timing of the raster calls, split into the three stages
// of the hot path: preprocess (projection, culling, colour), binning (depth
// sort, pair emission, tile sort, tile ranges) and blending (the tile
// renderer). Events are recorded on the launching stream only while enabled;
// stage_timing_read drains them. Not part of the reference ABI.
struct StageTimer {
    static constexpr size_t kMaxPending = 4096;
    bool enabled = false;
    std::vector<std::array<cudaEvent_t, 4>> pool;
    size_t used = 0;
    uint64_t dropped = 0;
    double total_ms[3] = {0.0, 0.0, 0.0};
    uint64_t calls = 0;
};

// Marks the stage boundaries of one raster call. Boundaries a call does not
// reach (early exits) are recorded when the marker goes out of scope, so
// every drained event set is complete.
class StageMarks {
public:
    StageMarks() = default;
    StageMarks(StageTimer& timer, cudaStream_t stream) { start(timer, stream); }
    StageMarks(const StageMarks&) = delete;
    StageMarks& operator=(const StageMarks&) = delete;
    ~StageMarks();
    void start(StageTimer& timer, cudaStream_t stream);  // records boundary 0
    void mark(int boundary);  // 0 = start, 1 = after preprocess, 2 = before blend, 3 = end
private:
    std::array<cudaEvent_t, 4>* set_ = nullptr;
    cudaStream_t stream_ = nullptr;
    int next_ = 0;
};

cudaError_t stage_timing_read(StageTimer& timer, double out_ms[3], uint64_t* calls);

// Allocates and zeroes context->device_error on first use.
cudaError_t ensure_device_error(HsRasterizerContext* context);
void stage_timing_destroy(StageTimer& timer);

}  // namespace hs

struct HsRasterizerContext {
    explicit HsRasterizerContext(int32_t device_id) : device(device_id) {}

    int32_t device;
    std::mutex mutex;

    // standard five-channel backend
    hs::DeviceBuffer std_geometry;  // per-Gaussian state
    hs::DeviceBuffer std_binning;   // pairs + sort scratch
    hs::DeviceBuffer std_image;     // tile ranges
    uint64_t std_peak_bytes = 0;
    uint64_t std_growth_count = 0;
    uint32_t* std_total_host = nullptr;  // pinned readback of the pair count

    // deterministic FlashGS backend
    hs::DeviceBuffer fg_gaussian;   // records, keys, counts, depth order
    hs::DeviceBuffer fg_pairs;      // tile ids / Gaussian ids (+ ping-pong)
    hs::DeviceBuffer fg_sort;       // radix-sort and scan scratch
    hs::DeviceBuffer fg_ranges;     // int2 per tile
    uint32_t* fg_total_host = nullptr;
    uint64_t fg_gaussian_capacity = 0;
    uint64_t fg_pair_capacity = 0;
    uint64_t fg_range_capacity = 0;
    uint64_t fg_peak_bytes = 0;
    uint64_t fg_growth_count = 0;
    uint64_t fg_overflow_retry_count = 0;
    uint64_t fg_forward_calls = 0;
    uint64_t fg_last_point_count = 0;
    uint64_t fg_last_num_rendered = 0;
    uint64_t fg_last_tile_count = 0;
    int32_t fg_last_width = 0;
    int32_t fg_last_height = 0;

    // camera / matrix helpers (cuBLAS, cuSOLVER library calls)
    cublasHandle_t math_tf32_blas = nullptr;
    cublasHandle_t math_default_blas = nullptr;
    cusolverDnHandle_t math_solver = nullptr;
    void* math_workspace = nullptr;
    uint64_t math_workspace_bytes = 0;
    uint64_t math_peak_bytes = 0;
    uint64_t math_growth_count = 0;
    int32_t math_inverse_workspace_count = 0;
    int32_t math_solve_info[16] = {};
    uint64_t math_handle_create_count = 0;
    uint64_t math_camera_center_calls = 0;
    uint64_t math_general_inverse_calls = 0;
    uint64_t math_matmul_calls = 0;
    uint64_t math_pixel_world_calls = 0;

    hs::StageTimer timer;

    // Device status word shared by the look-back waits of every sort and scan
    // of this context (bit 0: a wait gave up). Allocated and zeroed once.
    uint32_t* device_error = nullptr;
    cudaEvent_t std_count_event = nullptr;  // marks the standard totals readback
    cudaEvent_t fg_count_event = nullptr;   // marks the FlashGS totals readback
};

namespace hs {

uint64_t flashgs_current_bytes(const HsRasterizerContext* context);
uint64_t standard_current_bytes(const HsRasterizerContext* context);
cudaError_t flashgs_release(HsRasterizerContext* context);
cudaError_t standard_release(HsRasterizerContext* context);

// FlashGS forward (flashgs.cu). Arguments as in hs_flashgs_forward_f32_v1;
// only 16x16 tile rows [row_begin, row_end) (clamped to the frame) are
// binned and rendered, other output rows are left untouched.
cudaError_t flashgs_forward(HsRasterizerContext* context, int32_t point_count, int32_t width,
                            int32_t height, const float* positions3, const float* shs48,
                            const float* colors3, bool use_sh, const float* opacities1,
                            const float* covariance6, const float* scales2, float scale_modifier,
                            const float* rotations4, const float* specular1,
                            const float* roughness1, const float camera_position3[3],
                            const float camera_rotation9[9], float focal_x, float focal_y,
                            float z_far, float z_near, const float background3[3],
                            uint64_t initial_pair_capacity, float* output_color3,
                            float* output_other2, float* output_depth1, float* output_alpha1,
                            float* output_normal3, float* output_median_depth1,
                            float* output_distortion1, int32_t* output_num_rendered,
                            cudaStream_t stream, uint32_t row_begin = 0,
                            uint32_t row_end = UINT32_MAX);

cudaError_t flashgs_debug_copy(HsRasterizerContext* context, uint64_t point_capacity,
                               uint64_t pair_capacity, uint64_t tile_capacity,
                               float* points_xy2, float* rgb3, float* other2,
                               float* conic_opacity4, float* normal_opacity4, float* tu3,
                               float* tv3, float* tw3, uint64_t* sorted_keys,
                               uint32_t* sorted_values, int32_t* tile_ranges2);

// Standard five-channel forward (standard.cu); row_begin/row_end as for
// flashgs_forward.
cudaError_t standard_forward(HsRasterizerContext* context, int32_t point_count,
                             const float* background5, int32_t width, int32_t height,
                             const float* means3d, const float* colors5, const float* opacities,
                             const float* scales2, float scale_modifier, const float* rotations4,
                             const float* viewmatrix4x4, const float* projmatrix4x4,
                             const float* camera_position3, float tan_fovx, float tan_fovy,
                             bool prefiltered, float* output_color5, float* output_aux7,
                             float* output_weight, int32_t* output_radii,
                             int32_t* output_rendered, cudaStream_t stream,
                             uint32_t row_begin = 0, uint32_t row_end = UINT32_MAX);

// FlashGS host-side camera matrices (preprocess.cu:599-627), column-major.
void flashgs_camera_matrices(const float position[3], const float rotation9[9], int width,
                             int height, float focal_x, float focal_y, float z_far,
                             float z_near, float view[16], float proj[16]);

}  // namespace hs
