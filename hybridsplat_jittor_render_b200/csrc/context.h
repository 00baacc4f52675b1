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
// Creates context->side_stream, side_event and fork_event on first use.
cudaError_t ensure_side_stream(HsRasterizerContext* context);
// The stream and events of the per-view entry's postprocess camera terms.
cudaError_t ensure_post_stream(HsRasterizerContext* context);
// The stream and events of the per-view entry's graph replays.
cudaError_t ensure_graph_streams(HsRasterizerContext* context);
// Destroys the context's captured view graphs (waits for nothing: a launched
// graph completes after its executable is destroyed).
void destroy_view_graphs(HsRasterizerContext* context);
void destroy_side_stream(HsRasterizerContext* context);
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
    uint32_t* std_total_host = nullptr;    // mapped pinned readback of the pair totals
    uint32_t* std_total_mapped = nullptr;  // its device address
    uint64_t std_last_point_count = 0;     // Gaussians of the last forward (debug copy)

    // deterministic FlashGS backend
    hs::DeviceBuffer fg_gaussian;   // records, keys, counts, depth order
    hs::DeviceBuffer fg_pairs;      // tile ids / Gaussian ids (+ ping-pong)
    hs::DeviceBuffer fg_sort;       // radix-sort and scan scratch
    hs::DeviceBuffer fg_ranges;     // int2 per tile
    uint32_t* fg_total_host = nullptr;    // mapped pinned readback of the pair count
    uint32_t* fg_total_mapped = nullptr;  // its device address
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
    cudaEvent_t view_camera_event = nullptr;  // end of the last view-camera call (its workspace region)
    uint64_t math_handle_create_count = 0;
    uint64_t math_camera_center_calls = 0;
    uint64_t math_general_inverse_calls = 0;
    uint64_t math_matmul_calls = 0;
    uint64_t math_pixel_world_calls = 0;

    hs::StageTimer timer;

    // Device status word shared by the bounded waits of every sort and scan
    // of this context (bit 0: a wait gave up). Allocated once, cleared at the
    // start of every raster call and read back after its binning.
    uint32_t* device_error = nullptr;
    // Test hook (hs_b200_test_stall_lookback_v1): the tile of the next raster
    // call's first depth-sort pass that never publishes its look-back status.
    uint32_t test_stall_tile = 0xffffffffu;
    cudaEvent_t std_count_event = nullptr;  // marks the standard totals readback
    cudaEvent_t fg_count_event = nullptr;   // marks the FlashGS totals readback

    // Reflection trace (hs_optix_*): the scene BVH and its build scratch.
    hs::DeviceBuffer tr_scene;     // BVH nodes + triangle records (the GAS)
    hs::DeviceBuffer tr_scratch;   // build scratch (boxes, codes, sort, tree)
    hs::DeviceBuffer tr_rays;      // per-call ray order (keys, sort scratch)
    uint64_t tr_triangles = 0;     // triangles of the built scene (0: none)
    uint32_t tr_root = 0;
    uint64_t tr_signature = 0;
    uint64_t tr_build_count = 0;
    uint64_t tr_pipeline_count = 0;
    uint64_t tr_growth_count = 0;
    uint64_t tr_peak_bytes = 0;

    // Concurrent calls (forward_many): this context's calls run on its own
    // non-blocking stream, ordered against the caller's stream by events.
    cudaStream_t side_stream = nullptr;
    cudaEvent_t side_event = nullptr;  // phase marks on side_stream
    cudaStream_t post_stream = nullptr;      // the per-view entry's postprocess camera terms
    cudaEvent_t post_fork_event = nullptr;   // recorded on the view's stream before them
    cudaEvent_t post_done_event = nullptr;   // recorded on post_stream after them
    cudaEvent_t fork_event = nullptr;  // recorded on the caller's stream

    // Per-view entry replays (hs_b200_standard_view_v2 on the base handle): a
    // view whose arguments and buffers match an earlier call's runs as one
    // captured CUDA graph, sized for pair_capacity pairs per raster call,
    // with no host wait before its renderers are queued.
    struct ViewGraph {
        std::vector<unsigned char> key;    // the call's arguments and both contexts' buffer generations
        cudaGraphExec_t exec = nullptr;     // null: capture failed for this key, run the call directly
        uint32_t capacity[2] = {0, 0};      // pairs each raster call was captured for
        uint64_t last_use = 0;
    };
    std::vector<ViewGraph> view_graphs;    // at most kMaxViewGraphs
    std::vector<std::vector<unsigned char>> view_recent_keys;  // keys seen once (captured when seen again)
    uint64_t view_graph_clock = 0;
    uint64_t view_graph_captures = 0;
    uint64_t view_graph_replays = 0;
    uint64_t view_graph_reruns = 0;        // replays whose pair count overflowed, rendered again directly
    uint64_t std_last_emitted = 0;         // pairs of the last standard call that read its totals
    uint32_t std_recent_emitted[16] = {};  // pair counts of the last 16 such calls (ring)
    uint32_t std_recent_next = 0;
    cudaStream_t signal_stream = nullptr;  // a replay's host publication branch
    cudaEvent_t signal_event = nullptr;    // recorded (external) after that publication
    cudaEvent_t graph_fork_event = nullptr;
    cudaEvent_t graph_join_event = nullptr;
};

namespace hs {

// Status of a raster call whose bounded device wait gave up (a sort or scan
// look-back, or a bulk copy, that did not complete within its bound).
constexpr cudaError_t kWaitGaveUp = cudaErrorLaunchTimeout;

uint64_t flashgs_current_bytes(const HsRasterizerContext* context);
uint64_t standard_current_bytes(const HsRasterizerContext* context);
cudaError_t flashgs_release(HsRasterizerContext* context);
cudaError_t standard_release(HsRasterizerContext* context);

// Arguments of one FlashGS raster call, as in hs_flashgs_forward_f32_v1
// (host camera position, rotation and background are copied in). Only the
// 16x16 tile rows [row_begin, row_end) (clamped to the frame) are binned and
// rendered; other output rows are left untouched.
struct FlashgsCall {
    int32_t point_count = 0;
    int32_t width = 0, height = 0;
    const float* positions3 = nullptr;
    const float* shs48 = nullptr;
    const float* colors3 = nullptr;
    bool use_sh = false;
    const float* opacities1 = nullptr;
    const float* covariance6 = nullptr;
    const float* scales2 = nullptr;
    float scale_modifier = 1.0f;
    const float* rotations4 = nullptr;
    const float* specular1 = nullptr;
    const float* roughness1 = nullptr;
    float camera_position3[3] = {};
    float camera_rotation9[9] = {};
    float focal_x = 0.0f, focal_y = 0.0f, z_far = 0.0f, z_near = 0.0f;
    float background3[3] = {};
    uint64_t initial_pair_capacity = 1;
    float* output_color3 = nullptr;
    float* output_other2 = nullptr;
    float* output_depth1 = nullptr;
    float* output_alpha1 = nullptr;
    float* output_normal3 = nullptr;
    float* output_median_depth1 = nullptr;
    float* output_distortion1 = nullptr;
    int32_t* output_num_rendered = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t row_begin = 0, row_end = UINT32_MAX;
};

// Arguments of one standard raster call, as in hs_rasterizer_forward_f32_v1,
// with the same tile-row restriction.
struct StandardCall {
    int32_t point_count = 0;
    const float* background5 = nullptr;
    int32_t width = 0, height = 0;
    const float* means3d = nullptr;
    const float* colors5 = nullptr;
    const float* opacities = nullptr;
    const float* scales2 = nullptr;
    float scale_modifier = 1.0f;
    const float* rotations4 = nullptr;
    const float* viewmatrix4x4 = nullptr;
    const float* projmatrix4x4 = nullptr;
    const float* camera_position3 = nullptr;
    float tan_fovx = 0.0f, tan_fovy = 0.0f;
    bool prefiltered = false;
    float* output_color5 = nullptr;
    float* output_aux7 = nullptr;
    float* output_weight = nullptr;
    int32_t* output_radii = nullptr;
    int32_t* output_rendered = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t row_begin = 0, row_end = UINT32_MAX;
    // Non-zero: the call is being captured into a graph and never waits on
    // the host. Its binning is sized for pair_capacity pairs (the context's
    // pair buffers must hold them: standard_reserve_pairs); emission, tile
    // sort and ranges read the pair count from device memory and stop at the
    // capacity. Nothing is published to the host and finish() is not run:
    // the capturer publishes the totals (view_status_kernel) and checks them
    // after every replay.
    uint32_t pair_capacity = 0;
};

// FlashGS forward (flashgs.cu) on call.stream.
cudaError_t flashgs_forward(HsRasterizerContext* context, const FlashgsCall& call);

// Independent FlashGS calls, one context each (distinct contexts), run
// concurrently on the contexts' side streams: all preprocess and binning
// stages are queued before any tile renderer, and `stream` (the caller's)
// is ordered before and after all of them. Each call's stream field is
// ignored. Outputs are identical to flashgs_forward of each call.
// raster_begin, when given, is recorded once all binning is done, before the
// tile renderers.
cudaError_t flashgs_forward_many(HsRasterizerContext* const* contexts, const FlashgsCall* calls,
                                 uint32_t count, cudaStream_t stream, cudaEvent_t raster_begin = nullptr);

cudaError_t flashgs_debug_copy(HsRasterizerContext* context, uint64_t point_capacity,
                               uint64_t pair_capacity, uint64_t tile_capacity,
                               float* points_xy2, float* rgb3, float* other2,
                               float* conic_opacity4, float* normal_opacity4, float* tu3,
                               float* tv3, float* tw3, uint64_t* sorted_keys,
                               uint32_t* sorted_values, int32_t* tile_ranges2);

// Synchronous copy of the last standard forward's per-Gaussian blend state
// (centre, Tu|Tv|Tw, normal|opacity) to host buffers. Entries of Gaussians
// with radius 0 are unspecified.
cudaError_t standard_debug_copy(HsRasterizerContext* context, uint64_t point_capacity,
                                float* points_xy2, float* transmats9, float* normal_opacity4);

// Standard five-channel forward (standard.cu) on call.stream.
cudaError_t standard_forward(HsRasterizerContext* context, const StandardCall& call);

// Independent standard calls run as flashgs_forward_many runs FlashGS calls.
// With finish false (captured calls, pair_capacity set) the calls are queued
// and joined to `stream` without the host reading their wait status.
cudaError_t standard_forward_many(HsRasterizerContext* const* contexts,
                                  const StandardCall* calls, uint32_t count,
                                  cudaStream_t stream, cudaEvent_t raster_begin = nullptr,
                                  bool finish = true);

// Publishes the totals and wait status of captured standard calls (one per
// context, 1 or 2, each of point_counts[i] > 0 Gaussians) to the contexts'
// mapped totals blocks, on `stream`: the host reads them after a replay.
cudaError_t standard_view_status(HsRasterizerContext* const* contexts, const uint64_t* point_counts,
                                 uint32_t count, cudaStream_t stream);

// The most pairs one standard call sorts (the radix sort's 30-bit counts).
constexpr uint32_t kMaxStandardPairs = (1u << 30) - 1u;

// Records a standard call's pair count (last and recent counts).
inline void note_standard_pairs(HsRasterizerContext* ctx, uint32_t pairs) {
    ctx->std_last_emitted = pairs;
    ctx->std_recent_emitted[ctx->std_recent_next++ % 16] = pairs;
}

// The largest pair count of the context's last 16 standard calls.
inline uint32_t recent_standard_pairs(const HsRasterizerContext* ctx) {
    uint32_t most = 0;
    for (uint32_t v : ctx->std_recent_emitted) most = v > most ? v : most;
    return most;
}

// Pairs the context's standard pair buffers hold (0 before the first call).
uint32_t standard_pair_capacity(const HsRasterizerContext* context);
// Grows the standard pair buffers to hold at least `pairs` pairs.
cudaError_t standard_reserve_pairs(HsRasterizerContext* context, uint64_t pairs);

// Arguments of one hs_optix_trace_f32_v1 call (device pointers; checked by
// the entry point).
struct TraceCall {
    uint64_t ray_count = 0;
    const float* ray_origins3 = nullptr;
    const float* ray_directions3 = nullptr;
    const float* background3 = nullptr;
    const float* means3d = nullptr;
    const float* shs_m3 = nullptr;
    uint32_t coefficient_count = 0;
    uint32_t degree = 0;
    const float* others2 = nullptr;
    const float* opacities = nullptr;
    const float* scales2 = nullptr;
    float scale_modifier = 1.0f;
    const float* rotations4 = nullptr;
    const float* viewmatrix4x4 = nullptr;
    const float* projmatrix4x4 = nullptr;
    const float* camera_position3 = nullptr;
    int32_t start_from_first = 0;
    int32_t max_trace_depth = 0;
    float specular_threshold = 0.0f;
    int32_t use_others = 0;
    float* output_rgb3 = nullptr;
    float* output_depth1 = nullptr;
    float* output_acc1 = nullptr;
    float* output_normal3 = nullptr;
    float* output_dist1 = nullptr;
    float* output_aux2 = nullptr;
    float* output_mid32 = nullptr;
    float* output_wet1 = nullptr;
    cudaStream_t stream = nullptr;
};

// Builds the trace scene (BVH) of `triangle_count` triangles over
// `vertex_count` vertices (trace.cu); *bad_index is set (and
// cudaErrorInvalidValue returned) when a triangle names a vertex outside the
// vertex range. Synchronous.
cudaError_t trace_build_scene(HsRasterizerContext* context, const float* vertices3, uint64_t vertex_count,
                              const int32_t* triangles3, uint64_t triangle_count, bool* bad_index);
// Traces call.ray_count rays against the built scene on call.stream.
cudaError_t trace_rays(HsRasterizerContext* context, const TraceCall& call);
cudaError_t trace_release(HsRasterizerContext* context);
uint64_t trace_current_bytes(const HsRasterizerContext* context);

// FlashGS host-side camera matrices (preprocess.cu:599-627), column-major.
void flashgs_camera_matrices(const float position[3], const float rotation9[9], int width,
                             int height, float focal_x, float focal_y, float z_far,
                             float z_near, float view[16], float proj[16]);

}  // namespace hs
