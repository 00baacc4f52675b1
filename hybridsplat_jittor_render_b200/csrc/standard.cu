// Standard five-channel 2DGS forward for sm_100a.
//
// Pipeline (reference full_rasterizer.cu:203-394):
//   preprocess  one thread per Gaussian: near cull, 2DGS transform, facing
//               flip, screen-space AABB and tile rectangle (radii[P]); writes
//               an 80-byte blend record and a 48-byte cull shape (the region
//               where the Gaussian can reach alpha >= 1/255); counts the
//               reference's pairs (`rendered`) and the pairs it will emit.
//               One 12-byte readback of those totals replaces the reference's
//               D2H copy of num_rendered (full_rasterizer.cu:309-320); the
//               host waits for it while the depth sort runs.
//   depth sort  stable onesweep radix sort by the depth bits (ties keep
//               index order).
//   scan+emit   one kernel: exclusive scan of the emitted counts in depth
//               order and warp-cooperative emission of (tile, index | quadrant
//               mask) pairs.
//   tile sort   stable radix sort by tile id: per tile, the Gaussians keep the
//               reference's (depth key, index) order (full_rasterizer.cu:
//               127-153, 345-355).
//   ranges      per-tile [start, end).
//   render      128 threads per 16x16 tile, one warp per 8x8 quadrant, two
//               pixels per lane, per-pixel termination as in
//               forward.cu:323-422; pairs whose quadrant bit is clear are
//               skipped (they cannot reach alpha >= 1/255 there).
#include <algorithm>
#include <climits>

#include "context.h"

// Rounding policy of the kernels: the pinned forms that reproduce the
// reference build. Diagnostic builds may define this to a runtime table.
#ifndef HS_STANDARD_ROUNDING
#define HS_STANDARD_ROUNDING PinnedRounding
#endif
#include "sort.cuh"
#include "standard_kernels.cuh"

namespace hs {
namespace st {
namespace {

uint64_t geometry_bytes(uint64_t count) {
    Carver c(nullptr);
    c.take<float4>(count * kRecordQuads);
    c.take<float4>(count * kCullQuads);
    for (int k = 0; k < 5; ++k) c.take<uint32_t>(count);
    c.take<uint32_t>(64);
    return c.offset;
}

struct GeometryViews {
    float4* records;
    float4* cull;
    uint32_t* keys;
    uint32_t* order;
    uint32_t* counts;
    uint32_t* alt_keys;
    uint32_t* alt_order;
    uint32_t* totals;  // [0] reference pairs, [1] prefiltered violation, [2] emitted pairs, [3] errors
};

GeometryViews geometry_views(void* base, uint64_t count) {
    Carver c(base);
    GeometryViews v;
    v.records = c.take<float4>(count * kRecordQuads);
    v.cull = c.take<float4>(count * kCullQuads);
    v.keys = c.take<uint32_t>(count);
    v.order = c.take<uint32_t>(count);
    v.counts = c.take<uint32_t>(count);
    v.alt_keys = c.take<uint32_t>(count);
    v.alt_order = c.take<uint32_t>(count);
    v.totals = c.take<uint32_t>(64);
    return v;
}

uint64_t binning_bytes(uint64_t pairs) {
    Carver c(nullptr);
    for (int k = 0; k < 4; ++k) c.take<uint32_t>(pairs);
    c.offset += sort::sort_scratch_bytes(static_cast<uint32_t>(pairs > 0 ? pairs : 1)) + 256;
    return c.offset;
}

}  // namespace
}  // namespace st

uint64_t standard_current_bytes(const HsRasterizerContext* ctx) {
    return ctx->std_geometry.bytes + ctx->std_binning.bytes + ctx->std_image.bytes;
}

// Returned when prefiltered is set and a Gaussian fails the near cull; the
// reference traps the device in that case (auxiliary.h:218-224), this
// library reports the violation instead.
constexpr cudaError_t kPrefilteredViolation = cudaErrorInvalidValue;

cudaError_t standard_release(HsRasterizerContext* ctx) {
    cudaError_t first = cudaSuccess;
    for (DeviceBuffer* b : {&ctx->std_geometry, &ctx->std_binning, &ctx->std_image}) {
        const cudaError_t e = release_buffer(*b);
        if (first == cudaSuccess) first = e;
    }
    if (ctx->std_total_host != nullptr) {
        const cudaError_t e = cudaFreeHost(ctx->std_total_host);
        if (first == cudaSuccess) first = e;
        ctx->std_total_host = nullptr;
    }
    return first;
}

cudaError_t standard_forward(HsRasterizerContext* ctx, int32_t point_count,
                             const float* background5, int32_t width, int32_t height,
                             const float* means3d, const float* colors5, const float* opacities,
                             const float* scales2, float scale_modifier, const float* rotations4,
                             const float* viewmatrix4x4, const float* projmatrix4x4,
                             const float* camera_position3, float tan_fovx, float tan_fovy,
                             bool prefiltered, float* output_color5, float* output_aux7,
                             float* output_weight, int32_t* output_radii,
                             int32_t* output_rendered, cudaStream_t stream, uint32_t row_begin,
                             uint32_t row_end) {
    using namespace st;
    // Only the matrices drive the 2DGS projection; the camera position and
    // field of view are accepted for ABI compatibility (the reference passes
    // them through without using them when colours are precomputed).
    (void)camera_position3;
    (void)tan_fovx;
    (void)tan_fovy;
    const uint64_t pixels = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
    const uint32_t grid_x = static_cast<uint32_t>((width + 15) / 16);
    const uint32_t grid_y = static_cast<uint32_t>((height + 15) / 16);
    row_end = std::min(row_end, grid_y);
    if (row_begin >= row_end) return cudaErrorInvalidValue;
    const bool full_frame = row_begin == 0 && row_end == grid_y;
    if (point_count == 0) {
        // zero_outputs (full_rasterizer.cu:178-199) and nothing else.
        cudaError_t st = cudaMemsetAsync(output_rendered, 0, sizeof(int32_t), stream);
        if (full_frame) {
            if (st == cudaSuccess) st = cudaMemsetAsync(output_color5, 0, 5 * pixels * sizeof(float), stream);
            if (st == cudaSuccess) st = cudaMemsetAsync(output_aux7, 0, 7 * pixels * sizeof(float), stream);
            return st;
        }
        const uint64_t y0 = uint64_t(row_begin) * 16, y1 = std::min<uint64_t>(uint64_t(row_end) * 16, height);
        for (int c = 0; c < 12 && st == cudaSuccess; ++c) {
            float* plane = c < 5 ? output_color5 + c * pixels : output_aux7 + (c - 5) * pixels;
            st = cudaMemsetAsync(plane + y0 * width, 0, (y1 - y0) * width * sizeof(float), stream);
        }
        return st;
    }
    const uint64_t tiles = static_cast<uint64_t>(grid_x) * grid_y;
    const uint64_t count = static_cast<uint64_t>(point_count);
    StageMarks marks(ctx->timer, stream);

    // Geometry: per-Gaussian views followed by the depth-sort / scan scratch.
    const uint64_t geometry_used = geometry_bytes(count);
    const uint64_t geometry_scratch_bytes =
        std::max(sort::sort_scratch_bytes(point_count), bin::scan_scratch_bytes(point_count));
    cudaError_t st = ensure_buffer(ctx->std_geometry, geometry_used + geometry_scratch_bytes,
                                   &ctx->std_growth_count, true);
    if (st != cudaSuccess) return st;
    // image buffer: ranges, rasterisation order of the tiles, work counter
    st = ensure_buffer(ctx->std_image, tiles * (sizeof(uint2) + sizeof(uint32_t)) + 256,
                       &ctx->std_growth_count, true);
    if (st != cudaSuccess) return st;
    if (ctx->std_total_host == nullptr) {
        st = cudaHostAlloc(reinterpret_cast<void**>(&ctx->std_total_host), 4 * sizeof(uint32_t),
                           cudaHostAllocPortable);
        if (st != cudaSuccess) return st;
    }
    st = ensure_device_error(ctx);
    if (st != cudaSuccess) return st;
    if (ctx->std_count_event == nullptr) {
        st = cudaEventCreateWithFlags(&ctx->std_count_event, cudaEventDisableTiming);
        if (st != cudaSuccess) return st;
    }
    ctx->std_peak_bytes = std::max(ctx->std_peak_bytes, standard_current_bytes(ctx));
    const GeometryViews gv = geometry_views(ctx->std_geometry.ptr, count);
    void* geometry_scratch = static_cast<unsigned char*>(ctx->std_geometry.ptr) + geometry_used;
    uint2* ranges = static_cast<uint2*>(ctx->std_image.ptr);
    uint32_t* tile_order = reinterpret_cast<uint32_t*>(ranges + tiles);
    uint32_t* work_counter = tile_order + tiles;

    st = cudaMemsetAsync(output_weight, 0, count * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(gv.totals, 0, 4 * sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(ranges, 0, tiles * sizeof(uint2), stream);
    if (st != cudaSuccess) return st;
    const int blocks = (point_count + kPreThreads - 1) / kPreThreads;
    PreprocessOut po{gv.records, gv.cull, gv.keys, gv.order, gv.counts, output_radii, gv.totals,
                     ctx->device_error};
    preprocess_kernel<HS_STANDARD_ROUNDING><<<blocks, kPreThreads, 0, stream>>>(
        point_count, viewmatrix4x4, projmatrix4x4, width, height, grid_x, grid_y, means3d,
        colors5, opacities, scales2, scale_modifier, rotations4, prefiltered ? 1 : 0, row_begin,
        row_end, po);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    st = cudaMemcpyAsync(ctx->std_total_host, gv.totals, 4 * sizeof(uint32_t),
                         cudaMemcpyDeviceToHost, stream);
    if (st == cudaSuccess) st = cudaEventRecord(ctx->std_count_event, stream);
    if (st != cudaSuccess) return st;
    marks.mark(1);
    // The depth sort does not depend on the totals: queue it before waiting.
    st = sort::sort_pairs(gv.keys, gv.order, gv.alt_keys, gv.alt_order, point_count, 0, 32,
                          geometry_scratch, stream, ctx->device_error);
    if (st != cudaSuccess) return st;
    st = cudaEventSynchronize(ctx->std_count_event);
    if (st != cudaSuccess) return st;
    const uint32_t rendered = ctx->std_total_host[0];
    const uint32_t emitted = ctx->std_total_host[2];
    if (ctx->std_total_host[3] != 0) return cudaErrorLaunchTimeout;  // a look-back wait gave up
    if (ctx->std_total_host[1] != 0) return kPrefilteredViolation;
    if (rendered > static_cast<uint32_t>(INT_MAX) || emitted > sort::kMaxItems) {
        return cudaErrorInvalidValue;
    }
    st = cudaMemcpyAsync(output_rendered, gv.totals, sizeof(int32_t), cudaMemcpyDeviceToDevice,
                         stream);
    if (st != cudaSuccess) return st;

    const bool masked = count <= static_cast<uint64_t>(kIndexMask) + 1u;
    uint32_t* values = nullptr;
    if (emitted > 0) {
        st = ensure_buffer(ctx->std_binning, binning_bytes(emitted), &ctx->std_growth_count, true);
        if (st != cudaSuccess) return st;
        ctx->std_peak_bytes = std::max(ctx->std_peak_bytes, standard_current_bytes(ctx));
        Carver c(ctx->std_binning.ptr);
        uint32_t* tile_ids = c.take<uint32_t>(emitted);
        values = c.take<uint32_t>(emitted);
        uint32_t* alt_tiles = c.take<uint32_t>(emitted);
        uint32_t* alt_values = c.take<uint32_t>(emitted);
        void* scratch = c.take<unsigned char>(sort::sort_scratch_bytes(emitted));
        st = cudaMemsetAsync(geometry_scratch, 0, bin::scan_scratch_bytes(point_count), stream);
        if (st != cudaSuccess) return st;
        // alt_keys is free once the depth sort has finished: it receives the
        // first pair slot of every Gaussian.
        uint32_t* first_pair = gv.alt_keys;
        bin::offsets_kernel<<<bin::scan_tiles(point_count), bin::kScanThreads, 0, stream>>>(
            static_cast<uint32_t>(point_count), gv.order, gv.counts,
            static_cast<uint32_t*>(geometry_scratch), ctx->device_error, first_pair);
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
        const Emitter em{gv.cull, grid_x, masked};
        bin::emit_flat_kernel<Emitter>
            <<<(point_count + bin::kEmitThreads - 1) / bin::kEmitThreads, bin::kEmitThreads, 0,
               stream>>>(static_cast<uint32_t>(point_count), gv.counts, first_pair, em, tile_ids,
                         values);
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
        st = sort::sort_pairs(tile_ids, values, alt_tiles, alt_values, emitted, 0,
                              sort::bits_for_tiles(static_cast<uint32_t>(tiles)), scratch, stream,
                              ctx->device_error);
        if (st != cudaSuccess) return st;
        bin::ranges_kernel<uint2><<<(emitted + 255) / 256, 256, 0, stream>>>(
            emitted, static_cast<uint32_t>(tiles), tile_ids, ranges);
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
    }
    const uint32_t strip_tiles = (row_end - row_begin) * grid_x;
    bin::tile_order_kernel<uint2><<<1, bin::kOrderThreads, 0, stream>>>(
        row_begin * grid_x, strip_tiles, ranges, tile_order, work_counter);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    marks.mark(2);
    const uint32_t items = strip_tiles * 4u;
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
    if (masked) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, render_kernel<HS_STANDARD_ROUNDING, true>, kRenderThreads, 0);
    } else {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, render_kernel<HS_STANDARD_ROUNDING, false>, kRenderThreads, 0);
    }
    const uint32_t wanted = (items + kRenderThreads / 32 - 1) / (kRenderThreads / 32);
    const uint32_t render_blocks =
        std::min<uint32_t>(wanted, static_cast<uint32_t>(sms * std::max(per_sm, 1)));
    if (masked) {
        render_kernel<HS_STANDARD_ROUNDING, true><<<render_blocks, kRenderThreads, 0, stream>>>(
            ranges, tile_order, items, work_counter, values, gv.records, width, height, grid_x,
            background5, output_color5, output_aux7, output_weight);
    } else {
        render_kernel<HS_STANDARD_ROUNDING, false><<<render_blocks, kRenderThreads, 0, stream>>>(
            ranges, tile_order, items, work_counter, values, gv.records, width, height, grid_x,
            background5, output_color5, output_aux7, output_weight);
    }
    return cudaGetLastError();
}

}  // namespace hs
