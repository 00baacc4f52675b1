// Deterministic FlashGS forward for sm_100a.
//
// Pipeline for one view (reference flashgs_backend.cu:339-607):
//   1. preprocess   one thread per Gaussian: projection, EWA conic, SH colour,
//                   2DGS transform, exact tile/ellipse test count. Writes a
//                   96-byte blend record, a 32-byte emit record, the depth key
//                   and the pair count (preprocess.cu:364-597).
//   2. depth sort   stable radix sort of the visible Gaussians by the IEEE bits
//                   of view-space depth (ties keep Gaussian index order).
//   3. offsets      exclusive scan of pair counts in depth order; the total is
//                   the reference's num_rendered. One 4-byte readback sizes the
//                   pair buffers (the reference reads its atomic counter back
//                   at the same point, flashgs_backend.cu:480-488).
//   4. emit         each visible Gaussian writes its (tile, index) pairs at its
//                   offset, in depth order.
//   5. tile sort    stable radix sort of the pairs by tile id. Because step 4
//                   wrote pairs in (depth, index) order, the result is exactly
//                   the reference's lexicographic (tile|depth key, index) order
//                   produced by its two CUB sorts (sort.cu:160-189).
//   6. ranges       per-tile [start, end) (render.cu:46-68).
//   7. render       one 128-thread block per 16x16 tile, 2 pixels per thread,
//                   32-Gaussian batches staged in shared memory; tile-wide
//                   termination reproduces render.cu:499-698 exactly (see
//                   render_kernel). Writes the channel-first outputs directly,
//                   replacing the HWC workspace + pack_channels pass.
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>

#include "context.h"

// Rounding policy of the kernels: the pinned forms that reproduce the
// reference build. Diagnostic builds may define this to a runtime table.
#ifndef HS_FLASHGS_ROUNDING
#define HS_FLASHGS_ROUNDING PinnedRounding
#endif
#include "flashgs_kernels.cuh"
#include "sort.cuh"

namespace hs {
namespace fg {
namespace {

uint64_t gaussian_bytes(uint64_t count) {
    Carver c(nullptr);
    c.take<float4>(count * kRecordQuads);
    c.take<float4>(count * kEmitQuads);
    for (int k = 0; k < 6; ++k) c.take<uint32_t>(count);  // keys, order, counts, alt x2, offsets
    c.take<uint32_t>(64);                                  // device total
    return c.offset;
}

struct GaussianViews {
    float4* records;
    float4* emit;
    uint32_t* keys;
    uint32_t* order;
    uint32_t* counts;
    uint32_t* alt_keys;
    uint32_t* alt_order;
    uint32_t* offsets;
    uint32_t* total;
};

GaussianViews gaussian_views(void* base, uint64_t count) {
    Carver c(base);
    GaussianViews v;
    v.records = c.take<float4>(count * kRecordQuads);
    v.emit = c.take<float4>(count * kEmitQuads);
    v.keys = c.take<uint32_t>(count);
    v.order = c.take<uint32_t>(count);
    v.counts = c.take<uint32_t>(count);
    v.alt_keys = c.take<uint32_t>(count);
    v.alt_order = c.take<uint32_t>(count);
    v.offsets = c.take<uint32_t>(count);
    v.total = c.take<uint32_t>(64);
    return v;
}

uint64_t pair_bytes(uint64_t capacity) {
    Carver c(nullptr);
    for (int k = 0; k < 4; ++k) c.take<uint32_t>(capacity);
    return c.offset;
}

struct PairViews {
    uint32_t* tiles;
    uint32_t* ids;
    uint32_t* alt_tiles;
    uint32_t* alt_ids;
};

PairViews pair_views(void* base, uint64_t capacity) {
    Carver c(base);
    PairViews v;
    v.tiles = c.take<uint32_t>(capacity);
    v.ids = c.take<uint32_t>(capacity);
    v.alt_tiles = c.take<uint32_t>(capacity);
    v.alt_ids = c.take<uint32_t>(capacity);
    return v;
}

void update_peak(HsRasterizerContext* ctx) {
    ctx->fg_peak_bytes = std::max(ctx->fg_peak_bytes, flashgs_current_bytes(ctx));
}

}  // namespace
}  // namespace fg

uint64_t flashgs_current_bytes(const HsRasterizerContext* ctx) {
    return ctx->fg_gaussian.bytes + ctx->fg_pairs.bytes + ctx->fg_sort.bytes +
           ctx->fg_ranges.bytes + (ctx->fg_total_host != nullptr ? sizeof(uint32_t) : 0);
}

cudaError_t flashgs_release(HsRasterizerContext* ctx) {
    cudaError_t first = cudaSuccess;
    for (DeviceBuffer* b : {&ctx->fg_gaussian, &ctx->fg_pairs, &ctx->fg_sort, &ctx->fg_ranges}) {
        const cudaError_t e = release_buffer(*b);
        if (first == cudaSuccess) first = e;
    }
    if (ctx->fg_total_host != nullptr) {
        const cudaError_t e = cudaFreeHost(ctx->fg_total_host);
        if (first == cudaSuccess) first = e;
        ctx->fg_total_host = nullptr;
    }
    ctx->fg_gaussian_capacity = 0;
    ctx->fg_pair_capacity = 0;
    ctx->fg_range_capacity = 0;
    return first;
}

cudaError_t flashgs_forward(HsRasterizerContext* ctx, int32_t point_count, int32_t width,
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
                            cudaStream_t stream, uint32_t row_begin, uint32_t row_end) {
    using namespace fg;
    const int grid_x = (width + 15) / 16, grid_y = (height + 15) / 16;
    const uint64_t tiles = static_cast<uint64_t>(grid_x) * grid_y;
    row_end = std::min(row_end, static_cast<uint32_t>(grid_y));
    if (row_begin >= row_end) return cudaErrorInvalidValue;

    Camera cam;
    flashgs_camera_matrices(camera_position3, camera_rotation9, width, height, focal_x, focal_y,
                            z_far, z_near, cam.view, cam.proj);
    for (int k = 0; k < 3; ++k) cam.campos[k] = camera_position3[k];
    cam.tan_fovx = static_cast<float>(width) / (2.0f * focal_x);
    cam.tan_fovy = static_cast<float>(height) / (2.0f * focal_y);
    cam.focal_x = focal_x;
    cam.focal_y = focal_y;
    cam.width = width;
    cam.height = height;
    cam.grid_x = grid_x;
    cam.grid_y = grid_y;

    StageMarks marks(ctx->timer, stream);
    // ranges, rasterisation order of the tiles, work counter
    cudaError_t st = ensure_buffer(ctx->fg_ranges, tiles * (sizeof(int2) + sizeof(uint32_t)) + 256,
                                   &ctx->fg_growth_count);
    if (st != cudaSuccess) return st;
    ctx->fg_range_capacity = std::max<uint64_t>(ctx->fg_range_capacity, tiles);
    int2* ranges = static_cast<int2*>(ctx->fg_ranges.ptr);
    uint32_t* tile_order = reinterpret_cast<uint32_t*>(ranges + tiles);
    uint32_t* work_counter = tile_order + tiles;
    st = cudaMemsetAsync(ranges, 0, tiles * sizeof(int2), stream);
    if (st != cudaSuccess) return st;

    uint32_t num_rendered = 0;
    GaussianViews gv{};
    if (point_count > 0) {
        if (ctx->fg_total_host == nullptr) {
            st = cudaHostAlloc(reinterpret_cast<void**>(&ctx->fg_total_host), 4 * sizeof(uint32_t),
                               cudaHostAllocPortable);
            if (st != cudaSuccess) return st;
            ++ctx->fg_growth_count;
        }
        st = ensure_device_error(ctx);
        if (st != cudaSuccess) return st;
        if (ctx->fg_count_event == nullptr) {
            st = cudaEventCreateWithFlags(&ctx->fg_count_event, cudaEventDisableTiming);
            if (st != cudaSuccess) return st;
        }
        const uint64_t count = static_cast<uint64_t>(point_count);
        if (count > ctx->fg_gaussian_capacity || ctx->fg_gaussian.ptr == nullptr) {
            st = ensure_buffer(ctx->fg_gaussian, gaussian_bytes(count), &ctx->fg_growth_count);
            if (st != cudaSuccess) return st;
            ctx->fg_gaussian_capacity = count;
        }
        gv = gaussian_views(ctx->fg_gaussian.ptr, ctx->fg_gaussian_capacity);
        const uint64_t sort_need = std::max(sort::sort_scratch_bytes(point_count),
                                            bin::scan_scratch_bytes(point_count));
        st = ensure_buffer(ctx->fg_sort, sort_need, &ctx->fg_growth_count);
        if (st != cudaSuccess) return st;
        st = cudaMemsetAsync(gv.total, 0, 4 * sizeof(uint32_t), stream);
        if (st != cudaSuccess) return st;

        const int blocks = (point_count + kPreThreads - 1) / kPreThreads;
        preprocess_kernel<HS_FLASHGS_ROUNDING><<<blocks, kPreThreads, 0, stream>>>(
            point_count, cam, positions3, shs48, colors3, use_sh ? 1 : 0, opacities1,
            covariance6, scales2, scale_modifier, rotations4, specular1, roughness1, gv.records,
            gv.emit, gv.keys, gv.order, gv.counts, gv.total, ctx->device_error,
            static_cast<int>(row_begin), static_cast<int>(row_end));
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
        st = cudaMemcpyAsync(ctx->fg_total_host, gv.total, 4 * sizeof(uint32_t),
                             cudaMemcpyDeviceToHost, stream);
        if (st == cudaSuccess) st = cudaEventRecord(ctx->fg_count_event, stream);
        if (st != cudaSuccess) return st;
        marks.mark(1);
        // The depth sort does not depend on the pair count: queue it, then
        // wait for the count (the reference reads its counter back here,
        // flashgs_backend.cu:480-488).
        st = sort::sort_pairs(gv.keys, gv.order, gv.alt_keys, gv.alt_order, point_count, 0, 32,
                              ctx->fg_sort.ptr, stream, ctx->device_error);
        if (st != cudaSuccess) return st;
        st = cudaEventSynchronize(ctx->fg_count_event);
        if (st != cudaSuccess) return st;
        num_rendered = ctx->fg_total_host[0];
        if (ctx->fg_total_host[1] != 0) return cudaErrorLaunchTimeout;  // a look-back wait gave up
        if (num_rendered > static_cast<uint32_t>(INT_MAX) || num_rendered > sort::kMaxItems) {
            return cudaErrorInvalidValue;
        }

        // Pair capacity follows the reference's growth rule: start at the
        // caller's initial capacity and, whenever the pair count reaches it,
        // grow to max(count + 1, 1.25 x capacity) (flashgs_backend.cu:415-500).
        if (ctx->fg_pair_capacity == 0) {
            ctx->fg_pair_capacity = std::max<uint64_t>(initial_pair_capacity, 1);
        }
        if (num_rendered >= ctx->fg_pair_capacity) {
            ctx->fg_pair_capacity = std::max<uint64_t>(
                static_cast<uint64_t>(num_rendered) + 1,
                ctx->fg_pair_capacity + ctx->fg_pair_capacity / 4);
            ++ctx->fg_overflow_retry_count;
        }
        if (ctx->fg_pair_capacity > static_cast<uint64_t>(INT_MAX)) return cudaErrorInvalidValue;
        st = ensure_buffer(ctx->fg_pairs, pair_bytes(ctx->fg_pair_capacity), &ctx->fg_growth_count);
        if (st != cudaSuccess) return st;
        if (num_rendered > 0) {
            // sized by the pair capacity, so it grows only when the capacity does
            st = ensure_buffer(ctx->fg_sort,
                               std::max(sort_need, sort::sort_scratch_bytes(static_cast<uint32_t>(
                                                       ctx->fg_pair_capacity))),
                               &ctx->fg_growth_count);
            if (st != cudaSuccess) return st;
            const PairViews pv = pair_views(ctx->fg_pairs.ptr, ctx->fg_pair_capacity);
            st = cudaMemsetAsync(ctx->fg_sort.ptr, 0, bin::scan_scratch_bytes(point_count),
                                 stream);
            if (st != cudaSuccess) return st;
            // alt_keys is free once the depth sort has finished: it receives
            // the first pair slot of every Gaussian.
            uint32_t* first_pair = gv.alt_keys;
            bin::offsets_kernel<<<bin::scan_tiles(point_count), bin::kScanThreads, 0, stream>>>(
                static_cast<uint32_t>(point_count), gv.order, gv.counts,
                static_cast<uint32_t*>(ctx->fg_sort.ptr), ctx->device_error, first_pair);
            st = cudaGetLastError();
            if (st != cudaSuccess) return st;
            const Emitter<HS_FLASHGS_ROUNDING> em{gv.emit, grid_x};
            bin::emit_flat_compact_kernel<Emitter<HS_FLASHGS_ROUNDING>>
                <<<(point_count + bin::kEmitThreads - 1) / bin::kEmitThreads, bin::kEmitThreads, 0,
                   stream>>>(static_cast<uint32_t>(point_count), gv.counts, first_pair, em,
                             pv.tiles, pv.ids);
            st = cudaGetLastError();
            if (st != cudaSuccess) return st;
            st = sort::sort_pairs(pv.tiles, pv.ids, pv.alt_tiles, pv.alt_ids, num_rendered, 0,
                                  sort::bits_for_tiles(static_cast<uint32_t>(tiles)),
                                  ctx->fg_sort.ptr, stream, ctx->device_error);
            if (st != cudaSuccess) return st;
            bin::ranges_kernel<int2><<<(num_rendered + 255) / 256, 256, 0, stream>>>(
                num_rendered, static_cast<uint32_t>(tiles), pv.tiles, ranges);
            st = cudaGetLastError();
            if (st != cudaSuccess) return st;
        }
    }

    Outputs out{output_color3, output_other2, output_depth1, output_alpha1,
                output_normal3, output_median_depth1, output_distortion1};
    const float3 bg = make_float3(background3[0], background3[1], background3[2]);
    auto encode = [](float v) {
        const float c = std::min(std::max(0.0f, v * 255.0f), 255.0f);
        return static_cast<float>(static_cast<unsigned char>(c));
    };
    const float3 bg_encoded = make_float3(encode(bg.x), encode(bg.y), encode(bg.z));
    const uint32_t* ids = nullptr;
    if (num_rendered > 0) ids = pair_views(ctx->fg_pairs.ptr, ctx->fg_pair_capacity).ids;
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    const uint32_t strip_tiles = (row_end - row_begin) * static_cast<uint32_t>(grid_x);
    bin::tile_order_kernel<int2><<<1, bin::kOrderThreads, 0, stream>>>(
        row_begin * static_cast<uint32_t>(grid_x), strip_tiles, ranges, tile_order, work_counter);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    marks.mark(2);
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, render_kernel<HS_FLASHGS_ROUNDING>,
                                                  kRenderThreads, 0);
    const uint32_t render_blocks = static_cast<uint32_t>(
        std::min<uint64_t>(strip_tiles, static_cast<uint64_t>(sms) * std::max(per_sm, 1)));
    render_kernel<HS_FLASHGS_ROUNDING><<<render_blocks, kRenderThreads, 0, stream>>>(
        ranges, tile_order, strip_tiles, work_counter, ids, gv.records, width, height, grid_x, bg,
        bg_encoded, out);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    marks.mark(3);
    if (num_rendered > 0) {
        st = cudaMemcpyAsync(output_num_rendered, gv.total, sizeof(int32_t),
                             cudaMemcpyDeviceToDevice, stream);
    } else {
        st = cudaMemsetAsync(output_num_rendered, 0, sizeof(int32_t), stream);
    }
    if (st != cudaSuccess) return st;

    ++ctx->fg_forward_calls;
    ctx->fg_last_point_count = static_cast<uint64_t>(point_count);
    ctx->fg_last_num_rendered = num_rendered;
    ctx->fg_last_tile_count = tiles;
    ctx->fg_last_width = width;
    ctx->fg_last_height = height;
    update_peak(ctx);
    return cudaSuccess;
}

cudaError_t flashgs_debug_copy(HsRasterizerContext* ctx, uint64_t point_capacity,
                               uint64_t pair_capacity, uint64_t tile_capacity,
                               float* points_xy2, float* rgb3, float* other2,
                               float* conic_opacity4, float* normal_opacity4, float* tu3,
                               float* tv3, float* tw3, uint64_t* sorted_keys,
                               uint32_t* sorted_values, int32_t* tile_ranges2) {
    using namespace fg;
    if (ctx->fg_gaussian.ptr == nullptr || ctx->fg_pairs.ptr == nullptr ||
        ctx->fg_ranges.ptr == nullptr) {
        return cudaErrorInvalidResourceHandle;
    }
    const uint64_t points = ctx->fg_last_point_count;
    const uint64_t pairs = ctx->fg_last_num_rendered;
    const uint64_t tiles = ctx->fg_last_tile_count;
    if (point_capacity < points || pair_capacity < pairs || tile_capacity < tiles ||
        points_xy2 == nullptr || rgb3 == nullptr || other2 == nullptr ||
        conic_opacity4 == nullptr || normal_opacity4 == nullptr || tu3 == nullptr ||
        tv3 == nullptr || tw3 == nullptr || sorted_keys == nullptr || sorted_values == nullptr ||
        tile_ranges2 == nullptr) {
        return cudaErrorInvalidValue;
    }
    cudaError_t st = cudaDeviceSynchronize();
    if (st != cudaSuccess) return st;
    const GaussianViews gv = gaussian_views(ctx->fg_gaussian.ptr, ctx->fg_gaussian_capacity);
    std::vector<float> rec(points * kRecordQuads * 4);
    std::vector<uint32_t> keys(points), order(points);
    if (points > 0) {
        st = cudaMemcpy(rec.data(), gv.records, rec.size() * sizeof(float), cudaMemcpyDeviceToHost);
        if (st == cudaSuccess)
            st = cudaMemcpy(keys.data(), gv.keys, points * 4, cudaMemcpyDeviceToHost);
        if (st == cudaSuccess)
            st = cudaMemcpy(order.data(), gv.order, points * 4, cudaMemcpyDeviceToHost);
        if (st != cudaSuccess) return st;
    }
    std::vector<uint32_t> depth_bits(points, 0);
    for (uint64_t s = 0; s < points; ++s) depth_bits[order[s]] = keys[s];
    for (uint64_t i = 0; i < points; ++i) {
        const float* q = rec.data() + i * kRecordQuads * 4;
        points_xy2[2 * i] = q[0];
        points_xy2[2 * i + 1] = q[1];
        normal_opacity4[4 * i] = q[2];
        normal_opacity4[4 * i + 1] = q[3];
        normal_opacity4[4 * i + 2] = q[4];
        normal_opacity4[4 * i + 3] = q[5];
        rgb3[3 * i] = q[6];
        rgb3[3 * i + 1] = q[7];
        rgb3[3 * i + 2] = q[8];
        other2[2 * i] = q[9];
        other2[2 * i + 1] = q[10];
        tu3[3 * i] = q[11];
        tu3[3 * i + 1] = q[12];
        tu3[3 * i + 2] = q[13];
        tv3[3 * i] = q[14];
        tv3[3 * i + 1] = q[15];
        tv3[3 * i + 2] = q[16];
        tw3[3 * i] = q[17];
        tw3[3 * i + 1] = q[18];
        tw3[3 * i + 2] = q[19];
        conic_opacity4[4 * i] = q[20];
        conic_opacity4[4 * i + 1] = q[21];
        conic_opacity4[4 * i + 2] = q[22];
        conic_opacity4[4 * i + 3] = q[23];
    }
    if (pairs > 0) {
        const PairViews pv = pair_views(ctx->fg_pairs.ptr, ctx->fg_pair_capacity);
        std::vector<uint32_t> tile_ids(pairs);
        st = cudaMemcpy(tile_ids.data(), pv.tiles, pairs * 4, cudaMemcpyDeviceToHost);
        if (st == cudaSuccess)
            st = cudaMemcpy(sorted_values, pv.ids, pairs * 4, cudaMemcpyDeviceToHost);
        if (st != cudaSuccess) return st;
        for (uint64_t i = 0; i < pairs; ++i) {
            sorted_keys[i] = (static_cast<uint64_t>(tile_ids[i]) << 32) |
                             depth_bits[sorted_values[i]];
        }
    }
    if (tiles > 0) {
        st = cudaMemcpy(tile_ranges2, ctx->fg_ranges.ptr, tiles * sizeof(int2),
                        cudaMemcpyDeviceToHost);
    }
    return st;
}

}  // namespace hs
