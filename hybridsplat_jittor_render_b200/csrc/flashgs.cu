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

#include "concurrent.h"
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
        ctx->fg_total_mapped = nullptr;
    }
    ctx->fg_gaussian_capacity = 0;
    ctx->fg_pair_capacity = 0;
    ctx->fg_range_capacity = 0;
    return first;
}

namespace fg {
namespace {

// One FlashGS raster call in the three phases of run_many (concurrent.h).
class FlashgsPass {
public:
    FlashgsPass(HsRasterizerContext* ctx, const FlashgsCall& call) : ctx_(ctx), c_(call) {}
    cudaError_t begin();
    cudaError_t bin();
    cudaError_t render();
    cudaError_t finish();

private:
    HsRasterizerContext* ctx_;
    FlashgsCall c_;
    StageMarks marks_;
    Camera cam_{};
    int grid_x_ = 0, grid_y_ = 0;
    uint64_t tiles_ = 0;
    int2* ranges_ = nullptr;
    uint32_t* tile_order_ = nullptr;
    uint32_t* work_counter_ = nullptr;
    uint32_t num_rendered_ = 0;
    GaussianViews gv_{};
    uint64_t sort_need_ = 0;
    bool published_ = false;  // the error word follows binning (finish() reads it)
};

cudaError_t FlashgsPass::begin() {
    const cudaStream_t stream = c_.stream;
    grid_x_ = (c_.width + 15) / 16;
    grid_y_ = (c_.height + 15) / 16;
    tiles_ = static_cast<uint64_t>(grid_x_) * grid_y_;
    c_.row_end = std::min(c_.row_end, static_cast<uint32_t>(grid_y_));
    if (c_.row_begin >= c_.row_end) return cudaErrorInvalidValue;

    flashgs_camera_matrices(c_.camera_position3, c_.camera_rotation9, c_.width, c_.height,
                            c_.focal_x, c_.focal_y, c_.z_far, c_.z_near, cam_.view, cam_.proj);
    for (int k = 0; k < 3; ++k) cam_.campos[k] = c_.camera_position3[k];
    cam_.tan_fovx = static_cast<float>(c_.width) / (2.0f * c_.focal_x);
    cam_.tan_fovy = static_cast<float>(c_.height) / (2.0f * c_.focal_y);
    cam_.focal_x = c_.focal_x;
    cam_.focal_y = c_.focal_y;
    cam_.width = c_.width;
    cam_.height = c_.height;
    cam_.grid_x = grid_x_;
    cam_.grid_y = grid_y_;

    marks_.start(ctx_->timer, stream);
    // ranges, rasterisation order of the tiles, work counter
    cudaError_t st = ensure_buffer(ctx_->fg_ranges, tiles_ * (sizeof(int2) + sizeof(uint32_t)) + 256,
                                   &ctx_->fg_growth_count);
    if (st != cudaSuccess) return st;
    ctx_->fg_range_capacity = std::max<uint64_t>(ctx_->fg_range_capacity, tiles_);
    ranges_ = static_cast<int2*>(ctx_->fg_ranges.ptr);
    tile_order_ = reinterpret_cast<uint32_t*>(ranges_ + tiles_);
    work_counter_ = tile_order_ + tiles_;
    st = cudaMemsetAsync(ranges_, 0, tiles_ * sizeof(int2), stream);
    if (st != cudaSuccess || c_.point_count == 0) return st;

    if (ctx_->fg_total_host == nullptr) {
        st = bin::alloc_mapped_totals(&ctx_->fg_total_host, &ctx_->fg_total_mapped);
        if (st != cudaSuccess) return st;
        ++ctx_->fg_growth_count;
    }
    st = ensure_device_error(ctx_);
    if (st != cudaSuccess) return st;
    if (ctx_->fg_count_event == nullptr) {
        st = cudaEventCreateWithFlags(&ctx_->fg_count_event, cudaEventDisableTiming);
        if (st != cudaSuccess) return st;
    }
    const uint64_t count = static_cast<uint64_t>(c_.point_count);
    if (count > ctx_->fg_gaussian_capacity || ctx_->fg_gaussian.ptr == nullptr) {
        st = ensure_buffer(ctx_->fg_gaussian, gaussian_bytes(count), &ctx_->fg_growth_count);
        if (st != cudaSuccess) return st;
        ctx_->fg_gaussian_capacity = count;
    }
    gv_ = gaussian_views(ctx_->fg_gaussian.ptr, ctx_->fg_gaussian_capacity);
    sort_need_ = std::max(sort::sort_scratch_bytes(c_.point_count),
                          bin::scan_scratch_bytes(c_.point_count));
    st = ensure_buffer(ctx_->fg_sort, sort_need_, &ctx_->fg_growth_count);
    if (st != cudaSuccess) return st;
    // A wait that gave up in an earlier call must not fail this one.
    st = cudaMemsetAsync(ctx_->device_error, 0, sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(gv_.total, 0, 8 * sizeof(uint32_t), stream);
    if (st != cudaSuccess) return st;

    const int blocks = (c_.point_count + kPreThreads - 1) / kPreThreads;
    preprocess_kernel<HS_FLASHGS_ROUNDING><<<blocks, kPreThreads, 0, stream>>>(
        c_.point_count, cam_, c_.positions3, c_.shs48, c_.colors3, c_.use_sh ? 1 : 0,
        c_.opacities1, c_.covariance6, c_.scales2, c_.scale_modifier, c_.rotations4, c_.specular1,
        c_.roughness1, gv_.records, gv_.emit, gv_.keys, gv_.order, gv_.counts, gv_.total,
        static_cast<int>(c_.row_begin), static_cast<int>(c_.row_end));
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    bin::publish_totals_kernel<<<1, 32, 0, stream>>>(gv_.total, ctx_->fg_total_mapped);
    st = cudaGetLastError();
    if (st == cudaSuccess) st = cudaEventRecord(ctx_->fg_count_event, stream);
    if (st != cudaSuccess) return st;
    marks_.mark(1);
    // The depth sort does not depend on the pair count: queue it, then wait
    // for the count in bin() (the reference reads its counter back at this
    // point, flashgs_backend.cu:480-488).
    const uint32_t stall = ctx_->test_stall_tile;  // test hook, one call only
    ctx_->test_stall_tile = sort::kNoStall;
    // Gaussians without pairs are left out of it (total[4] counts the others).
    return sort::sort_pairs(gv_.keys, gv_.order, gv_.alt_keys, gv_.alt_order, c_.point_count, 0,
                            32, ctx_->fg_sort.ptr, stream, ctx_->device_error, stall, gv_.total + 4);
}

cudaError_t FlashgsPass::bin() {
    const cudaStream_t stream = c_.stream;
    cudaError_t st = cudaSuccess;
    if (c_.point_count > 0) {
        st = cudaEventSynchronize(ctx_->fg_count_event);
        if (st != cudaSuccess) return st;
        num_rendered_ = ctx_->fg_total_host[0];
        if (num_rendered_ > static_cast<uint32_t>(INT_MAX) || num_rendered_ > sort::kMaxItems) {
            return cudaErrorInvalidValue;
        }

        // Pair capacity follows the reference's growth rule: start at the
        // caller's initial capacity and, whenever the pair count reaches it,
        // grow to max(count + 1, 1.25 x capacity) (flashgs_backend.cu:415-500).
        if (ctx_->fg_pair_capacity == 0) {
            ctx_->fg_pair_capacity = std::max<uint64_t>(c_.initial_pair_capacity, 1);
        }
        if (num_rendered_ >= ctx_->fg_pair_capacity) {
            ctx_->fg_pair_capacity = std::max<uint64_t>(
                static_cast<uint64_t>(num_rendered_) + 1,
                ctx_->fg_pair_capacity + ctx_->fg_pair_capacity / 4);
            ++ctx_->fg_overflow_retry_count;
        }
        if (ctx_->fg_pair_capacity > static_cast<uint64_t>(INT_MAX)) return cudaErrorInvalidValue;
        st = ensure_buffer(ctx_->fg_pairs, pair_bytes(ctx_->fg_pair_capacity),
                           &ctx_->fg_growth_count);
        if (st != cudaSuccess) return st;
        if (num_rendered_ > 0) {
            // sized by the pair capacity, so it grows only when the capacity does
            st = ensure_buffer(ctx_->fg_sort,
                               std::max(sort_need_, sort::sort_scratch_bytes(static_cast<uint32_t>(
                                                        ctx_->fg_pair_capacity))),
                               &ctx_->fg_growth_count);
            if (st != cudaSuccess) return st;
            const PairViews pv = pair_views(ctx_->fg_pairs.ptr, ctx_->fg_pair_capacity);
            st = cudaMemsetAsync(ctx_->fg_sort.ptr, 0, bin::scan_scratch_bytes(c_.point_count),
                                 stream);
            if (st != cudaSuccess) return st;
            // alt_keys is free once the depth sort has finished: it receives
            // the first pair slot of every Gaussian.
            uint32_t* first_pair = gv_.alt_keys;
            bin::offsets_kernel<<<bin::scan_tiles(c_.point_count), bin::kScanThreads, 0, stream>>>(
                static_cast<uint32_t>(c_.point_count), gv_.total + 4, gv_.order, gv_.counts,
                static_cast<uint32_t*>(ctx_->fg_sort.ptr), ctx_->device_error, first_pair);
            st = cudaGetLastError();
            if (st != cudaSuccess) return st;
            const Emitter<HS_FLASHGS_ROUNDING> em{gv_.emit, grid_x_};
            bin::emit_flat_compact_kernel<Emitter<HS_FLASHGS_ROUNDING>>
                <<<(c_.point_count + bin::kEmitThreads - 1) / bin::kEmitThreads, bin::kEmitThreads,
                   0, stream>>>(static_cast<uint32_t>(c_.point_count), gv_.counts, first_pair, em,
                                pv.tiles, pv.ids, ctx_->device_error);
            st = cudaGetLastError();
            if (st != cudaSuccess) return st;
            st = sort::sort_pairs(pv.tiles, pv.ids, pv.alt_tiles, pv.alt_ids, num_rendered_, 0,
                                  sort::bits_for_tiles(static_cast<uint32_t>(tiles_)),
                                  ctx_->fg_sort.ptr, stream, ctx_->device_error);
            if (st != cudaSuccess) return st;
            bin::ranges_kernel<int2><<<bin::ranges_grid(num_rendered_), bin::kRangeThreads, 0, stream>>>(
                num_rendered_, static_cast<uint32_t>(tiles_), pv.tiles, ranges_);
            st = cudaGetLastError();
            if (st != cudaSuccess) return st;
        }
    }
    const uint32_t strip_tiles = (c_.row_end - c_.row_begin) * static_cast<uint32_t>(grid_x_);
    // The waits of the depth sort, offset scan and tile sort are over: the
    // tile order kernel also sends their error word to the host (non-empty
    // calls), read by finish().
    bin::tile_order_kernel<int2><<<1, bin::kOrderThreads, 0, stream>>>(
        c_.row_begin * static_cast<uint32_t>(grid_x_), strip_tiles, ranges_, tile_order_,
        work_counter_, ctx_->device_error, c_.point_count > 0 ? ctx_->fg_total_mapped + 1 : nullptr);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    if (c_.point_count > 0) {
        if (st == cudaSuccess) st = cudaEventRecord(ctx_->fg_count_event, stream);
        if (st != cudaSuccess) return st;
        published_ = true;
    }
    marks_.mark(2);
    return cudaSuccess;
}

cudaError_t FlashgsPass::render() {
    const cudaStream_t stream = c_.stream;
    Outputs out{c_.output_color3, c_.output_other2, c_.output_depth1, c_.output_alpha1,
                c_.output_normal3, c_.output_median_depth1, c_.output_distortion1};
    const float3 bg = make_float3(c_.background3[0], c_.background3[1], c_.background3[2]);
    auto encode = [](float v) {
        const float c = std::min(std::max(0.0f, v * 255.0f), 255.0f);
        return static_cast<float>(static_cast<unsigned char>(c));
    };
    const float3 bg_encoded = make_float3(encode(bg.x), encode(bg.y), encode(bg.z));
    const uint32_t* ids = nullptr;
    if (num_rendered_ > 0) ids = pair_views(ctx_->fg_pairs.ptr, ctx_->fg_pair_capacity).ids;
    const uint32_t strip_tiles = (c_.row_end - c_.row_begin) * static_cast<uint32_t>(grid_x_);
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx_->device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, render_kernel<HS_FLASHGS_ROUNDING>,
                                                  kRenderThreads, 0);
    const uint32_t render_blocks = static_cast<uint32_t>(
        std::min<uint64_t>(strip_tiles, static_cast<uint64_t>(sms) * std::max(per_sm, 1)));
    render_kernel<HS_FLASHGS_ROUNDING><<<render_blocks, kRenderThreads, 0, stream>>>(
        ranges_, tile_order_, strip_tiles, work_counter_, ids, gv_.records, c_.width, c_.height,
        grid_x_, bg, bg_encoded, out, published_ ? ctx_->device_error : nullptr);
    cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    marks_.mark(3);
    if (num_rendered_ > 0) {
        st = cudaMemcpyAsync(c_.output_num_rendered, gv_.total, sizeof(int32_t),
                             cudaMemcpyDeviceToDevice, stream);
    } else {
        st = cudaMemsetAsync(c_.output_num_rendered, 0, sizeof(int32_t), stream);
    }
    if (st != cudaSuccess) return st;

    ++ctx_->fg_forward_calls;
    ctx_->fg_last_point_count = static_cast<uint64_t>(c_.point_count);
    ctx_->fg_last_num_rendered = num_rendered_;
    ctx_->fg_last_tile_count = tiles_;
    ctx_->fg_last_width = c_.width;
    ctx_->fg_last_height = c_.height;
    update_peak(ctx_);
    return cudaSuccess;
}

// Fails the call when one of its bounded waits gave up. The host waits for
// the end of binning here, with the renderer already queued behind it.
cudaError_t FlashgsPass::finish() {
    if (!published_) return cudaSuccess;
    const cudaError_t st = cudaEventSynchronize(ctx_->fg_count_event);
    if (st != cudaSuccess) return st;
    return ctx_->fg_total_host[1] != 0 ? kWaitGaveUp : cudaSuccess;
}

}  // namespace
}  // namespace fg

cudaError_t flashgs_forward(HsRasterizerContext* ctx, const FlashgsCall& call) {
    fg::FlashgsPass pass(ctx, call);
    cudaError_t e = pass.begin();
    if (e == cudaSuccess) e = pass.bin();
    if (e == cudaSuccess) e = pass.render();
    if (e == cudaSuccess) e = pass.finish();
    return e;
}

cudaError_t flashgs_forward_many(HsRasterizerContext* const* contexts, const FlashgsCall* calls,
                                 uint32_t count, cudaStream_t stream, cudaEvent_t raster_begin) {
    return run_many<fg::FlashgsPass>(contexts, calls, count, stream, raster_begin);
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
