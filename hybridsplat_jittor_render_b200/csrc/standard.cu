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

#include "concurrent.h"
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
    uint32_t* totals;  // [0] reference pairs, [1] prefiltered violation, [2] emitted pairs,
                       // [4] Gaussians with pairs
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

cudaError_t standard_debug_copy(HsRasterizerContext* ctx, uint64_t point_capacity,
                                float* points_xy2, float* transmats9, float* normal_opacity4) {
    using namespace st;
    const uint64_t points = ctx->std_last_point_count;
    if (points > 0 && ctx->std_geometry.ptr == nullptr) return cudaErrorInvalidResourceHandle;
    if (point_capacity < points || points_xy2 == nullptr || transmats9 == nullptr ||
        normal_opacity4 == nullptr) {
        return cudaErrorInvalidValue;
    }
    cudaError_t st = cudaDeviceSynchronize();
    if (st != cudaSuccess || points == 0) return st;
    std::vector<float> rec(points * kRecordQuads * 4);
    st = cudaMemcpy(rec.data(), geometry_views(ctx->std_geometry.ptr, points).records,
                    rec.size() * sizeof(float), cudaMemcpyDeviceToHost);
    if (st != cudaSuccess) return st;
    // record layout: xy, n.xy | n.z, op, c0, c1 | c2, c3, c4, Tu.x | Tu.yz, Tv.xy | Tv.z, Tw
    for (uint64_t i = 0; i < points; ++i) {
        const float* q = rec.data() + i * kRecordQuads * 4;
        points_xy2[2 * i] = q[0];
        points_xy2[2 * i + 1] = q[1];
        normal_opacity4[4 * i] = q[2];
        normal_opacity4[4 * i + 1] = q[3];
        normal_opacity4[4 * i + 2] = q[4];
        normal_opacity4[4 * i + 3] = q[5];
        float* t = transmats9 + 9 * i;
        t[0] = q[11]; t[1] = q[12]; t[2] = q[13];
        t[3] = q[14]; t[4] = q[15]; t[5] = q[16];
        t[6] = q[17]; t[7] = q[18]; t[8] = q[19];
    }
    return cudaSuccess;
}

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
        ctx->std_total_mapped = nullptr;
    }
    return first;
}

namespace st {
namespace {

// One standard raster call in the three phases of run_many (concurrent.h).
class StandardPass {
public:
    StandardPass(HsRasterizerContext* ctx, const StandardCall& call) : ctx_(ctx), c_(call) {}
    cudaError_t begin();
    cudaError_t bin();
    cudaError_t render();
    cudaError_t finish();

private:
    HsRasterizerContext* ctx_;
    StandardCall c_;
    StageMarks marks_;
    bool done_ = false;  // empty input: begin() wrote the outputs
    uint32_t grid_x_ = 0, grid_y_ = 0;
    uint64_t tiles_ = 0, count_ = 0;
    GeometryViews gv_{};
    void* geometry_scratch_ = nullptr;
    uint2* ranges_ = nullptr;
    uint32_t* tile_order_ = nullptr;
    uint32_t* work_counter_ = nullptr;
    uint32_t* values_ = nullptr;
    bool masked_ = false;
    bool published_ = false;  // the error word follows binning (finish() reads it)
};

cudaError_t StandardPass::begin() {
    // Only the matrices drive the 2DGS projection; the camera position and
    // field of view are accepted for ABI compatibility (the reference passes
    // them through without using them when colours are precomputed).
    const cudaStream_t stream = c_.stream;
    const uint64_t pixels = static_cast<uint64_t>(c_.width) * static_cast<uint64_t>(c_.height);
    grid_x_ = static_cast<uint32_t>((c_.width + 15) / 16);
    grid_y_ = static_cast<uint32_t>((c_.height + 15) / 16);
    c_.row_end = std::min(c_.row_end, grid_y_);
    if (c_.row_begin >= c_.row_end) return cudaErrorInvalidValue;
    const bool full_frame = c_.row_begin == 0 && c_.row_end == grid_y_;
    if (c_.point_count == 0) {
        // zero_outputs (full_rasterizer.cu:178-199) and nothing else.
        done_ = true;
        cudaError_t st = cudaMemsetAsync(c_.output_rendered, 0, sizeof(int32_t), stream);
        if (full_frame) {
            if (st == cudaSuccess)
                st = cudaMemsetAsync(c_.output_color5, 0, 5 * pixels * sizeof(float), stream);
            if (st == cudaSuccess)
                st = cudaMemsetAsync(c_.output_aux7, 0, 7 * pixels * sizeof(float), stream);
            return st;
        }
        const uint64_t y0 = uint64_t(c_.row_begin) * 16;
        const uint64_t y1 = std::min<uint64_t>(uint64_t(c_.row_end) * 16, c_.height);
        for (int c = 0; c < 12 && st == cudaSuccess; ++c) {
            float* plane = c < 5 ? c_.output_color5 + c * pixels : c_.output_aux7 + (c - 5) * pixels;
            st = cudaMemsetAsync(plane + y0 * c_.width, 0, (y1 - y0) * c_.width * sizeof(float), stream);
        }
        return st;
    }
    tiles_ = static_cast<uint64_t>(grid_x_) * grid_y_;
    count_ = static_cast<uint64_t>(c_.point_count);
    marks_.start(ctx_->timer, stream);

    // Geometry: per-Gaussian views followed by the depth-sort / scan scratch.
    const uint64_t geometry_used = geometry_bytes(count_);
    const uint64_t geometry_scratch_bytes =
        std::max(sort::sort_scratch_bytes(c_.point_count), bin::scan_scratch_bytes(c_.point_count));
    cudaError_t st = ensure_buffer(ctx_->std_geometry, geometry_used + geometry_scratch_bytes,
                                   &ctx_->std_growth_count, true);
    if (st != cudaSuccess) return st;
    // image buffer: ranges, rasterisation order of the tiles, work counter
    st = ensure_buffer(ctx_->std_image, tiles_ * (sizeof(uint2) + sizeof(uint32_t)) + 256,
                       &ctx_->std_growth_count, true);
    if (st != cudaSuccess) return st;
    if (ctx_->std_total_host == nullptr) {
        st = bin::alloc_mapped_totals(&ctx_->std_total_host, &ctx_->std_total_mapped);
        if (st != cudaSuccess) return st;
    }
    st = ensure_device_error(ctx_);
    if (st != cudaSuccess) return st;
    if (ctx_->std_count_event == nullptr) {
        st = cudaEventCreateWithFlags(&ctx_->std_count_event, cudaEventDisableTiming);
        if (st != cudaSuccess) return st;
    }
    ctx_->std_peak_bytes = std::max(ctx_->std_peak_bytes, standard_current_bytes(ctx_));
    gv_ = geometry_views(ctx_->std_geometry.ptr, count_);
    ctx_->std_last_point_count = count_;
    geometry_scratch_ = static_cast<unsigned char*>(ctx_->std_geometry.ptr) + geometry_used;
    ranges_ = static_cast<uint2*>(ctx_->std_image.ptr);
    tile_order_ = reinterpret_cast<uint32_t*>(ranges_ + tiles_);
    work_counter_ = tile_order_ + tiles_;

    // A wait that gave up in an earlier call must not fail this one.
    st = cudaMemsetAsync(ctx_->device_error, 0, sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c_.output_weight, 0, count_ * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(gv_.totals, 0, 8 * sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(ranges_, 0, tiles_ * sizeof(uint2), stream);
    if (st != cudaSuccess) return st;
    const int blocks = (c_.point_count + kPreThreads - 1) / kPreThreads;
    PreprocessOut po{gv_.records, gv_.cull, gv_.keys, gv_.order, gv_.counts, c_.output_radii,
                     gv_.totals};
    preprocess_kernel<HS_STANDARD_ROUNDING><<<blocks, kPreThreads, 0, stream>>>(
        c_.point_count, c_.viewmatrix4x4, c_.projmatrix4x4, c_.width, c_.height, grid_x_, grid_y_,
        c_.means3d, c_.colors5, c_.opacities, c_.scales2, c_.scale_modifier, c_.rotations4,
        c_.prefiltered ? 1 : 0, c_.row_begin, c_.row_end, po);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    if (c_.pair_capacity == 0) {
        bin::publish_totals_kernel<<<1, 32, 0, stream>>>(gv_.totals, ctx_->std_total_mapped);
        st = cudaGetLastError();
        if (st == cudaSuccess) st = cudaEventRecord(ctx_->std_count_event, stream);
        if (st != cudaSuccess) return st;
    }
    marks_.mark(1);
    // The depth sort does not depend on the totals: queue it before waiting.
    // It leaves out the Gaussians that emit no pair (totals[4] counts the
    // others, which alone enter the offset scan).
    const uint32_t stall = ctx_->test_stall_tile;  // test hook, one call only
    ctx_->test_stall_tile = sort::kNoStall;
    return sort::sort_pairs(gv_.keys, gv_.order, gv_.alt_keys, gv_.alt_order, c_.point_count, 0, 32,
                            geometry_scratch_, stream, ctx_->device_error, stall, gv_.totals + 4);
}

cudaError_t StandardPass::bin() {
    if (done_) return cudaSuccess;
    const cudaStream_t stream = c_.stream;
    const bool captured = c_.pair_capacity != 0;
    cudaError_t st = cudaSuccess;
    uint32_t emitted = c_.pair_capacity;
    // captured: the pair count stays on the device and bounds the tile sort
    // and the ranges; the buffers are sized for the capacity
    const uint32_t* bound = captured ? gv_.totals + 2 : nullptr;
    if (!captured) {
        st = cudaEventSynchronize(ctx_->std_count_event);
        if (st != cudaSuccess) return st;
        const uint32_t rendered = ctx_->std_total_host[0];
        emitted = ctx_->std_total_host[2];
        if (ctx_->std_total_host[1] != 0) return kPrefilteredViolation;
        if (rendered > static_cast<uint32_t>(INT_MAX) || emitted > sort::kMaxItems) {
            return cudaErrorInvalidValue;
        }
        note_standard_pairs(ctx_, emitted);
    } else if (ctx_->std_binning.bytes < binning_bytes(emitted)) {
        return cudaErrorInvalidValue;  // standard_reserve_pairs first
    }
    st = cudaMemcpyAsync(c_.output_rendered, gv_.totals, sizeof(int32_t), cudaMemcpyDeviceToDevice,
                         stream);
    if (st != cudaSuccess) return st;

    masked_ = count_ <= static_cast<uint64_t>(kIndexMask) + 1u;
    if (emitted > 0) {
        st = ensure_buffer(ctx_->std_binning, binning_bytes(emitted), &ctx_->std_growth_count, true);
        if (st != cudaSuccess) return st;
        ctx_->std_peak_bytes = std::max(ctx_->std_peak_bytes, standard_current_bytes(ctx_));
        Carver c(ctx_->std_binning.ptr);
        uint32_t* tile_ids = c.take<uint32_t>(emitted);
        values_ = c.take<uint32_t>(emitted);
        uint32_t* alt_tiles = c.take<uint32_t>(emitted);
        uint32_t* alt_values = c.take<uint32_t>(emitted);
        void* scratch = c.take<unsigned char>(sort::sort_scratch_bytes(emitted));
        st = cudaMemsetAsync(geometry_scratch_, 0, bin::scan_scratch_bytes(c_.point_count), stream);
        if (st != cudaSuccess) return st;
        // alt_keys is free once the depth sort has finished: it receives the
        // first pair slot of every Gaussian.
        uint32_t* first_pair = gv_.alt_keys;
        bin::offsets_kernel<<<bin::scan_tiles(c_.point_count), bin::kScanThreads, 0, stream>>>(
            static_cast<uint32_t>(c_.point_count), gv_.totals + 4, gv_.order, gv_.counts,
            static_cast<uint32_t*>(geometry_scratch_), ctx_->device_error, first_pair);
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
        emit_rows_kernel<<<(c_.point_count + kEmitRowThreads - 1) / kEmitRowThreads,
                           kEmitRowThreads, 0, stream>>>(
            static_cast<uint32_t>(c_.point_count), gv_.counts, first_pair, gv_.cull, grid_x_,
            masked_ ? 1 : 0, tile_ids, values_, ctx_->device_error, emitted);
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
        st = sort::sort_pairs(tile_ids, values_, alt_tiles, alt_values, emitted, 0,
                              sort::bits_for_tiles(static_cast<uint32_t>(tiles_)), scratch, stream,
                              ctx_->device_error, sort::kNoStall, nullptr, bound);
        if (st != cudaSuccess) return st;
        bin::ranges_kernel<uint2><<<bin::ranges_grid(emitted), bin::kRangeThreads, 0, stream>>>(
            emitted, static_cast<uint32_t>(tiles_), tile_ids, ranges_, bound);
        st = cudaGetLastError();
        if (st != cudaSuccess) return st;
    }
    const uint32_t strip_tiles = (c_.row_end - c_.row_begin) * grid_x_;
    // The waits of the depth sort, offset scan and tile sort are over: the tile
    // order kernel also sends their error word to the host, read by finish()
    // once the renderer is queued.
    bin::tile_order_kernel<uint2><<<1, bin::kOrderThreads, 0, stream>>>(
        c_.row_begin * grid_x_, strip_tiles, ranges_, tile_order_, work_counter_, ctx_->device_error,
        captured ? nullptr : ctx_->std_total_mapped + 3);
    st = cudaGetLastError();
    if (st == cudaSuccess && !captured) st = cudaEventRecord(ctx_->std_count_event, stream);
    if (st != cudaSuccess) return st;
    published_ = !captured;
    marks_.mark(2);
    return cudaSuccess;
}

cudaError_t StandardPass::render() {
    if (done_) return cudaSuccess;
    const uint32_t items = (c_.row_end - c_.row_begin) * grid_x_ * 4u;
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx_->device);
    if (masked_) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, render_kernel<HS_STANDARD_ROUNDING, true>, kRenderThreads, 0);
    } else {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, render_kernel<HS_STANDARD_ROUNDING, false>, kRenderThreads, 0);
    }
    const uint32_t wanted = (items + kRenderThreads / 32 - 1) / (kRenderThreads / 32);
    const uint32_t render_blocks =
        std::min<uint32_t>(wanted, static_cast<uint32_t>(sms * std::max(per_sm, 1)));
    if (masked_) {
        render_kernel<HS_STANDARD_ROUNDING, true><<<render_blocks, kRenderThreads, 0, c_.stream>>>(
            ranges_, tile_order_, items, work_counter_, values_, gv_.records, c_.width, c_.height,
            grid_x_, c_.background5, c_.output_color5, c_.output_aux7, c_.output_weight,
            ctx_->device_error);
    } else {
        render_kernel<HS_STANDARD_ROUNDING, false><<<render_blocks, kRenderThreads, 0, c_.stream>>>(
            ranges_, tile_order_, items, work_counter_, values_, gv_.records, c_.width, c_.height,
            grid_x_, c_.background5, c_.output_color5, c_.output_aux7, c_.output_weight,
            ctx_->device_error);
    }
    const cudaError_t st = cudaGetLastError();
    marks_.mark(3);
    return st;
}

// Fails the call when one of its bounded waits gave up. The host waits for
// the end of binning here, with the renderer already queued behind it.
cudaError_t StandardPass::finish() {
    if (!published_) return cudaSuccess;
    const cudaError_t st = cudaEventSynchronize(ctx_->std_count_event);
    if (st != cudaSuccess) return st;
    return ctx_->std_total_host[3] != 0 ? kWaitGaveUp : cudaSuccess;
}

}  // namespace
}  // namespace st

cudaError_t standard_forward(HsRasterizerContext* ctx, const StandardCall& call) {
    st::StandardPass pass(ctx, call);
    cudaError_t e = pass.begin();
    if (e == cudaSuccess) e = pass.bin();
    if (e == cudaSuccess) e = pass.render();
    if (e == cudaSuccess) e = pass.finish();
    return e;
}

cudaError_t standard_forward_many(HsRasterizerContext* const* contexts, const StandardCall* calls,
                                  uint32_t count, cudaStream_t stream, cudaEvent_t raster_begin,
                                  bool finish) {
    return run_many<st::StandardPass>(contexts, calls, count, stream, raster_begin, finish);
}

cudaError_t standard_view_status(HsRasterizerContext* const* contexts, const uint64_t* point_counts,
                                 uint32_t count, cudaStream_t stream) {
    if (count == 0 || count > 2) return cudaErrorInvalidValue;
    bin::ViewStatusArgs a{};
    for (uint32_t i = 0; i < count; ++i) {
        HsRasterizerContext* ctx = contexts[i];
        if (ctx->std_total_mapped == nullptr || ctx->device_error == nullptr || point_counts[i] == 0)
            return cudaErrorInvalidValue;
        a.call[i].totals = st::geometry_views(ctx->std_geometry.ptr, point_counts[i]).totals;
        a.call[i].error = ctx->device_error;
        a.call[i].host = ctx->std_total_mapped;
    }
    bin::view_status_kernel<<<count, 32, 0, stream>>>(a);
    return cudaGetLastError();
}

static_assert(kMaxStandardPairs == sort::kMaxItems, "the pair limit is the sort's");

uint32_t standard_pair_capacity(const HsRasterizerContext* ctx) {
    // the largest pair count whose binning layout fits the buffer
    uint64_t lo = 0, hi = sort::kMaxItems;
    if (ctx->std_binning.bytes < st::binning_bytes(1)) return 0;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo + 1) / 2;
        if (st::binning_bytes(mid) <= ctx->std_binning.bytes) lo = mid; else hi = mid - 1;
    }
    return static_cast<uint32_t>(lo);
}

cudaError_t standard_reserve_pairs(HsRasterizerContext* ctx, uint64_t pairs) {
    if (pairs > sort::kMaxItems) return cudaErrorInvalidValue;
    return ensure_buffer(ctx->std_binning, st::binning_bytes(pairs), &ctx->std_growth_count, true);
}

}  // namespace hs
