// Standard five-channel forward that allocates nothing.
//
// hs_rasterizer_forward_f32_v1 grows per-context device workspaces with
// cudaMalloc and keeps a pinned host word for the pair count. Some callers
// cannot allow that: a host whose caching allocator already owns nearly all
// device memory (a library cudaMalloc then fails or fragments the pool), a
// serving loop that must not pay allocation or implicit device-wide
// synchronisation (freeing a grown buffer synchronises the device) once it is
// running, or code that runs where allocation is not permitted. This entry
// point serves them for small views: every scratch buffer is carved from one
// file-scope device array of kScratchBytes bytes, so the call issues no
// cudaMalloc, cudaFree, cudaHostAlloc or allocating library call. It runs the
// same kernels as the context path (standard_kernels.cuh, sort.cu,
// binning.cuh) in the same order, so its outputs equal that path's.
//
// Limits (checked, violations return a range error with the limit named):
// point_count <= kMaxPoints, tiles <= kMaxTiles, emitted pairs <= kMaxPairs.
// The emitted-pair limit is only known after preprocessing; when it is
// exceeded the outputs are left incomplete.
//
// The scratch array lives in this translation unit's module; with CUDA's
// lazy module loading it occupies device memory only once this entry point
// has been used on a device. Its address is fetched with
// cudaGetSymbolAddress the first time the entry point runs on each device
// (with that device current), so a caller should make its first call on each
// device before any stream capture and before any phase in which the runtime
// must not be asked to load modules.
//
// What must start at zero: the wait-status word at the start of the array
// (set when a bounded wait of a sort or scan gave up) and the per-call
// counters; the call clears them itself before its first kernel, so a failed
// call does not affect the next one. All other scratch is written before it is
// read. A wait that gives up fails the same call: the word is read back after
// the renderer is queued.
//
// Concurrency: all calls on one device share the array. A process-wide lock
// serialises the host side and all work goes to the legacy default stream,
// so the GPU work of consecutive calls is ordered; a caller must not run this
// entry point's work on its own streams concurrently (there is no stream
// argument).
#include <algorithm>
#include <climits>
#include <cstdio>
#include <mutex>

#include "context.h"

#ifndef HS_STANDARD_ROUNDING
#define HS_STANDARD_ROUNDING PinnedRounding
#endif
#include "sort.cuh"
#include "standard_kernels.cuh"

namespace hs {
namespace st_noalloc {

constexpr uint32_t kMaxPoints = 16384;
constexpr uint32_t kMaxPairs = 262144;
constexpr uint32_t kMaxTiles = 4096;
constexpr uint64_t kScratchBytes = 8ull << 20;  // 8 MiB

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
unsigned char* g_scratch_address[kMaxDevices] = {};

struct Layout {
    // [error word][totals] [geometry][geometry scratch] [pairs x4][pair sort scratch] [image]
    uint32_t* error;
    uint32_t* totals;
    float4* records;
    float4* cull;
    uint32_t* keys;
    uint32_t* order;
    uint32_t* counts;
    uint32_t* alt_keys;
    uint32_t* alt_order;
    void* geometry_scratch;
    uint32_t* tile_ids;
    uint32_t* values;
    uint32_t* alt_tiles;
    uint32_t* alt_values;
    void* pair_scratch;
    uint2* ranges;
    uint32_t* tile_order;
    uint32_t* work_counter;
    uint64_t used;
};

Layout carve(unsigned char* base, uint64_t points, uint64_t pairs, uint64_t tiles) {
    Carver c(base);
    Layout l;
    l.error = c.take<uint32_t>(64);
    l.totals = c.take<uint32_t>(64);
    l.records = c.take<float4>(points * st::kRecordQuads);
    l.cull = c.take<float4>(points * st::kCullQuads);
    l.keys = c.take<uint32_t>(points);
    l.order = c.take<uint32_t>(points);
    l.counts = c.take<uint32_t>(points);
    l.alt_keys = c.take<uint32_t>(points);
    l.alt_order = c.take<uint32_t>(points);
    l.geometry_scratch = c.take<unsigned char>(
        std::max(sort::sort_scratch_bytes(static_cast<uint32_t>(points)),
                 bin::scan_scratch_bytes(static_cast<uint32_t>(points))));
    l.tile_ids = c.take<uint32_t>(pairs);
    l.values = c.take<uint32_t>(pairs);
    l.alt_tiles = c.take<uint32_t>(pairs);
    l.alt_values = c.take<uint32_t>(pairs);
    l.pair_scratch = c.take<unsigned char>(sort::sort_scratch_bytes(static_cast<uint32_t>(pairs)));
    l.ranges = c.take<uint2>(tiles);
    l.tile_order = c.take<uint32_t>(tiles);
    l.work_counter = c.take<uint32_t>(64);
    l.used = c.offset;
    return l;
}

struct Result {
    cudaError_t status;
    const char* limit;  // non-null: a size limit was exceeded
    uint64_t value;
    uint64_t bound;
};

Result forward(int device, int32_t point_count, const float* background5, int32_t width,
               int32_t height, const float* means3d, const float* colors5, const float* opacities,
               const float* scales2, float scale_modifier, const float* rotations4,
               const float* viewmatrix4x4, const float* projmatrix4x4, bool prefiltered,
               float* output_color5, float* output_aux7, float* output_weight,
               int32_t* output_radii, int32_t* output_rendered) {
    using namespace st;
    const cudaStream_t stream = nullptr;
    const uint32_t grid_x = static_cast<uint32_t>((width + 15) / 16);
    const uint32_t grid_y = static_cast<uint32_t>((height + 15) / 16);
    const uint64_t tiles = static_cast<uint64_t>(grid_x) * grid_y;
    if (static_cast<uint64_t>(point_count) > kMaxPoints) {
        return {cudaSuccess, "point_count", static_cast<uint64_t>(point_count), kMaxPoints};
    }
    if (tiles > kMaxTiles) return {cudaSuccess, "16x16 tile count", tiles, kMaxTiles};
    if (device < 0 || device >= kMaxDevices) return {cudaErrorInvalidDevice, nullptr, 0, 0};
    unsigned char*& base = g_scratch_address[device];
    if (base == nullptr) {
        void* address = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&address, g_scratch);
        if (e != cudaSuccess) return {e, nullptr, 0, 0};
        base = static_cast<unsigned char*>(address);
    }
    const uint64_t pixels = static_cast<uint64_t>(width) * static_cast<uint64_t>(height);
    if (point_count == 0) {
        cudaError_t e = cudaMemsetAsync(output_color5, 0, 5 * pixels * sizeof(float), stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(output_aux7, 0, 7 * pixels * sizeof(float), stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(output_rendered, 0, sizeof(int32_t), stream);
        return {e, nullptr, 0, 0};
    }
    const Layout l = carve(base, kMaxPoints, kMaxPairs, kMaxTiles);
    if (l.used > kScratchBytes) return {cudaErrorInvalidValue, "scratch layout", l.used, kScratchBytes};

    cudaError_t st = cudaMemsetAsync(l.error, 0, sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(output_weight, 0, point_count * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(l.totals, 0, 8 * sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(l.ranges, 0, tiles * sizeof(uint2), stream);
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    const int blocks = (point_count + kPreThreads - 1) / kPreThreads;
    PreprocessOut po{l.records, l.cull, l.keys, l.order, l.counts, output_radii, l.totals};
    preprocess_kernel<HS_STANDARD_ROUNDING><<<blocks, kPreThreads, 0, stream>>>(
        point_count, viewmatrix4x4, projmatrix4x4, width, height, grid_x, grid_y, means3d,
        colors5, opacities, scales2, scale_modifier, rotations4, prefiltered ? 1 : 0, 0u, grid_y,
        po);
    st = cudaGetLastError();
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    st = sort::sort_pairs(l.keys, l.order, l.alt_keys, l.alt_order, point_count, 0, 32,
                          l.geometry_scratch, stream, l.error);
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    uint32_t totals[4] = {};
    st = cudaMemcpy(totals, l.totals, sizeof(totals), cudaMemcpyDeviceToHost);  // pageable: no pinned buffer
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    const uint32_t rendered = totals[0];
    const uint32_t emitted = totals[2];
    if (totals[1] != 0) return {cudaErrorInvalidValue, nullptr, 0, 0};
    if (emitted > kMaxPairs) return {cudaSuccess, "emitted pair count", emitted, kMaxPairs};
    if (rendered > static_cast<uint32_t>(INT_MAX)) return {cudaErrorInvalidValue, nullptr, 0, 0};
    st = cudaMemcpyAsync(output_rendered, l.totals, sizeof(int32_t), cudaMemcpyDeviceToDevice,
                         stream);
    if (st != cudaSuccess) return {st, nullptr, 0, 0};

    if (emitted > 0) {
        st = cudaMemsetAsync(l.geometry_scratch, 0, bin::scan_scratch_bytes(point_count), stream);
        if (st != cudaSuccess) return {st, nullptr, 0, 0};
        uint32_t* first_pair = l.alt_keys;
        bin::offsets_kernel<<<bin::scan_tiles(point_count), bin::kScanThreads, 0, stream>>>(
            static_cast<uint32_t>(point_count), nullptr, l.order, l.counts,
            static_cast<uint32_t*>(l.geometry_scratch), l.error, first_pair);
        st = cudaGetLastError();
        if (st != cudaSuccess) return {st, nullptr, 0, 0};
        emit_rows_kernel<<<(point_count + kEmitRowThreads - 1) / kEmitRowThreads, kEmitRowThreads, 0,
                           stream>>>(static_cast<uint32_t>(point_count), l.counts, first_pair,
                                     l.cull, grid_x, 1, l.tile_ids, l.values, l.error,
                                     emitted);
        st = cudaGetLastError();
        if (st != cudaSuccess) return {st, nullptr, 0, 0};
        st = sort::sort_pairs(l.tile_ids, l.values, l.alt_tiles, l.alt_values, emitted, 0,
                              sort::bits_for_tiles(static_cast<uint32_t>(tiles)), l.pair_scratch,
                              stream, l.error);
        if (st != cudaSuccess) return {st, nullptr, 0, 0};
        bin::ranges_kernel<uint2><<<bin::ranges_grid(emitted), bin::kRangeThreads, 0, stream>>>(
            emitted, static_cast<uint32_t>(tiles), l.tile_ids, l.ranges);
        st = cudaGetLastError();
        if (st != cudaSuccess) return {st, nullptr, 0, 0};
    }
    bin::tile_order_kernel<uint2><<<1, bin::kOrderThreads, 0, stream>>>(
        0u, static_cast<uint32_t>(tiles), l.ranges, l.tile_order, l.work_counter, l.error, nullptr);
    st = cudaGetLastError();
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    const uint32_t items = static_cast<uint32_t>(tiles) * 4u;
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, render_kernel<HS_STANDARD_ROUNDING, true>, kRenderThreads, 0);
    const uint32_t wanted = (items + kRenderThreads / 32 - 1) / (kRenderThreads / 32);
    const uint32_t render_blocks =
        std::min<uint32_t>(wanted, static_cast<uint32_t>(sms * std::max(per_sm, 1)));
    render_kernel<HS_STANDARD_ROUNDING, true><<<render_blocks, kRenderThreads, 0, stream>>>(
        l.ranges, l.tile_order, items, l.work_counter, l.values, l.records, width, height,
        grid_x, background5, output_color5, output_aux7, output_weight, l.error);
    st = cudaGetLastError();
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    // The wait-status word of this call's sorts and scan (a blocking copy on
    // the legacy stream: it completes after the renderer).
    uint32_t gave_up = 0;
    st = cudaMemcpy(&gave_up, l.error, sizeof(gave_up), cudaMemcpyDeviceToHost);
    if (st != cudaSuccess) return {st, nullptr, 0, 0};
    return {gave_up != 0 ? kWaitGaveUp : cudaSuccess, nullptr, 0, 0};
}

}  // namespace st_noalloc

// Entry-point body for hs_b200_rasterizer_forward_noalloc_f32_v1 (c_api.cpp
// validates the arguments and maps the result to a status).
cudaError_t standard_forward_noalloc(int32_t device, int32_t point_count,
                                    const float* background5, int32_t width, int32_t height,
                                    const float* means3d, const float* colors5,
                                    const float* opacities, const float* scales2,
                                    float scale_modifier, const float* rotations4,
                                    const float* viewmatrix4x4, const float* projmatrix4x4,
                                    bool prefiltered, float* output_color5, float* output_aux7,
                                    float* output_weight, int32_t* output_radii,
                                    int32_t* output_rendered, char* limit_text,
                                    uint64_t limit_capacity) {
    std::lock_guard<std::mutex> lock(st_noalloc::g_lock);
    const st_noalloc::Result r = st_noalloc::forward(
        device, point_count, background5, width, height, means3d, colors5, opacities, scales2,
        scale_modifier, rotations4, viewmatrix4x4, projmatrix4x4, prefiltered, output_color5,
        output_aux7, output_weight, output_radii, output_rendered);
    if (r.limit != nullptr && limit_text != nullptr && limit_capacity != 0) {
        std::snprintf(limit_text, limit_capacity,
                      "no-alloc rasterizer: %s %llu exceeds the fixed scratch limit of %llu",
                      r.limit, static_cast<unsigned long long>(r.value),
                      static_cast<unsigned long long>(r.bound));
    }
    return r.limit != nullptr ? cudaErrorNotSupported : r.status;
}

}  // namespace hs
