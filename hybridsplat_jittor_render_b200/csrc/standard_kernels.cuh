// Standard-backend kernels (templates over the rounding policy). Instantiated
// by standard.cu with the pinned policy; see standard.cu for the pipeline.
#pragma once

#include "binning.cuh"
#include "standard_math.cuh"

namespace hs {
namespace st {

constexpr int kPreThreads = 128;
constexpr int kRenderThreads = 128;  // 4 warps, one 8x8 quadrant each
constexpr int kRecordQuads = 5;      // 80-byte blend record
constexpr int kCullQuads = 4;        // 64-byte cull shape + clipped rectangle
// Pair values carry the Gaussian index in the low 28 bits and the quadrant
// mask in the top 4 when the point count allows it.
constexpr uint32_t kIndexBits = 28;
constexpr uint32_t kIndexMask = (1u << kIndexBits) - 1u;

struct PreprocessOut {
    float4* records;
    float4* cull;            // kCullQuads per Gaussian
    uint32_t* depth_keys;
    uint32_t* order;
    uint32_t* counts;        // pairs emitted per Gaussian
    int32_t* radii;
    uint32_t* totals;        // [0] reference pair count, [1] prefiltered violation, [2] emitted,
                             // [4] Gaussians that emit pairs (kept by the depth sort)
};

__device__ __forceinline__ void warp_add(uint32_t* dst, uint32_t v) {
    v = bin::warp_sum(v);
    if ((threadIdx.x & 31) == 0 && v != 0u) atomicAdd(dst, v);
}

// Live tiles of each lane's Gaussian (clipped box [x0, x1) x [y0, y1), cull
// shape c), counted by the whole warp: the rows of the 32 boxes are dealt to
// the lanes in chunks of 32 (Gaussian, row) units, a lane reading its unit's
// shape from the owning lane by shuffles, and each unit's row_columns count is
// added to the owner's total in `sums` (this warp's 32 words of shared
// memory). These are the functions and inputs emit_rows_kernel lists the
// tiles with, so the counts match the emission exactly. Every lane of the
// warp must call this.
__device__ __forceinline__ uint32_t warp_live_tiles(const CullShape& c, int x0, int y0, int x1,
                                                    int y1, bool valid, uint32_t* sums) {
    const int lane = threadIdx.x & 31;
    const bool test = valid && c.mode == kCullEllipse && x1 > x0;
    sums[lane] = (valid && c.mode == kCullNever) ? static_cast<uint32_t>((x1 - x0) * (y1 - y0)) : 0u;
    uint32_t incl = test ? static_cast<uint32_t>(y1 - y0) : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    __syncwarp();
    for (uint32_t u0 = 0; u0 < total; u0 += 32) {
        const uint32_t u = u0 + lane;
        int j = 0;
#pragma unroll
        for (int step = 16; step >= 1; step >>= 1) {
            if (__shfl_sync(0xffffffffu, incl, j + step - 1) <= u) j += step;
        }
        const uint32_t before = __shfl_sync(0xffffffffu, incl, j > 0 ? j - 1 : 0);
        CullShape o;
        o.mx = __shfl_sync(0xffffffffu, c.mx, j);
        o.my = __shfl_sync(0xffffffffu, c.my, j);
        o.k = __shfl_sync(0xffffffffu, c.k, j);
        o.w0 = __shfl_sync(0xffffffffu, c.w0, j);
        o.hx = __shfl_sync(0xffffffffu, c.hx, j);
        o.hy = __shfl_sync(0xffffffffu, c.hy, j);
        o.yr = __shfl_sync(0xffffffffu, c.yr, j);
        o.ihy = __shfl_sync(0xffffffffu, c.ihy, j);
        o.gx = __shfl_sync(0xffffffffu, c.gx, j);
        o.gy = __shfl_sync(0xffffffffu, c.gy, j);
        o.r2 = __shfl_sync(0xffffffffu, c.r2, j);
        o.mode = kCullEllipse;
        const int ox0 = __shfl_sync(0xffffffffu, x0, j), ox1 = __shfl_sync(0xffffffffu, x1, j);
        const int oy0 = __shfl_sync(0xffffffffu, y0, j);
        if (u < total) {
            const int ty = oy0 + static_cast<int>(u - (j > 0 ? before : 0u));
            const BandSpans row =
                row_spans(quadrant_band_spans(o, ty, 0), quadrant_band_spans(o, ty, 1));
            const int n = row_columns(row, ox0, ox1).count();
            if (n != 0) atomicAdd(&sums[j], static_cast<uint32_t>(n));
        }
    }
    __syncwarp();
    return sums[lane];
}

// preprocessCUDA<5> (forward.cu:148-251) plus the cull shape. A Gaussian
// emits the tiles of its reference rectangle (getRect) that also lie in the
// bounding box of its live region; `rendered` still counts the whole
// rectangle, as the reference does. Only tile rows [row_begin, row_end) are
// rendered (the whole frame unless a caller renders a strip of it).
template <class R>
__global__ void __launch_bounds__(kPreThreads) preprocess_kernel(
    int point_count, const float* __restrict__ viewmatrix, const float* __restrict__ projmatrix,
    int width, int height, uint32_t grid_x, uint32_t grid_y, const float* __restrict__ means,
    const float* __restrict__ colors5, const float* __restrict__ opacities,
    const float* __restrict__ scales, float scale_modifier, const float* __restrict__ rotations,
    int prefiltered, uint32_t row_begin, uint32_t row_end, PreprocessOut out) {
    const int idx = blockIdx.x * kPreThreads + threadIdx.x;
    const bool active = idx < point_count;
    const R r;
    __shared__ float m[32];
    __shared__ uint32_t live_sums[kPreThreads];
    if (threadIdx.x < 16) m[threadIdx.x] = viewmatrix[threadIdx.x];
    else if (threadIdx.x < 32) m[threadIdx.x] = projmatrix[threadIdx.x - 16];
    __syncthreads();
    float view[16], proj[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        view[k] = m[k];
        proj[k] = m[16 + k];
    }
    uint32_t area = 0, emitted = 0, violation = 0;
    CullShape cs;
    cs.mode = kCullAlways;
    cs.mx = cs.my = cs.k = cs.w0 = cs.hx = cs.hy = cs.yr = cs.ihy = cs.gx = cs.gy = cs.r2 = 0.0f;
    int x0 = 0, y0 = 0, x1 = 0, y1 = 0;
    bool valid = false;
    float depth = 0.0f;
    if (active) {
        // All inputs are requested before any arithmetic; scales and
        // rotations use 64/128-bit loads when their rows are aligned.
        const float3 p = make_float3(means[3 * idx], means[3 * idx + 1], means[3 * idx + 2]);
        const float2 scale = (reinterpret_cast<uintptr_t>(scales) & 7u) == 0
                                 ? reinterpret_cast<const float2*>(scales)[idx]
                                 : make_float2(scales[2 * idx], scales[2 * idx + 1]);
        const float4 rot = (reinterpret_cast<uintptr_t>(rotations) & 15u) == 0
                               ? reinterpret_cast<const float4*>(rotations)[idx]
                               : make_float4(rotations[4 * idx], rotations[4 * idx + 1],
                                             rotations[4 * idx + 2], rotations[4 * idx + 3]);
        const float op_in = opacities[idx];
        float col[5];
#pragma unroll
        for (int k = 0; k < 5; ++k) col[k] = colors5[5 * static_cast<size_t>(idx) + k];
        const Projected g = project_gaussian(r, view, proj, p, scale, scale_modifier, rot, width,
                                             height, grid_x, grid_y);
        violation = (g.behind && prefiltered) ? 1u : 0u;
        out.order[idx] = static_cast<uint32_t>(idx);
        if (!g.valid) {
            out.radii[idx] = 0;
            out.counts[idx] = 0;
            out.depth_keys[idx] = 0xffffffffu;
        } else {
            const float op = op_in;
            const float* c = col;
            float4* rec = out.records + static_cast<size_t>(idx) * kRecordQuads;
            rec[0] = make_float4(g.xy.x, g.xy.y, g.normal.x, g.normal.y);
            rec[1] = make_float4(g.normal.z, op, c[0], c[1]);
            rec[2] = make_float4(c[2], c[3], c[4], g.tu.x);
            rec[3] = make_float4(g.tu.y, g.tu.z, g.tv.x, g.tv.y);
            rec[4] = make_float4(g.tv.z, g.tw.x, g.tw.y, g.tw.z);
            // pairs of the reference rectangle inside the rendered tile rows
            const uint32_t ry0 = max(g.rect_min.y, row_begin), ry1 = min(g.rect_max.y, row_end);
            area = ry1 > ry0 ? (g.rect_max.x - g.rect_min.x) * (ry1 - ry0) : 0u;
            cs = cull_shape(op, g.xy.x, g.xy.y, g.tu, g.tv, g.tw);
            valid = true;
            depth = g.depth;
            int bx0, by0, bx1, by1;
            if (cull_tile_box(cs, bx0, by0, bx1, by1)) {
                x0 = max(static_cast<int>(g.rect_min.x), bx0);
                y0 = max(static_cast<int>(max(g.rect_min.y, row_begin)), by0);
                x1 = min(static_cast<int>(g.rect_max.x), bx1 + 1);
                y1 = min(static_cast<int>(min(g.rect_max.y, row_end)), by1 + 1);
                if (x1 <= x0 || y1 <= y0) x0 = y0 = x1 = y1 = 0;
            }
            float4* cu = out.cull + static_cast<size_t>(idx) * kCullQuads;
            cu[0] = make_float4(cs.mx, cs.my, cs.k, cs.w0);
            cu[1] = make_float4(cs.hx, cs.hy, cs.yr, cs.gx);
            cu[2] = make_float4(cs.gy, cs.r2, __int_as_float(cs.mode), cs.ihy);
            cu[3] = make_float4(__uint_as_float(static_cast<uint32_t>(x0) | (static_cast<uint32_t>(y0) << 16)),
                                __uint_as_float(static_cast<uint32_t>(x1) | (static_cast<uint32_t>(y1) << 16)),
                                0.0f, 0.0f);
            out.radii[idx] = static_cast<int32_t>(g.radius);
        }
    }
    // pairs to emit: the live tiles of the clipped box (counted by the warp)
    emitted = warp_live_tiles(cs, x0, y0, x1, y1, valid, live_sums + (threadIdx.x & ~31));
    if (valid) {
        out.counts[idx] = emitted;
        // a Gaussian without pairs takes the depth sort's dropped key; one with
        // pairs never does (a NaN depth's bits are at most 0xfffffffe here)
        out.depth_keys[idx] = emitted != 0 ? min(__float_as_uint(depth), sort::kDropKey - 1u)
                                           : sort::kDropKey;
    }
    warp_add(out.totals + 0, area);
    warp_add(out.totals + 1, violation);
    warp_add(out.totals + 2, emitted);
    warp_add(out.totals + 4, emitted != 0 ? 1u : 0u);  // Gaussians the depth sort keeps
}

// Pair emission by rows. Each warp owns 32 Gaussians (in index order) and
// walks the rows of their clipped boxes in chunks of 32 (Gaussian, row)
// units: a lane takes one unit, computes the row's quadrant-band spans and
// live columns with the same functions the preprocess counted them with
// (row_columns), then the warp deals the chunk's live tiles to its lanes
// round-robin. A lane finds the unit of a tile by binary search over the
// units' inclusive tile counts, its column with RowColumns::at and its
// quadrant mask from the unit's spans, and takes the next slot of the
// Gaussian (one shared-memory counter per Gaussian; the slots of one
// Gaussian are filled in any order, which the stable tile sort makes
// irrelevant: each tile appears once per Gaussian). The value of a pair is
// the Gaussian index | quadrant mask << kIndexBits (masked) or the index.
struct RowUnit {
    BandSpans top, bottom;
    RowColumns cols;
    int ty;
    uint32_t owner;   // Gaussian within the block
    uint32_t tiles;   // inclusive live-tile count over the chunk
    int never;        // kCullNever: every tile, all quadrants
};

__device__ __forceinline__ CullShape load_cull_shape(const float4* cull, uint32_t gid, int& x0,
                                                     int& y0, int& x1, int& y1) {
    const float4* p = cull + static_cast<size_t>(gid) * kCullQuads;
    const float4 a = p[0], b = p[1], c = p[2], d = p[3];
    CullShape s;
    s.mx = a.x; s.my = a.y; s.k = a.z; s.w0 = a.w;
    s.hx = b.x; s.hy = b.y; s.yr = b.z; s.gx = b.w;
    s.gy = c.x; s.r2 = c.y; s.mode = __float_as_int(c.z); s.ihy = c.w;
    const uint32_t lo = __float_as_uint(d.x), hi = __float_as_uint(d.y);
    x0 = lo & 0xffff;
    y0 = lo >> 16;
    x1 = hi & 0xffff;
    y1 = hi >> 16;
    return s;
}

constexpr int kEmitRowThreads = 128;

static __global__ void __launch_bounds__(kEmitRowThreads) emit_rows_kernel(
    uint32_t count, const uint32_t* __restrict__ counts, const uint32_t* __restrict__ first_pair,
    const float4* __restrict__ cull, uint32_t grid_x, int masked, uint32_t* __restrict__ tile_ids,
    uint32_t* __restrict__ values, const uint32_t* __restrict__ error, uint32_t capacity) {
    if (sort::wait_failed(error)) return;  // first_pair is not a valid offset table
    __shared__ RowUnit units[kEmitRowThreads];
    __shared__ uint32_t cursor[kEmitRowThreads], counted[kEmitRowThreads],
        offsets[kEmitRowThreads], rows_incl[kEmitRowThreads];
    const uint32_t gid = blockIdx.x * kEmitRowThreads + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const uint32_t base = threadIdx.x & ~31u;
    const uint32_t cnt = gid < count ? counts[gid] : 0u;
    int bx0 = 0, by0 = 0, bx1 = 0, by1 = 0;
    if (cnt != 0u) load_cull_shape(cull, gid, bx0, by0, bx1, by1);
    cursor[threadIdx.x] = 0;
    const uint32_t first = cnt != 0u ? first_pair[gid] : 0u;
    // Slots from `capacity` on are not written: a call whose buffers were
    // sized before its pair count was known (a graph replay) checks the count
    // afterwards and renders again when it did not fit.
    const uint32_t room = first < capacity ? capacity - first : 0u;
    counted[threadIdx.x] = cnt < room ? cnt : room;
    offsets[threadIdx.x] = first;
    uint32_t incl = cnt != 0u ? static_cast<uint32_t>(by1 - by0) : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    rows_incl[threadIdx.x] = incl;
    const uint32_t total_rows = __shfl_sync(0xffffffffu, incl, 31);
    __syncwarp();
    RowUnit* my_units = units + base;
    for (uint32_t u0 = 0; u0 < total_rows; u0 += 32) {
        // 1. one (Gaussian, row) unit per lane
        const uint32_t u = u0 + lane;
        uint32_t n = 0;
        RowUnit unit;
        unit.cols = RowColumns{1, 0, 1, 0};
        unit.never = 0;
        unit.owner = 0;
        unit.ty = 0;
        if (u < total_rows) {
            uint32_t j = 0;
#pragma unroll
            for (uint32_t step = 16; step >= 1; step >>= 1) {
                if (rows_incl[base + j + step - 1] <= u) j += step;
            }
            const uint32_t owner = base + j;
            const uint32_t r = u - (j == 0 ? 0u : rows_incl[owner - 1]);
            int x0, y0, x1, y1;
            const CullShape c = load_cull_shape(cull, blockIdx.x * kEmitRowThreads + owner, x0, y0,
                                                x1, y1);
            unit.owner = owner;
            unit.ty = y0 + static_cast<int>(r);
            if (c.mode == kCullNever) {
                unit.never = 1;
                unit.cols = RowColumns{x0, x1 - 1, 1, 0};
            } else {
                unit.top = quadrant_band_spans(c, unit.ty, 0);
                unit.bottom = quadrant_band_spans(c, unit.ty, 1);
                unit.cols = row_columns(row_spans(unit.top, unit.bottom), x0, x1);
            }
            n = static_cast<uint32_t>(unit.cols.count());
        }
        uint32_t tiles = n;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, tiles, off);
            if (lane >= off) tiles += t;
        }
        unit.tiles = tiles;
        my_units[lane] = unit;
        const uint32_t chunk_tiles = __shfl_sync(0xffffffffu, tiles, 31);
        __syncwarp();
        // 2. the chunk's live tiles, round-robin over the lanes
        for (uint32_t t = lane; t < chunk_tiles; t += 32) {
            uint32_t j = 0;
#pragma unroll
            for (uint32_t step = 16; step >= 1; step >>= 1) {
                if (my_units[j + step - 1].tiles <= t) j += step;
            }
            const RowUnit& w = my_units[j];
            const int i = static_cast<int>(t - (j == 0 ? 0u : my_units[j - 1].tiles));
            const int tx = w.cols.at(i);
            uint32_t tag = 0;
            if (masked) tag = (w.never ? 0xfu : quadrant_mask(w.top, w.bottom, tx)) << kIndexBits;
            const uint32_t owner = w.owner;
            const uint32_t slot = bin::take_slot(cursor, owner);
            if (slot < counted[owner]) {
                const uint32_t at = offsets[owner] + slot;
                tile_ids[at] = static_cast<uint32_t>(w.ty) * grid_x + static_cast<uint32_t>(tx);
                values[at] = (blockIdx.x * kEmitRowThreads + owner) | tag;
            }
        }
        __syncwarp();
    }
}

__device__ __forceinline__ BlendRecord load_record(const float4* q) {
    const float4 a = q[0], b = q[1], c = q[2], d = q[3], e = q[4];
    BlendRecord g;
    g.x = a.x; g.y = a.y; g.nx = a.z; g.ny = a.w;
    g.nz = b.x; g.op = b.y; g.c[0] = b.z; g.c[1] = b.w;
    g.c[2] = c.x; g.c[3] = c.y; g.c[4] = c.z; g.tux = c.w;
    g.tuy = d.x; g.tuz = d.y; g.tvx = d.z; g.tvy = d.w;
    g.tvz = e.x; g.twx = e.y; g.twy = e.z; g.twz = e.w;
    return g;
}

template <class R>
__device__ __forceinline__ void store_pixel(const R& r, const PixelState& s,
                                            const float* bg, float* color, float* aux,
                                            size_t plane, size_t pix) {
    const int vo = r(S_OUT);
#pragma unroll
    for (int k = 0; k < 5; ++k) color[k * plane + pix] = mad(vo, s.t, bg[k], s.c[k]);
    aux[pix] = s.d;
    aux[plane + pix] = sub(1.0f, s.t);
    aux[2 * plane + pix] = s.n[0];
    aux[3 * plane + pix] = s.n[1];
    aux[4 * plane + pix] = s.n[2];
    aux[5 * plane + pix] = s.median;
    aux[6 * plane + pix] = s.dist;
}

// renderCUDA<5> (forward.cu:256-445). Every pixel blends its tile's list in
// order and stops on its own (forward.cu:323-328, 398-402), so each 8x8
// quadrant of a tile is an independent work item. The kernel is persistent:
// each warp takes items (tile order[i / 4], quadrant i % 4) from a global
// counter, longest tiles first, two pixels per lane (rows ly and ly + 4). A
// warp walks its tile's list 32 pairs at a time, keeps the pairs whose
// quadrant bit is set, stages their records in its shared-memory slots and
// blends them in list order; it stops when its 64 pixels are done. Blend
// weights are summed across the warp before one atomicAdd per Gaussian.
template <class R, bool kMasked>
__global__ void __launch_bounds__(kRenderThreads, 7) render_kernel(
    const uint2* __restrict__ ranges, const uint32_t* __restrict__ tile_order, uint32_t items,
    uint32_t* __restrict__ work_counter, const uint32_t* __restrict__ pair_values,
    const float4* __restrict__ records, int width, int height, uint32_t grid_x,
    const float* __restrict__ background5, float* __restrict__ color, float* __restrict__ aux,
    float* __restrict__ weight, const uint32_t* __restrict__ error) {
    // A bounded wait of this call gave up: the pair lists may hold any value.
    if (sort::wait_failed(error)) return;
    __shared__ float4 slots[kRenderThreads / 32][32 * kRecordQuads];
    __shared__ uint32_t slot_ids[kRenderThreads / 32][32];
    const R r;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    float4* my_slots = slots[warp];
    uint32_t* my_ids = slot_ids[warp];
    float bg[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) bg[k] = background5[k];
    const size_t plane = static_cast<size_t>(width) * height;
    for (;;) {
        uint32_t item = 0;
        if (lane == 0) item = atomicAdd(work_counter, 1u);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= items) break;
        const uint32_t tile = tile_order[item >> 2];
        const int quad = static_cast<int>(item & 3u);
        const int tx = tile % grid_x, ty = tile / grid_x;
        const int px = tx * 16 + (quad & 1) * 8 + (lane & 7);
        const int py0 = ty * 16 + (quad >> 1) * 8 + (lane >> 3), py1 = py0 + 4;
        const bool in0 = px < width && py0 < height;
        const bool in1 = px < width && py1 < height;
        const float fx = static_cast<float>(px);
        const float fy0 = static_cast<float>(py0), fy1 = static_cast<float>(py1);
        PixelState s0, s1;
        pixel_init(s0, in0);
        pixel_init(s1, in1);
        const uint2 range = ranges[tile];
        const uint32_t n = range.y - range.x;
        for (uint32_t base = 0; base < n; base += 32) {
            if (__all_sync(0xffffffffu, s0.done && s1.done)) break;
            const uint32_t j = base + lane;
            const uint32_t v = j < n ? pair_values[range.x + j] : 0u;
            const bool live = j < n && (!kMasked || ((v >> (kIndexBits + quad)) & 1u) != 0u);
            const uint32_t mask = __ballot_sync(0xffffffffu, live);
            if (live) {
                const uint32_t gid = kMasked ? (v & kIndexMask) : v;
                const uint32_t slot = __popc(mask & lt);
                const float4* src = records + static_cast<size_t>(gid) * kRecordQuads;
#pragma unroll
                for (int q = 0; q < kRecordQuads; ++q) my_slots[slot * kRecordQuads + q] = src[q];
                my_ids[slot] = gid;
            }
            __syncwarp();
            const int live_count = __popc(mask);
            for (int k = 0; k < live_count; ++k) {
                const BlendRecord g = load_record(my_slots + k * kRecordQuads);
                const ColumnTerms col = column_terms(r, fx, g);
                const float w = blend2(r, s0, s1, col, fy0, fy1, g);
                if (__any_sync(0xffffffffu, w != 0.0f)) {
                    // The Gaussian's blend weight over the warp's 64 pixels, summed
                    // exactly in 2^-24 fixed point by one warp reduction (each
                    // lane's w <= 2, so the sum stays below 2^31); the per-lane
                    // rounding (<= 2^-25) is of the order of the float atomics'
                    // own, which make this output order-dependent in both
                    // libraries. Only the weights use it; colours are untouched.
                    const uint32_t sum =
                        __reduce_add_sync(0xffffffffu, __float2uint_rn(w * 16777216.0f));
                    if (lane == 0 && sum != 0u)
                        atomicAdd(weight + my_ids[k], __uint2float_rn(sum) * (1.0f / 16777216.0f));
                }
            }
            __syncwarp();
        }
        if (in0) store_pixel(r, s0, bg, color, aux, plane, static_cast<size_t>(py0) * width + px);
        if (in1) store_pixel(r, s1, bg, color, aux, plane, static_cast<size_t>(py1) * width + px);
    }
}

}  // namespace st
}  // namespace hs
