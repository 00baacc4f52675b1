// FlashGS kernels (templates over the rounding policy). Instantiated by
// flashgs.cu with the pinned policy; see flashgs.cu for the pipeline.
#pragma once

#include <climits>

#include "binning.cuh"
#include "flashgs_math.cuh"

namespace hs {
namespace fg {


constexpr int kPreThreads = 128;
constexpr int kRenderThreads = 128;  // 4 warps, 2 pixels per thread
constexpr int kBatch = 32;           // Gaussians staged per shared-memory batch
constexpr int kRecordQuads = 6;      // 96-byte record: 5 blend quads + conic/opacity
constexpr int kEmitQuads = 2;        // 32-byte emit record

struct Camera {
    float view[16];
    float proj[16];
    float campos[3];
    float tan_fovx, tan_fovy;
    float focal_x, focal_y;
    int width, height, grid_x, grid_y;
};

__device__ __forceinline__ float4 f4(float a, float b, float c, float d) {
    return make_float4(a, b, c, d);
}

// Rectangles up to 2 * kSerialTiles tiles are emitted by their own lane,
// larger ones by the whole warp, 32 tiles per step.
constexpr int kSerialTiles = 4;

template <class R>
// 12 blocks per SM (40 registers, a few spills): the kernel waits on its
// input loads, and the extra resident warps hide more of that latency.
__global__ void __launch_bounds__(kPreThreads, 12) preprocess_kernel(
    int point_count, Camera cam, const float* __restrict__ positions,
    const float* __restrict__ shs, const float* __restrict__ colors, int use_sh,
    const float* __restrict__ opacities, const float* __restrict__ cov6,
    const float* __restrict__ scales, float scale_modifier, const float* __restrict__ rotations,
    const float* __restrict__ specular, const float* __restrict__ roughness,
    float4* __restrict__ records, float4* __restrict__ emit, uint32_t* __restrict__ depth_keys,
    uint32_t* __restrict__ order, uint32_t* __restrict__ pair_counts,
    uint32_t* __restrict__ totals, int row_begin, int row_end) {
    const int idx = blockIdx.x * kPreThreads + threadIdx.x;
    const bool active = idx < point_count;
    const int lane = threadIdx.x & 31;
    const R r;
    Projected g;
    g.in_front = false;
    g.touches = false;
    float3 p = make_float3(0.0f, 0.0f, 0.0f);
    float opacity = 0.0f;
    if (active) {
        p = make_float3(positions[3 * idx], positions[3 * idx + 1], positions[3 * idx + 2]);
        opacity = opacities[idx];
        float cov[6];
#pragma unroll
        for (int k = 0; k < 6; ++k) cov[k] = cov6[6 * idx + k];
        const float2 scale = make_float2(scales[2 * idx], scales[2 * idx + 1]);
        const float4 rot = make_float4(rotations[4 * idx], rotations[4 * idx + 1],
                                       rotations[4 * idx + 2], rotations[4 * idx + 3]);
        g = project_gaussian(r, cam.view, cam.proj, p, opacity, cov, scale, scale_modifier, rot,
                             cam.width, cam.height, cam.focal_x, cam.focal_y, cam.tan_fovx,
                             cam.tan_fovy, cam.grid_x, cam.grid_y);
    }
    // Exact tile/ellipse count (preprocess.cu:482-506). The rectangle tiles
    // of the warp's 32 Gaussians are numbered 0..total-1 and dealt to the
    // lanes round-robin; each lane finds the owning Gaussian by binary search
    // over the warp's inclusive tile counts and adds its hit to the owner's
    // shared-memory counter, so every lane does the same number of tests.
    __shared__ float s_shape[kPreThreads][6];      // xy, conic, power
    __shared__ int s_rect[kPreThreads][3];         // x0, y0, width
    __shared__ uint32_t s_incl[kPreThreads];
    __shared__ uint32_t s_hits[kPreThreads];
    const bool candidate = g.in_front && g.touches;
    const int gw = candidate ? g.rect_max.x - g.rect_min.x : 0;
    const uint32_t full_area =
        candidate ? static_cast<uint32_t>(gw * (g.rect_max.y - g.rect_min.y)) : 0u;
    // rows of the rectangle inside the rendered tile rows
    const int ry0 = max(g.rect_min.y, row_begin), ry1 = min(g.rect_max.y, row_end);
    const uint32_t area = candidate && ry1 > ry0 ? static_cast<uint32_t>(gw * (ry1 - ry0)) : 0u;
    s_shape[threadIdx.x][0] = g.xy.x;
    s_shape[threadIdx.x][1] = g.xy.y;
    s_shape[threadIdx.x][2] = g.conic.x;
    s_shape[threadIdx.x][3] = g.conic.y;
    s_shape[threadIdx.x][4] = g.conic.z;
    s_shape[threadIdx.x][5] = g.power;
    s_rect[threadIdx.x][0] = g.rect_min.x;
    s_rect[threadIdx.x][1] = ry0;
    s_rect[threadIdx.x][2] = gw;
    s_hits[threadIdx.x] = 0;
    uint32_t incl = area;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    s_incl[threadIdx.x] = incl;
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    const uint32_t wbase = threadIdx.x & ~31u;
    __syncwarp();
    for (uint32_t f = lane; f < total; f += 32) {
        uint32_t j = 0;
#pragma unroll
        for (uint32_t step = 16; step >= 1; step >>= 1) {
            if (s_incl[wbase + j + step - 1] <= f) j += step;
        }
        const uint32_t o = wbase + j;
        const uint32_t k = f - (j == 0 ? 0u : s_incl[o - 1]);
        const int w = s_rect[o][2];
        const int tx = s_rect[o][0] + static_cast<int>(k) % w;
        const int ty = s_rect[o][1] + static_cast<int>(k) / w;
        const float2 cxy = make_float2(s_shape[o][0], s_shape[o][1]);
        const float3 cc = make_float3(s_shape[o][2], s_shape[o][3], s_shape[o][4]);
        if (tile_hit(r, tx, ty, cxy, cc, s_shape[o][5])) atomicAdd(&s_hits[o], 1u);
    }
    __syncwarp();
    const uint32_t hits = s_hits[threadIdx.x];
    const uint32_t total_hits = bin::warp_sum(hits);
    if (lane == 0 && total_hits != 0u) atomicAdd(totals, total_hits);
    // Gaussians with pairs: the items the depth sort keeps (totals[4])
    const uint32_t kept = bin::warp_sum(hits > 0 ? 1u : 0u);
    if (lane == 0 && kept != 0u) atomicAdd(totals + 4, kept);
    if (!active) return;
    // Single-tile Gaussians always keep their record (preprocess.cu:482-506).
    const bool write = candidate && (full_area == 1u || hits > 0);
    float4* rec = records + static_cast<size_t>(idx) * kRecordQuads;
    if (write) {
        float3 rgb;
        if (use_sh) {
            rgb = sh_color(r, p, make_float3(cam.campos[0], cam.campos[1], cam.campos[2]),
                           shs + static_cast<size_t>(idx) * 48);
        } else {
            rgb = make_float3(colors[3 * idx], colors[3 * idx + 1], colors[3 * idx + 2]);
        }
        const float sp = specular[idx], ro = roughness[idx];
        rec[0] = f4(g.xy.x, g.xy.y, g.normal.x, g.normal.y);
        rec[1] = f4(g.normal.z, opacity, rgb.x, rgb.y);
        rec[2] = f4(rgb.z, sp, ro, g.tu.x);
        rec[3] = f4(g.tu.y, g.tu.z, g.tv.x, g.tv.y);
        rec[4] = f4(g.tv.z, g.tw.x, g.tw.y, g.tw.z);
        rec[5] = f4(mul(-0.5f * kLog2e, g.conic.x), mul(-kLog2e, g.conic.y),
                    mul(-0.5f * kLog2e, g.conic.z), g.log2_opacity);
    } else {
        const float4 z = f4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int q = 0; q < kRecordQuads; ++q) rec[q] = z;
    }
    float4* em = emit + static_cast<size_t>(idx) * kEmitQuads;
    em[0] = f4(g.xy.x, g.xy.y, g.conic.x, g.conic.y);
    const uint32_t lo = static_cast<uint32_t>(g.rect_min.x) | (static_cast<uint32_t>(area != 0u ? ry0 : 0) << 16);
    const uint32_t hi = static_cast<uint32_t>(g.rect_max.x) | (static_cast<uint32_t>(area != 0u ? ry1 : 0) << 16);
    em[1] = f4(g.conic.z, g.power, __uint_as_float(lo), __uint_as_float(hi));
    // without pairs: the depth sort's dropped key, which a Gaussian with pairs
    // never takes (a NaN depth's bits are at most 0xfffffffe here)
    depth_keys[idx] = hits > 0 ? min(__float_as_uint(g.depth), sort::kDropKey - 1u) : sort::kDropKey;
    order[idx] = static_cast<uint32_t>(idx);
    pair_counts[idx] = hits;
}

// Emits the (tile, index) pairs of one Gaussian: the tiles of its rectangle
// that pass the exact tile/ellipse test, compacted with a warp ballot.
template <class R>
struct Emitter {
    const float4* emit_records;
    int grid_x;

    struct Shape {
        float4 a, b;
    };
    __device__ __forceinline__ Shape load(uint32_t gid) const {
        const float4* q = emit_records + static_cast<size_t>(gid) * kEmitQuads;
        return Shape{q[0], q[1]};
    }
    __device__ __forceinline__ uint32_t slots(const Shape& s) const {
        const uint32_t lo = __float_as_uint(s.b.z), hi = __float_as_uint(s.b.w);
        return ((hi & 0xffff) - (lo & 0xffff)) * ((hi >> 16) - (lo >> 16));
    }
    struct Cache {};
    __device__ __forceinline__ bool pair_at(const Shape& s, uint32_t, uint32_t k, uint32_t& tile,
                                            uint32_t& tag, Cache&) const {
        tag = 0u;
        const R r;
        const uint32_t lo = __float_as_uint(s.b.z), hi = __float_as_uint(s.b.w);
        const int x0 = lo & 0xffff, y0 = lo >> 16, w = static_cast<int>(hi & 0xffff) - x0;
        const int tx = x0 + static_cast<int>(k) % w, ty = y0 + static_cast<int>(k) / w;
        tile = static_cast<uint32_t>(ty * grid_x + tx);
        return tile_hit(r, tx, ty, make_float2(s.a.x, s.a.y), make_float3(s.a.z, s.a.w, s.b.x), s.b.y);
    }
};

__device__ __forceinline__ BlendRecord load_record(const float4* q) {
    const float4 a = q[0], b = q[1], c = q[2], d = q[3], e = q[4];
    BlendRecord g;
    g.x = a.x; g.y = a.y; g.nx = a.z; g.ny = a.w;
    g.nz = b.x; g.op = b.y; g.r = b.z; g.g = b.w;
    g.b = c.x; g.spec = c.y; g.rough = c.z; g.tux = c.w;
    g.tuy = d.x; g.tuz = d.y; g.tvx = d.z; g.tvy = d.w;
    g.tvz = e.x; g.twx = e.y; g.twy = e.z; g.twz = e.w;
    return g;
}

struct Outputs {
    float* color;
    float* other;
    float* depth;
    float* alpha;
    float* normal;
    float* median;
    float* distortion;
};

template <class R>
__device__ __forceinline__ void store_pixel(const R& r, const PixelState& s, float3 bg,
                                            const Outputs& o, size_t plane, size_t pix) {
    float v[12];
    finish_pixel(r, s, bg, v);
    o.color[pix] = v[0];
    o.color[plane + pix] = v[1];
    o.color[2 * plane + pix] = v[2];
    o.other[pix] = v[3];
    o.other[plane + pix] = v[4];
    o.depth[pix] = v[5];
    o.alpha[pix] = v[6];
    o.normal[pix] = v[7];
    o.normal[plane + pix] = v[8];
    o.normal[2 * plane + pix] = v[9];
    o.median[pix] = v[10];
    o.distortion[pix] = v[11];
}

__device__ __forceinline__ void store_empty(float3 bg_encoded, const Outputs& o, size_t plane,
                                            size_t pix) {
    o.color[pix] = bg_encoded.x;
    o.color[plane + pix] = bg_encoded.y;
    o.color[2 * plane + pix] = bg_encoded.z;
    o.other[pix] = 0.0f;
    o.other[plane + pix] = 0.0f;
    o.depth[pix] = 0.0f;
    o.alpha[pix] = 0.0f;
    o.normal[pix] = 0.0f;
    o.normal[plane + pix] = 0.0f;
    o.normal[2 * plane + pix] = 0.0f;
    o.median[pix] = 0.0f;
    o.distortion[pix] = 0.0f;
}

// Tile-wide termination. The reference warp stops after Gaussian j when all
// 256 pixels of the tile (including pixels outside the image) have T < 1e-4,
// so the tile consumes n_tile = (first such j) + 1 Gaussians and every pixel
// blends exactly those. T never increases, so "warp w is done after j" is
// monotone and n_tile - 1 = max over warps of each warp's first done index.
// Per batch: phase A - every warp that is not yet done blends until it is
// done (recording the index) or the batch ends; barrier; if all warps are
// done the tile end is the maximum index, otherwise the batch end; phase B -
// warps that stopped early blend the remaining Gaussians up to that end.
template <class R>
__global__ void __launch_bounds__(kRenderThreads) render_kernel(
    const int2* __restrict__ ranges, const uint32_t* __restrict__ tile_order, uint32_t tile_count,
    uint32_t* __restrict__ work_counter, const uint32_t* __restrict__ gaussian_ids,
    const float4* __restrict__ records, int width, int height, int grid_x, float3 bg,
    float3 bg_encoded, Outputs out, const uint32_t* __restrict__ error) {
    // A bounded wait of this call gave up: the pair lists may hold any value.
    if (sort::wait_failed(error)) return;
    __shared__ float4 batch[kBatch * 5];
    __shared__ int done_at[kRenderThreads / 32];
    __shared__ uint32_t next_tile;
    const R r;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lx = threadIdx.x & 15, ly = threadIdx.x >> 4;
    const size_t plane = static_cast<size_t>(width) * height;
    // Persistent: each block takes tiles from the global counter, in the
    // longest-first order of tile_order.
    for (;;) {
        __syncthreads();  // the previous tile's readers of next_tile/done_at are finished
        if (threadIdx.x == 0) next_tile = atomicAdd(work_counter, 1u);
        __syncthreads();
        const uint32_t slot = next_tile;
        if (slot >= tile_count) break;
        const int tile = static_cast<int>(tile_order[slot]);
        const int tx = tile % grid_x, ty = tile / grid_x;
        const int px = tx * 16 + lx, py0 = ty * 16 + ly, py1 = py0 + 8;
        const bool in0 = px < width && py0 < height;
        const bool in1 = px < width && py1 < height;
        const int2 range = ranges[tile];
        if (range.x >= range.y) {
            if (in0) store_empty(bg_encoded, out, plane, static_cast<size_t>(py0) * width + px);
            if (in1) store_empty(bg_encoded, out, plane, static_cast<size_t>(py1) * width + px);
            continue;
        }
        const float fx = static_cast<float>(px);
        const float fy0 = static_cast<float>(py0), fy1 = static_cast<float>(py1);
        const float2 fy = make_float2(fy0, fy1);
        PixelPair sp;
        pair_init(sp);
        const int n = range.y - range.x;
        bool warp_done = false;
        int warp_done_at = 0;
        for (int base = 0; base < n; base += kBatch) {
            const int nb = min(kBatch, n - base);
            __syncthreads();
            for (int i = threadIdx.x; i < nb * 5; i += kRenderThreads) {
                const int j = i / 5, q = i - j * 5;
                const uint32_t gid = gaussian_ids[range.x + base + j];
                batch[i] = records[static_cast<size_t>(gid) * kRecordQuads + q];
            }
            __syncthreads();
            int cursor = 0;
            if (!warp_done) {
                cursor = nb;
                for (int j = 0; j < nb; ++j) {
                    const BlendRecord g = load_record(batch + j * 5);
                    const ColumnTerms col = column_terms(r, fx, g);
                    blend_pair(r, sp, col, fy, g);
                    if (__all_sync(0xffffffffu, sp.t.x < 0.0001f && sp.t.y < 0.0001f)) {
                        warp_done = true;
                        warp_done_at = base + j;
                        cursor = j + 1;
                        break;
                    }
                }
            }
            if (lane == 0) done_at[warp] = warp_done ? warp_done_at : INT_MAX;
            __syncthreads();
            int tile_end = done_at[0];
#pragma unroll
            for (int w = 1; w < kRenderThreads / 32; ++w) tile_end = max(tile_end, done_at[w]);
            const int stop = tile_end == INT_MAX ? nb : tile_end - base + 1;
            for (int j = cursor; j < stop; ++j) {
                const BlendRecord g = load_record(batch + j * 5);
                const ColumnTerms col = column_terms(r, fx, g);
                blend_pair(r, sp, col, fy, g);
            }
            if (tile_end != INT_MAX) break;
        }
        if (in0) store_pixel(r, pixel_of(sp, 0), bg, out, plane, static_cast<size_t>(py0) * width + px);
        if (in1) store_pixel(r, pixel_of(sp, 1), bg, out, plane, static_cast<size_t>(py1) * width + px);
    }
}

}  // namespace fg
}  // namespace hs
