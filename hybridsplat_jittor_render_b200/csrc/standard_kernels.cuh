// Standard-backend kernels (templates over the rounding policy). Instantiated
// by standard.cu with the pinned policy; see standard.cu for the pipeline.
#pragma once

#include "standard_math.cuh"

namespace hs {
namespace st {


constexpr int kPreThreads = 128;
constexpr int kRenderThreads = 128;
constexpr int kBatch = 32;
constexpr int kRecordQuads = 5;

template <class R>
__global__ void __launch_bounds__(kPreThreads) preprocess_kernel(
    int point_count, const float* __restrict__ viewmatrix, const float* __restrict__ projmatrix,
    int width, int height, uint32_t grid_x, uint32_t grid_y, const float* __restrict__ means,
    const float* __restrict__ colors5, const float* __restrict__ opacities,
    const float* __restrict__ scales, float scale_modifier, const float* __restrict__ rotations,
    int prefiltered, float4* __restrict__ records, uint2* __restrict__ rects,
    uint32_t* __restrict__ depth_keys, uint32_t* __restrict__ order,
    uint32_t* __restrict__ pair_counts, int32_t* __restrict__ radii,
    uint32_t* __restrict__ error_flag) {
    const int idx = blockIdx.x * kPreThreads + threadIdx.x;
    if (idx >= point_count) return;
    const R r;
    float view[16], proj[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        view[k] = viewmatrix[k];
        proj[k] = projmatrix[k];
    }
    const float3 p = make_float3(means[3 * idx], means[3 * idx + 1], means[3 * idx + 2]);
    const float2 scale = make_float2(scales[2 * idx], scales[2 * idx + 1]);
    const float4 rot = make_float4(rotations[4 * idx], rotations[4 * idx + 1],
                                   rotations[4 * idx + 2], rotations[4 * idx + 3]);
    const Projected g =
        project_gaussian(r, view, proj, p, scale, scale_modifier, rot, width, height, grid_x, grid_y);
    if (g.behind && prefiltered) atomicOr(error_flag, 1u);
    order[idx] = static_cast<uint32_t>(idx);
    if (!g.valid) {
        radii[idx] = 0;
        pair_counts[idx] = 0;
        depth_keys[idx] = 0xffffffffu;
        return;
    }
    const float op = opacities[idx];
    const float* c = colors5 + 5 * static_cast<size_t>(idx);
    float4* rec = records + static_cast<size_t>(idx) * kRecordQuads;
    rec[0] = make_float4(g.xy.x, g.xy.y, g.normal.x, g.normal.y);
    rec[1] = make_float4(g.normal.z, op, c[0], c[1]);
    rec[2] = make_float4(c[2], c[3], c[4], g.tu.x);
    rec[3] = make_float4(g.tu.y, g.tu.z, g.tv.x, g.tv.y);
    rec[4] = make_float4(g.tv.z, g.tw.x, g.tw.y, g.tw.z);
    rects[idx] = make_uint2(g.rect_min.x | (g.rect_min.y << 16), g.rect_max.x | (g.rect_max.y << 16));
    radii[idx] = static_cast<int32_t>(g.radius);
    pair_counts[idx] = (g.rect_max.x - g.rect_min.x) * (g.rect_max.y - g.rect_min.y);
    depth_keys[idx] = __float_as_uint(g.depth);
}

__global__ void __launch_bounds__(kPreThreads) emit_kernel(
    int point_count, uint32_t grid_x, const uint32_t* __restrict__ order,
    const uint32_t* __restrict__ pair_counts, const uint32_t* __restrict__ offsets,
    const uint2* __restrict__ rects, uint32_t* __restrict__ tile_ids,
    uint32_t* __restrict__ gaussian_ids) {
    const int s = blockIdx.x * kPreThreads + threadIdx.x;
    if (s >= point_count) return;
    const uint32_t gid = order[s];
    if (pair_counts[gid] == 0) return;
    const uint2 rc = rects[gid];
    const uint32_t x0 = rc.x & 0xffff, y0 = rc.x >> 16, x1 = rc.y & 0xffff, y1 = rc.y >> 16;
    uint32_t out = offsets[s];
    for (uint32_t y = y0; y < y1; ++y) {
        for (uint32_t x = x0; x < x1; ++x) {
            tile_ids[out] = y * grid_x + x;
            gaussian_ids[out] = gid;
            ++out;
        }
    }
}

__global__ void ranges_kernel(uint32_t pair_count, const uint32_t* __restrict__ tile_ids,
                              uint2* __restrict__ ranges) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pair_count) return;
    const uint32_t t = tile_ids[i];
    if (i == 0) {
        ranges[t].x = 0;
    } else {
        const uint32_t prev = tile_ids[i - 1];
        if (t != prev) {
            ranges[prev].y = i;
            ranges[t].x = i;
        }
    }
    if (i == pair_count - 1) ranges[t].y = pair_count;
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

template <class R>
__global__ void __launch_bounds__(kRenderThreads) render_kernel(
    const uint2* __restrict__ ranges, const uint32_t* __restrict__ gaussian_ids,
    const float4* __restrict__ records, int width, int height, uint32_t grid_x,
    const float* __restrict__ background5, float* __restrict__ color, float* __restrict__ aux,
    float* __restrict__ weight) {
    __shared__ float4 batch[kBatch * kRecordQuads];
    __shared__ uint32_t batch_ids[kBatch];
    const R r;
    const uint32_t tile = blockIdx.x;
    const int tx = tile % grid_x, ty = tile / grid_x;
    const int lx = threadIdx.x & 15, ly = threadIdx.x >> 4;
    const int px = tx * 16 + lx, py0 = ty * 16 + ly, py1 = py0 + 8;
    const bool in0 = px < width && py0 < height;
    const bool in1 = px < width && py1 < height;
    const float fx = static_cast<float>(px);
    const float fy0 = static_cast<float>(py0), fy1 = static_cast<float>(py1);
    float bg[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) bg[k] = background5[k];
    PixelState s0, s1;
    pixel_init(s0, in0);
    pixel_init(s1, in1);
    const uint2 range = ranges[tile];
    const int n = static_cast<int>(range.y - range.x);
    const int lane = threadIdx.x & 31;
    for (int base = 0; base < n; base += kBatch) {
        // Stop once every pixel of the tile is done (forward.cu:326-328).
        if (__syncthreads_and(s0.done && s1.done)) break;
        const int nb = min(kBatch, n - base);
        for (int i = threadIdx.x; i < nb * kRecordQuads; i += kRenderThreads) {
            const int j = i / kRecordQuads, q = i - j * kRecordQuads;
            const uint32_t gid = gaussian_ids[range.x + base + j];
            if (q == 0) batch_ids[j] = gid;
            batch[i] = records[static_cast<size_t>(gid) * kRecordQuads + q];
        }
        __syncthreads();
        if (!__all_sync(0xffffffffu, s0.done && s1.done)) {
            for (int j = 0; j < nb; ++j) {
                const BlendRecord g = load_record(batch + j * kRecordQuads);
                float w = blend(r, s0, fx, fy0, g);
                w += blend(r, s1, fx, fy1, g);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) w += __shfl_xor_sync(0xffffffffu, w, off);
                if (lane == 0 && w != 0.0f) atomicAdd(weight + batch_ids[j], w);
            }
        }
        __syncthreads();
    }
    const size_t plane = static_cast<size_t>(width) * height;
    if (in0) store_pixel(r, s0, bg, color, aux, plane, static_cast<size_t>(py0) * width + px);
    if (in1) store_pixel(r, s1, bg, color, aux, plane, static_cast<size_t>(py1) * width + px);
}

}  // namespace st
}  // namespace hs
