// Elementwise kernels with fixed FP32 rounding: activations, SH colour, view
// direction, reflection-ray generation (prefix/suffix), disk rotation and the
// two-branch fusion.
//
// Each kernel restates the rounding steps of the reference kernel named in
// its comment. This file is compiled with --fmad=false (as the reference
// compiles rasterizer/precise_{activation,direction,disk_rotation,
// reflection_trace,sh}.cu, CMakeLists.txt:109-120), and every step is an
// explicit *_rn operation, so the results are bit-identical. The kernels are
// HBM-bound grid-stride loops sized to the SM count.
#include <cuda_runtime.h>

#include <cstdint>

#include "fp.cuh"
#include "fuse.cuh"
#include "precise.h"

namespace hs {
namespace precise {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float norm3_torch(float x, float y, float z) {
    // PyTorch's length-3 inner reduction adds (x^2 + z^2) + y^2
    // (precise_reflection_trace.cu:35-42).
    return __fsqrt_rn(add(add(mul(x, x), mul(z, z)), mul(y, y)));
}

__device__ __forceinline__ float norm4_torch(float a, float b, float c, float d) {
    // (a^2 + b^2) + (c^2 + d^2) (precise_reflection_trace.cu:44-55).
    return __fsqrt_rn(add(add(mul(a, a), mul(b, b)), add(mul(c, c), mul(d, d))));
}

__device__ __forceinline__ void normalize4_clamp(float& a, float& b, float& c, float& d,
                                                 float eps) {
    const float n = norm4_torch(a, b, c, d);
    const float den = n < eps ? eps : n;
    a = div(a, den);
    b = div(b, den);
    c = div(c, den);
    d = div(d, den);
}

// Two F.normalize-style passes of build_rotation (precise_reflection_trace.cu:
// 129-151, precise_disk_rotation.cu:68-92).
__device__ __forceinline__ void twice_normalized(const float* q, float& w, float& x, float& y,
                                                 float& z) {
    w = q[0];
    x = q[1];
    y = q[2];
    z = q[3];
    normalize4_clamp(w, x, y, z, 1.0e-12f);
    const float n = norm4_torch(w, x, y, z);
    w = div(w, n);
    x = div(x, n);
    y = div(y, n);
    z = div(z, n);
}

__global__ void sigmoid_kernel(const float* __restrict__ in, float* __restrict__ out,
                               uint64_t count) {
    // precise_activation.cu:11-17
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        out[i] = div(1.0f, add(1.0f, expf(sub(0.0f, in[i]))));
    }
}

__global__ void normalize4_kernel(const float* __restrict__ in, float* __restrict__ out,
                                  uint64_t count) {
    // precise_activation.cu:19-34
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        float a = in[4 * i], b = in[4 * i + 1], c = in[4 * i + 2], d = in[4 * i + 3];
        normalize4_clamp(a, b, c, d, 1.0e-12f);
        out[4 * i] = a;
        out[4 * i + 1] = b;
        out[4 * i + 2] = c;
        out[4 * i + 3] = d;
    }
}

__global__ void fuse_maps_kernel(const float* __restrict__ base, const float* __restrict__ refl,
                                 const float* __restrict__ specular, float* __restrict__ diffuse,
                                 float* __restrict__ final_rgb, float* __restrict__ stored,
                                 uint64_t values) {
    // precise_activation.cu:36-55
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < values;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const float s = specular[i / 3];
        const float dv = mul(base[i], sub(1.0f, s));
        const float rv = mul(mul(refl[i], s), 2.0f);
        diffuse[i] = dv;
        stored[i] = rv;
        final_rgb[i] = add(dv, mul(0.5f, rv));
    }
}

__global__ void direction_kernel(const float* __restrict__ points,
                                 const float* __restrict__ center, uint64_t count,
                                 float* __restrict__ out) {
    // precise_direction.cu:11-35
    const float cx = center[0], cy = center[1], cz = center[2];
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const float x = sub(points[3 * i], cx);
        const float y = sub(points[3 * i + 1], cy);
        const float z = sub(points[3 * i + 2], cz);
        const float n = norm3_torch(x, y, z);
        out[3 * i] = div(x, n);
        out[3 * i + 1] = div(y, n);
        out[3 * i + 2] = div(z, n);
    }
}

// One colour channel of precise_sh.cu:11-138: every product and sum rounded
// in source order. c points at the channel's coefficients.
__device__ __forceinline__ float sh_channel(const float* c, float x, float y, float z, float xx,
                                            float yy, float zz, float xy, float yz, float xz,
                                            uint32_t degree) {
    float r = mul(0.28209479177387814f, c[0]);
    if (degree > 0) {
        const float c1 = 0.4886025119029199f;
        r = sub(r, mul(mul(c1, y), c[1]));
        r = add(r, mul(mul(c1, z), c[2]));
        r = sub(r, mul(mul(c1, x), c[3]));
    }
    if (degree > 1) {
        r = add(r, mul(mul(1.0925484305920792f, xy), c[4]));
        r = add(r, mul(mul(-1.0925484305920792f, yz), c[5]));
        const float p6 = sub(sub(mul(2.0f, zz), xx), yy);
        r = add(r, mul(mul(0.31539156525252005f, p6), c[6]));
        r = add(r, mul(mul(-1.0925484305920792f, xz), c[7]));
        r = add(r, mul(mul(0.5462742152960396f, sub(xx, yy)), c[8]));
    }
    if (degree > 2) {
        const float p9 = sub(mul(3.0f, xx), yy);
        r = add(r, mul(mul(mul(-0.5900435899266435f, y), p9), c[9]));
        r = add(r, mul(mul(mul(2.890611442640554f, xy), z), c[10]));
        const float p11 = sub(sub(mul(4.0f, zz), xx), yy);
        r = add(r, mul(mul(mul(-0.4570457994644658f, y), p11), c[11]));
        const float p12 = sub(sub(mul(2.0f, zz), mul(3.0f, xx)), mul(3.0f, yy));
        r = add(r, mul(mul(mul(0.3731763325901154f, z), p12), c[12]));
        r = add(r, mul(mul(mul(-0.4570457994644658f, x), p11), c[13]));
        r = add(r, mul(mul(mul(1.445305721320277f, z), sub(xx, yy)), c[14]));
        const float p15 = sub(xx, mul(3.0f, yy));
        r = add(r, mul(mul(mul(-0.5900435899266435f, x), p15), c[15]));
    }
    return fmaxf(add(r, 0.5f), 0.0f);
}

// Any coefficient count and alignment.
__global__ void sh_to_rgb_kernel(const float* __restrict__ sh, const float* __restrict__ dirs,
                                 uint64_t count, uint32_t coefficients, uint32_t degree,
                                 float* __restrict__ out) {
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        const float x = dirs[3 * i], y = dirs[3 * i + 1], z = dirs[3 * i + 2];
        const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
        const float xy = mul(x, y), yz = mul(y, z), xz = mul(x, z);
        for (uint32_t ch = 0; ch < 3; ++ch) {
            out[3 * i + ch] = sh_channel(sh + (i * 3 + ch) * coefficients, x, y, z, xx, yy, zz,
                                         xy, yz, xz, degree);
        }
    }
}

// 16 coefficients per channel, 16-byte aligned rows. A block stages the
// 192-byte rows of its 128 Gaussians in shared memory with coalesced 128-bit
// loads (rows padded to 49 words so the per-thread reads do not conflict),
// then each thread evaluates its own Gaussian.
constexpr int kShThreads = 128;
constexpr int kShStride = 49;

template <uint32_t kDegree>
__global__ void __launch_bounds__(kShThreads) sh16_to_rgb_kernel(
    const float4* __restrict__ sh, const float* __restrict__ dirs, uint64_t count,
    float* __restrict__ out) {
    __shared__ float rows[kShThreads * kShStride];
    const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kShThreads;
    const uint64_t left = count - first;
    const uint32_t n = left < kShThreads ? static_cast<uint32_t>(left) : kShThreads;
    for (uint32_t f = threadIdx.x; f < n * 12; f += kShThreads) {
        const float4 v = sh[first * 12 + f];
        float* d = rows + (f / 12) * kShStride + (f % 12) * 4;
        d[0] = v.x;
        d[1] = v.y;
        d[2] = v.z;
        d[3] = v.w;
    }
    __syncthreads();
    if (threadIdx.x >= n) return;
    const uint64_t i = first + threadIdx.x;
    const float* c = rows + threadIdx.x * kShStride;
    const float x = dirs[3 * i], y = dirs[3 * i + 1], z = dirs[3 * i + 2];
    const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
    const float xy = mul(x, y), yz = mul(y, z), xz = mul(x, z);
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        out[3 * i + ch] = sh_channel(c + 16 * ch, x, y, z, xx, yy, zz, xy, yz, xz, kDegree);
    }
}

// View direction of one Gaussian, as direction_kernel computes it.
__device__ __forceinline__ void view_direction(const float* p, float cx, float cy, float cz,
                                               float& x, float& y, float& z) {
    const float dx = sub(p[0], cx), dy = sub(p[1], cy), dz = sub(p[2], cz);
    const float n = norm3_torch(dx, dy, dz);
    x = div(dx, n);
    y = div(dy, n);
    z = div(dz, n);
}

// The standard branch's colours in one pass: view direction (direction_kernel),
// SH colour (sh_to_rgb_kernel) and the [rgb, specular, roughness] concatenation
// that the reference performs in Jittor (renderer.py:260-266). Same rounding
// as the three steps, so colours5 is bit-identical to them.
__global__ void sh_colors5_kernel(const float* __restrict__ sh, uint32_t coefficients,
                                  uint32_t degree, const float* __restrict__ points,
                                  const float* __restrict__ center,
                                  const float* __restrict__ specular,
                                  const float* __restrict__ roughness, uint64_t count,
                                  float* __restrict__ out5) {
    const float cx = center[0], cy = center[1], cz = center[2];
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        float x, y, z;
        view_direction(points + 3 * i, cx, cy, cz, x, y, z);
        const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
        const float xy = mul(x, y), yz = mul(y, z), xz = mul(x, z);
        for (uint32_t ch = 0; ch < 3; ++ch) {
            out5[5 * i + ch] = sh_channel(sh + (i * 3 + ch) * coefficients, x, y, z, xx, yy, zz,
                                          xy, yz, xz, degree);
        }
        out5[5 * i + 3] = specular[i];
        out5[5 * i + 4] = roughness[i];
    }
}

// sh_colors5_kernel for 16 coefficients per channel in 16-byte aligned rows,
// staged through shared memory as in sh16_to_rgb_kernel: the work of one
// block (`block`, `rows` its kShThreads * kShStride shared floats).
struct ShColorsArgs {
    const float4* sh;
    const float* points;
    const float* center;
    const float* specular;
    const float* roughness;
    uint64_t count;
    float* out5;
};

template <uint32_t kDegree>
__device__ __forceinline__ void sh16_colors5_block(const ShColorsArgs& a, uint32_t block, float* rows) {
    const uint64_t first = static_cast<uint64_t>(block) * kShThreads;
    const uint64_t left = a.count - first;
    const uint32_t n = left < kShThreads ? static_cast<uint32_t>(left) : kShThreads;
    for (uint32_t f = threadIdx.x; f < n * 12; f += kShThreads) {
        const float4 v = a.sh[first * 12 + f];
        float* d = rows + (f / 12) * kShStride + (f % 12) * 4;
        d[0] = v.x;
        d[1] = v.y;
        d[2] = v.z;
        d[3] = v.w;
    }
    __syncthreads();
    if (threadIdx.x >= n) return;
    const uint64_t i = first + threadIdx.x;
    const float* c = rows + threadIdx.x * kShStride;
    float x, y, z;
    view_direction(a.points + 3 * i, a.center[0], a.center[1], a.center[2], x, y, z);
    const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
    const float xy = mul(x, y), yz = mul(y, z), xz = mul(x, z);
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        a.out5[5 * i + ch] = sh_channel(c + 16 * ch, x, y, z, xx, yy, zz, xy, yz, xz, kDegree);
    }
    a.out5[5 * i + 3] = a.specular[i];
    a.out5[5 * i + 4] = a.roughness[i];
}

template <uint32_t kDegree>
__global__ void __launch_bounds__(kShThreads) sh16_colors5_kernel(ShColorsArgs a) {
    __shared__ float rows[kShThreads * kShStride];
    sh16_colors5_block<kDegree>(a, blockIdx.x, rows);
}

// fuse_maps_kernel with channel-first inputs: base and reflection colours as
// three planes of `pixels` values each, the specular plane; the outputs are
// interleaved [pixels, 3] exactly as fuse_maps_kernel writes them. This
// replaces the three HWC transposes that precede fuse_maps in the reference
// session (renderer.py, math.py:301-311).
__global__ void fuse_maps_planar_kernel(const float* __restrict__ base,
                                        const float* __restrict__ refl,
                                        const float* __restrict__ specular,
                                        float* __restrict__ diffuse, float* __restrict__ final_rgb,
                                        float* __restrict__ stored, uint64_t pixels) {
    for (uint64_t p = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; p < pixels;
         p += uint64_t(gridDim.x) * blockDim.x) {
        fuse_planar_pixel(base, refl, specular[p], pixels, p, diffuse, final_rgb, stored);
    }
}

// precise_reflection_trace.cu:119-183: the matrix entries contract the
// leading product with the following add/sub (one fma each).
__device__ __forceinline__ void prefix_matrix(const float* q, float o[9]) {
    float w, x, y, z;
    twice_normalized(q, w, x, y, z);
    const float wz = mul(w, z), wy = mul(w, y), wx = mul(w, x);
    const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
    o[0] = sub(1.0f, mul(2.0f, fma(y, y, zz)));
    o[1] = mul(2.0f, fma(x, y, sub(0.0f, wz)));
    o[2] = mul(2.0f, fma(x, z, wy));
    o[3] = mul(2.0f, fma(x, y, wz));
    o[4] = sub(1.0f, mul(2.0f, fma(x, x, zz)));
    o[5] = mul(2.0f, fma(y, z, sub(0.0f, wx)));
    o[6] = mul(2.0f, fma(x, z, sub(0.0f, wy)));
    o[7] = mul(2.0f, fma(y, z, wx));
    o[8] = sub(1.0f, mul(2.0f, fma(x, x, yy)));
}

__global__ void reflection_prefix_kernel(const float* __restrict__ rot, uint64_t count,
                                         float* __restrict__ out) {
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        float o[9];
        prefix_matrix(rot + 4 * i, o);
#pragma unroll
        for (int k = 0; k < 9; ++k) out[9 * i + k] = o[k];
    }
}

__global__ void disk_rotation_kernel(const float* __restrict__ rot, uint64_t count,
                                     float* __restrict__ out) {
    // precise_disk_rotation.cu:58-125: every stage rounded separately.
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += uint64_t(gridDim.x) * blockDim.x) {
        float w, x, y, z;
        twice_normalized(rot + 4 * i, w, x, y, z);
        const float xy = mul(x, y), xz = mul(x, z), yz = mul(y, z);
        const float wz = mul(w, z), wy = mul(w, y), wx = mul(w, x);
        const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
        float* o = out + 9 * i;
        o[0] = sub(1.0f, mul(2.0f, add(yy, zz)));
        o[1] = mul(2.0f, sub(xy, wz));
        o[2] = mul(2.0f, add(xz, wy));
        o[3] = mul(2.0f, add(xy, wz));
        o[4] = sub(1.0f, mul(2.0f, add(xx, zz)));
        o[5] = mul(2.0f, sub(yz, wx));
        o[6] = mul(2.0f, sub(xz, wy));
        o[7] = mul(2.0f, add(yz, wx));
        o[8] = sub(1.0f, mul(2.0f, add(xx, yy)));
    }
}

// normalize with "+ eps" in the denominator (math_utils normalize).
__device__ __forceinline__ float normalize3_add(float& x, float& y, float& z) {
    const float den = add(norm3_torch(x, y, z), 1.0e-8f);
    x = div(x, den);
    y = div(y, den);
    z = div(z, den);
    return den;
}

// One thread per reflective Gaussian; the block's 36-float output rows are
// staged in shared memory (padded to 37 words) and written with coalesced
// stores.
constexpr int kSuffixThreads = 128;
constexpr int kSuffixStride = 37;

// precise_reflection_trace.cu:185-330: the 36-float row of one reflective
// Gaussian at p with raw normal n, seen from camera centre c.
__device__ __forceinline__ void suffix_row(float px, float py, float pz, float cx, float cy, float cz,
                                           float inx, float iny, float inz, float values[36]) {
    float vx = sub(cx, px), vy = sub(cy, py), vz = sub(cz, pz);
    normalize3_add(vx, vy, vz);
    // Facing flip against -(p - c), dot reduced as (x + z) + y.
    const float tx = sub(0.0f, sub(px, cx));
    const float ty = sub(0.0f, sub(py, cy));
    const float tz = sub(0.0f, sub(pz, cz));
    const float flip_dot = add(add(mul(inx, tx), mul(inz, tz)), mul(iny, ty));
    const bool positive = flip_dot >= 0.0f;
    const float sign = positive ? 1.0f : -1.0f;
    const float nrx = mul(inx, sign), nry = mul(iny, sign), nrz = mul(inz, sign);
    const float nn = norm3_torch(nrx, nry, nrz);
    const float nden = nn < 1.0e-20f ? 1.0e-20f : nn;
    const float nx = div(nrx, nden), ny = div(nry, nden), nz = div(nrz, nden);
    const float rpx = mul(nx, vx), rpy = mul(ny, vy), rpz = mul(nz, vz);
    const float dot_nv = add(add(rpx, rpz), rpy);
    const float two_dot = mul(2.0f, dot_nv);
    const float snx = mul(two_dot, nx), sny = mul(two_dot, ny), snz = mul(two_dot, nz);
    const float rx = sub(snx, vx), ry = sub(sny, vy), rz = sub(snz, vz);
    float dx = rx, dy = ry, dz = rz;
    const float ray_den = normalize3_add(dx, dy, dz);
    const float ox = mul(0.05f, dx), oy = mul(0.05f, dy), oz = mul(0.05f, dz);
    const float row[36] = {vx,  vy,  vz,  nx,  ny,  nz,  rx,  ry,  rz,
                           dx,  dy,  dz,  add(px, ox), add(py, oy), add(pz, oz),
                           positive ? 1.0f : 0.0f,
                           inx, iny, inz, nrx, nry, nrz, nden, rpx, rpy, rpz,
                           dot_nv, two_dot, snx, sny, snz, ray_den, ox, oy, oz,
                           flip_dot};
#pragma unroll
    for (int k = 0; k < 36; ++k) values[k] = row[k];
}

// The block's 36-float rows, staged in shared memory (padded to 37 words),
// written with coalesced stores.
__device__ __forceinline__ void store_rows(const float* rows, uint64_t first, uint32_t n, float* out36) {
    float* dst = out36 + first * 36;
    for (uint32_t f = threadIdx.x; f < n * 36; f += kSuffixThreads) {
        dst[f] = rows[(f / 36) * kSuffixStride + f % 36];
    }
}

__global__ void __launch_bounds__(kSuffixThreads) reflection_suffix_kernel(
    const float* __restrict__ xyz, const float* __restrict__ center,
    const float* __restrict__ normal_raw, uint64_t count, float* __restrict__ out36) {
    __shared__ float rows[kSuffixThreads * kSuffixStride];
    const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kSuffixThreads;
    const uint64_t left = count - first;
    const uint32_t n = left < kSuffixThreads ? static_cast<uint32_t>(left) : kSuffixThreads;
    if (threadIdx.x < n) {
        const uint64_t i = first + threadIdx.x;
        float values[36];
        suffix_row(xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], center[0], center[1], center[2],
                   normal_raw[3 * i], normal_raw[3 * i + 1], normal_raw[3 * i + 2], values);
        float* row = rows + threadIdx.x * kSuffixStride;
#pragma unroll
        for (int k = 0; k < 36; ++k) row[k] = values[k];
    }
    __syncthreads();
    store_rows(rows, first, n, out36);
}

// One view's reflection preparation in one pass (renderer.py:267-280): the
// prefix rotation rot9, its third column normal3 (the raw normal), the
// suffix row out36 and, when the pointers are given, the trace's ray origins
// (row columns 12..14) and directions (9..11) and the raster colours
// colors5 = [rgb3, specular, roughness]. Each value is computed by the same
// functions as the separate kernels, so they are bit-identical to them.
struct ReflectionViewArgs {
    const float* rot_raw;
    const float* xyz;
    const float* center;
    uint64_t count;
    float* rot9;
    float* normal3;
    float* out36;
    float* origins3;
    float* directions3;
    const float* rgb3;
    const float* specular;
    const float* roughness;
    float* colors5;
};

// The work of one block (`rows`: kSuffixThreads * kSuffixStride shared floats).
__device__ __forceinline__ void reflection_view_block(const ReflectionViewArgs& a, uint32_t block, float* rows) {
    const uint64_t first = static_cast<uint64_t>(block) * kSuffixThreads;
    const uint64_t left = a.count - first;
    const uint32_t n = left < kSuffixThreads ? static_cast<uint32_t>(left) : kSuffixThreads;
    if (threadIdx.x < n) {
        const uint64_t i = first + threadIdx.x;
        float o[9];
        prefix_matrix(a.rot_raw + 4 * i, o);
#pragma unroll
        for (int k = 0; k < 9; ++k) a.rot9[9 * i + k] = o[k];
        a.normal3[3 * i] = o[2];
        a.normal3[3 * i + 1] = o[5];
        a.normal3[3 * i + 2] = o[8];
        float values[36];
        suffix_row(a.xyz[3 * i], a.xyz[3 * i + 1], a.xyz[3 * i + 2], a.center[0], a.center[1], a.center[2], o[2],
                   o[5], o[8], values);
        if (a.origins3 != nullptr) {
            for (int c = 0; c < 3; ++c) {
                a.origins3[3 * i + c] = values[12 + c];
                a.directions3[3 * i + c] = values[9 + c];
            }
        }
        if (a.colors5 != nullptr) {
            a.colors5[5 * i] = a.rgb3[3 * i];
            a.colors5[5 * i + 1] = a.rgb3[3 * i + 1];
            a.colors5[5 * i + 2] = a.rgb3[3 * i + 2];
            a.colors5[5 * i + 3] = a.specular[i];
            a.colors5[5 * i + 4] = a.roughness[i];
        }
        float* row = rows + threadIdx.x * kSuffixStride;
#pragma unroll
        for (int k = 0; k < 36; ++k) row[k] = values[k];
    }
    __syncthreads();
    store_rows(rows, first, n, a.out36);
}

__global__ void __launch_bounds__(kSuffixThreads) reflection_view_kernel(ReflectionViewArgs a) {
    __shared__ float rows[kSuffixThreads * kSuffixStride];
    reflection_view_block(a, blockIdx.x, rows);
}

// A view's prologue in one grid: blocks [0, sh_blocks) compute the base
// colours (sh16_colors5_block), the rest the reflection preparation
// (reflection_view_block); the two are independent and run side by side.
static_assert(kShThreads == kSuffixThreads, "one block size for both parts of the prologue");
constexpr int kPrologueRows =
    kShThreads * kShStride > kSuffixThreads * kSuffixStride ? kShThreads * kShStride : kSuffixThreads * kSuffixStride;

template <uint32_t kDegree>
__global__ void __launch_bounds__(kShThreads) view_prologue_kernel(ShColorsArgs a, ReflectionViewArgs b,
                                                                   uint32_t sh_blocks) {
    __shared__ float rows[kPrologueRows];
    if (blockIdx.x < sh_blocks) {
        sh16_colors5_block<kDegree>(a, blockIdx.x, rows);
    } else {
        reflection_view_block(b, blockIdx.x - sh_blocks, rows);
    }
}

unsigned grid_for(uint64_t count) {
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    const uint64_t needed = (count + kThreads - 1) / kThreads;
    const uint64_t cap = static_cast<uint64_t>(sms) * 8;
    return static_cast<unsigned>(needed < cap ? (needed > 0 ? needed : 1) : cap);
}

}  // namespace

cudaError_t sigmoid(const float* in, float* out, uint64_t count, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    sigmoid_kernel<<<grid_for(count), kThreads, 0, s>>>(in, out, count);
    return cudaGetLastError();
}

cudaError_t normalize4(const float* in, float* out, uint64_t count, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    normalize4_kernel<<<grid_for(count), kThreads, 0, s>>>(in, out, count);
    return cudaGetLastError();
}

cudaError_t fuse_maps(const float* base, const float* refl, const float* specular,
                      float* diffuse, float* final_rgb, float* stored, uint64_t pixels,
                      cudaStream_t s) {
    if (pixels == 0) return cudaSuccess;
    if (pixels > UINT64_MAX / 3) return cudaErrorInvalidValue;
    fuse_maps_kernel<<<grid_for(pixels * 3), kThreads, 0, s>>>(base, refl, specular, diffuse,
                                                                final_rgb, stored, pixels * 3);
    return cudaGetLastError();
}

cudaError_t direction(const float* points, const float* center, uint64_t count, float* out,
                      cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    direction_kernel<<<grid_for(count), kThreads, 0, s>>>(points, center, count, out);
    return cudaGetLastError();
}

cudaError_t sh_to_rgb(const float* sh, const float* dirs, uint64_t count, uint32_t coefficients,
                      uint32_t degree, float* out, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    if (coefficients == 16 && (reinterpret_cast<uintptr_t>(sh) & 15u) == 0 && degree <= 3) {
        const unsigned blocks = static_cast<unsigned>((count + kShThreads - 1) / kShThreads);
        const float4* sh4 = reinterpret_cast<const float4*>(sh);
        switch (degree) {
            case 0: sh16_to_rgb_kernel<0><<<blocks, kShThreads, 0, s>>>(sh4, dirs, count, out); break;
            case 1: sh16_to_rgb_kernel<1><<<blocks, kShThreads, 0, s>>>(sh4, dirs, count, out); break;
            case 2: sh16_to_rgb_kernel<2><<<blocks, kShThreads, 0, s>>>(sh4, dirs, count, out); break;
            default: sh16_to_rgb_kernel<3><<<blocks, kShThreads, 0, s>>>(sh4, dirs, count, out); break;
        }
        return cudaGetLastError();
    }
    sh_to_rgb_kernel<<<grid_for(count), kThreads, 0, s>>>(sh, dirs, count, coefficients, degree,
                                                           out);
    return cudaGetLastError();
}

cudaError_t sh_colors5(const float* sh, uint32_t coefficients, uint32_t degree,
                      const float* points, const float* center, const float* specular,
                      const float* roughness, uint64_t count, float* out5, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    if (coefficients == 16 && (reinterpret_cast<uintptr_t>(sh) & 15u) == 0 && degree <= 3) {
        const unsigned blocks = static_cast<unsigned>((count + kShThreads - 1) / kShThreads);
        const ShColorsArgs a{reinterpret_cast<const float4*>(sh), points, center, specular, roughness, count, out5};
        switch (degree) {
            case 0: sh16_colors5_kernel<0><<<blocks, kShThreads, 0, s>>>(a); break;
            case 1: sh16_colors5_kernel<1><<<blocks, kShThreads, 0, s>>>(a); break;
            case 2: sh16_colors5_kernel<2><<<blocks, kShThreads, 0, s>>>(a); break;
            default: sh16_colors5_kernel<3><<<blocks, kShThreads, 0, s>>>(a); break;
        }
        return cudaGetLastError();
    }
    sh_colors5_kernel<<<grid_for(count), kThreads, 0, s>>>(sh, coefficients, degree, points, center,
                                                            specular, roughness, count, out5);
    return cudaGetLastError();
}

cudaError_t fuse_maps_planar(const float* base, const float* refl, const float* specular,
                             float* diffuse, float* final_rgb, float* stored, uint64_t pixels,
                             cudaStream_t s) {
    if (pixels == 0) return cudaSuccess;
    if (pixels > UINT64_MAX / 3) return cudaErrorInvalidValue;
    fuse_maps_planar_kernel<<<grid_for(pixels), kThreads, 0, s>>>(base, refl, specular, diffuse,
                                                                    final_rgb, stored, pixels);
    return cudaGetLastError();
}

cudaError_t reflection_prefix(const float* rot, uint64_t count, float* out, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    reflection_prefix_kernel<<<grid_for(count), kThreads, 0, s>>>(rot, count, out);
    return cudaGetLastError();
}

cudaError_t disk_rotation(const float* rot, uint64_t count, float* out, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    disk_rotation_kernel<<<grid_for(count), kThreads, 0, s>>>(rot, count, out);
    return cudaGetLastError();
}

cudaError_t reflection_suffix(const float* xyz, const float* center, const float* normal_raw,
                              uint64_t count, float* out36, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    reflection_suffix_kernel<<<static_cast<unsigned>((count + kSuffixThreads - 1) / kSuffixThreads),
                               kSuffixThreads, 0, s>>>(xyz, center, normal_raw, count, out36);
    return cudaGetLastError();
}

cudaError_t reflection_view(const float* rot_raw, const float* xyz, const float* center, uint64_t count,
                            float* rot9, float* normal3, float* out36, float* origins3, float* directions3,
                            const float* rgb3, const float* specular, const float* roughness, float* colors5,
                            cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    const ReflectionViewArgs a{rot_raw, xyz,         center, count,    rot9,      normal3, out36,
                               origins3, directions3, rgb3,  specular, roughness, colors5};
    reflection_view_kernel<<<static_cast<unsigned>((count + kSuffixThreads - 1) / kSuffixThreads),
                             kSuffixThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t view_prologue(const float* sh, uint32_t coefficients, uint32_t degree, const float* points,
                          const float* center, const float* specular, const float* roughness, uint64_t count,
                          float* out5, const float* rot_raw, const float* xyz, uint64_t reflection_count,
                          float* rot9, float* normal3, float* out36, float* origins3, float* directions3,
                          const float* rgb3, const float* reflection_specular, const float* reflection_roughness,
                          float* colors5, cudaStream_t s) {
    const uint64_t sh_blocks = (count + kShThreads - 1) / kShThreads;
    const uint64_t refl_blocks = (reflection_count + kSuffixThreads - 1) / kSuffixThreads;
    const bool fused = coefficients == 16 && (reinterpret_cast<uintptr_t>(sh) & 15u) == 0 && degree <= 3 &&
                       count != 0 && reflection_count != 0 && sh_blocks + refl_blocks <= 0x7fffffffu;
    if (!fused) {
        cudaError_t e = sh_colors5(sh, coefficients, degree, points, center, specular, roughness, count, out5, s);
        if (e == cudaSuccess) {
            e = reflection_view(rot_raw, xyz, center, reflection_count, rot9, normal3, out36, origins3,
                                directions3, rgb3, reflection_specular, reflection_roughness, colors5, s);
        }
        return e;
    }
    const ShColorsArgs a{reinterpret_cast<const float4*>(sh), points, center, specular, roughness, count, out5};
    const ReflectionViewArgs b{rot_raw,  xyz,         center, reflection_count,    rot9,
                               normal3,  out36,       origins3, directions3,       rgb3,
                               reflection_specular, reflection_roughness, colors5};
    const unsigned blocks = static_cast<unsigned>(sh_blocks + refl_blocks);
    const uint32_t split = static_cast<uint32_t>(sh_blocks);
    switch (degree) {
        case 0: view_prologue_kernel<0><<<blocks, kShThreads, 0, s>>>(a, b, split); break;
        case 1: view_prologue_kernel<1><<<blocks, kShThreads, 0, s>>>(a, b, split); break;
        case 2: view_prologue_kernel<2><<<blocks, kShThreads, 0, s>>>(a, b, split); break;
        default: view_prologue_kernel<3><<<blocks, kShThreads, 0, s>>>(a, b, split); break;
    }
    return cudaGetLastError();
}

}  // namespace precise
}  // namespace hs
