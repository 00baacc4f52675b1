// Raw-map postprocess of one view: the session's per-pixel steps after the
// raster calls, fused into one pass per backend.
//
// Standard backend, postprocess_raster (math.py:426-463) with depth_to_normal
// (math.py:351-423): from color[5,H,W] and aux[7,H,W] (depth, alpha,
// normal[3], median depth, distortion) it writes the session's flattened HWC
// maps
//   rgb[HW,3], acc[HW], dpt[HW], norm[HW,3], surf_norm[HW,3], dist[HW],
//   spec[HW], rough[HW]
// where
//   dpt        = precise_depth_divide(depth, alpha) * (1 - ratio)
//                + nan_to_num(median) * ratio
//   norm       = normal @ B           (B = world_view_transform[:3,:3]^T)
//   xyz        = dpt * ray + origin   (ray: the per-view world-space pixel rays
//                                      from the two TF32 GEMMs of
//                                      depth_to_normal, origin = c2w[:3,3])
//   surf_norm  = safe_normalize((xyz[y+1]-xyz[y-1]) x (xyz[x+1]-xyz[x-1]),
//                               eps 1e-12) * alpha, zero on the image border
// The divide, the non-finite mappings, the ray scaling and offset and the
// finite differences are the reference's exactly rounded operations (each a
// separate PyTorch/Jittor kernel there). The reference leaves the contraction
// of the 3-term normal rotation, the cross product and the squared norm to
// Jittor's code generator; here they are written as explicitly rounded
// products and sums (no fused multiply-add).
//
// FlashGS backend, _flashgs_postprocess (renderer.py:176-202): rgb, acc, dpt
// (nan_to_num(precise_depth_divide(depth, alpha))), norm (normal @ B), spec
// (other[0]); surf_norm and dist are zero.
#include <cuda_runtime.h>

#include <cstdint>

#include "fp.cuh"
#include "fuse.cuh"
#include "postprocess.h"

namespace hs {
namespace post {
namespace {

constexpr int kThreads = 256;

// _nan_to_num_like_pytorch (math.py:331-336): NaN and +inf -> 0, -inf -> -FLT_MAX.
__device__ __forceinline__ float nan_to_num_session(float v) {
    const uint32_t b = __float_as_uint(v);
    if ((b & 0x7f800000u) != 0x7f800000u) return v;
    return ((b & 0x007fffffu) != 0u || (b & 0x80000000u) == 0u) ? 0.0f : __uint_as_float(0xff7fffffu);
}

// precise_depth_divide (ops/jittor/precise_depth_divide_op.cc): the correctly
// rounded quotient with the same non-finite mapping.
__device__ __forceinline__ float depth_divide(float numerator, float denominator) {
    return nan_to_num_session(div(numerator, denominator));
}

__device__ __forceinline__ float surface_depth(const float* aux, size_t plane, size_t p,
                                               float keep, float ratio) {
    const float expected = depth_divide(aux[p], aux[plane + p]);
    const float median = nan_to_num_session(aux[5 * plane + p]);
    return add(mul(expected, keep), mul(median, ratio));
}

// xyz = depth * ray + origin of pixel q (the two rounded steps of
// depth_to_normal, math.py:409-413).
__device__ __forceinline__ void world_point(const float* aux, const float* rays, size_t plane,
                                            size_t q, float keep, float ratio, const float o[3],
                                            float out[3]) {
    const float d = surface_depth(aux, plane, q, keep, ratio);
#pragma unroll
    for (int c = 0; c < 3; ++c) out[c] = add(mul(d, rays[3 * q + c]), o[c]);
}

// n @ B for a row vector n and a row-major 3x3 B.
__device__ __forceinline__ void rotate(const float n[3], const float* b, float out[3]) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        out[j] = add(add(mul(n[0], b[j]), mul(n[1], b[3 + j])), mul(n[2], b[6 + j]));
    }
}

__global__ void __launch_bounds__(kThreads) pixel_grid_kernel(int width, int height,
                                                              float* __restrict__ out3) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    for (uint64_t p = blockIdx.x * uint64_t(kThreads) + threadIdx.x; p < pixels;
         p += uint64_t(gridDim.x) * kThreads) {
        out3[3 * p] = static_cast<float>(p % width);
        out3[3 * p + 1] = static_cast<float>(p / width);
        out3[3 * p + 2] = 1.0f;
    }
}

// One pixel of the standard maps (see the file comment).
__device__ __forceinline__ void standard_pixel(int width, int height, size_t plane, size_t p,
                                               const float* __restrict__ color, const float* __restrict__ aux,
                                               const float* __restrict__ rays, const float* o, const float* b,
                                               float keep, float ratio, const StandardMaps& maps) {
    const int x = static_cast<int>(p % width), y = static_cast<int>(p / width);
    const float alpha = aux[plane + p];
    const float depth = surface_depth(aux, plane, p, keep, ratio);
    const float n[3] = {aux[2 * plane + p], aux[3 * plane + p], aux[4 * plane + p]};
    float nr[3];
    rotate(n, b, nr);
    float s[3] = {0.0f, 0.0f, 0.0f};
    if (x > 0 && y > 0 && x < width - 1 && y < height - 1) {
        // xyz of the four neighbours, then the central differences
        float up[3], down[3], left[3], right[3];
        world_point(aux, rays, plane, p - width, keep, ratio, o, up);
        world_point(aux, rays, plane, p + width, keep, ratio, o, down);
        world_point(aux, rays, plane, p - 1, keep, ratio, o, left);
        world_point(aux, rays, plane, p + 1, keep, ratio, o, right);
        float dx[3], dy[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            dx[c] = sub(down[c], up[c]);
            dy[c] = sub(right[c], left[c]);
        }
        const float cr[3] = {sub(mul(dx[1], dy[2]), mul(dx[2], dy[1])),
                             sub(mul(dx[2], dy[0]), mul(dx[0], dy[2])),
                             sub(mul(dx[0], dy[1]), mul(dx[1], dy[0]))};
        // norm.maximum(eps) with PyTorch's NaN propagation (fmaxf would drop a NaN)
        const float length = __fsqrt_rn(add(add(mul(cr[0], cr[0]), mul(cr[1], cr[1])), mul(cr[2], cr[2])));
        const float norm = isnan(length) ? length : fmaxf(length, 1e-12f);
#pragma unroll
        for (int c = 0; c < 3; ++c) s[c] = div(cr[c], norm);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        maps.rgb3[3 * p + c] = color[c * plane + p];
        maps.norm3[3 * p + c] = nr[c];
        maps.surf_norm3[3 * p + c] = mul(s[c], alpha);
    }
    maps.acc[p] = alpha;
    maps.dpt[p] = depth;
    maps.dist[p] = aux[6 * plane + p];
    maps.spec[p] = color[3 * plane + p];
    maps.rough[p] = color[4 * plane + p];
}

// The maps alone (kFuse false) or, for the one-view entry, with the colour
// fusion of the same pixel from the base call's colour planes 0..3 and the
// reflection call's planes 0..2 (fuse_planar_pixel), in one pass.
template <bool kFuse>
__global__ void __launch_bounds__(kThreads) standard_kernel(
    int width, int height, const float* __restrict__ color, const float* __restrict__ aux,
    const float* __restrict__ rays, const float* __restrict__ origin3,
    const float* __restrict__ rotation9, float keep, float ratio, StandardMaps maps,
    const float* __restrict__ refl_color, float* __restrict__ diffuse, float* __restrict__ final_rgb,
    float* __restrict__ stored) {
    const size_t plane = static_cast<size_t>(width) * height;
    float b[9], o[3];
#pragma unroll
    for (int k = 0; k < 9; ++k) b[k] = rotation9[k];
#pragma unroll
    for (int k = 0; k < 3; ++k) o[k] = origin3[k];
    for (size_t p = blockIdx.x * size_t(kThreads) + threadIdx.x; p < plane;
         p += size_t(gridDim.x) * kThreads) {
        standard_pixel(width, height, plane, p, color, aux, rays, o, b, keep, ratio, maps);
        if (kFuse) fuse_planar_pixel(color, refl_color, color[3 * plane + p], plane, p, diffuse, final_rgb, stored);
    }
}

// kFromView: `rotation` is the row-major world_view_transform (4 x 4) and the
// normal rotation world_view[:3,:3]^T is read from it in place.
// kFuse: also the colour fusion of the pixel from color3, refl_color3 and the
// specular plane other2[0] (fuse_planar_pixel), for the one-view entry.
template <bool kFromView, bool kFuse>
__global__ void __launch_bounds__(kThreads) flashgs_kernel(
    int width, int height, const float* __restrict__ color3, const float* __restrict__ other2,
    const float* __restrict__ depth1, const float* __restrict__ alpha1,
    const float* __restrict__ normal3, const float* __restrict__ rotation, FlashgsMaps maps,
    const float* __restrict__ refl_color3, float* __restrict__ diffuse, float* __restrict__ final_rgb,
    float* __restrict__ stored) {
    const size_t plane = static_cast<size_t>(width) * height;
    float b[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) b[k] = kFromView ? rotation[4 * (k % 3) + k / 3] : rotation[k];
    for (size_t p = blockIdx.x * size_t(kThreads) + threadIdx.x; p < plane;
         p += size_t(gridDim.x) * kThreads) {
        const float alpha = alpha1[p];
        const float n[3] = {normal3[p], normal3[plane + p], normal3[2 * plane + p]};
        float nr[3];
        rotate(n, b, nr);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            maps.rgb3[3 * p + c] = color3[c * plane + p];
            maps.norm3[3 * p + c] = nr[c];
            if (maps.surf_norm3 != nullptr) maps.surf_norm3[3 * p + c] = 0.0f;
        }
        maps.acc[p] = alpha;
        maps.dpt[p] = depth_divide(depth1[p], alpha);
        maps.spec[p] = other2[p];
        if (maps.dist != nullptr) maps.dist[p] = 0.0f;
        if (kFuse) fuse_planar_pixel(color3, refl_color3, other2[p], plane, p, diffuse, final_rgb, stored);
    }
}

// ---- N x 3 by 3 x 3 products on the tensor cores (TF32) ----
//
// The reference forms these products with cublasSgemm(OP_T, OP_N, m = 3,
// n = N, k = 3) under CUBLAS_TF32_TENSOR_OP_MATH (precise_matmul_nt_n3k3,
// c_api.cpp:1673); on B200 that runs a CUTLASS-style TF32 tensor-op GEMM
// with m16n8k8 MMAs. Its results are reproduced bit for bit by: operands
// rounded from FP32 to TF32 to nearest, ties to even (CUTLASS's
// round_to_nearest conversion for these targets; measured against the
// reference library's cuBLAS results, where rounding half away from zero
// and truncation both disagree), one m16n8k8 MMA per output block with the
// three products in k slots 0..2 and zeros after them, FP32 accumulation
// from zero, alpha = 1 and beta = 0. The warp below issues that instruction
// with the GEMM's operand placement: A = the 3 x 3 matrix (rows = output
// components, the GEMM's m), B = eight rows of the N x 3 operand (the
// GEMM's n). For fewer than kMmaMinRows rows cuBLAS takes another path, and
// the callers keep cuBLAS there.

// FP32 -> TF32 (10-bit mantissa), round to nearest even; infinities and NaNs
// pass unchanged (the MMA reads only the top 19 bits).
__device__ __forceinline__ uint32_t tf32_rne(float x) {
    const uint32_t b = __float_as_uint(x);
    if ((b & 0x7f800000u) == 0x7f800000u) return b;
    return (b + 0xfffu + ((b >> 13) & 1u)) & 0xffffe000u;
}

// D = A(16x8, rows g / g+8, cols t / t+4) * B(8x8, rows t / t+4, col g), C = 0.
__device__ __forceinline__ void mma_tf32_k8(float d[4], uint32_t a0, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(0u), "r"(0u), "r"(0u), "r"(b0), "r"(0u), "f"(0.0f));
}

// Lane (g = lane / 4, t = lane % 4) holds A[g][t] of the 3 x 3 matrix.
__device__ __forceinline__ uint32_t matrix_fragment(const float* m3x3, int lane) {
    const int g = lane >> 2, t = lane & 3;
    return (g < 3 && t < 3) ? tf32_rne(m3x3[3 * g + t]) : 0u;
}

// After mma_tf32_k8, lane (g, t) holds out[row 2t][g] in d[0] and
// out[row 2t + 1][g] in d[1] for g < 3. Returns component t of row g (the B
// fragment of a following product; t == 3 gives 0).
__device__ __forceinline__ float transpose_fragment(const float d[4], int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int src = (t < 3 ? t : 0) * 4 + (g >> 1);
    const float v0 = __shfl_sync(0xffffffffu, d[0], src);
    const float v1 = __shfl_sync(0xffffffffu, d[1], src);
    return t < 3 ? ((g & 1) ? v1 : v0) : 0.0f;
}

__device__ __forceinline__ void store_fragment(const float d[4], uint64_t row0, uint64_t rows,
                                               float* __restrict__ out3, int lane) {
    const int g = lane >> 2, t = lane & 3;
    if (g >= 3) return;
    const uint64_t r0 = row0 + 2u * t, r1 = r0 + 1u;
    if (r0 < rows) out3[3 * r0 + g] = d[0];
    if (r1 < rows) out3[3 * r1 + g] = d[1];
}

constexpr int kMmaRowsPerWarp = 32;  // four groups of eight rows per loop trip

// out[i] = left[i] @ right^T for N rows, or, when kPixels, the world rays of
// the pixel grid: ((x, y, 1) @ first^T) @ second^T, both products rounded as
// above and the intermediate kept in FP32 between them (the reference's two
// GEMMs through a scratch buffer).
template <bool kPixels>
__global__ void __launch_bounds__(kThreads) tf32_rows3_kernel(
    uint64_t rows, int width, const float* __restrict__ left3, const float* __restrict__ first,
    const float* __restrict__ second, float* __restrict__ out3) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t a_first = matrix_fragment(first, lane);
    const uint32_t a_second = kPixels ? matrix_fragment(second, lane) : 0u;
    const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (kThreads / 32);
    for (uint64_t base = (static_cast<uint64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5)) *
                         kMmaRowsPerWarp;
         base < rows; base += warps * kMmaRowsPerWarp) {
#pragma unroll
        for (int group = 0; group < kMmaRowsPerWarp / 8; ++group) {
            const uint64_t row0 = base + 8u * group;
            const uint64_t row = row0 + g;  // this lane's B row
            uint32_t b0 = 0u;
            if (row < rows && t < 3) {
                float v;
                if (kPixels) {
                    // pixel images hold fewer than 2^32 pixels (pixel_rays), so
                    // the column and row come from a 32-bit division
                    const uint32_t r32 = static_cast<uint32_t>(row), w32 = static_cast<uint32_t>(width);
                    v = t == 0 ? static_cast<float>(r32 % w32) : (t == 1 ? static_cast<float>(r32 / w32) : 1.0f);
                } else {
                    v = left3[3 * row + t];
                }
                b0 = tf32_rne(v);
            }
            float d[4];
            mma_tf32_k8(d, a_first, b0);
            if (kPixels) {
                const float cam = transpose_fragment(d, lane);
                const uint32_t b1 = (row < rows && t < 3) ? tf32_rne(cam) : 0u;
                mma_tf32_k8(d, a_second, b1);
            }
            store_fragment(d, row0, rows, out3, lane);
        }
    }
}

__global__ void camera_inputs_kernel(float fx, float cx, float fy, float cy, const float* __restrict__ wv,
                                     float* __restrict__ k9, float* __restrict__ wt16) {
    const int i = threadIdx.x;
    if (i < 9) {
        const float k[9] = {fx, 0.0f, cx, 0.0f, fy, cy, 0.0f, 0.0f, 1.0f};
        k9[i] = k[i];
    }
    if (i < 16) wt16[i] = wv[4 * (i % 4) + i / 4];
}

__global__ void camera_pack_kernel(const float* __restrict__ c2w, const float* __restrict__ wv,
                                   float* __restrict__ out) {
    const int i = threadIdx.x;
    if (i < 9) {
        const int r = i / 3, c = i % 3;
        out[9 + i] = c2w[4 * r + c];    // rotation c2w[:3,:3]
        out[21 + i] = wv[4 * c + r];    // normal rotation world_view[:3,:3]^T
    }
    if (i < 3) out[18 + i] = c2w[4 * i + 3];  // origin c2w[:3,3]
}

unsigned mma_grid_for(uint64_t rows) {
    const uint64_t warps = (rows + kMmaRowsPerWarp - 1) / kMmaRowsPerWarp;
    const uint64_t blocks = (warps + kThreads / 32 - 1) / (kThreads / 32);
    return static_cast<unsigned>(blocks < 148u * 8u ? (blocks > 0 ? blocks : 1) : 148u * 8u);
}

unsigned grid_for(uint64_t items) {
    const uint64_t blocks = (items + kThreads - 1) / kThreads;
    return static_cast<unsigned>(blocks < 148u * 16u ? (blocks > 0 ? blocks : 1) : 148u * 16u);
}

}  // namespace

cudaError_t pixel_grid(int width, int height, float* out3, cudaStream_t s) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    if (pixels == 0) return cudaSuccess;
    pixel_grid_kernel<<<grid_for(pixels), kThreads, 0, s>>>(width, height, out3);
    return cudaGetLastError();
}

cudaError_t pixel_rays(int width, int height, const float* inverse_intrinsics3x3,
                       const float* rotation3x3, float* rays3, cudaStream_t s) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    if (pixels == 0) return cudaSuccess;
    if (pixels > UINT32_MAX) return cudaErrorInvalidValue;
    tf32_rows3_kernel<true><<<mma_grid_for(pixels), kThreads, 0, s>>>(
        pixels, width, nullptr, inverse_intrinsics3x3, rotation3x3, rays3);
    return cudaGetLastError();
}

cudaError_t matmul_nt_n3k3(const float* left_n3, const float* right3x3, uint64_t rows,
                           float* out_n3, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    tf32_rows3_kernel<false><<<mma_grid_for(rows), kThreads, 0, s>>>(rows, 1, left_n3, right3x3,
                                                                     nullptr, out_n3);
    return cudaGetLastError();
}

cudaError_t camera_inputs(float fx, float cx, float fy, float cy, const float* world_view4x4, float* k9,
                          float* wt16, cudaStream_t s) {
    camera_inputs_kernel<<<1, 32, 0, s>>>(fx, cx, fy, cy, world_view4x4, k9, wt16);
    return cudaGetLastError();
}

cudaError_t camera_pack(const float* c2w16, const float* world_view4x4, float* out30, cudaStream_t s) {
    camera_pack_kernel<<<1, 32, 0, s>>>(c2w16, world_view4x4, out30);
    return cudaGetLastError();
}

cudaError_t standard(int width, int height, const float* color5, const float* aux7,
                     const float* rays3, const float* origin3, const float* rotation9, float keep,
                     float ratio, const StandardMaps& maps, cudaStream_t s) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    if (pixels == 0) return cudaSuccess;
    standard_kernel<false><<<grid_for(pixels), kThreads, 0, s>>>(width, height, color5, aux7, rays3, origin3,
                                                                 rotation9, keep, ratio, maps, nullptr, nullptr,
                                                                 nullptr, nullptr);
    return cudaGetLastError();
}

cudaError_t standard_with_fusion(int width, int height, const float* color5, const float* aux7, const float* rays3,
                                 const float* origin3, const float* rotation9, float keep, float ratio,
                                 const StandardMaps& maps, const float* reflection_color5, float* diffuse3,
                                 float* final_rgb3, float* stored3, cudaStream_t s) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    if (pixels == 0) return cudaSuccess;
    standard_kernel<true><<<grid_for(pixels), kThreads, 0, s>>>(width, height, color5, aux7, rays3, origin3,
                                                                rotation9, keep, ratio, maps, reflection_color5,
                                                                diffuse3, final_rgb3, stored3);
    return cudaGetLastError();
}

cudaError_t flashgs(int width, int height, const float* color3, const float* other2,
                    const float* depth1, const float* alpha1, const float* normal3,
                    const float* rotation9, const FlashgsMaps& maps, cudaStream_t s) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    if (pixels == 0) return cudaSuccess;
    flashgs_kernel<false, false><<<grid_for(pixels), kThreads, 0, s>>>(
        width, height, color3, other2, depth1, alpha1, normal3, rotation9, maps, nullptr, nullptr, nullptr, nullptr);
    return cudaGetLastError();
}

cudaError_t flashgs_from_view(int width, int height, const float* color3, const float* other2,
                              const float* depth1, const float* alpha1, const float* normal3,
                              const float* world_view4x4, const FlashgsMaps& maps, const float* reflection_color3,
                              float* diffuse3, float* final_rgb3, float* stored3, cudaStream_t s) {
    const uint64_t pixels = static_cast<uint64_t>(width) * height;
    if (pixels == 0) return cudaSuccess;
    if (reflection_color3 != nullptr) {
        flashgs_kernel<true, true><<<grid_for(pixels), kThreads, 0, s>>>(
            width, height, color3, other2, depth1, alpha1, normal3, world_view4x4, maps, reflection_color3, diffuse3,
            final_rgb3, stored3);
    } else {
        flashgs_kernel<true, false><<<grid_for(pixels), kThreads, 0, s>>>(
            width, height, color3, other2, depth1, alpha1, normal3, world_view4x4, maps, nullptr, nullptr, nullptr,
            nullptr);
    }
    return cudaGetLastError();
}

}  // namespace post
}  // namespace hs
