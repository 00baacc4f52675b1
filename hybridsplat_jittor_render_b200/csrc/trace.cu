// Reflection trace on CUDA cores: scene build (BVH over the disk triangles)
// and the per-ray trace of the reference OptiX programs.
//
// Scene build (hs_optix_build_scene_v1; reference optix_backend.cpp:375-458
// builds an OptiX GAS over the same triangles):
//   boxes      one thread per triangle: vertex indices checked, box of its
//              three vertices (widened by a relative 2^-20 and 1e-7), centroid
//              bounds of the scene (block reduction + ordered-int atomics);
//   morton     30-bit Morton code of each centroid in the scene bounds;
//   sort       the onesweep radix sort (sort.cu) of (code, triangle);
//   hierarchy  one thread per internal node: Karras' parallel binary radix
//              tree over the sorted codes (T. Karras, "Maximizing parallelism
//              in the construction of BVHs, octrees, and k-d trees", HPG
//              2012), equal codes split by their sorted position;
//   leaves     the triangles' vertices in sorted order (48 bytes each);
//   refit      one thread per leaf walks up; the second thread to reach a
//              node writes both children's boxes into it (64 bytes per node)
//              and continues;
//   widen      each binary node's two children, the larger internal ones
//              expanded by surface area until there are four, become the
//              children of a wide node (128 bytes: one float4 per box
//              coordinate of the four children, then their references), so a
//              traversal fetches four boxes per node.
// Trace (hs_optix_trace_f32_v1; reference optix_backend.cpp:460-617 and the
// programs of vendor/optix_tracer/forward.cu:219-660): one thread per ray;
// each trace step is a stack traversal of the wide BVH (children pushed
// farthest first) that keeps the 16 nearest hits in a sorted per-thread
// buffer (shared memory), pruning boxes beyond the 16th; the hits are then
// shaded front to back exactly as the reference raygen program does, and the
// step restarts behind the last processed hit while 16 or more hits were
// found. Which hits a step keeps does not depend on the traversal order.
#include <math_constants.h>

#include <algorithm>
#include <climits>
#include <cstring>

#include "context.h"
#include "sort.cuh"
#include "trace.cuh"

namespace hs {
namespace tr {
namespace {

constexpr int kBuildThreads = 256;
constexpr int kTraceThreads = 128;

__device__ __forceinline__ uint32_t ordered(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unordered(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// Widening of every triangle box: the slab test's rounding can never reject
// a box whose triangle the watertight test hits.
__device__ __forceinline__ float widen_lo(float v) { return v - (fabsf(v) * 9.5367431640625e-07f + 1e-7f); }
__device__ __forceinline__ float widen_hi(float v) { return v + (fabsf(v) * 9.5367431640625e-07f + 1e-7f); }

// status bit of a scene build: a triangle names a vertex outside [0, vertex_count)
constexpr uint32_t kBadIndex = 1u;

__global__ void __launch_bounds__(kBuildThreads) boxes_kernel(
    uint32_t n, const float* __restrict__ vertices, uint64_t vertex_count,
    const int32_t* __restrict__ triangles, float4* __restrict__ lo, float4* __restrict__ hi,
    uint32_t* __restrict__ bounds, uint32_t* __restrict__ status) {
    const uint32_t i = blockIdx.x * kBuildThreads + threadIdx.x;
    float cx = CUDART_INF_F, cy = CUDART_INF_F, cz = CUDART_INF_F;
    float mx = -CUDART_INF_F, my = -CUDART_INF_F, mz = -CUDART_INF_F;
    if (i < n) {
        float3 v[3];
        bool valid = true;
        for (int k = 0; k < 3; ++k) {
            const int32_t idx = triangles[3 * static_cast<uint64_t>(i) + k];
            if (idx < 0 || static_cast<uint64_t>(idx) >= vertex_count) {
                valid = false;
                atomicOr(status, kBadIndex);
                v[k] = make_float3(0.0f, 0.0f, 0.0f);
            } else {
                const float* p = vertices + 3 * static_cast<uint64_t>(idx);
                v[k] = make_float3(p[0], p[1], p[2]);
            }
        }
        float4 a = make_float4(fminf(fminf(v[0].x, v[1].x), v[2].x), fminf(fminf(v[0].y, v[1].y), v[2].y),
                               fminf(fminf(v[0].z, v[1].z), v[2].z), 0.0f);
        float4 b = make_float4(fmaxf(fmaxf(v[0].x, v[1].x), v[2].x), fmaxf(fmaxf(v[0].y, v[1].y), v[2].y),
                               fmaxf(fmaxf(v[0].z, v[1].z), v[2].z), 0.0f);
        bool finite = true;
        for (int k = 0; k < 3; ++k)
            finite = finite && isfinite(v[k].x) && isfinite(v[k].y) && isfinite(v[k].z);
        if (!valid || !finite) {
            // never hit: an empty box, and a centroid that does not widen the bounds
            a = make_float4(CUDART_INF_F, CUDART_INF_F, CUDART_INF_F, 0.0f);
            b = make_float4(-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, 0.0f);
        } else {
            a = make_float4(widen_lo(a.x), widen_lo(a.y), widen_lo(a.z), 0.0f);
            b = make_float4(widen_hi(b.x), widen_hi(b.y), widen_hi(b.z), 0.0f);
            cx = mx = 0.5f * (a.x + b.x);
            cy = my = 0.5f * (a.y + b.y);
            cz = mz = 0.5f * (a.z + b.z);
        }
        lo[i] = a;
        hi[i] = b;
    }
    // block reduction of the centroid bounds
    __shared__ float red[6][kBuildThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float vals[6] = {cx, cy, cz, mx, my, mz};
    for (int k = 0; k < 6; ++k) {
        float x = vals[k];
        for (int off = 16; off > 0; off >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, x, off);
            x = k < 3 ? fminf(x, y) : fmaxf(x, y);
        }
        if (lane == 0) red[k][warp] = x;
    }
    __syncthreads();
    if (threadIdx.x < 6) {
        const int k = threadIdx.x;
        float x = red[k][0];
        for (int w = 1; w < kBuildThreads / 32; ++w) x = k < 3 ? fminf(x, red[k][w]) : fmaxf(x, red[k][w]);
        if (k < 3) atomicMin(bounds + k, ordered(x));
        else atomicMax(bounds + k, ordered(x));
    }
}

__device__ __forceinline__ uint32_t spread10(uint32_t v) {
    v &= 0x3ffu;
    v = (v | (v << 16)) & 0x030000ffu;
    v = (v | (v << 8)) & 0x0300f00fu;
    v = (v | (v << 4)) & 0x030c30c3u;
    v = (v | (v << 2)) & 0x09249249u;
    return v;
}

__global__ void __launch_bounds__(kBuildThreads) morton_kernel(
    uint32_t n, const float4* __restrict__ lo, const float4* __restrict__ hi,
    const uint32_t* __restrict__ bounds, uint32_t* __restrict__ keys, uint32_t* __restrict__ vals) {
    const uint32_t i = blockIdx.x * kBuildThreads + threadIdx.x;
    if (i >= n) return;
    const float b0 = unordered(bounds[0]), b1 = unordered(bounds[1]), b2 = unordered(bounds[2]);
    const float e0 = unordered(bounds[3]) - b0, e1 = unordered(bounds[4]) - b1, e2 = unordered(bounds[5]) - b2;
    const float4 a = lo[i], b = hi[i];
    uint32_t code = 0xffffffffu;  // empty boxes sort last
    if (a.x <= b.x) {
        auto cell = [](float c, float origin, float extent) -> uint32_t {
            const float u = extent > 0.0f ? (c - origin) / extent : 0.0f;
            return static_cast<uint32_t>(fminf(fmaxf(u * 1024.0f, 0.0f), 1023.0f));
        };
        code = (spread10(cell(0.5f * (a.x + b.x), b0, e0)) << 2) |
               (spread10(cell(0.5f * (a.y + b.y), b1, e1)) << 1) | spread10(cell(0.5f * (a.z + b.z), b2, e2));
    }
    keys[i] = code;
    vals[i] = i;
}

// Common-prefix length of the sorted codes at positions i and j (-1 out of
// range); equal codes compare their positions (32 more bits) instead. The
// prefixes of the internal nodes on any root-to-leaf path strictly increase
// within [0, 64), so the tree is at most 64 internal nodes deep.
__device__ __forceinline__ int common_prefix(const uint32_t* keys, int64_t n, int64_t i, int64_t j) {
    if (j < 0 || j >= n) return -1;
    const uint32_t a = keys[i], b = keys[j];
    if (a != b) return __clz(a ^ b);
    return 32 + __clz(static_cast<uint32_t>(i) ^ static_cast<uint32_t>(j));
}

__global__ void __launch_bounds__(kBuildThreads) hierarchy_kernel(
    uint32_t n, const uint32_t* __restrict__ keys, uint32_t* __restrict__ children,
    uint32_t* __restrict__ parents) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kBuildThreads + threadIdx.x;
    const int64_t count = n;
    if (i >= count - 1) return;
    const int d = common_prefix(keys, count, i, i + 1) - common_prefix(keys, count, i, i - 1) >= 0 ? 1 : -1;
    const int min_prefix = common_prefix(keys, count, i, i - d);
    int64_t span = 2;
    while (common_prefix(keys, count, i, i + span * d) > min_prefix) span *= 2;
    int64_t length = 0;
    for (int64_t t = span / 2; t >= 1; t /= 2) {
        if (common_prefix(keys, count, i, i + (length + t) * d) > min_prefix) length += t;
    }
    const int64_t j = i + length * d;
    const int node_prefix = common_prefix(keys, count, i, j);
    int64_t split = 0;
    for (int64_t div = 2;; div *= 2) {
        const int64_t t = (length + div - 1) / div;
        if (common_prefix(keys, count, i, i + (split + t) * d) > node_prefix) split += t;
        if (t == 1) break;
    }
    const int64_t gamma = i + split * d + (d < 0 ? -1 : 0);
    const int64_t first = d > 0 ? i : j, last = d > 0 ? j : i;
    const uint32_t left = first == gamma ? (kLeafBit | static_cast<uint32_t>(gamma)) : static_cast<uint32_t>(gamma);
    const uint32_t right = last == gamma + 1 ? (kLeafBit | static_cast<uint32_t>(gamma + 1))
                                             : static_cast<uint32_t>(gamma + 1);
    children[2 * i] = left;
    children[2 * i + 1] = right;
    // parents: internal nodes at [0, n - 1), leaf slots at [n - 1, 2n - 1)
    parents[(left & kLeafBit) ? (count - 1 + (left & ~kLeafBit)) : left] = static_cast<uint32_t>(i);
    parents[(right & kLeafBit) ? (count - 1 + (right & ~kLeafBit)) : right] = static_cast<uint32_t>(i);
}

__global__ void __launch_bounds__(kBuildThreads) leaves_kernel(
    uint32_t n, const uint32_t* __restrict__ order, const float* __restrict__ vertices,
    uint64_t vertex_count, const int32_t* __restrict__ triangles, float4* __restrict__ tris) {
    const uint32_t s = blockIdx.x * kBuildThreads + threadIdx.x;
    if (s >= n) return;
    const uint32_t t = order[s];
    float3 v[3];
    for (int k = 0; k < 3; ++k) {
        const int32_t idx = triangles[3 * static_cast<uint64_t>(t) + k];
        if (idx < 0 || static_cast<uint64_t>(idx) >= vertex_count) {
            v[k] = make_float3(CUDART_NAN_F, CUDART_NAN_F, CUDART_NAN_F);
        } else {
            const float* p = vertices + 3 * static_cast<uint64_t>(idx);
            v[k] = make_float3(p[0], p[1], p[2]);
        }
    }
    float4* dst = tris + 3 * static_cast<uint64_t>(s);
    dst[0] = make_float4(v[0].x, v[0].y, v[0].z, __uint_as_float(t));
    dst[1] = make_float4(v[1].x, v[1].y, v[1].z, 0.0f);
    dst[2] = make_float4(v[2].x, v[2].y, v[2].z, 0.0f);
}

__global__ void __launch_bounds__(kBuildThreads) refit_kernel(
    uint32_t n, const uint32_t* __restrict__ order, const float4* __restrict__ lo,
    const float4* __restrict__ hi, const uint32_t* __restrict__ children,
    const uint32_t* __restrict__ parents, uint32_t* __restrict__ visits, float4* node_boxes,
    float4* __restrict__ nodes) {
    const uint32_t s = blockIdx.x * kBuildThreads + threadIdx.x;
    if (s >= n || n < 2) return;
    uint32_t node = parents[n - 1 + s];
    for (;;) {
        __threadfence();
        if (atomicAdd(visits + node, 1u) == 0u) return;  // the sibling subtree is not finished
        __threadfence();
        float4 box[2][2];
        for (int c = 0; c < 2; ++c) {
            const uint32_t ref = children[2 * node + c];
            if (ref & kLeafBit) {
                const uint32_t t = order[ref & ~kLeafBit];
                box[c][0] = lo[t];
                box[c][1] = hi[t];
            } else {
                box[c][0] = __ldcg(node_boxes + 2 * ref);
                box[c][1] = __ldcg(node_boxes + 2 * ref + 1);
            }
        }
        float4* out = nodes + 4 * static_cast<uint64_t>(node);
        out[0] = make_float4(box[0][0].x, box[0][0].y, box[0][0].z, __uint_as_float(children[2 * node]));
        out[1] = make_float4(box[0][1].x, box[0][1].y, box[0][1].z, __uint_as_float(children[2 * node + 1]));
        out[2] = box[1][0];
        out[3] = box[1][1];
        __stcg(node_boxes + 2 * node,
               make_float4(fminf(box[0][0].x, box[1][0].x), fminf(box[0][0].y, box[1][0].y),
                           fminf(box[0][0].z, box[1][0].z), 0.0f));
        __stcg(node_boxes + 2 * node + 1,
               make_float4(fmaxf(box[0][1].x, box[1][1].x), fmaxf(box[0][1].y, box[1][1].y),
                           fmaxf(box[0][1].z, box[1][1].z), 0.0f));
        if (node == 0) return;
        node = parents[node];
    }
}

// Single-triangle scene: a root node whose second child is empty.
__global__ void single_root_kernel(const float4* __restrict__ lo, const float4* __restrict__ hi,
                                   float4* __restrict__ nodes) {
    nodes[0] = make_float4(lo[0].x, lo[0].y, lo[0].z, __uint_as_float(kLeafBit));
    nodes[1] = make_float4(hi[0].x, hi[0].y, hi[0].z, __uint_as_float(kNoChild));
    nodes[2] = make_float4(CUDART_INF_F, CUDART_INF_F, CUDART_INF_F, 0.0f);
    nodes[3] = make_float4(CUDART_INF_F, CUDART_INF_F, CUDART_INF_F, 0.0f);
}

// The wide tree: wide node i holds up to four binary nodes that together
// cover binary node i's subtree: its two children, then, while a slot is
// free, the internal one of largest box surface area replaced by its two
// children (leaves and empty children stand for themselves). One thread per
// binary node; nodes that the traversal never reaches are written too.
// Empty slots get the box [+inf, +inf], which the slab test rejects, and the
// reference kNoChild.
__global__ void __launch_bounds__(kBuildThreads) widen_kernel(uint32_t internal,
                                                              const float4* __restrict__ binary,
                                                              float4* __restrict__ wide) {
    const uint32_t i = blockIdx.x * kBuildThreads + threadIdx.x;
    if (i >= internal) return;
    float lx[4], ly[4], lz[4], hx[4], hy[4], hz[4];
    uint32_t ref[4];
    int k = 0;
    auto take = [&](const float4* node, int c) {
        const float4 lo = node[2 * c], hi = node[2 * c + 1];
        lx[k] = lo.x; ly[k] = lo.y; lz[k] = lo.z;
        hx[k] = hi.x; hy[k] = hi.y; hz[k] = hi.z;
        ref[k++] = __float_as_uint(c == 0 ? node[0].w : node[1].w);
    };
    const float4* node = binary + 4 * static_cast<uint64_t>(i);
    take(node, 0);
    take(node, 1);
    // greedy: expand the internal child with the largest surface area
    while (k < 4) {
        int best = -1;
        float best_area = -1.0f;
        for (int j = 0; j < k; ++j) {
            if (ref[j] == kNoChild || (ref[j] & kLeafBit) != 0u) continue;
            const float dx = hx[j] - lx[j], dy = hy[j] - ly[j], dz = hz[j] - lz[j];
            const float area = dx * dy + dy * dz + dz * dx;
            if (area > best_area) {
                best_area = area;
                best = j;
            }
        }
        if (best < 0) break;
        const float4* child = binary + 4 * static_cast<uint64_t>(ref[best]);
        // the expanded child's slot takes its first child, a new slot its second
        const int last = k;
        take(child, 1);
        k = best;
        take(child, 0);
        k = last + 1;
    }
    for (; k < 4; ++k) {
        lx[k] = ly[k] = lz[k] = hx[k] = hy[k] = hz[k] = CUDART_INF_F;
        ref[k] = kNoChild;
    }
    float4* out = wide + kWideQuads * static_cast<uint64_t>(i);
    out[0] = make_float4(lx[0], lx[1], lx[2], lx[3]);
    out[1] = make_float4(hx[0], hx[1], hx[2], hx[3]);
    out[2] = make_float4(ly[0], ly[1], ly[2], ly[3]);
    out[3] = make_float4(hy[0], hy[1], hy[2], hy[3]);
    out[4] = make_float4(lz[0], lz[1], lz[2], lz[3]);
    out[5] = make_float4(hz[0], hz[1], hz[2], hz[3]);
    out[6] = make_float4(__uint_as_float(ref[0]), __uint_as_float(ref[1]), __uint_as_float(ref[2]),
                         __uint_as_float(ref[3]));
    out[7] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

// ------------------------------------------------------------------- trace

struct TraceArgs {
    uint32_t rays;
    const float* ray_o;
    const float* ray_d;
    const float* background;
    const float* means;
    const float* shs;
    uint32_t coeffs;
    int degree;
    const float* others;  // null unless use_others
    const float* opacities;
    const float* scales;
    float scale_modifier;
    const float* rotations;
    const float* projmatrix;
    const float* campos;
    int start_from_first;
    int max_depth;
    float specular_threshold;
    float* out_rgb;
    float* out_depth;
    float* out_acc;
    float* out_normal;
    float* out_dist;
    float* out_aux;
    float* out_mid;
    Bvh bvh;
};

struct Segment {
    float c[3];
    float d, a, dist, m1, m2, t;
    float n[3];
    float o[2];
    float3 e;
};

// The image-plane terms of the first trace when start_from_first is set
// (compute_transmat_xy, forward.cu:112-169) with the reference's launch
// geometry W = 3, H = ray count; false when the projected centre is undefined.
__device__ bool transmat_xy(const float3& p, const float2& scale, float mod, const float4& rot,
                            const float* proj, int W, int H, float cutoff, float& s2p_z, float2& xy) {
    float3 R[3];
    rotation_rows(rot, R);
    const float sx = mul(mod, scale.x), sy = mul(mod, scale.y);
    // L = R * diag(sx, sy, 1): the first two columns scale, the third stays
    const float3 L[3] = {f3(mul(R[0].x, sx), mul(R[0].y, sy), R[0].z), f3(mul(R[1].x, sx), mul(R[1].y, sy), R[1].z),
                         f3(mul(R[2].x, sx), mul(R[2].y, sy), R[2].z)};
    const float3 s2w[4] = {f3(L[0].x, L[0].y, p.x), f3(L[1].x, L[1].y, p.y), f3(L[2].x, L[2].y, p.z),
                           f3(0.0f, 0.0f, 1.0f)};
    const float4 w2n[4] = {make_float4(proj[0], proj[4], proj[8], proj[12]),
                           make_float4(proj[1], proj[5], proj[9], proj[13]),
                           make_float4(proj[2], proj[6], proj[10], proj[14]),
                           make_float4(proj[3], proj[7], proj[11], proj[15])};
    const float4 n2p[3] = {make_float4(static_cast<float>(W / 2.0), 0.0f, 0.0f, static_cast<float>((W - 1) / 2.0)),
                           make_float4(0.0f, static_cast<float>(H / 2.0), 0.0f, static_cast<float>((H - 1) / 2.0)),
                           make_float4(0.0f, 0.0f, 0.0f, 1.0f)};
    float4 P[3];
    for (int r = 0; r < 3; ++r) {
        const float4 m = n2p[r];
        auto col = [&](float a0, float a1, float a2, float a3) {
            return fma(m.w, a3, fma(m.z, a2, fma(m.y, a1, mul(m.x, a0))));
        };
        P[r] = make_float4(col(w2n[0].x, w2n[1].x, w2n[2].x, w2n[3].x), col(w2n[0].y, w2n[1].y, w2n[2].y, w2n[3].y),
                           col(w2n[0].z, w2n[1].z, w2n[2].z, w2n[3].z), col(w2n[0].w, w2n[1].w, w2n[2].w, w2n[3].w));
    }
    float3 S[3];
    for (int r = 0; r < 3; ++r) {
        const float4 m = P[r];
        auto col = [&](float a0, float a1, float a2, float a3) {
            return fma(m.w, a3, fma(m.z, a2, fma(m.y, a1, mul(m.x, a0))));
        };
        S[r] = f3(col(s2w[0].x, s2w[1].x, s2w[2].x, s2w[3].x), col(s2w[0].y, s2w[1].y, s2w[2].y, s2w[3].y),
                  col(s2w[0].z, s2w[1].z, s2w[2].z, s2w[3].z));
    }
    s2p_z = S[2].z;
    const float c2 = mul(cutoff, cutoff);
    const float3 t = f3(c2, c2, -1.0f);
    const float d = dot3f(t, f3(mul(S[2].x, S[2].x), mul(S[2].y, S[2].y), mul(S[2].z, S[2].z)));
    if (d == 0.0f) return false;
    const float3 f = f3(div(t.x, d), div(t.y, d), div(t.z, d));
    auto sum3 = [](const float3& v) { return add(add(v.x, v.y), v.z); };
    xy = make_float2(sum3(f3(mul(mul(f.x, S[0].x), S[2].x), mul(mul(f.y, S[0].y), S[2].y), mul(mul(f.z, S[0].z), S[2].z))),
                     sum3(f3(mul(mul(f.x, S[1].x), S[2].x), mul(mul(f.y, S[1].y), S[2].y), mul(mul(f.z, S[1].z), S[2].z))));
    return true;
}

// The 16 nearest hits (distance, leaf slot) of one trace step, sorted, in
// this thread's columns of shared memory (stride kTraceThreads).
struct Buffer {
    float* t;
    uint32_t* s;
    __device__ __forceinline__ float& t_at(int k) const { return t[k * kTraceThreads]; }
    __device__ __forceinline__ uint32_t& s_at(int k) const { return s[k * kTraceThreads]; }
    // sorted insertion (ties: smaller slot first)
    __device__ __forceinline__ void insert(float v, uint32_t slot) const {
        int k = kChunk - 1;
        while (k > 0) {
            const float pt = t_at(k - 1);
            const uint32_t ps = s_at(k - 1);
            if (!(pt > v || (pt == v && ps > slot))) break;
            t_at(k) = pt;
            s_at(k) = ps;
            --k;
        }
        t_at(k) = v;
        s_at(k) = slot;
    }
};

// One trace step: a BVH traversal from `o` that keeps the 16 nearest hits,
// pruning boxes beyond the 16th once the buffer is full. Returns the number
// of hits that entered the buffer (at least 16 when the ray has 16 or more).
__device__ uint32_t collect(const Bvh& bvh, const float3& o, const float3& inv, const RayShear& shear,
                            const Buffer& hits) {
    uint32_t stack[kStackDepth];
    for (int k = 0; k < kChunk; ++k) {
        hits.t_at(k) = kDepthInfinity;
        hits.s_at(k) = 0xffffffffu;
    }
    uint32_t found = 0;
    float limit = kDepthInfinity;
    int sp = 0;
    stack[sp++] = bvh.root;
    while (sp > 0) {
        const uint32_t ref = stack[--sp];
        if (ref & kLeafBit) {
            const uint32_t slot = ref & ~kLeafBit;
            const float4* tri = bvh.tris + 3 * static_cast<uint64_t>(slot);
            const float4 v0 = __ldg(tri), v1 = __ldg(tri + 1), v2 = __ldg(tri + 2);
            const float t = hit_triangle(o, shear, f3(v0.x, v0.y, v0.z), f3(v1.x, v1.y, v1.z), f3(v2.x, v2.y, v2.z));
            if (t >= 0.0f && t < limit) {
                ++found;
                hits.insert(t, slot);
                limit = hits.t_at(kChunk - 1);
            }
            continue;
        }
        const float4* node = bvh.nodes + kWideQuads * static_cast<uint64_t>(ref);
        const float4 minx = __ldg(node), maxx = __ldg(node + 1), miny = __ldg(node + 2),
                     maxy = __ldg(node + 3), minz = __ldg(node + 4), maxz = __ldg(node + 5);
        const uint4 refs = __ldg(reinterpret_cast<const uint4*>(node + 6));
        const float box_limit = limit * 1.000244140625f;
        // the children whose box the ray enters before box_limit, by entry
        // distance (a 4-element sorting network; missed ones at +inf)
        float e[4];
        uint32_t c[4] = {refs.x, refs.y, refs.z, refs.w};
        e[0] = hit_box(o, inv, minx.x, miny.x, minz.x, maxx.x, maxy.x, maxz.x, box_limit, e[0]) ? e[0] : CUDART_INF_F;
        e[1] = hit_box(o, inv, minx.y, miny.y, minz.y, maxx.y, maxy.y, maxz.y, box_limit, e[1]) ? e[1] : CUDART_INF_F;
        e[2] = hit_box(o, inv, minx.z, miny.z, minz.z, maxx.z, maxy.z, maxz.z, box_limit, e[2]) ? e[2] : CUDART_INF_F;
        e[3] = hit_box(o, inv, minx.w, miny.w, minz.w, maxx.w, maxy.w, maxz.w, box_limit, e[3]) ? e[3] : CUDART_INF_F;
        auto order2 = [&](int a, int b) {
            if (e[b] < e[a]) {
                const float te = e[a];
                e[a] = e[b];
                e[b] = te;
                const uint32_t tc = c[a];
                c[a] = c[b];
                c[b] = tc;
            }
        };
        order2(0, 1);
        order2(2, 3);
        order2(0, 2);
        order2(1, 3);
        order2(1, 2);
        // Never taken: at most 3 entries per wide level above this node (at
        // most 64 levels) plus these four.
        if (sp + 4 > kStackDepth) break;
        // farthest first, so that the nearest is popped next
        for (int k = 3; k >= 0; --k) {
            if (e[k] != CUDART_INF_F && c[k] != kNoChild) stack[sp++] = c[k];
        }
    }
    return found;
}

// One traceRay of the reference (forward.cu:219-405) from `o` along `d`.
__device__ void trace_segment(const TraceArgs& a, const float3& o, const float3& d, float min_depth,
                              int depth_index, Segment& s, const Buffer& hit_buffer) {
    const float3 inv = f3(div(1.0f, d.x), div(1.0f, d.y), div(1.0f, d.z));
    const RayShear shear = ray_shear(d);
    const float bg[3] = {a.background[0], a.background[1], a.background[2]};
    const float3 campos = f3(a.campos[0], a.campos[1], a.campos[2]);
    const float far_ratio = div(kFar, sub(kFar, kNear));
    float t_prev = 1.0f, t_next = 1.0f, dpt = 0.0f, pdpt = 0.0f;
    int last = -1, contributors = 0;
    float3 ot = o;
    const Buffer* hits = &hit_buffer;
    // Trace steps are bounded: far from the origin the restart offset can
    // vanish in float rounding and a step could repeat itself.
    for (int step_count = 0; step_count < kMaxTraceSteps; ++step_count) {
        const uint32_t found = collect(a.bvh, ot, inv, shear, hit_buffer);
        // --- shade the buffer front to back (forward.cu:281-385)
        const int n = found < kChunk ? static_cast<int>(found) : kChunk;
        bool stop = false;
        for (int i = 0; i < n; ++i) {
            const uint32_t prim = __float_as_uint(__ldg(a.bvh.tris + 3 * static_cast<uint64_t>(hits->s_at(i))).w);
            const int g = static_cast<int>(prim / 2u);
            if (g == last) continue;
            const float tm = hits->t_at(i);
            dpt = static_cast<float>(static_cast<double>(add(tm, pdpt)) + (pdpt == 0.0f ? 0.0 : kStepEpsilon));
            // A scene with more than two triangles per ray names Gaussians the
            // call has no data for: such hits are skipped.
            if (static_cast<uint32_t>(g) >= a.rays) continue;
            const float3 xyz = f3(fma(dpt, d.x, o.x), fma(dpt, d.y, o.y), fma(dpt, d.z, o.z));
            const float* q = a.rotations + 4 * static_cast<uint64_t>(g);
            const float4 rot = make_float4(q[0], q[1], q[2], q[3]);
            const float3 p = f3(a.means[3 * g], a.means[3 * g + 1], a.means[3 * g + 2]);
            const float2 sc = make_float2(a.scales[2 * g], a.scales[2 * g + 1]);
            float3 R[3];
            rotation_rows_t(rot, R);
            const float tx = dot3f(R[0], p), ty = dot3f(R[1], p);
            const float u1 = add(dot3f(R[0], xyz), -tx), v1 = add(dot3f(R[1], xyz), -ty);
            const float2 uv = make_float2(div(u1, sc.x), div(v1, sc.y));
            const float rho3d = fma(uv.y, uv.y, mul(uv.x, uv.x));
            float3 normal = R[2];
            const float3 dir = f3(sub(p.x, campos.x), sub(p.y, campos.y), sub(p.z, campos.z));
            const float cosv = -dot3f(dir, normal);
            if (cosv == 0.0f) continue;
            if (!(cosv > 0.0f)) normal = f3(-normal.x, -normal.y, -normal.z);
            float rho2d, cmd;
            if (depth_index == 0 && a.start_from_first) {
                float s2pz = 0.0f;
                float2 xy = make_float2(0.0f, 0.0f);
                const bool ok = transmat_xy(p, sc, a.scale_modifier, rot, a.projmatrix, 3,
                                            static_cast<int>(a.rays), 3.0f, s2pz, xy);
                rho2d = mul(fma(xy.y, xy.y, mul(xy.x, xy.x)), kFilterInvSquare);
                if (!ok && rho3d > rho2d) continue;
                cmd = rho3d <= rho2d ? dpt : s2pz;
            } else {
                rho2d = add(rho3d, 1.0f);
                cmd = dpt;
            }
            if (cmd < min_depth) continue;
            const float power = mul(-0.5f, fminf(rho3d, rho2d));
            if (power > 0.0f) continue;
            const float alpha = fminf(0.99f, mul(a.opacities[g], expf(power)));
            if (alpha < 1.0f / 255.0f) continue;
            t_next = mul(t_prev, sub(1.0f, alpha));
            if (t_next < kTThreshold) {
                stop = true;
                break;
            }
            if (++contributors > kMaxContributors) {
                stop = true;
                break;
            }
            last = g;
            const float w = mul(alpha, t_prev);
            const float3 col = sh_color(a.degree, a.shs + static_cast<uint64_t>(g) * a.coeffs * 3, d);
            s.c[0] = fma(w, col.x, s.c[0]);
            s.c[1] = fma(w, col.y, s.c[1]);
            s.c[2] = fma(w, col.z, s.c[2]);
            if (a.others != nullptr) {
                s.o[0] = fma(w, a.others[2 * g], s.o[0]);
                s.o[1] = fma(w, a.others[2 * g + 1], s.o[1]);
            }
            const float aa = sub(1.0f, t_prev);
            const float m = mul(far_ratio, sub(1.0f, div(kNear, cmd)));
            s.dist = fma(w, fma(-mul(2.0f, m), s.m1, fma(mul(m, m), aa, s.m2)), s.dist);
            s.m1 = fma(w, m, s.m1);
            s.m2 = fma(mul(w, m), m, s.m2);
            s.d = fma(w, cmd, s.d);
            s.n[0] = fma(w, normal.x, s.n[0]);
            s.n[1] = fma(w, normal.y, s.n[1]);
            s.n[2] = fma(w, normal.z, s.n[2]);
            t_prev = t_next;
        }
        if (stop || t_next < kTThreshold || found < static_cast<uint32_t>(kChunk) || contributors > kMaxContributors)
            break;
        pdpt = dpt;
        const float step = static_cast<float>(static_cast<double>(pdpt) + kStepEpsilon);
        ot = f3(fma(step, d.x, o.x), fma(step, d.y, o.y), fma(step, d.z, o.z));
    }
    for (int ch = 0; ch < 3; ++ch) s.c[ch] = fma(t_prev, bg[ch], s.c[ch]);
    s.a = sub(1.0f, t_prev);
    s.t = t_prev;
    s.e = f3(fma(s.d, d.x, o.x), fma(s.d, d.y, o.y), fma(s.d, d.z, o.z));
}

__device__ __forceinline__ void trace_one(const TraceArgs& a, uint32_t r, const Buffer& hits);

// Persistent: every thread takes the next ray of the spatial order from a
// global counter whenever its ray is done, so the short rays of a warp do not
// wait for its longest one. The traversal waits on dependent node fetches, so
// occupancy matters more than the few registers spilled to fit 8 blocks/SM
// (measured 5% faster than 5 blocks/SM at 96 registers).
__global__ void __launch_bounds__(kTraceThreads, 8) trace_kernel(TraceArgs a, const uint32_t* __restrict__ order,
                                                              uint32_t* __restrict__ next_ray) {
    __shared__ float hit_t[kChunk * kTraceThreads];
    __shared__ uint32_t hit_s[kChunk * kTraceThreads];
    const Buffer hits{hit_t + threadIdx.x, hit_s + threadIdx.x};
    for (;;) {
        const uint32_t slot = atomicAdd(next_ray, 1u);
        if (slot >= a.rays) break;
        trace_one(a, order[slot], hits);
    }
}

// Spatial order of the rays: 27-bit Morton code of the origin in the scene's
// bounds, then the direction's octant (3 low bits); ties by ray index.
__global__ void __launch_bounds__(kBuildThreads) ray_keys_kernel(
    uint32_t rays, const float* __restrict__ ray_o, const float* __restrict__ ray_d,
    const float* __restrict__ bounds, uint32_t* __restrict__ keys, uint32_t* __restrict__ vals) {
    const uint32_t r = blockIdx.x * kBuildThreads + threadIdx.x;
    if (r >= rays) return;
    auto cell = [](float c, float lo, float hi) -> uint32_t {
        const float e = hi - lo;
        const float u = e > 0.0f ? (c - lo) / e : 0.0f;
        return static_cast<uint32_t>(fminf(fmaxf(u * 512.0f, 0.0f), 511.0f));  // NaN -> 0
    };
    const float ox = ray_o[3 * static_cast<uint64_t>(r)], oy = ray_o[3 * static_cast<uint64_t>(r) + 1],
                oz = ray_o[3 * static_cast<uint64_t>(r) + 2];
    const uint32_t m = (spread10(cell(ox, bounds[0], bounds[3])) << 2) |
                       (spread10(cell(oy, bounds[1], bounds[4])) << 1) | spread10(cell(oz, bounds[2], bounds[5]));
    const uint32_t oct = (ray_d[3 * static_cast<uint64_t>(r)] < 0.0f ? 4u : 0u) |
                         (ray_d[3 * static_cast<uint64_t>(r) + 1] < 0.0f ? 2u : 0u) |
                         (ray_d[3 * static_cast<uint64_t>(r) + 2] < 0.0f ? 1u : 0u);
    keys[r] = (m << 3) | oct;
    vals[r] = r;
}

__global__ void scene_bounds_kernel(const uint32_t* __restrict__ ordered_bounds, float* __restrict__ bounds) {
    if (threadIdx.x < 6) bounds[threadIdx.x] = unordered(ordered_bounds[threadIdx.x]);
}

// tracePath + __raygen__ot (forward.cu:408-620) for ray r.
__device__ __forceinline__ void trace_one(const TraceArgs& a, uint32_t r, const Buffer& hits) {
    float3 o = f3(a.ray_o[3 * static_cast<uint64_t>(r)], a.ray_o[3 * static_cast<uint64_t>(r) + 1],
                  a.ray_o[3 * static_cast<uint64_t>(r) + 2]);
    float3 d = f3(a.ray_d[3 * static_cast<uint64_t>(r)], a.ray_d[3 * static_cast<uint64_t>(r) + 1],
                  a.ray_d[3 * static_cast<uint64_t>(r) + 2]);
    float rgb[3] = {0.0f, 0.0f, 0.0f};
    float s_prod = 1.0f;
    float* mid = a.out_mid + 32 * static_cast<uint64_t>(r);
    for (int i = 0; i < a.max_depth + 1; ++i) {
        Segment s{};
        s.t = 1.0f;
        const float min_depth = (i == 0 && a.start_from_first) ? kNear : kStartOffset;
        trace_segment(a, o, d, min_depth, i, s, hits);
        if (i == 0) {
            a.out_depth[r] = s.d;
            a.out_acc[r] = s.a;
            a.out_normal[3 * static_cast<uint64_t>(r)] = s.n[0];
            a.out_normal[3 * static_cast<uint64_t>(r) + 1] = s.n[1];
            a.out_normal[3 * static_cast<uint64_t>(r) + 2] = s.n[2];
            a.out_dist[r] = s.dist;
            a.out_aux[2 * static_cast<uint64_t>(r)] = s.o[0];
            a.out_aux[2 * static_cast<uint64_t>(r) + 1] = s.o[1];
        }
        const float f_this = i == a.max_depth ? 1.0f : sub(1.0f, s.o[0]);
        for (int ch = 0; ch < 3; ++ch) rgb[ch] = add(rgb[ch], mul(mul(s.c[ch], f_this), s_prod));
        s_prod = mul(s_prod, s.o[0]);
        float* m = mid + i * kMidChannels;
        m[0] = o.x; m[1] = o.y; m[2] = o.z;
        m[3] = d.x; m[4] = d.y; m[5] = d.z;
        m[6] = s.d;
        m[7] = s.a;
        m[8] = s.n[0]; m[9] = s.n[1]; m[10] = s.n[2];
        m[11] = s.o[0]; m[12] = s.o[1];
        m[13] = s.c[0]; m[14] = s.c[1]; m[15] = s.c[2];
        const float3 nn = f3(s.n[0], s.n[1], s.n[2]);
        if (__fsqrt_rn(dot3f(nn, nn)) == 0.0f || s.o[0] <= a.specular_threshold) break;
        const float3 n = normalize3(nn);
        const float k = mul(2.0f, dot3f(n, d));
        d = f3(fma(-k, n.x, d.x), fma(-k, n.y, d.y), fma(-k, n.z, d.z));
        o = f3(fma(static_cast<float>(kStepEpsilon), d.x, s.e.x), fma(static_cast<float>(kStepEpsilon), d.y, s.e.y),
               fma(static_cast<float>(kStepEpsilon), d.z, s.e.z));
    }
    for (int ch = 0; ch < 3; ++ch) a.out_rgb[3 * static_cast<uint64_t>(r) + ch] = rgb[ch];
}

struct BuildLayout {
    float4* lo;
    float4* hi;
    uint32_t* keys;
    uint32_t* vals;
    uint32_t* alt_keys;
    uint32_t* alt_vals;
    uint32_t* children;
    uint32_t* parents;
    uint32_t* visits;
    float4* node_boxes;
    float4* binary;  // binary radix tree: 4 float4 per internal node
    uint32_t* bounds;
    uint32_t* status;
    void* sort_scratch;
    uint64_t bytes;
};

BuildLayout build_layout(void* base, uint64_t n) {
    Carver c(base);
    BuildLayout l;
    l.lo = c.take<float4>(n);
    l.hi = c.take<float4>(n);
    l.keys = c.take<uint32_t>(n);
    l.vals = c.take<uint32_t>(n);
    l.alt_keys = c.take<uint32_t>(n);
    l.alt_vals = c.take<uint32_t>(n);
    l.children = c.take<uint32_t>(2 * n);
    l.parents = c.take<uint32_t>(2 * n);
    l.visits = c.take<uint32_t>(n);
    l.node_boxes = c.take<float4>(2 * n);
    l.binary = c.take<float4>(4 * std::max<uint64_t>(n > 0 ? n - 1 : 1, 1));
    l.bounds = c.take<uint32_t>(64);
    l.status = c.take<uint32_t>(64);
    l.sort_scratch = c.take<unsigned char>(sort::sort_scratch_bytes(static_cast<uint32_t>(n)));
    l.bytes = c.offset;
    return l;
}

struct SceneLayout {
    float4* nodes;
    float4* tris;
    float* bounds;  // centroid bounds of the scene: min xyz, max xyz
    uint64_t bytes;
};

SceneLayout scene_layout(void* base, uint64_t n) {
    Carver c(base);
    SceneLayout l;
    l.nodes = c.take<float4>(kWideQuads * std::max<uint64_t>(n > 0 ? n - 1 : 1, 1));
    l.tris = c.take<float4>(3 * n);
    l.bounds = c.take<float>(64);
    l.bytes = c.offset;
    return l;
}

// Per-call scratch of the trace: the ray order and its sort.
struct RayLayout {
    uint32_t* keys;
    uint32_t* vals;
    uint32_t* alt_keys;
    uint32_t* alt_vals;
    uint32_t* counter;
    void* sort_scratch;
    uint64_t bytes;
};

RayLayout ray_layout(void* base, uint64_t rays) {
    Carver c(base);
    RayLayout l;
    l.keys = c.take<uint32_t>(rays);
    l.vals = c.take<uint32_t>(rays);
    l.alt_keys = c.take<uint32_t>(rays);
    l.alt_vals = c.take<uint32_t>(rays);
    l.counter = c.take<uint32_t>(64);
    l.sort_scratch = c.take<unsigned char>(sort::sort_scratch_bytes(static_cast<uint32_t>(rays)));
    l.bytes = c.offset;
    return l;
}

}  // namespace
}  // namespace tr

uint64_t trace_current_bytes(const HsRasterizerContext* ctx) {
    return ctx->tr_scene.bytes + ctx->tr_scratch.bytes + ctx->tr_rays.bytes;
}

cudaError_t trace_release(HsRasterizerContext* ctx) {
    cudaError_t first = cudaDeviceSynchronize();
    for (DeviceBuffer* b : {&ctx->tr_scene, &ctx->tr_scratch, &ctx->tr_rays}) {
        const cudaError_t e = release_buffer(*b);
        if (first == cudaSuccess) first = e;
    }
    ctx->tr_triangles = 0;
    ctx->tr_root = 0;
    ctx->tr_signature = 0;
    return first;
}

cudaError_t trace_build_scene(HsRasterizerContext* ctx, const float* vertices3, uint64_t vertex_count,
                              const int32_t* triangles3, uint64_t triangle_count, bool* bad_index) {
    using namespace tr;
    *bad_index = false;
    const cudaStream_t stream = nullptr;
    const uint64_t n = triangle_count;
    const BuildLayout need = build_layout(nullptr, n);
    cudaError_t st = ensure_buffer(ctx->tr_scratch, need.bytes, &ctx->tr_growth_count, true);
    if (st != cudaSuccess) return st;
    const SceneLayout scene_need = scene_layout(nullptr, n);
    st = ensure_buffer(ctx->tr_scene, scene_need.bytes, &ctx->tr_growth_count, true);
    if (st != cudaSuccess) return st;
    ctx->tr_peak_bytes = std::max(ctx->tr_peak_bytes, trace_current_bytes(ctx));
    const BuildLayout l = build_layout(ctx->tr_scratch.ptr, n);
    const SceneLayout sl = scene_layout(ctx->tr_scene.ptr, n);
    const uint32_t n32 = static_cast<uint32_t>(n);
    const unsigned blocks = static_cast<unsigned>((n + kBuildThreads - 1) / kBuildThreads);
    // bounds: min words start at the largest ordered value, max words at 0
    const uint32_t init[8] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0u, 0u, 0u, 0u, 0u};
    st = cudaMemcpyAsync(l.bounds, init, sizeof(init), cudaMemcpyHostToDevice, stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(l.status, 0, sizeof(uint32_t), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(l.visits, 0, n * sizeof(uint32_t), stream);
    if (st != cudaSuccess) return st;
    boxes_kernel<<<blocks, kBuildThreads, 0, stream>>>(n32, vertices3, vertex_count, triangles3, l.lo, l.hi,
                                                       l.bounds, l.status);
    morton_kernel<<<blocks, kBuildThreads, 0, stream>>>(n32, l.lo, l.hi, l.bounds, l.keys, l.vals);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    st = sort::sort_pairs(l.keys, l.vals, l.alt_keys, l.alt_vals, n32, 0, 32, l.sort_scratch, stream,
                          ctx->device_error);
    if (st != cudaSuccess) return st;
    if (n >= 2) {
        hierarchy_kernel<<<static_cast<unsigned>((n - 1 + kBuildThreads - 1) / kBuildThreads), kBuildThreads, 0,
                           stream>>>(n32, l.keys, l.children, l.parents);
        refit_kernel<<<blocks, kBuildThreads, 0, stream>>>(n32, l.vals, l.lo, l.hi, l.children, l.parents,
                                                           l.visits, l.node_boxes, l.binary);
    } else {
        single_root_kernel<<<1, 1, 0, stream>>>(l.lo, l.hi, l.binary);
    }
    const uint32_t internal = n >= 2 ? n32 - 1 : 1u;
    widen_kernel<<<(internal + kBuildThreads - 1) / kBuildThreads, kBuildThreads, 0, stream>>>(internal, l.binary,
                                                                                              sl.nodes);
    leaves_kernel<<<blocks, kBuildThreads, 0, stream>>>(n32, l.vals, vertices3, vertex_count, triangles3, sl.tris);
    scene_bounds_kernel<<<1, 32, 0, stream>>>(l.bounds, sl.bounds);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    uint32_t status = 0, gave_up = 0;
    st = cudaMemcpyAsync(&status, l.status, sizeof(status), cudaMemcpyDeviceToHost, stream);
    if (st == cudaSuccess) st = cudaMemcpyAsync(&gave_up, ctx->device_error, sizeof(gave_up), cudaMemcpyDeviceToHost, stream);
    if (st == cudaSuccess) st = cudaStreamSynchronize(stream);
    if (st != cudaSuccess) return st;
    if (gave_up != 0) return kWaitGaveUp;
    if (status & kBadIndex) {
        *bad_index = true;
        return cudaErrorInvalidValue;
    }
    ctx->tr_triangles = n;
    ctx->tr_root = 0u;  // internal node 0 (a single triangle: a node with one leaf child)
    return cudaSuccess;
}

cudaError_t trace_rays(HsRasterizerContext* ctx, const TraceCall& c) {
    using namespace tr;
    const cudaStream_t stream = c.stream;
    if (c.ray_count == 0) return cudaSuccess;
    const SceneLayout sl = scene_layout(ctx->tr_scene.ptr, ctx->tr_triangles);
    TraceArgs a{};
    a.rays = static_cast<uint32_t>(c.ray_count);
    a.ray_o = c.ray_origins3;
    a.ray_d = c.ray_directions3;
    a.background = c.background3;
    a.means = c.means3d;
    a.shs = c.shs_m3;
    a.coeffs = c.coefficient_count;
    a.degree = static_cast<int>(c.degree);
    a.others = c.use_others ? c.others2 : nullptr;
    a.opacities = c.opacities;
    a.scales = c.scales2;
    a.scale_modifier = c.scale_modifier;
    a.rotations = c.rotations4;
    a.projmatrix = c.projmatrix4x4;
    a.campos = c.camera_position3;
    a.start_from_first = c.start_from_first;
    a.max_depth = c.max_trace_depth;
    a.specular_threshold = c.specular_threshold;
    a.out_rgb = c.output_rgb3;
    a.out_depth = c.output_depth1;
    a.out_acc = c.output_acc1;
    a.out_normal = c.output_normal3;
    a.out_dist = c.output_dist1;
    a.out_aux = c.output_aux2;
    a.out_mid = c.output_mid32;
    a.bvh = Bvh{sl.nodes, sl.tris, ctx->tr_root};
    // outputs start at zero, as in the reference (optix_backend.cpp:565-573)
    const uint64_t r = c.ray_count;
    cudaError_t st = cudaMemsetAsync(c.output_rgb3, 0, r * 3 * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_depth1, 0, r * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_acc1, 0, r * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_normal3, 0, r * 3 * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_dist1, 0, r * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_aux2, 0, r * 2 * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_mid32, 0, r * 32 * sizeof(float), stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(c.output_wet1, 0, r * sizeof(float), stream);
    if (st != cudaSuccess) return st;
    StageMarks marks(ctx->timer, stream);
    // the rays in spatial order
    const RayLayout need = ray_layout(nullptr, r);
    st = ensure_buffer(ctx->tr_rays, need.bytes, &ctx->tr_growth_count, true);
    if (st != cudaSuccess) return st;
    ctx->tr_peak_bytes = std::max(ctx->tr_peak_bytes, trace_current_bytes(ctx));
    const RayLayout rl = ray_layout(ctx->tr_rays.ptr, r);
    st = cudaMemsetAsync(rl.counter, 0, sizeof(uint32_t), stream);
    if (st != cudaSuccess) return st;
    ray_keys_kernel<<<static_cast<unsigned>((r + kBuildThreads - 1) / kBuildThreads), kBuildThreads, 0, stream>>>(
        a.rays, c.ray_origins3, c.ray_directions3, sl.bounds, rl.keys, rl.vals);
    st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    // sort_pairs' bounded waits report into the trace's own status word
    st = cudaMemsetAsync(rl.counter + 1, 0, sizeof(uint32_t), stream);
    if (st != cudaSuccess) return st;
    st = sort::sort_pairs(rl.keys, rl.vals, rl.alt_keys, rl.alt_vals, a.rays, 0, 32, rl.sort_scratch, stream,
                          rl.counter + 1);
    if (st != cudaSuccess) return st;
    marks.mark(1);
    marks.mark(2);
    int sms = 148, per_sm = 1;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, trace_kernel, kTraceThreads, 0);
    const uint64_t wanted = (r + kTraceThreads - 1) / kTraceThreads;
    const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>(wanted, static_cast<uint64_t>(sms) * std::max(per_sm, 1)));
    trace_kernel<<<blocks, kTraceThreads, 0, stream>>>(a, rl.vals, rl.counter);
    st = cudaGetLastError();
    marks.mark(3);
    return st;
}

}  // namespace hs
