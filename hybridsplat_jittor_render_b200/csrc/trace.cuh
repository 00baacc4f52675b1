// Reflection trace: ray/triangle test, BVH layout and the per-hit 2DGS
// shading of the reference OptiX programs, as device code.
//
// The reference traces one ray per reflective Gaussian against a GAS built
// from two triangles per reflective Gaussian (the 6-sigma square of its
// disk, math.py:253-298) with an any-hit program that keeps the CHUNK_SIZE =
// 16 nearest hits of each optixTrace in a sorted buffer and a raygen program
// that shades them front to back, restarting the trace behind the last
// processed hit while the buffer came back full
// (vendor/optix_tracer/forward.cu:219-405, 563-660; config.h:31-45;
// auxiliary.h:31-55, 230-243, 265-272, 386-441). Here the GAS is a BVH built
// by this library (trace.cu) and each trace step is a BVH traversal that
// collects the same 16 nearest hits; hits are ordered by distance, ties by
// primitive index. Every product and sum is an explicitly rounded operation
// (fp.cuh) so that the CPU oracle (oracle/cpu_oracle.c) restates it exactly;
// only expf differs between the two.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fp.cuh"

namespace hs {
namespace tr {

constexpr int kChunk = 16;                 // CHUNK_SIZE
constexpr float kDepthInfinity = 1e16f;    // DEPTH_INFINTY, also the trace's tmax
constexpr int kMaxContributors = 256;      // MAX_INTERSECTION
constexpr double kStepEpsilon = 0.00001;   // STEP_EPSILON (a double constant)
constexpr float kStartOffset = 0.06f;      // START_OFFSET as the float min_depth
constexpr float kNear = 0.2f;              // near_n
constexpr float kFar = 100.0f;             // far_n
constexpr float kFilterInvSquare = 2.0f;
constexpr float kTThreshold = 0.0001f;
constexpr int kMidChannels = 16;           // MID_CHANNELS per trace depth
constexpr uint32_t kLeafBit = 0x80000000u; // child reference: leaf slot
constexpr uint32_t kNoChild = 0xffffffffu; // empty child slot of a wide node
// Traversal stack: a wide node's children lie at least one binary level below
// it and the binary tree is at most 64 internal nodes deep, so the path of
// wide nodes being traversed is at most 64 long; each leaves at most 3
// siblings on the stack, plus the 4 children of the node being expanded.
constexpr int kStackDepth = 3 * 64 + 4;
constexpr int kMaxTraceSteps = 4096;    // trace steps (16 hits each) per segment

// BVH over the scene triangles, 4 children per node (the binary radix tree
// with every second level collapsed; children's boxes stored in the parent,
// one coordinate of the four children per float4): node k = 8 float4
// {min x, max x, min y, max y, min z, max z, child references, unused}; a
// child reference with kLeafBit names a leaf slot, whose triangle is
// 3 float4 {v0 | primitive index, v1, v2} in `tris`; kNoChild an empty slot
// (its box is empty).
constexpr int kWideQuads = 8;
struct Bvh {
    const float4* nodes;
    const float4* tris;
    uint32_t root;  // reference of the root node
};

__device__ __forceinline__ float3 f3(float x, float y, float z) { return make_float3(x, y, z); }
__device__ __forceinline__ float comp(const float3& v, int k) { return k == 0 ? v.x : (k == 1 ? v.y : v.z); }

// Per-ray constants of the watertight ray/triangle test (Woop, Benthin and
// Wald, "Watertight Ray/Triangle Intersection", JCGT 2(1), 2013): the
// dominant axis kz, the shear (sx, sy) and the scale sz.
struct RayShear {
    int kx, ky, kz;
    float sx, sy, sz;
};

__device__ __forceinline__ RayShear ray_shear(const float3& d) {
    const float ax = fabsf(d.x), ay = fabsf(d.y), az = fabsf(d.z);
    RayShear r;
    r.kz = (ax > ay) ? (ax > az ? 0 : 2) : (ay > az ? 1 : 2);
    r.kx = r.kz == 2 ? 0 : r.kz + 1;
    r.ky = r.kx == 2 ? 0 : r.kx + 1;
    if (comp(d, r.kz) < 0.0f) {
        const int t = r.kx;
        r.kx = r.ky;
        r.ky = t;
    }
    const float dz = comp(d, r.kz);
    r.sx = div(comp(d, r.kx), dz);
    r.sy = div(comp(d, r.ky), dz);
    r.sz = div(1.0f, dz);
    return r;
}

// Distance t of the hit of ray (o, shear) with triangle (a, b, c), or a
// negative value for a miss; both faces count. Edges shared by two
// triangles are hit by at least one of them.
__device__ __forceinline__ float hit_triangle(const float3& o, const RayShear& r, const float3& a,
                                              const float3& b, const float3& c) {
    const float3 A = f3(sub(a.x, o.x), sub(a.y, o.y), sub(a.z, o.z));
    const float3 B = f3(sub(b.x, o.x), sub(b.y, o.y), sub(b.z, o.z));
    const float3 C = f3(sub(c.x, o.x), sub(c.y, o.y), sub(c.z, o.z));
    const float ax = sub(comp(A, r.kx), mul(r.sx, comp(A, r.kz)));
    const float ay = sub(comp(A, r.ky), mul(r.sy, comp(A, r.kz)));
    const float bx = sub(comp(B, r.kx), mul(r.sx, comp(B, r.kz)));
    const float by = sub(comp(B, r.ky), mul(r.sy, comp(B, r.kz)));
    const float cx = sub(comp(C, r.kx), mul(r.sx, comp(C, r.kz)));
    const float cy = sub(comp(C, r.ky), mul(r.sy, comp(C, r.kz)));
    float u = sub(mul(cx, by), mul(cy, bx));
    float v = sub(mul(ax, cy), mul(ay, cx));
    float w = sub(mul(bx, ay), mul(by, ax));
    if (u == 0.0f || v == 0.0f || w == 0.0f) {
        // edge cases: the 2x2 determinants in double (exact for float inputs)
        u = static_cast<float>(static_cast<double>(cx) * by - static_cast<double>(cy) * bx);
        v = static_cast<float>(static_cast<double>(ax) * cy - static_cast<double>(ay) * cx);
        w = static_cast<float>(static_cast<double>(bx) * ay - static_cast<double>(by) * ax);
    }
    if ((u < 0.0f || v < 0.0f || w < 0.0f) && (u > 0.0f || v > 0.0f || w > 0.0f)) return -1.0f;
    const float det = add(add(u, v), w);
    if (det == 0.0f) return -1.0f;
    const float az = mul(r.sz, comp(A, r.kz));
    const float bz = mul(r.sz, comp(B, r.kz));
    const float cz = mul(r.sz, comp(C, r.kz));
    const float t = div(add(add(mul(u, az), mul(v, bz)), mul(w, cz)), det);
    return t >= 0.0f ? t : -1.0f;  // NaN compares false: a miss
}

// Slab test of the box [lo, hi] against [0, limit]; inv = 1 / d per axis.
__device__ __forceinline__ bool hit_box(const float3& o, const float3& inv, float lx, float ly, float lz,
                                        float hx, float hy, float hz, float limit, float& entry) {
    const float tx0 = mul(sub(lx, o.x), inv.x), tx1 = mul(sub(hx, o.x), inv.x);
    const float ty0 = mul(sub(ly, o.y), inv.y), ty1 = mul(sub(hy, o.y), inv.y);
    const float tz0 = mul(sub(lz, o.z), inv.z), tz1 = mul(sub(hz, o.z), inv.z);
    const float tn = fmaxf(fmaxf(fminf(tx0, tx1), fminf(ty0, ty1)), fmaxf(fminf(tz0, tz1), 0.0f));
    const float tf = fminf(fminf(fmaxf(tx0, tx1), fmaxf(ty0, ty1)), fminf(fmaxf(tz0, tz1), limit));
    entry = tn;
    return tn <= tf;
}

// ---------------------------------------------------------------- shading

__device__ __forceinline__ float dot3f(const float3& a, const float3& b) {
    return fma(a.z, b.z, fma(a.y, b.y, mul(a.x, b.x)));
}

// normalize (auxiliary.h:242): v / sqrt(v.v)
__device__ __forceinline__ float3 normalize3(const float3& v) {
    const float n = __fsqrt_rn(dot3f(v, v));
    return f3(div(v.x, n), div(v.y, n), div(v.z, n));
}

// Rows of the transposed rotation of quaternion (w, x, y, z) =
// (q.x, q.y, q.z, q.w) after normalisation (quat_to_rotmat_transpose,
// auxiliary.h:414-441); 1/sqrt instead of rsqrtf.
__device__ __forceinline__ void rotation_rows_t(const float4& q, float3 R[3]) {
    const float s = div(1.0f, __fsqrt_rn(fma(q.z, q.z, fma(q.y, q.y, fma(q.x, q.x, mul(q.w, q.w))))));
    const float w = mul(q.x, s), x = mul(q.y, s), y = mul(q.z, s), z = mul(q.w, s);
    R[0] = f3(sub(1.0f, mul(2.0f, fma(z, z, mul(y, y)))), mul(2.0f, fma(w, z, mul(x, y))),
              mul(2.0f, fma(-w, y, mul(x, z))));
    R[1] = f3(mul(2.0f, fma(-w, z, mul(x, y))), sub(1.0f, mul(2.0f, fma(z, z, mul(x, x)))),
              mul(2.0f, fma(w, x, mul(y, z))));
    R[2] = f3(mul(2.0f, fma(w, y, mul(x, z))), mul(2.0f, fma(-w, x, mul(y, z))),
              sub(1.0f, mul(2.0f, fma(y, y, mul(x, x)))));
}

// Rows of the rotation itself (quat_to_rotmat, auxiliary.h:386-412).
__device__ __forceinline__ void rotation_rows(const float4& q, float3 R[3]) {
    float3 T[3];
    rotation_rows_t(q, T);
    R[0] = f3(T[0].x, T[1].x, T[2].x);
    R[1] = f3(T[0].y, T[1].y, T[2].y);
    R[2] = f3(T[0].z, T[1].z, T[2].z);
}

// computeColorFromSH of the tracer (forward.cu:25-69), degree <= 3, in the
// direction `dir_orig` (normalised here).
__device__ __forceinline__ float3 sh_color(int deg, const float* sh, const float3& dir_orig) {
    constexpr float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
    constexpr float C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                             -1.0925484305920792f, 0.5462742152960396f};
    constexpr float C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                             0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                             -0.5900435899266435f};
    auto coef = [&](int k, int ch) { return sh[3 * k + ch]; };
    float res[3];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) res[ch] = mul(C0, coef(0, ch));
    const float3 d = normalize3(dir_orig);
    if (deg > 0) {
        const float x = d.x, y = d.y, z = d.z;
        const float c1y = mul(C1, y), c1z = mul(C1, z), c1x = mul(C1, x);
#pragma unroll
        for (int ch = 0; ch < 3; ++ch)
            res[ch] = fma(-c1x, coef(3, ch), fma(c1z, coef(2, ch), fma(-c1y, coef(1, ch), res[ch])));
        if (deg > 1) {
            const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
            const float xy = mul(x, y), yz = mul(y, z), xz = mul(x, z);
            const float f4 = mul(C2[0], xy), f5 = mul(C2[1], yz);
            const float f6 = mul(C2[2], sub(sub(mul(2.0f, zz), xx), yy));
            const float f7 = mul(C2[3], xz), f8 = mul(C2[4], sub(xx, yy));
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                float t = fma(f4, coef(4, ch), res[ch]);
                t = fma(f5, coef(5, ch), t);
                t = fma(f6, coef(6, ch), t);
                t = fma(f7, coef(7, ch), t);
                res[ch] = fma(f8, coef(8, ch), t);
            }
            if (deg > 2) {
                const float g9 = mul(mul(C3[0], y), sub(mul(3.0f, xx), yy));
                const float g10 = mul(mul(C3[1], xy), z);
                const float g11 = mul(mul(C3[2], y), sub(sub(mul(4.0f, zz), xx), yy));
                const float g12 = mul(mul(C3[3], z), sub(sub(mul(2.0f, zz), mul(3.0f, xx)), mul(3.0f, yy)));
                const float g13 = mul(mul(C3[4], x), sub(sub(mul(4.0f, zz), xx), yy));
                const float g14 = mul(mul(C3[5], z), sub(xx, yy));
                const float g15 = mul(mul(C3[6], x), sub(xx, mul(3.0f, yy)));
#pragma unroll
                for (int ch = 0; ch < 3; ++ch) {
                    float t = fma(g9, coef(9, ch), res[ch]);
                    t = fma(g10, coef(10, ch), t);
                    t = fma(g11, coef(11, ch), t);
                    t = fma(g12, coef(12, ch), t);
                    t = fma(g13, coef(13, ch), t);
                    t = fma(g14, coef(14, ch), t);
                    res[ch] = fma(g15, coef(15, ch), t);
                }
            }
        }
    }
    return f3(fmaxf(add(res[0], 0.5f), 0.0f), fmaxf(add(res[1], 0.5f), 0.0f), fmaxf(add(res[2], 0.5f), 0.0f));
}

}  // namespace tr
}  // namespace hs
