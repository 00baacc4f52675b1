// Standard five-channel backend: per-Gaussian preprocess and per-pixel blend.
//
// Restates, operation by operation, vendor/standard_rasterizer/forward.cu:
//   preprocessCUDA<5>  forward.cu:148-251 (in_frustum auxiliary.h:203-228,
//                      compute_transmat forward.cu:75-115, compute_aabb
//                      forward.cu:119-145, getRect auxiliary.h:85-95)
//   renderCUDA<5>      forward.cu:256-445 (per-pixel blend forward.cu:345-421)
// with the splat transform shared with FlashGS (splat_math.cuh). The
// reference compiles this backend with nvcc defaults (-O3, --fmad=true), so
// it has its own pinned rounding policy.
#pragma once

#include "splat_math.cuh"

namespace hs {
namespace st {

// Forms reproducing the reference standard build (see splat_math.cuh for the
// site list). Unlisted sites use the first variant of their helper.
__host__ __device__ constexpr int pinned_site(int site) {
    switch (site) {
        case S_QN_PAIR: return 1;      // x*x fused onto the rounded w*w
        case S_R00: return 2;          // 1 - 2(y*y + z*z) with both squares rounded
        case S_AABB_D_PAIR: return 1;  // 9*Tw.y^2 fused onto the rounded 9*Tw.x^2
        case S_AABB_P_PAIR: return 2;  // f.x*(Tu.x*Tw.x) + f.y*(...), both rounded
        case S_RHO2: return 1;         // d.y*d.y fused onto the rounded d.x*d.x
        default: return 0;
    }
}

struct PinnedRounding {
    __device__ __forceinline__ int operator()(int site) const { return pinned_site(site); }
};

struct Projected {
    bool valid;         // survived the near cull, facing test and AABB, non-empty rect
    bool behind;        // failed the near cull (the reference traps when prefiltered)
    float depth;
    float2 xy;
    float radius;
    float3 normal;
    float3 tu, tv, tw;
    uint2 rect_min, rect_max;
};

// glm::max(x, y) = (x < y) ? y : x (glm/detail/func_common.inl:25-30).
__device__ __forceinline__ float glm_max(float x, float y) { return (x < y) ? y : x; }

template <class R>
__device__ __forceinline__ Projected project_gaussian(const R& r, const float* view,
                                                      const float* proj, float3 p, float2 scale,
                                                      float scale_modifier, float4 rot,
                                                      int width, int height, uint32_t grid_x,
                                                      uint32_t grid_y) {
    Projected g;
    g.valid = false;
    g.behind = false;
    const float pvx = affine_row(r, S_PVIEW_PAIR, S_PVIEW_TAIL, view, 0, p.x, p.y, p.z);
    const float pvy = affine_row(r, S_PVIEW_PAIR, S_PVIEW_TAIL, view, 1, p.x, p.y, p.z);
    const float pvz = affine_row(r, S_PVIEW_PAIR, S_PVIEW_TAIL, view, 2, p.x, p.y, p.z);
    g.depth = pvz;
    if (pvz <= 0.2f) {
        g.behind = true;
        return g;
    }
    float3 n;
    splat_transform(r, view, proj, p, scale, scale_modifier, rot, width, height, g.tu, g.tv,
                    g.tw, n);
    const float cosv = -dot3(r(S_COS_PAIR), r(S_COS_TAIL), pvx, n.x, pvy, n.y, pvz, n.z);
    if (cosv == 0.0f) return g;
    const float sign = cosv > 0.0f ? 1.0f : -1.0f;
    g.normal = make_float3(mul(sign, n.x), mul(sign, n.y), mul(sign, n.z));

    // compute_aabb with cutoff 3: t = (9, 9, -1).
    const float sqx = mul(g.tw.x, g.tw.x), sqy = mul(g.tw.y, g.tw.y), sqz = mul(g.tw.z, g.tw.z);
    const float dpair = dot2(r(S_AABB_D_PAIR), 9.0f, sqx, 9.0f, sqy);
    const float d = r(S_AABB_D_TAIL) == 0 ? fma(-g.tw.z, g.tw.z, dpair) : sub(dpair, sqz);
    if (d == 0.0f) return g;
    const float inv = div(1.0f, d);
    const float fx = mul(inv, 9.0f), fy = mul(inv, 9.0f), fz = -inv;
    const float px = dot3(r(S_AABB_P_PAIR), r(S_AABB_P_TAIL), fx, mul(g.tu.x, g.tw.x), fy,
                          mul(g.tu.y, g.tw.y), fz, mul(g.tu.z, g.tw.z));
    const float py = dot3(r(S_AABB_P_PAIR), r(S_AABB_P_TAIL), fx, mul(g.tv.x, g.tw.x), fy,
                          mul(g.tv.y, g.tw.y), fz, mul(g.tv.z, g.tw.z));
    const float qx = dot3(r(S_AABB_Q_PAIR), r(S_AABB_Q_TAIL), fx, mul(g.tu.x, g.tu.x), fy,
                          mul(g.tu.y, g.tu.y), fz, mul(g.tu.z, g.tu.z));
    const float qy = dot3(r(S_AABB_Q_PAIR), r(S_AABB_Q_TAIL), fx, mul(g.tv.x, g.tv.x), fy,
                          mul(g.tv.y, g.tv.y), fz, mul(g.tv.z, g.tv.z));
    const float h0x = msub(r(S_AABB_H), px, px, qx);
    const float h0y = msub(r(S_AABB_H), py, py, qy);
    const float hx = __fsqrt_rn(glm_max(1e-4f, h0x));
    const float hy = __fsqrt_rn(glm_max(1e-4f, h0y));
    g.xy = make_float2(px, py);
    g.radius = ceilf(fmaxf(fmaxf(hx, hy), 3.0f * 0.707106f));

    // getRect with BLOCK_X = BLOCK_Y = 16 and an int radius.
    const float rad = static_cast<float>(static_cast<int>(g.radius));
    g.rect_min.x = min(grid_x, static_cast<uint32_t>(max(0, __float2int_rz(div(sub(px, rad), 16.0f)))));
    g.rect_min.y = min(grid_y, static_cast<uint32_t>(max(0, __float2int_rz(div(sub(py, rad), 16.0f)))));
    g.rect_max.x = min(grid_x, static_cast<uint32_t>(max(
                                   0, __float2int_rz(div(sub(add(add(px, rad), 16.0f), 1.0f), 16.0f)))));
    g.rect_max.y = min(grid_y, static_cast<uint32_t>(max(
                                   0, __float2int_rz(div(sub(add(add(py, rad), 16.0f), 1.0f), 16.0f)))));
    g.valid = (g.rect_max.x - g.rect_min.x) * (g.rect_max.y - g.rect_min.y) != 0;
    return g;
}

struct PixelState {
    float c[5];
    float t;
    float d;
    float m1, m2;
    float dist;
    float median;
    float n[3];
    bool done;
};

__device__ __forceinline__ void pixel_init(PixelState& s, bool inside) {
#pragma unroll
    for (int k = 0; k < 5; ++k) s.c[k] = 0.0f;
    s.t = 1.0f;
    s.d = 0.0f;
    s.m1 = s.m2 = 0.0f;
    s.dist = 0.0f;
    s.median = 0.0f;
    s.n[0] = s.n[1] = s.n[2] = 0.0f;
    s.done = !inside;
}

// Per-Gaussian blend record (same 80-byte layout as FlashGS: xy, normal,
// opacity, five colour channels, Tu, Tv, Tw).
struct BlendRecord {
    float x, y;
    float nx, ny, nz, op;
    float c[5];
    float tux, tuy, tuz;
    float tvx, tvy, tvz;
    float twx, twy, twz;
};

// One pixel, one Gaussian (forward.cu:345-421). Returns the blend weight w
// (0 when the Gaussian was skipped for this pixel).
template <class R>
__device__ __forceinline__ float blend(const R& r, PixelState& s, float px, float py,
                                       const BlendRecord& g) {
    if (s.done) return 0.0f;
    const int vk = r(S_K);
    const float kx = msub(vk, px, g.twx, g.tux);
    const float ky = msub(vk, px, g.twy, g.tuy);
    const float kz = msub(vk, px, g.twz, g.tuz);
    const float lx = msub(vk, py, g.twx, g.tvx);
    const float ly = msub(vk, py, g.twy, g.tvy);
    const float lz = msub(vk, py, g.twz, g.tvz);
    const int vc = r(S_CROSS);
    const float pzv = diff2(vc, kx, ly, ky, lx);
    if (pzv == 0.0f) return 0.0f;
    const float pxv = diff2(vc, ky, lz, kz, ly);
    const float pyv = diff2(vc, kz, lx, kx, lz);
    const float sx = div(pxv, pzv);
    const float sy = div(pyv, pzv);
    const float rho3d = dot2(r(S_RHO3), sx, sx, sy, sy);
    const float dx = sub(g.x, px);
    const float dy = sub(g.y, py);
    const float rho2d = mul(2.0f, dot2(r(S_RHO2), dx, dx, dy, dy));
    const float rho = fminf(rho3d, rho2d);
    const float depth =
        rho3d <= rho2d ? add(dot2(r(S_DEPTH), sx, g.twx, sy, g.twy), g.twz) : g.twz;
    if (depth < kNear) return 0.0f;
    const float power = mul(-0.5f, rho);
    if (power > 0.0f) return 0.0f;
    const float alpha = fminf(0.99f, mul(g.op, expf(power)));
    if (alpha < 1.0f / 255.0f) return 0.0f;
    const float test_t = mul(s.t, sub(1.0f, alpha));
    if (test_t < 0.0001f) {
        s.done = true;
        return 0.0f;
    }
    const float w = mul(alpha, s.t);
    const float a = sub(1.0f, s.t);
    const float m = mul(kFar / (kFar - kNear), sub(1.0f, div(kNear, depth)));
    const float mm = mul(m, m);
    const int va = r(S_ACC);
    const float dd = nmad(r(S_D2), mad(r(S_D1), mm, a, s.m2), mul(2.0f, m), s.m1);
    s.dist = mad(va, dd, w, s.dist);
    s.d = mad(va, depth, w, s.d);
    s.m1 = mad(va, m, w, s.m1);
    s.m2 = mad(va, mm, w, s.m2);
    if (s.t > 0.5f) s.median = depth;
    s.n[0] = mad(va, g.nx, w, s.n[0]);
    s.n[1] = mad(va, g.ny, w, s.n[1]);
    s.n[2] = mad(va, g.nz, w, s.n[2]);
#pragma unroll
    for (int k = 0; k < 5; ++k) s.c[k] = mad(va, g.c[k], w, s.c[k]);
    s.t = test_t;
    return w;
}

}  // namespace st
}  // namespace hs
