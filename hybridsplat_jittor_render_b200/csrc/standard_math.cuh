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

#include <climits>

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
        case S_AABB_PX_PAIR: return 1; // centre x: f.y*(Tu.y*Tw.y) fused onto the rounded f.x*(...)
        case S_AABB_QX_PAIR: return 1; // extent x: f.y*(Tu.y*Tu.y) fused onto the rounded f.x*(...)
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
    const float px = dot3(r(S_AABB_PX_PAIR), r(S_AABB_P_TAIL), fx, mul(g.tu.x, g.tw.x), fy,
                          mul(g.tu.y, g.tw.y), fz, mul(g.tu.z, g.tw.z));
    const float py = dot3(r(S_AABB_PY_PAIR), r(S_AABB_P_TAIL), fx, mul(g.tv.x, g.tw.x), fy,
                          mul(g.tv.y, g.tw.y), fz, mul(g.tv.z, g.tw.z));
    const float qx = dot3(r(S_AABB_QX_PAIR), r(S_AABB_Q_TAIL), fx, mul(g.tu.x, g.tu.x), fy,
                          mul(g.tu.y, g.tu.y), fz, mul(g.tu.z, g.tu.z));
    const float qy = dot3(r(S_AABB_QY_PAIR), r(S_AABB_Q_TAIL), fx, mul(g.tv.x, g.tv.x), fy,
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

// The terms of an evaluation that depend only on the pixel column: the
// k = x Tw - Tu vector of the ray-splat intersection and x's offset from the
// centre. A lane's two pixels share their column, so these are formed once.
struct ColumnTerms {
    float kx, ky, kz, dx;
};

template <class R>
__device__ __forceinline__ ColumnTerms column_terms(const R& r, float px, const BlendRecord& g) {
    const int vk = r(S_K);
    return ColumnTerms{msub(vk, px, g.twx, g.tux), msub(vk, px, g.twy, g.tuy),
                       msub(vk, px, g.twz, g.tuz), sub(g.x, px)};
}

// One pixel, one Gaussian (forward.cu:345-421). Returns the blend weight w
// (0 when the Gaussian was skipped for this pixel).
template <class R>
__device__ __forceinline__ float blend(const R& r, PixelState& s, const ColumnTerms& col, float py,
                                       const BlendRecord& g) {
    if (s.done) return 0.0f;
    const int vk = r(S_K);
    const float kx = col.kx, ky = col.ky, kz = col.kz;
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
    const float dx = col.dx;
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

// The alpha of one pixel x Gaussian evaluation, with the operations of blend()
// up to its alpha test but no early exit: `live` is false exactly where
// blend() returns before its transmittance test (a done pixel, p.z == 0,
// depth < near, power > 0, alpha < 1/255; NaNs pass as they do there).
template <class R>
__device__ __forceinline__ float alpha_of(const R& r, const PixelState& s, const ColumnTerms& col, float py,
                                          const BlendRecord& g, float& depth, bool& live) {
    const int vk = r(S_K);
    const float lx = msub(vk, py, g.twx, g.tvx);
    const float ly = msub(vk, py, g.twy, g.tvy);
    const float lz = msub(vk, py, g.twz, g.tvz);
    const int vc = r(S_CROSS);
    const float pzv = diff2(vc, col.kx, ly, col.ky, lx);
    const float pxv = diff2(vc, col.ky, lz, col.kz, ly);
    const float pyv = diff2(vc, col.kz, lx, col.kx, lz);
    const float sx = div(pxv, pzv);
    const float sy = div(pyv, pzv);
    const float rho3d = dot2(r(S_RHO3), sx, sx, sy, sy);
    const float dy = sub(g.y, py);
    const float rho2d = mul(2.0f, dot2(r(S_RHO2), col.dx, col.dx, dy, dy));
    const float rho = fminf(rho3d, rho2d);
    depth = rho3d <= rho2d ? add(dot2(r(S_DEPTH), sx, g.twx, sy, g.twy), g.twz) : g.twz;
    const float power = mul(-0.5f, rho);
    const float alpha = fminf(0.99f, mul(g.op, expf(power)));
    live = !s.done && pzv != 0.0f && !(depth < kNear) && !(power > 0.0f) && !(alpha < 1.0f / 255.0f);
    return alpha;
}

// alpha_of for a lane's two pixels (rows py0 and py1 of one column), with
// every operation the two pixels share issued once as a packed pair (fp.cuh:
// each component rounds as the scalar instruction of alpha_of); the
// divisions, expf and the minima stay per pixel. Outputs as alpha_of's, for
// pixel 0 and pixel 1.
template <class R>
__device__ __forceinline__ void alpha_of2(const R& r, const PixelState& s0, const PixelState& s1,
                                          const ColumnTerms& col, float py0, float py1, const BlendRecord& g,
                                          float& a0, float& a1, float& d0, float& d1, bool& live0, bool& live1) {
    const float2 py = make_float2(py0, py1);
    const int vk = r(S_K);
    const float2 lx = msub_x2(vk, py, pair(g.twx), pair(g.tvx));
    const float2 ly = msub_x2(vk, py, pair(g.twy), pair(g.tvy));
    const float2 lz = msub_x2(vk, py, pair(g.twz), pair(g.tvz));
    const int vc = r(S_CROSS);
    const float2 kx = pair(col.kx), ky = pair(col.ky), kz = pair(col.kz);
    const float2 pzv = diff2_x2(vc, kx, ly, ky, lx);
    const float2 pxv = diff2_x2(vc, ky, lz, kz, ly);
    const float2 pyv = diff2_x2(vc, kz, lx, kx, lz);
    const float2 sx = make_float2(div(pxv.x, pzv.x), div(pxv.y, pzv.y));
    const float2 sy = make_float2(div(pyv.x, pzv.x), div(pyv.y, pzv.y));
    const float2 rho3d = dot2_x2(r(S_RHO3), sx, sx, sy, sy);
    const float2 dy = sub2(pair(g.y), py);
    const float2 rho2d = mul2(pair(2.0f), dot2_x2(r(S_RHO2), pair(col.dx), pair(col.dx), dy, dy));
    const float2 rho = make_float2(fminf(rho3d.x, rho2d.x), fminf(rho3d.y, rho2d.y));
    const float2 on_plane = add2(dot2_x2(r(S_DEPTH), sx, pair(g.twx), sy, pair(g.twy)), pair(g.twz));
    d0 = rho3d.x <= rho2d.x ? on_plane.x : g.twz;
    d1 = rho3d.y <= rho2d.y ? on_plane.y : g.twz;
    const float2 power = mul2(pair(-0.5f), rho);
    const float2 scaled = mul2(pair(g.op), make_float2(expf(power.x), expf(power.y)));
    a0 = fminf(0.99f, scaled.x);
    a1 = fminf(0.99f, scaled.y);
    live0 = !s0.done && pzv.x != 0.0f && !(d0 < kNear) && !(power.x > 0.0f) && !(a0 < 1.0f / 255.0f);
    live1 = !s1.done && pzv.y != 0.0f && !(d1 < kNear) && !(power.y > 0.0f) && !(a1 < 1.0f / 255.0f);
}

// The state update of blend() after its alpha test. Returns w.
template <class R>
__device__ __forceinline__ float apply(const R& r, PixelState& s, float alpha, float depth, const BlendRecord& g) {
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

// blend() for a lane's two pixels (same column, rows py0 and py1): both
// alphas are computed without branches, so their dependency chains
// interleave; each update is applied where blend() would apply it. Returns
// the sum of the two weights.
template <class R>
__device__ __forceinline__ float blend2(const R& r, PixelState& s0, PixelState& s1, const ColumnTerms& col,
                                        float py0, float py1, const BlendRecord& g) {
    float a0, a1, d0, d1;
    bool live0, live1;
    alpha_of2(r, s0, s1, col, py0, py1, g, a0, a1, d0, d1, live0, live1);
    float w = 0.0f;
    if (live0) w = apply(r, s0, a0, d0, g);
    if (live1) w += apply(r, s1, a1, d1, g);
    return w;
}

// ---------------------------------------------------------------- culling
//
// A pixel x Gaussian evaluation changes the pixel state only when
// alpha = min(0.99, op * expf(-rho / 2)) >= 1/255 (forward.cu:392-393; the
// median, depth, normal and colour updates all follow that test). Since
// 0.99 > 1/255 this needs rho <= c = 2 ln(255 op), and rho = min(rho3d, rho2d)
// with rho3d = s.s (the ray-splat intersection in splat units) and
// rho2d = 2 |xy - pixel|^2. So the pixels that can change are inside
//   * the image of the disc s.s <= c under the splat's homography: an ellipse
//     with centre m and matrix S, (p - m)^T S^-1 (p - m) <= 1, whenever the
//     splat plane's horizon stays off the disc (otherwise: no culling); and
//   * the disc |p - xy|^2 <= c / 2.
// m and S come from the dual conic of the disc, the same construction the
// reference uses for its cutoff-3 AABB (forward.cu:119-145) with the cutoff
// replaced by sqrt(c). The shape is computed in double precision with c
// widened to 1.02 c + 0.05, and quadrant rectangles are widened by kCullPad,
// so rounding in the per-pixel arithmetic cannot make a culled evaluation
// live. Culling therefore never changes an output value; it only skips
// evaluations that would have returned early.
enum CullMode : int { kCullEllipse = 0, kCullNever = 1, kCullAlways = 2 };

// The ellipse is stored by its horizontal chords: with Y the height above
// the centre, the chord at Y is centred at mx + k Y and has half-width
// w0 sqrt(1 - (Y / hy)^2) for |Y| <= hy; its extreme points are x = mx +- hx
// at heights +-yr. These parameters are computed in double from the dual
// conic and scaled together by 1.0003 about the centre (a uniform widening
// that dwarfs their float rounding). The x-extent of the ellipse over a band
// of rows then costs two square roots (the chord ends at the band's edges, or
// the extreme point when its height is inside the band), so each band of a
// Gaussian is reduced to two x-intervals (ellipse, disc) and a tile or
// quadrant is live when its widened x-range meets one of them. The square
// roots are the approximate hardware ones (relative error ~1e-7, far inside
// the widening); every other step is an explicitly rounded operation, so the
// preprocess (which counts the live tiles) and the emission (which writes
// them) compute the same bits and take identical decisions.
struct CullShape {
    float mx, my;     // ellipse centre (pixels)
    float k;          // chord-centre slope
    float w0;         // chord half-width at the centre height
    float hx, hy;     // half extents of the ellipse's bounding box
    float yr;         // height of the rightmost point (the leftmost is at -yr)
    float ihy;        // 1 / hy
    float gx, gy, r2; // disc centre and squared radius
    int mode;         // kCullEllipse: test; kCullNever: every pixel may be live; kCullAlways: none
};

__device__ __forceinline__ CullShape cull_shape(float op, float x, float y, float3 tu, float3 tv,
                                                float3 tw) {
    CullShape c;
    c.mx = c.my = c.k = c.w0 = c.hx = c.hy = c.yr = c.ihy = 0.0f;
    c.gx = x;
    c.gy = y;
    c.r2 = 0.0f;
    if (!(op > 1.0f / 255.0f)) {  // op * expf(.) < 1/255 everywhere (NaN opacity included)
        c.mode = kCullAlways;
        return c;
    }
    // The widening (2% + 0.05) dwarfs the error of logf here.
    const float cwf = 1.02f * (2.0f * logf(255.0f * op)) + 0.05f;
    const double cw = static_cast<double>(cwf) * 1.0001;
    c.r2 = static_cast<float>(0.5 * cw * 1.0001);
    const double twx = tw.x, twy = tw.y, twz = tw.z;
    const double d = cw * (twx * twx + twy * twy) - twz * twz;
    c.mode = kCullNever;
    if (!(d < -1e-6 * twz * twz)) return c;  // unbounded image of the disc
    // Dual-conic moments in double: m^2 - q cancels to the ellipse size.
    const double fxy = cw / d, fz = -1.0 / d;
    const double mx = fxy * (double(tu.x) * twx + double(tu.y) * twy) + fz * double(tu.z) * twz;
    const double my = fxy * (double(tv.x) * twx + double(tv.y) * twy) + fz * double(tv.z) * twz;
    const double quu = fxy * (double(tu.x) * tu.x + double(tu.y) * tu.y) + fz * double(tu.z) * tu.z;
    const double qvv = fxy * (double(tv.x) * tv.x + double(tv.y) * tv.y) + fz * double(tv.z) * tv.z;
    const double quv = fxy * (double(tu.x) * tv.x + double(tu.y) * tv.y) + fz * double(tu.z) * tv.z;
    // (p - m)^T S^-1 (p - m) <= 1 with S = [[sxx, sxy], [sxy, syy]]
    const double sxx = mx * mx - quu, syy = my * my - qvv, sxy = mx * my - quv;
    const double det = sxx * syy - sxy * sxy;
    if (!(sxx > 0.0 && syy > 0.0 && det > 0.0) || !(fabs(mx) < 1e7 && fabs(my) < 1e7)) return c;
    constexpr double kWiden = 1.0003;
    c.mx = static_cast<float>(mx);
    c.my = static_cast<float>(my);
    c.k = static_cast<float>(sxy / syy);
    c.w0 = static_cast<float>(sqrt(det / syy) * kWiden);
    c.hx = static_cast<float>(sqrt(sxx) * kWiden);
    c.hy = static_cast<float>(sqrt(syy) * kWiden);
    c.yr = static_cast<float>(sxy / sqrt(sxx) * kWiden);
    c.ihy = static_cast<float>(1.0 / (sqrt(syy) * kWiden));
    c.mode = kCullEllipse;
    return c;
}

// x-interval [l, r] (pixels) of the ellipse within rows [ya, yb]; empty
// (l > r) when the band misses it.
__device__ __forceinline__ void ellipse_span(const CullShape& c, float ya, float yb, float& l,
                                             float& r) {
    const float y0 = fmaxf(sub(ya, c.my), -c.hy), y1 = fminf(sub(yb, c.my), c.hy);
    if (!(y0 <= y1)) {
        l = 1.0f;
        r = 0.0f;
        return;
    }
    const float t0 = fminf(fmaxf(mul(y0, c.ihy), -1.0f), 1.0f);
    const float t1 = fminf(fmaxf(mul(y1, c.ihy), -1.0f), 1.0f);
    const float h0 = mul(c.w0, approx_sqrt(mul(sub(1.0f, t0), add(1.0f, t0))));
    const float h1 = mul(c.w0, approx_sqrt(mul(sub(1.0f, t1), add(1.0f, t1))));
    const float c0 = mul(c.k, y0), c1 = mul(c.k, y1);
    float xl = fminf(sub(c0, h0), sub(c1, h1));
    float xr = fmaxf(add(c0, h0), add(c1, h1));
    if (y0 <= -c.yr && -c.yr <= y1) xl = fminf(xl, -c.hx);
    if (y0 <= c.yr && c.yr <= y1) xr = fmaxf(xr, c.hx);
    l = add(c.mx, xl);
    r = add(c.mx, xr);
}

// x-interval of the disc within rows [ya, yb].
__device__ __forceinline__ void disc_span(const CullShape& c, float ya, float yb, float& l,
                                          float& r) {
    const float dy = fmaxf(fmaxf(sub(ya, c.gy), sub(c.gy, yb)), 0.0f);
    const float q = sub(c.r2, mul(dy, dy));
    if (!(q >= 0.0f)) {
        l = 1.0f;
        r = 0.0f;
        return;
    }
    const float w = approx_sqrt(q);
    l = sub(c.gx, w);
    r = add(c.gx, w);
}

// Does [x0, x1] meet [l, r]? (False for an empty or NaN interval.)
__device__ __forceinline__ bool meets(float l, float r, float x0, float x1) {
    return x0 <= r && x1 >= l && l <= r;
}

// Culling intervals of one band of rows: ellipse and disc.
struct BandSpans {
    float el, er, dl, dr;
};

__device__ __forceinline__ BandSpans band_spans(const CullShape& c, float ya, float yb) {
    BandSpans s;
    ellipse_span(c, ya, yb, s.el, s.er);
    disc_span(c, ya, yb, s.dl, s.dr);
    return s;
}

// Pixels whose evaluation can be live lie inside the culling shapes, which
// are already widened in their threshold and scale; tiles and quadrants are
// further widened by kCullPad pixels on each side to cover the float rounding
// of the span arithmetic (below 1e-3 px at screen coordinates under 4e6).
// Every bound is an integer plus or minus kCullPad, exact in float.
constexpr float kCullPad = 0.25f;

// Spans of the two 8-row quadrant bands of tile row ty, widened by kCullPad:
// rows [16 ty + 8 qy - pad, 16 ty + 8 qy + 7 + pad].
__device__ __forceinline__ BandSpans quadrant_band_spans(const CullShape& c, int ty, int qy) {
    const float y = static_cast<float>(ty * 16 + qy * 8);
    return band_spans(c, y - kCullPad, y + (7.0f + kCullPad));
}

__device__ __forceinline__ void hull(float al, float ar, float bl, float br, float& l, float& r) {
    const bool a = al <= ar, b = bl <= br;
    l = a && b ? fminf(al, bl) : (a ? al : (b ? bl : 1.0f));
    r = a && b ? fmaxf(ar, br) : (a ? ar : (b ? br : 0.0f));
}

// Spans of a tile row: the hulls of its two quadrant bands' ellipse and disc
// spans (the row, widened by kCullPad, is the union of the two bands); tile
// tx is live when [16 tx - pad, 16 tx + 15 + pad] meets one of them.
__device__ __forceinline__ BandSpans row_spans(const BandSpans& top, const BandSpans& bottom) {
    BandSpans s;
    hull(top.el, top.er, bottom.el, bottom.er, s.el, s.er);
    hull(top.dl, top.dr, bottom.dl, bottom.dr, s.dl, s.dr);
    return s;
}

// Tile columns [lo, hi] whose widened range [16 tx - pad, 16 tx + 15 + pad]
// meets [l, r]: the first column with 16 lo + 15 + pad >= l and the last with
// 16 hi - pad <= r, found from the quotients and corrected by those exact
// comparisons.
__device__ __forceinline__ void span_columns(float l, float r, int& lo, int& hi) {
    const float lc = fminf(fmaxf(l, -4.0e6f), 4.0e6f), rc = fminf(fmaxf(r, -4.0e6f), 4.0e6f);
    lo = static_cast<int>(ceilf(mul(sub(lc, 15.0f + kCullPad), 0.0625f)));
    hi = static_cast<int>(floorf(mul(add(rc, kCullPad), 0.0625f)));
    if (!(static_cast<float>(lo * 16) + (15.0f + kCullPad) >= l)) ++lo;
    if (static_cast<float>((lo - 1) * 16) + (15.0f + kCullPad) >= l) --lo;
    if (!(static_cast<float>(hi * 16) - kCullPad <= r)) --hi;
    if (static_cast<float>((hi + 1) * 16) - kCullPad <= r) ++hi;
}

// The live tiles of one row of a clipped box [x0, x1): the columns whose
// widened range meets the ellipse span, [elo, ehi], and those meeting the disc
// span, [dlo, dhi] (either may be empty: lo > hi). The row's live tiles are
// their union, listed ellipse columns first, then the disc columns outside
// them (RowColumns::at).
struct RowColumns {
    int elo, ehi, dlo, dhi;
    __device__ __forceinline__ int ellipse_count() const { return max(ehi - elo + 1, 0); }
    __device__ __forceinline__ int disc_count() const { return max(dhi - dlo + 1, 0); }
    // disc columns before the ellipse range that are not in it
    __device__ __forceinline__ int disc_before() const {
        return ellipse_count() == 0 ? disc_count() : max(min(dhi, elo - 1) - dlo + 1, 0);
    }
    __device__ __forceinline__ int count() const {
        const int ne = ellipse_count(), nd = disc_count();
        const int both = max(min(ehi, dhi) - max(elo, dlo) + 1, 0);
        return ne + nd - (ne > 0 && nd > 0 ? both : 0);
    }
    // column of the i-th live tile, 0 <= i < count()
    __device__ __forceinline__ int at(int i) const {
        const int ne = ellipse_count();
        if (i < ne) return elo + i;
        const int j = i - ne, before = disc_before();
        if (j < before) return dlo + j;
        return max(dlo, ehi + 1) + (j - before);
    }
};

__device__ __forceinline__ RowColumns row_columns(const BandSpans& s, int x0, int x1) {
    RowColumns r{1, 0, 1, 0};
    if (s.el <= s.er) span_columns(s.el, s.er, r.elo, r.ehi);
    if (s.dl <= s.dr) span_columns(s.dl, s.dr, r.dlo, r.dhi);
    r.elo = max(r.elo, x0);
    r.ehi = min(r.ehi, x1 - 1);
    r.dlo = max(r.dlo, x0);
    r.dhi = min(r.dhi, x1 - 1);
    return r;
}

// 4-bit mask of the 8x8 quadrants of live tile tx that may hold a live pixel,
// from the spans of its row's two quadrant bands; bit (qy * 2 + qx).
// Never empty for a live tile: a rounding disagreement between the tile and
// quadrant tests falls back to all four quadrants.
__device__ __forceinline__ uint32_t quadrant_mask(const BandSpans& top, const BandSpans& bottom,
                                                  int tx) {
    uint32_t mask = 0;
#pragma unroll
    for (int qx = 0; qx < 2; ++qx) {
        const float x = static_cast<float>(tx * 16 + qx * 8);
        const float x0 = x - kCullPad, x1 = x + (7.0f + kCullPad);
        if (meets(top.el, top.er, x0, x1) || meets(top.dl, top.dr, x0, x1)) mask |= 1u << qx;
        if (meets(bottom.el, bottom.er, x0, x1) || meets(bottom.dl, bottom.dr, x0, x1))
            mask |= 1u << (2 + qx);
    }
    return mask != 0u ? mask : 0xfu;
}

// Tiles (16 px) that may hold a live pixel: the bounding box of the ellipse
// and the disc, widened by one pixel. Returns false when there are none.
__device__ __forceinline__ bool cull_tile_box(const CullShape& c, int& tx0, int& ty0, int& tx1,
                                              int& ty1) {
    if (c.mode == kCullAlways) return false;
    if (c.mode == kCullNever) {
        tx0 = ty0 = INT_MIN / 2;
        tx1 = ty1 = INT_MAX / 2;
        return true;
    }
    const float rd = sqrtf(c.r2) + 1.0f;
    const float ex = c.hx + 1.0f, ey = c.hy + 1.0f;
    const float bx0 = fminf(c.gx - rd, c.mx - ex), bx1 = fmaxf(c.gx + rd, c.mx + ex);
    const float by0 = fminf(c.gy - rd, c.my - ey), by1 = fmaxf(c.gy + rd, c.my + ey);
    tx0 = static_cast<int>(floorf(fmaxf(bx0, -1e6f) * (1.0f / 16.0f)));
    ty0 = static_cast<int>(floorf(fmaxf(by0, -1e6f) * (1.0f / 16.0f)));
    tx1 = static_cast<int>(floorf(fminf(bx1, 1e6f) * (1.0f / 16.0f)));
    ty1 = static_cast<int>(floorf(fminf(by1, 1e6f) * (1.0f / 16.0f)));
    return true;
}

}  // namespace st
}  // namespace hs
