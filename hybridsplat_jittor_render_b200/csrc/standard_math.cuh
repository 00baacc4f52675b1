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
// widened to 1.02 c + 0.05, and quadrant rectangles are widened by one pixel,
// so rounding in the per-pixel arithmetic cannot make a culled evaluation
// live. Culling therefore never changes an output value; it only skips
// evaluations that would have returned early.
enum CullMode : int { kCullEllipse = 0, kCullNever = 1, kCullAlways = 2 };

// The ellipse is stored in its axis frame: with X, Y relative to the centre,
// (u, v) = (cs X + sn Y, cs Y - sn X) and u^2 ia + v^2 ib <= 1. Evaluating
// squares in the axis frame keeps thin (edge-on) ellipses well conditioned in
// single precision: rounding moves the boundary by about 1e-7 of the
// distance to the centre, far below the one-pixel widening of the tested
// rectangles. ryx and rxy locate the minimum of the form along a vertical or
// horizontal edge (Y = ryx X, X = rxy Y).
struct CullShape {
    float mx, my;     // ellipse centre (pixels)
    float cs, sn;     // major-axis direction
    float ia, ib;     // inverse squared semi-axes
    float ryx, rxy;   // edge minimisers
    float gx, gy, r2; // disc centre and squared radius
    int mode;         // kCullEllipse: test; kCullNever: every pixel may be live; kCullAlways: none
    float hx, hy;     // half extents of the ellipse's bounding box
};

__device__ __forceinline__ CullShape cull_shape(float op, float x, float y, float3 tu, float3 tv,
                                                float3 tw) {
    CullShape c;
    c.mx = c.my = c.sn = c.ia = c.ib = c.ryx = c.rxy = c.hx = c.hy = 0.0f;
    c.cs = 1.0f;
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
    const double sxx = mx * mx - quu, syy = my * my - qvv, sxy = mx * my - quv;
    const double det = sxx * syy - sxy * sxy;
    if (!(sxx > 0.0 && syy > 0.0 && det > 0.0) || !(fabs(mx) < 1e7 && fabs(my) < 1e7)) return c;
    // Eigen-decomposition of [[sxx, sxy], [sxy, syy]] without trigonometry:
    // r = la - lb, (cos 2t, sin 2t) = (sxx - syy, 2 sxy) / r, and the
    // half-angle formulas taken on the side that avoids cancellation.
    const double dxy = sxx - syy;
    const double r = sqrt(dxy * dxy + 4.0 * sxy * sxy);
    const double la = 0.5 * (sxx + syy + r);
    const double lb = det / la;
    double cs = 1.0, sn = 0.0;
    if (r > 0.0) {
        if (dxy >= 0.0) {
            cs = sqrt(0.5 * (1.0 + dxy / r));
            sn = sxy / (r * cs);
        } else {
            sn = sqrt(0.5 * (1.0 - dxy / r));
            if (sxy < 0.0) sn = -sn;
            cs = sxy / (r * sn);
        }
    }
    // widen the axes slightly to absorb the rounding of the stored direction
    const double ia = 1.0 / (la * 1.0002), ib = 1.0 / (lb * 1.0002 + 1e-8 * la);
    const double axx = cs * cs * ia + sn * sn * ib, ayy = sn * sn * ia + cs * cs * ib;
    const double axy = cs * sn * (ia - ib);
    c.mx = static_cast<float>(mx);
    c.my = static_cast<float>(my);
    c.cs = static_cast<float>(cs);
    c.sn = static_cast<float>(sn);
    c.ia = static_cast<float>(ia);
    c.ib = static_cast<float>(ib);
    c.ryx = static_cast<float>(-axy / ayy);
    c.rxy = static_cast<float>(-axy / axx);
    c.hx = static_cast<float>(sqrt(sxx) * 1.0003);
    c.hy = static_cast<float>(sqrt(syy) * 1.0003);
    c.mode = kCullEllipse;
    return c;
}

__device__ __forceinline__ float cull_form(const CullShape& c, float X, float Y) {
    const float u = c.cs * X + c.sn * Y, v = c.cs * Y - c.sn * X;
    return u * u * c.ia + v * v * c.ib;
}

// Can any pixel of [x0, x1] x [y0, y1] (already widened) be live? Written
// without early exits so that the lanes of a warp, each testing a different
// Gaussian, stay converged.
__device__ __forceinline__ bool cull_rect_live(const CullShape& c, float x0, float y0, float x1,
                                               float y1) {
    const float cx = fminf(fmaxf(c.gx, x0), x1), cy = fminf(fmaxf(c.gy, y0), y1);
    const float ddx = cx - c.gx, ddy = cy - c.gy;
    const bool disc = ddx * ddx + ddy * ddy <= c.r2;
    const float X0 = x0 - c.mx, X1 = x1 - c.mx, Y0 = y0 - c.my, Y1 = y1 - c.my;
    const bool centre = X0 <= 0.0f && X1 >= 0.0f && Y0 <= 0.0f && Y1 >= 0.0f;
    // Minimum of the form along each edge of the rectangle.
    const float fa = cull_form(c, X0, fminf(fmaxf(c.ryx * X0, Y0), Y1));
    const float fb = cull_form(c, X1, fminf(fmaxf(c.ryx * X1, Y0), Y1));
    const float fc = cull_form(c, fminf(fmaxf(c.rxy * Y0, X0), X1), Y0);
    const float fd = cull_form(c, fminf(fmaxf(c.rxy * Y1, X0), X1), Y1);
    const bool edge = fminf(fminf(fa, fb), fminf(fc, fd)) <= 1.0f;
    const bool tested = disc || centre || edge;
    return c.mode == kCullNever || (c.mode == kCullEllipse && tested);
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

// 4-bit mask of the 8x8 quadrants of tile (tx, ty) that may hold a live
// pixel; bit (qy * 2 + qx).
__device__ __forceinline__ uint32_t cull_quadrants(const CullShape& c, int tx, int ty) {
    uint32_t mask = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float x0 = static_cast<float>(tx * 16 + (q & 1) * 8) - 1.0f;
        const float y0 = static_cast<float>(ty * 16 + (q >> 1) * 8) - 1.0f;
        if (cull_rect_live(c, x0, y0, x0 + 9.0f, y0 + 9.0f)) mask |= 1u << q;
    }
    return mask;
}

}  // namespace st
}  // namespace hs
