// FlashGS per-Gaussian preprocess and per-pixel blend arithmetic.
//
// Every function here restates one reference function operation by operation
// so that results are bit-identical:
//   preprocess  vendor/flashgs/cuda_rasterizer/preprocess.cu:64-241,246-362,
//               364-597 (the kernel body, computeCov2D, computeColorFromSH,
//               block_intersect_ellipse, quat_to_rotmat, compute_transmat)
//   blend       vendor/flashgs/cuda_rasterizer/render.cu:77-136,143-183
// GLM products are expanded in the column/row order of the vendored GLM
// (glm/detail/type_mat3x3.inl:486-519, type_mat4x3.inl:506-563).
//
// Wherever the reference source leaves the choice of fused multiply-add to
// the compiler, the expression is a numbered rounding site (hs::Site, see
// splat_math.cuh) whose form is selected by a Rounding policy R. The FlashGS
// `PinnedRounding` holds the forms that reproduce the reference FlashGS build;
// they are guarded by the bit-exact parity tests against the reference library.
#pragma once

#include "splat_math.cuh"

namespace hs {
namespace fg {

// Forms reproducing the reference FlashGS build. Unlisted sites use the
// first variant of their helper.
__host__ __device__ constexpr int pinned_site(int site) {
    switch (site) {
        case S_QN_PAIR: return 1;   // x*x fused onto the rounded w*w
        case S_R00: return 2;       // 1 - 2(y*y + z*z) with both squares rounded
        case S_SH_P6B: return 1;    // (2zz - xx) - yy with yy rounded
        case S_SH_P8: return 2;     // xx - yy, both squares rounded
        case S_SH_P11B: return 1;   // (4zz - xx) - yy with yy rounded
        case S_SH_P12A: return 1;   // 2zz - 3xx with 3*xx fused
        case S_SH_P15: return 1;    // xx - 3yy with 3*yy fused
        case S_T: return 1;         // T - alpha*T, product rounded
        default: return 0;
    }
}

struct PinnedRounding {
    __device__ __forceinline__ int operator()(int site) const { return pinned_site(site); }
};

constexpr float kLog2e = 1.4426950216293334961f;
constexpr float kLn2 = 0.69314718055f;

// Per-Gaussian outputs of the preprocess.
struct Projected {
    bool in_front;      // survived the depth / opacity culls and the facing test
    bool touches;       // non-empty tile rectangle ("point_valid" before tile tests)
    float depth;        // p_view.z (sort key low word)
    float2 xy;          // pixel-space centre
    float3 conic;
    float power;
    float log2_opacity;
    float3 normal;
    float3 tu, tv, tw;
    int2 rect_min, rect_max;
};

// segment_intersect_ellipse (preprocess.cu:187-194).
template <class R>
__device__ __forceinline__ bool segment_hits(const R& r, float a, float b, float c, float d,
                                             float lo, float hi) {
    const float delta = diff2(r(S_EL_DELTA), b, b, mul(4.0f, a), c);
    const float a2 = mul(2.0f, a);
    const float t1 = mad(r(S_EL_T), sub(lo, d), a2, b);
    const float t2 = mad(r(S_EL_T), sub(hi, d), a2, b);
    return delta >= 0.0f && (t1 <= 0.0f || mul(t1, t1) <= delta) &&
           (t2 >= 0.0f || mul(t2, t2) <= delta);
}

// block_contains_center || block_intersect_ellipse for tile (tx, ty)
// (preprocess.cu:196-241, 485-488, 548-551).
template <class R>
__device__ __forceinline__ bool tile_hit(const R& r, int tx, int ty, float2 center, float3 conic,
                                         float power) {
    const int min_x = tx * 16, min_y = ty * 16;
    const int max_x = min_x + 15, max_y = min_y + 15;
    const float fminx = static_cast<float>(min_x), fminy = static_cast<float>(min_y);
    const float fmaxx = static_cast<float>(max_x), fmaxy = static_cast<float>(max_y);
    if (center.x >= fminx && center.x <= fmaxx && center.y >= fminy && center.y <= fmaxy) {
        return true;
    }
    const float w = mul(2.0f, power);
    const float dx = mul(center.x, 2.0f) < static_cast<float>(min_x + max_x)
                         ? sub(center.x, fminx)
                         : sub(center.x, fmaxx);
    {
        const float a = conic.z;
        const float b = mul(mul(-2.0f, conic.y), dx);
        const float c = msub(r(S_EL_C), mul(conic.x, dx), dx, w);
        if (segment_hits(r, a, b, c, center.y, fminy, fmaxy)) return true;
    }
    const float dy = mul(center.y, 2.0f) < static_cast<float>(min_y + max_y)
                         ? sub(center.y, fminy)
                         : sub(center.y, fmaxy);
    const float a = conic.x;
    const float b = mul(mul(-2.0f, conic.y), dy);
    const float c = msub(r(S_EL_C), mul(conic.z, dy), dy, w);
    return segment_hits(r, a, b, c, center.x, fminx, fmaxx);
}

// ndc2Pix with the reference's double-precision literals (preprocess.cu:64-67).
__device__ __forceinline__ float ndc_to_pixel(float v, int size) {
    const double t =
        __fma_rn(__dadd_rn(static_cast<double>(v), 1.0), static_cast<double>(size), -1.0);
    return __double2float_rn(__dmul_rn(t, 0.5));
}

__device__ __forceinline__ int trunc_to_int(float v) { return __float2int_rz(v); }

// "a - b*b"-style step where b*b is a shared rounded product bb: variant 0
// fuses the product (fma(-b, b, a)), variant 1 subtracts the rounded bb.
__device__ __forceinline__ float sub_square(int v, float a, float b, float bb) {
    return v == 0 ? fma(-b, b, a) : sub(a, bb);
}

// computeColorFromSH (preprocess.cu:145-185), degree 3, with clamp at 0.
template <class R>
__device__ __forceinline__ float3 sh_color(const R& r, float3 p, float3 campos,
                                           const float* __restrict__ sh /* 48 floats */) {
    float dx = sub(p.x, campos.x), dy = sub(p.y, campos.y), dz = sub(p.z, campos.z);
    const float l2 = dot3(r(S_SH_L2_PAIR), r(S_SH_L2_TAIL), dx, dx, dy, dy, dz, dz);
    const float rs = approx_rsqrt(l2);
    const float x = mul(dx, rs), y = mul(dy, rs), z = mul(dz, rs);
    const float xx = mul(x, x), yy = mul(y, y), zz = mul(z, z);
    const float xy = mul(x, y), yz = mul(y, z), xz = mul(x, z);
    const float zz2 = mul(2.0f, zz), zz4 = mul(4.0f, zz), xx3 = mul(3.0f, xx), yy3 = mul(3.0f, yy);

    const float p6a = r(S_SH_P6A) == 0 ? sub(zz2, xx) : fma(-x, x, zz2);
    const float p6 = sub_square(r(S_SH_P6B), p6a, y, yy);
    const float p8 = diff2(r(S_SH_P8), x, x, y, y);
    const float p9 = diff2(r(S_SH_P9), 3.0f, xx, y, y);
    const float p11a = r(S_SH_P11A) == 0 ? sub(zz4, xx) : fma(-x, x, zz4);
    const float p11 = sub_square(r(S_SH_P11B), p11a, y, yy);
    const float p12a = diff2(r(S_SH_P12A), 2.0f, zz, 3.0f, xx);
    const float p12 = r(S_SH_P12B) == 0 ? fma(-3.0f, yy, p12a) : sub(p12a, yy3);
    const float p15 = diff2(r(S_SH_P15), x, x, 3.0f, yy);
    (void)xx3;

    const float c1 = 0.4886025119029199f;
    const float s1 = mul(c1, y), s2 = mul(c1, z), s3 = mul(c1, x);
    const float s4 = mul(1.0925484305920792f, xy);
    const float s5 = mul(-1.0925484305920792f, yz);
    const float s6 = mul(0.31539156525252005f, p6);
    const float s7 = mul(-1.0925484305920792f, xz);
    const float s8 = mul(0.5462742152960396f, p8);
    const float s9 = mul(mul(-0.5900435899266435f, y), p9);
    const float s10 = mul(mul(2.890611442640554f, xy), z);
    const float s11 = mul(mul(-0.4570457994644658f, y), p11);
    const float s12 = mul(mul(0.3731763325901154f, z), p12);
    const float s13 = mul(mul(-0.4570457994644658f, x), p11);
    const float s14 = mul(mul(1.445305721320277f, z), p8);
    const float s15 = mul(mul(-0.5900435899266435f, x), p15);

    const int acc = r(S_SH_ACC);
    float out[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        float v = mad(r(S_SH_DC), 0.28209479177387814f, sh[c], 0.5f);
        v = nmad(acc, v, s1, sh[3 + c]);
        v = mad(acc, s2, sh[6 + c], v);
        v = nmad(acc, v, s3, sh[9 + c]);
        v = mad(acc, s4, sh[12 + c], v);
        v = mad(acc, s5, sh[15 + c], v);
        v = mad(acc, s6, sh[18 + c], v);
        v = mad(acc, s7, sh[21 + c], v);
        v = mad(acc, s8, sh[24 + c], v);
        v = mad(acc, s9, sh[27 + c], v);
        v = mad(acc, s10, sh[30 + c], v);
        v = mad(acc, s11, sh[33 + c], v);
        v = mad(acc, s12, sh[36 + c], v);
        v = mad(acc, s13, sh[39 + c], v);
        v = mad(acc, s14, sh[42 + c], v);
        v = mad(acc, s15, sh[45 + c], v);
        out[c] = ptx_max(v, 0.0f);
    }
    return make_float3(out[0], out[1], out[2]);
}

// Per-Gaussian projection (preprocess.cu:435-480 with computeCov2D and
// compute_transmat). `view`/`proj` are column-major 4x4 (GLM storage).
template <class R>
__device__ __forceinline__ Projected project_gaussian(
    const R& r, const float* view, const float* proj, float3 p, float opacity,
    const float cov3[6], float2 scale, float scale_modifier, float4 rot, int width, int height,
    float focal_x, float focal_y, float tan_fovx, float tan_fovy, int grid_x, int grid_y) {
    Projected g;
    g.in_front = false;
    g.touches = false;
    const float pvx = affine_row(r, S_PVIEW_PAIR, S_PVIEW_TAIL, view, 0, p.x, p.y, p.z);
    const float pvy = affine_row(r, S_PVIEW_PAIR, S_PVIEW_TAIL, view, 1, p.x, p.y, p.z);
    const float pvz = affine_row(r, S_PVIEW_PAIR, S_PVIEW_TAIL, view, 2, p.x, p.y, p.z);
    g.depth = pvz;
    if (pvz <= 0.2f) return g;
    if (mul(255.0f, opacity) < 1.0f) return g;

    const float phx = affine_row(r, S_PHOM_PAIR, S_PHOM_TAIL, proj, 0, p.x, p.y, p.z);
    const float phy = affine_row(r, S_PHOM_PAIR, S_PHOM_TAIL, proj, 1, p.x, p.y, p.z);
    const float phw = affine_row(r, S_PHOM_PAIR, S_PHOM_TAIL, proj, 3, p.x, p.y, p.z);
    const float pw = div(1.0f, add(phw, 0.0000001f));
    const float ppx = mul(phx, pw);
    const float ppy = mul(phy, pw);

    // computeCov2D (preprocess.cu:103-143)
    const float limx = mul(1.3f, tan_fovx);
    const float limy = mul(1.3f, tan_fovy);
    const float txtz = div(pvx, pvz);
    const float tytz = div(pvy, pvz);
    const float tx = mul(fminf(limx, fmaxf(-limx, txtz)), pvz);
    const float ty = mul(fminf(limy, fmaxf(-limy, tytz)), pvz);
    const float tz2 = mul(pvz, pvz);
    const float j00 = div(focal_x, pvz);
    const float j02 = div(-mul(focal_x, tx), tz2);
    const float j11 = div(focal_y, pvz);
    const float j12 = div(-mul(focal_y, ty), tz2);
    // W[c][i] = view[4*i + c]; T = W * J has a zero third column.
    float t0[3], t1[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const float w0 = view[4 * i + 0], w1 = view[4 * i + 1], w2 = view[4 * i + 2];
        t0[i] = mad(r(S_WJ_TAIL), w2, j02, mul(w0, j00));
        t1[i] = mad(r(S_WJ_TAIL), w2, j12, mul(w1, j11));
    }
    // M1 = T^T * Vrk: M1[c][i] = T[i][0]*V[c][0] + T[i][1]*V[c][1] + T[i][2]*V[c][2]
    const float v[3][3] = {{cov3[0], cov3[1], cov3[2]},
                           {cov3[1], cov3[3], cov3[4]},
                           {cov3[2], cov3[4], cov3[5]}};
    float m1[3][2];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        m1[c][0] = dot3(r(S_M1_PAIR), r(S_M1_TAIL), t0[0], v[c][0], t0[1], v[c][1], t0[2], v[c][2]);
        m1[c][1] = dot3(r(S_M1_PAIR), r(S_M1_TAIL), t1[0], v[c][0], t1[1], v[c][1], t1[2], v[c][2]);
    }
    // cov[c][i] = M1[0][i]*T[c][0] + M1[1][i]*T[c][1] + M1[2][i]*T[c][2]
    const float c00 = dot3(r(S_COV_PAIR), r(S_COV_TAIL), m1[0][0], t0[0], m1[1][0], t0[1],
                           m1[2][0], t0[2]);
    const float c01 = dot3(r(S_COV_PAIR), r(S_COV_TAIL), m1[0][1], t0[0], m1[1][1], t0[1],
                           m1[2][1], t0[2]);
    const float c11 = dot3(r(S_COV_PAIR), r(S_COV_TAIL), m1[0][1], t1[0], m1[1][1], t1[1],
                           m1[2][1], t1[2]);
    const float cx = add(c00, 0.3f);
    const float cy = c01;
    const float cz = add(c11, 0.3f);

    const float det = diff2(r(S_DET), cx, cz, cy, cy);
    const float det_inv = div(1.0f, det);
    g.conic = make_float3(mul(cz, det_inv), mul(-cy, det_inv), mul(cx, det_inv));

    g.log2_opacity = approx_lg2(opacity);
    g.power = mad(r(S_POWER), kLn2, g.log2_opacity, kLn2 * 8.0f);
    const int ext_w =
        trunc_to_int(mad(r(S_EXTENT), 1.414214f, approx_sqrt(mul(cx, g.power)), 1.0f));
    const int ext_h =
        trunc_to_int(mad(r(S_EXTENT), 1.414214f, approx_sqrt(mul(cz, g.power)), 1.0f));

    g.xy = make_float2(ndc_to_pixel(ppx, width), ndc_to_pixel(ppy, height));
    // getRect (preprocess.cu:90-100)
    const float ew = static_cast<float>(ext_w), eh = static_cast<float>(ext_h);
    g.rect_min.x = min(grid_x, max(0, trunc_to_int(div(sub(g.xy.x, ew), 16.0f))));
    g.rect_min.y = min(grid_y, max(0, trunc_to_int(div(sub(g.xy.y, eh), 16.0f))));
    g.rect_max.x = min(grid_x, max(0, trunc_to_int(div(add(g.xy.x, ew), 16.0f)) + 1));
    g.rect_max.y = min(grid_y, max(0, trunc_to_int(div(add(g.xy.y, eh), 16.0f)) + 1));
    g.touches = (g.rect_max.x - g.rect_min.x) * (g.rect_max.y - g.rect_min.y) > 0;

    // compute_transmat (preprocess.cu:322-362) and the camera-space normal.
    float3 n;
    splat_transform(r, view, proj, p, scale, scale_modifier, rot, width, height, g.tu, g.tv, g.tw, n);
    const float cosv = -dot3(r(S_COS_PAIR), r(S_COS_TAIL), pvx, n.x, pvy, n.y, pvz, n.z);
    if (cosv == 0.0f) {
        // The reference returns from the kernel here (preprocess.cu:476);
        // the Gaussian then produces no record and no pairs.
        g.touches = false;
        return g;
    }
    const float sign = cosv > 0.0f ? 1.0f : -1.0f;
    g.normal = make_float3(mul(sign, n.x), mul(sign, n.y), mul(sign, n.z));
    g.in_front = true;
    return g;
}

// Per-pixel blend state (render.cu:411-456).
struct PixelState {
    float cr, cg, cb;  // colour
    float o0, o1;      // other features (specular, roughness)
    float t;           // transmittance
    float d;           // depth
    float m1, m2;      // distortion moments
    float dist;        // distortion
    float median;      // median depth
    float nx, ny, nz;  // normal
};

__device__ __forceinline__ void pixel_init(PixelState& s) {
    s.cr = s.cg = s.cb = 0.0f;
    s.o0 = s.o1 = 0.0f;
    s.t = 1.0f;
    s.d = 0.0f;
    s.m1 = s.m2 = 0.0f;
    s.dist = 0.0f;
    s.median = 0.0f;
    s.nx = s.ny = s.nz = 0.0f;
}

// Per-Gaussian blend record read by the rasteriser (80 bytes).
struct BlendRecord {
    float x, y;           // pixel-space centre
    float nx, ny, nz, op; // normal and opacity
    float r, g, b;        // colour
    float spec, rough;    // other features
    float tux, tuy, tuz;
    float tvx, tvy, tvz;
    float twx, twy, twz;
};

// The terms of an evaluation that depend only on the pixel column (k =
// x Tw - Tu and x's offset from the centre), formed once for a lane's two
// pixels, which share their column.
struct ColumnTerms {
    float kx, ky, kz, dx;
};

template <class R>
__device__ __forceinline__ ColumnTerms column_terms(const R& r, float px, const BlendRecord& g) {
    const int vk = r(S_K);
    return ColumnTerms{msub(vk, px, g.twx, g.tux), msub(vk, px, g.twy, g.tuy),
                       msub(vk, px, g.twz, g.tuz), sub(g.x, px)};
}

// pixel_shader (render.cu:77-136).
template <class R>
__device__ __forceinline__ void blend(const R& r, PixelState& s, const ColumnTerms& col, float py,
                                      const BlendRecord& g) {
    const int vk = r(S_K);
    const float kx = col.kx, ky = col.ky, kz = col.kz;
    const float lx = msub(vk, py, g.twx, g.tvx);
    const float ly = msub(vk, py, g.twy, g.tvy);
    const float lz = msub(vk, py, g.twz, g.tvz);
    const int vc = r(S_CROSS);
    const float pxv = diff2(vc, ky, lz, kz, ly);
    const float pyv = diff2(vc, kz, lx, kx, lz);
    const float pzv = diff2(vc, kx, ly, ky, lx);
    const float sx = div(pxv, pzv);
    const float sy = div(pyv, pzv);
    const float rho3d = dot2(r(S_RHO3), sx, sx, sy, sy);
    const float dx = col.dx;
    const float dy = sub(g.y, py);
    const float rho2d = mul(2.0f, dot2(r(S_RHO2), dx, dx, dy, dy));
    const float rho = fminf(rho3d, rho2d);
    const float depth = rho3d <= rho2d ? add(dot2(r(S_DEPTH), sx, g.twx, sy, g.twy), g.twz) : g.twz;
    const float power = mul(-0.5f, rho);
    const float alpha = fminf(0.99f, mul(g.op, expf(power)));
    const float w = mul(alpha, s.t);
    const int va = r(S_ACC);
    s.cr = mad(va, g.r, w, s.cr);
    s.cg = mad(va, g.g, w, s.cg);
    s.cb = mad(va, g.b, w, s.cb);
    s.t = r(S_T) == 0 ? fma(-alpha, s.t, s.t) : sub(s.t, w);
    s.o0 = mad(va, g.spec, w, s.o0);
    s.o1 = mad(va, g.rough, w, s.o1);
    const float a = sub(1.0f, s.t);
    const float m = mul(kFar / (kFar - kNear), sub(1.0f, div(kNear, depth)));
    const float mm = mul(m, m);
    const float dd = nmad(r(S_D2), mad(r(S_D1), mm, a, s.m2), mul(2.0f, m), s.m1);
    s.dist = mad(va, dd, w, s.dist);
    s.m1 = mad(va, m, w, s.m1);
    s.m2 = mad(va, mm, w, s.m2);
    if (s.t > 0.5f) s.median = depth;
    s.d = mad(va, depth, w, s.d);
    s.nx = mad(va, g.nx, w, s.nx);
    s.ny = mad(va, g.ny, w, s.ny);
    s.nz = mad(va, g.nz, w, s.nz);
}

// The states of a lane's two pixels (rows py0 and py1 of one column), member
// by member as pairs (.x: py0, .y: py1), so that blend_pair can update both
// with packed FP32x2 instructions.
struct PixelPair {
    float2 cr, cg, cb, o0, o1, t, d, m1, m2, dist, median, nx, ny, nz;
};

__device__ __forceinline__ void pair_init(PixelPair& s) {
    s.cr = s.cg = s.cb = s.o0 = s.o1 = pair(0.0f);
    s.t = pair(1.0f);
    s.d = s.m1 = s.m2 = s.dist = s.median = pair(0.0f);
    s.nx = s.ny = s.nz = pair(0.0f);
}

// The state of pixel `which` (0: .x, 1: .y) of a pair.
__device__ __forceinline__ PixelState pixel_of(const PixelPair& p, int which) {
    auto c = [which](float2 v) { return which == 0 ? v.x : v.y; };
    PixelState s;
    s.cr = c(p.cr);
    s.cg = c(p.cg);
    s.cb = c(p.cb);
    s.o0 = c(p.o0);
    s.o1 = c(p.o1);
    s.t = c(p.t);
    s.d = c(p.d);
    s.m1 = c(p.m1);
    s.m2 = c(p.m2);
    s.dist = c(p.dist);
    s.median = c(p.median);
    s.nx = c(p.nx);
    s.ny = c(p.ny);
    s.nz = c(p.nz);
    return s;
}

// blend() of one Gaussian at both pixels of a pair: every operation of
// blend() issued once as a packed pair (fp.cuh: each component rounds as the
// scalar instruction), except the divisions, expf, the minima and the median
// selection, which stay per pixel. Each component equals blend() of that
// pixel.
template <class R>
__device__ __forceinline__ void blend_pair(const R& r, PixelPair& s, const ColumnTerms& col, float2 py,
                                           const BlendRecord& g) {
    const int vk = r(S_K);
    const float2 kx = pair(col.kx), ky = pair(col.ky), kz = pair(col.kz);
    const float2 lx = msub_x2(vk, py, pair(g.twx), pair(g.tvx));
    const float2 ly = msub_x2(vk, py, pair(g.twy), pair(g.tvy));
    const float2 lz = msub_x2(vk, py, pair(g.twz), pair(g.tvz));
    const int vc = r(S_CROSS);
    const float2 pxv = diff2_x2(vc, ky, lz, kz, ly);
    const float2 pyv = diff2_x2(vc, kz, lx, kx, lz);
    const float2 pzv = diff2_x2(vc, kx, ly, ky, lx);
    const float2 sx = make_float2(div(pxv.x, pzv.x), div(pxv.y, pzv.y));
    const float2 sy = make_float2(div(pyv.x, pzv.x), div(pyv.y, pzv.y));
    const float2 rho3d = dot2_x2(r(S_RHO3), sx, sx, sy, sy);
    const float2 dx = pair(col.dx);
    const float2 dy = sub2(pair(g.y), py);
    const float2 rho2d = mul2(pair(2.0f), dot2_x2(r(S_RHO2), dx, dx, dy, dy));
    const float2 rho = make_float2(fminf(rho3d.x, rho2d.x), fminf(rho3d.y, rho2d.y));
    const float2 on_plane = add2(dot2_x2(r(S_DEPTH), sx, pair(g.twx), sy, pair(g.twy)), pair(g.twz));
    const float2 depth = make_float2(rho3d.x <= rho2d.x ? on_plane.x : g.twz, rho3d.y <= rho2d.y ? on_plane.y : g.twz);
    const float2 power = mul2(pair(-0.5f), rho);
    const float2 scaled = mul2(pair(g.op), make_float2(expf(power.x), expf(power.y)));
    const float2 alpha = make_float2(fminf(0.99f, scaled.x), fminf(0.99f, scaled.y));
    const float2 w = mul2(alpha, s.t);
    const int va = r(S_ACC);
    s.cr = mad_x2(va, pair(g.r), w, s.cr);
    s.cg = mad_x2(va, pair(g.g), w, s.cg);
    s.cb = mad_x2(va, pair(g.b), w, s.cb);
    s.t = r(S_T) == 0 ? fma2(neg2(alpha), s.t, s.t) : sub2(s.t, w);
    s.o0 = mad_x2(va, pair(g.spec), w, s.o0);
    s.o1 = mad_x2(va, pair(g.rough), w, s.o1);
    const float2 a = sub2(pair(1.0f), s.t);
    const float2 m = mul2(pair(kFar / (kFar - kNear)),
                          sub2(pair(1.0f), make_float2(div(kNear, depth.x), div(kNear, depth.y))));
    const float2 mm = mul2(m, m);
    const float2 dd = nmad_x2(r(S_D2), mad_x2(r(S_D1), mm, a, s.m2), mul2(pair(2.0f), m), s.m1);
    s.dist = mad_x2(va, dd, w, s.dist);
    s.m1 = mad_x2(va, m, w, s.m1);
    s.m2 = mad_x2(va, mm, w, s.m2);
    if (s.t.x > 0.5f) s.median.x = depth.x;
    if (s.t.y > 0.5f) s.median.y = depth.y;
    s.d = mad_x2(va, depth, w, s.d);
    s.nx = mad_x2(va, pair(g.nx), w, s.nx);
    s.ny = mad_x2(va, pair(g.ny), w, s.ny);
    s.nz = mad_x2(va, pair(g.nz), w, s.nz);
}

// write_output (render.cu:143-183) for one pixel: returns the 12 output
// values in the channel order color3, other2, depth, alpha, normal3,
// median, distortion.
template <class R>
__device__ __forceinline__ void finish_pixel(const R& r, const PixelState& s, float3 bg,
                                             float out[12]) {
    const float t = s.t < 0.0001f ? 0.0f : s.t;
    const int vo = r(S_OUT);
    out[0] = mad(vo, t, bg.x, s.cr);
    out[1] = mad(vo, t, bg.y, s.cg);
    out[2] = mad(vo, t, bg.z, s.cb);
    out[3] = mad(vo, t, bg.x, s.o0);
    out[4] = mad(vo, t, bg.y, s.o1);
    out[5] = s.d;
    out[6] = sub(1.0f, t);
    out[7] = s.nx;
    out[8] = s.ny;
    out[9] = s.nz;
    out[10] = s.median;
    out[11] = s.dist;
}

// encode() of render.cu:138-141 and flashgs_backend.cu:307-310.
__device__ __forceinline__ float encode_background(float v) {
    const float c = fminf(fmaxf(0.0f, mul(v, 255.0f)), 255.0f);
    return static_cast<float>(static_cast<unsigned char>(__float2uint_rz(c)));
}

}  // namespace fg
}  // namespace hs
