/*
 * CPU restatement of the HybridSplat forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle that tests, the smoke
 * check and the CPU-baseline leg of bench.py compare the CUDA library with;
 * the product never links or calls it.
 *
 * It restates, in plain C, the reference algorithms:
 *   FlashGS preprocess    vendor/flashgs/cuda_rasterizer/preprocess.cu:64-597
 *   FlashGS camera        vendor/flashgs/cuda_rasterizer/preprocess.cu:599-651
 *   pair order            vendor/flashgs/cuda_rasterizer/sort.cu:160-189
 *   tile ranges           vendor/flashgs/cuda_rasterizer/render.cu:46-68
 *   FlashGS blend         vendor/flashgs/cuda_rasterizer/render.cu:77-183,358-732
 *   standard preprocess   vendor/standard_rasterizer/forward.cu:75-251,
 *                         auxiliary.h:80-228
 *   standard blend        vendor/standard_rasterizer/forward.cu:256-445
 *   orchestration         rasterizer/flashgs_backend.cu:339-607,
 *                         rasterizer/full_rasterizer.cu:203-394
 * Rounding: products and sums are evaluated in the reference's source order;
 * where the reference compiler fuses a multiply-add the restatement uses
 * fmaf() (same forms as the CUDA library). The GPU-only approximate
 * instructions have no CPU equivalent and are replaced by correctly rounded
 * functions (sqrt.approx -> sqrtf, rsqrt.approx/rsqrtf -> 1/sqrtf,
 * lg2.approx -> log2f) and CUDA expf by the C library expf, so agreement with
 * the reference is to a tolerance, not bit-exact; the exact bits are pinned
 * against the reference library itself on the GPU.
 *
 * Build: gcc -O2 -ffp-contract=off -fopenmp -shared -fPIC (oracle/build_oracle.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

#define API __attribute__((visibility("default")))

static float mad_f(float a, float b, float c) { return fmaf(a, b, c); }
/* a*b + c*d with the first product fused */
static float dot2_f(float a, float b, float c, float d) { return fmaf(a, b, c * d); }
/* a*b - c*d */
static float diff2_f(float a, float b, float c, float d) { return fmaf(a, b, -(c * d)); }
static float dot3_f(float a, float b, float c, float d, float e, float f) {
    return fmaf(e, f, dot2_f(a, b, c, d));
}
static float affine_row(const float* m, int i, float x, float y, float z) {
    return dot3_f(m[i], x, m[4 + i], y, m[8 + i], z) + m[12 + i];
}
static int trunc_i(float v) {
    if (!(v == v)) return 0;
    if (v >= 2147483648.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int)v;
}
static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* ---------------------------------------------------------------- camera */

/* getViewMatrix / getProjectionMatrix (preprocess.cu:599-627), column-major. */
API void oracle_flashgs_camera(const float position[3], const float rot9[9], int width,
                               int height, float fx, float fy, float zfar, float znear,
                               float view[16], float proj[16]) {
    memset(view, 0, 16 * sizeof(float));
    for (int c = 0; c < 3; ++c)
        for (int i = 0; i < 3; ++i) view[4 * c + i] = rot9[3 * c + i];
    for (int i = 0; i < 3; ++i) {
        float t = rot9[i] * -position[0];
        t = t + rot9[3 + i] * -position[1];
        t = t + rot9[6 + i] * -position[2];
        view[12 + i] = t;
    }
    view[15] = 1.0f;
    const float top = (float)height / (2.0f * fy) * znear, bottom = -top;
    const float right = (float)width / (2.0f * fx) * znear, left = -right;
    float p[16];
    memset(p, 0, sizeof(p));
    p[0] = 2.0f * znear / (right - left);
    p[5] = 2.0f * znear / (top - bottom);
    p[2] = (right + left) / (right - left);
    p[6] = (top + bottom) / (top - bottom);
    p[14] = 1.0f;
    p[10] = 1.0f * zfar / (zfar - znear);
    p[11] = -(zfar * znear) / (zfar - znear);
    float a[16];
    for (int c = 0; c < 4; ++c)
        for (int r = 0; r < 4; ++r) a[4 * c + r] = p[4 * r + c];
    for (int j = 0; j < 4; ++j)
        for (int r = 0; r < 4; ++r) {
            float t = a[r] * view[4 * j];
            t = t + a[4 + r] * view[4 * j + 1];
            t = t + a[8 + r] * view[4 * j + 2];
            t = t + a[12 + r] * view[4 * j + 3];
            proj[4 * j + r] = t;
        }
}

/* quat_to_rotmat + compute_transmat + normal (preprocess.cu:246-362). */
static void splat_transform(const float* view, const float* proj, const float p[3], float sx,
                            float sy, float mod, const float q[4], int W, int H, float tu[3],
                            float tv[3], float tw[3], float n[3]) {
    const float qn = fmaf(q[2], q[2], fmaf(q[1], q[1], dot2_f(q[3], q[3], q[0], q[0])));
    const float s = 1.0f / sqrtf(qn);
    const float qw = q[0] * s, qx = q[1] * s, qy = q[2] * s, qz = q[3] * s;
    float rm[3][3];
    rm[0][0] = 1.0f - 2.0f * dot2_f(qy, qy, qz, qz);
    rm[0][1] = 2.0f * dot2_f(qx, qy, qw, qz);
    rm[0][2] = 2.0f * diff2_f(qx, qz, qw, qy);
    rm[1][0] = 2.0f * diff2_f(qx, qy, qw, qz);
    rm[1][1] = 1.0f - 2.0f * dot2_f(qx, qx, qz, qz);
    rm[1][2] = 2.0f * dot2_f(qy, qz, qw, qx);
    rm[2][0] = 2.0f * dot2_f(qx, qz, qw, qy);
    rm[2][1] = 2.0f * diff2_f(qy, qz, qw, qx);
    rm[2][2] = 1.0f - 2.0f * dot2_f(qx, qx, qy, qy);
    /* GLM forms the products with the structural zeros of S, splat2world and
     * ndc2pix too: signed zeros (NaN for an infinite factor) that decide the
     * sign of a zero result and leave every other value unchanged. */
    const float s0 = mod * sx, s1 = mod * sy;
    float l0[3], l1[3], l2[3];
    for (int i = 0; i < 3; ++i) {
        const float z0 = rm[0][i] * 0.0f, z1 = rm[1][i] * 0.0f, z2 = rm[2][i] * 0.0f;
        l0[i] = rm[0][i] * s0 + z1 + z2;
        l1[i] = z0 + rm[1][i] * s1 + z2;
        l2[i] = z0 + z1 + rm[2][i];
    }
    float b[4][3];
    for (int c = 0; c < 4; ++c) {
        const float zp = 0.0f * proj[12 + c];
        b[c][0] = dot3_f(l0[0], proj[c], l0[1], proj[4 + c], l0[2], proj[8 + c]) + zp;
        b[c][1] = dot3_f(l1[0], proj[c], l1[1], proj[4 + c], l1[2], proj[8 + c]) + zp;
        b[c][2] = dot3_f(p[0], proj[c], p[1], proj[4 + c], p[2], proj[8 + c]) + proj[12 + c];
    }
    const float w2 = (float)W * 0.5f, wm = (float)(W - 1) * 0.5f;
    const float h2 = (float)H * 0.5f, hm = (float)(H - 1) * 0.5f;
    for (int i = 0; i < 3; ++i) {
        const float z0 = b[0][i] * 0.0f, z1 = b[1][i] * 0.0f, z2 = b[2][i] * 0.0f;
        tu[i] = fmaf(b[3][i], wm, b[0][i] * w2) + (z1 + z2);
        tv[i] = fmaf(b[3][i], hm, b[1][i] * h2) + (z0 + z2);
        tw[i] = b[3][i] + ((z0 + z1) + z2);
    }
    n[0] = dot3_f(view[0], l2[0], view[4], l2[1], view[8], l2[2]);
    n[1] = dot3_f(view[1], l2[0], view[5], l2[1], view[9], l2[2]);
    n[2] = dot3_f(view[2], l2[0], view[6], l2[1], view[10], l2[2]);
}

/* ---------------------------------------------------------------- FlashGS */

static int segment_hits(float a, float b, float c, float d, float lo, float hi) {
    const float delta = diff2_f(b, b, 4.0f * a, c);
    const float t1 = fmaf(lo - d, 2.0f * a, b);
    const float t2 = fmaf(hi - d, 2.0f * a, b);
    return delta >= 0.0f && (t1 <= 0.0f || t1 * t1 <= delta) && (t2 >= 0.0f || t2 * t2 <= delta);
}

/* block_contains_center || block_intersect_ellipse (preprocess.cu:187-241). */
static int tile_hit(int tx, int ty, const float xy[2], const float conic[3], float power) {
    const int x0 = tx * 16, y0 = ty * 16, x1 = x0 + 15, y1 = y0 + 15;
    if (xy[0] >= (float)x0 && xy[0] <= (float)x1 && xy[1] >= (float)y0 && xy[1] <= (float)y1) return 1;
    const float w = 2.0f * power;
    const float dx = xy[0] * 2.0f < (float)(x0 + x1) ? xy[0] - (float)x0 : xy[0] - (float)x1;
    if (segment_hits(conic[2], (-2.0f * conic[1]) * dx, fmaf(conic[0] * dx, dx, -w), xy[1], (float)y0, (float)y1))
        return 1;
    const float dy = xy[1] * 2.0f < (float)(y0 + y1) ? xy[1] - (float)y0 : xy[1] - (float)y1;
    return segment_hits(conic[0], (-2.0f * conic[1]) * dy, fmaf(conic[2] * dy, dy, -w), xy[0], (float)x0, (float)x1);
}

static float ndc_to_pixel(float v, int s) {
    return (float)(fma((double)v + 1.0, (double)s, -1.0) * 0.5);
}

/* computeColorFromSH (preprocess.cu:145-185). */
static void sh_color(const float p[3], const float campos[3], const float* sh, float out[3]) {
    float dx = p[0] - campos[0], dy = p[1] - campos[1], dz = p[2] - campos[2];
    const float l2 = dot3_f(dx, dx, dy, dy, dz, dz);
    const float rs = 1.0f / sqrtf(l2);
    const float x = dx * rs, y = dy * rs, z = dz * rs;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
    const float p6 = fmaf(-y, y, 2.0f * zz - xx);
    const float p8 = fmaf(x, x, -yy);
    const float p9 = fmaf(3.0f, xx, -yy);
    const float p11 = fmaf(-y, y, 4.0f * zz - xx);
    const float p12 = fmaf(-3.0f, yy, fmaf(2.0f, zz, -(3.0f * xx)));
    const float p15 = fmaf(-3.0f, yy, xx);
    const float c1 = 0.4886025119029199f;
    const float s1 = c1 * y, s2 = c1 * z, s3 = c1 * x;
    const float s4 = 1.0925484305920792f * xy, s5 = -1.0925484305920792f * yz;
    const float s6 = 0.31539156525252005f * p6, s7 = -1.0925484305920792f * xz;
    const float s8 = 0.5462742152960396f * p8;
    const float s9 = (-0.5900435899266435f * y) * p9, s10 = (2.890611442640554f * xy) * z;
    const float s11 = (-0.4570457994644658f * y) * p11, s12 = (0.3731763325901154f * z) * p12;
    const float s13 = (-0.4570457994644658f * x) * p11, s14 = (1.445305721320277f * z) * p8;
    const float s15 = (-0.5900435899266435f * x) * p15;
    const float sc[16] = {0, -s1, s2, -s3, s4, s5, s6, s7, s8, s9, s10, s11, s12, s13, s14, s15};
    for (int c = 0; c < 3; ++c) {
        float v = fmaf(0.28209479177387814f, sh[c], 0.5f);
        for (int k = 1; k < 16; ++k) v = fmaf(sc[k], sh[3 * k + c], v);
        out[c] = v > 0.0f ? v : 0.0f;
    }
}

typedef struct {
    uint64_t key;
    uint32_t value;
} Pair;

static int pair_less(const void* a, const void* b) {
    const Pair* x = (const Pair*)a;
    const Pair* y = (const Pair*)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->value < y->value ? -1 : (x->value > y->value);
}

typedef struct {
    float xy[2], conic[3], power, log2op, normal[3], tu[3], tv[3], tw[3], depth, rgb[3];
    int rmin[2], rmax[2];
    int write;
    uint32_t hits;
} FgGauss;

/* Per-Gaussian part of preprocessCUDA (preprocess.cu:402-597). */
static void fg_preprocess_one(int idx, const float* view, const float* proj, const float* campos,
                              int W, int H, float fx, float fy, int gx, int gy,
                              const float* pos, const float* shs, const float* colors, int use_sh,
                              const float* opac, const float* cov6, const float* scales,
                              float mod, const float* rot, FgGauss* g) {
    memset(g, 0, sizeof(*g));
    const float* p = pos + 3 * (size_t)idx;
    const float pvx = affine_row(view, 0, p[0], p[1], p[2]);
    const float pvy = affine_row(view, 1, p[0], p[1], p[2]);
    const float pvz = affine_row(view, 2, p[0], p[1], p[2]);
    g->depth = pvz;
    if (pvz <= 0.2f) return;
    const float op = opac[idx];
    if (255.0f * op < 1.0f) return;
    const float phx = affine_row(proj, 0, p[0], p[1], p[2]);
    const float phy = affine_row(proj, 1, p[0], p[1], p[2]);
    const float phw = affine_row(proj, 3, p[0], p[1], p[2]);
    const float pw = 1.0f / (phw + 0.0000001f);
    const float ppx = phx * pw, ppy = phy * pw;
    const float tanx = (float)W / (2.0f * fx), tany = (float)H / (2.0f * fy);
    const float limx = 1.3f * tanx, limy = 1.3f * tany;
    const float txtz = pvx / pvz, tytz = pvy / pvz;
    const float tx = fminf(limx, fmaxf(-limx, txtz)) * pvz;
    const float ty = fminf(limy, fmaxf(-limy, tytz)) * pvz;
    const float j00 = fx / pvz, j02 = -(fx * tx) / (pvz * pvz);
    const float j11 = fy / pvz, j12 = -(fy * ty) / (pvz * pvz);
    float t0[3], t1[3];
    for (int i = 0; i < 3; ++i) {
        t0[i] = fmaf(view[4 * i + 2], j02, view[4 * i] * j00);
        t1[i] = fmaf(view[4 * i + 2], j12, view[4 * i + 1] * j11);
    }
    const float* c6 = cov6 + 6 * (size_t)idx;
    const float v[3][3] = {{c6[0], c6[1], c6[2]}, {c6[1], c6[3], c6[4]}, {c6[2], c6[4], c6[5]}};
    float m1[3][2];
    for (int c = 0; c < 3; ++c) {
        m1[c][0] = dot3_f(t0[0], v[c][0], t0[1], v[c][1], t0[2], v[c][2]);
        m1[c][1] = dot3_f(t1[0], v[c][0], t1[1], v[c][1], t1[2], v[c][2]);
    }
    const float cx = dot3_f(m1[0][0], t0[0], m1[1][0], t0[1], m1[2][0], t0[2]) + 0.3f;
    const float cy = dot3_f(m1[0][1], t0[0], m1[1][1], t0[1], m1[2][1], t0[2]);
    const float cz = dot3_f(m1[0][1], t1[0], m1[1][1], t1[1], m1[2][1], t1[2]) + 0.3f;
    const float det = diff2_f(cx, cz, cy, cy);
    const float det_inv = 1.0f / det;
    g->conic[0] = cz * det_inv;
    g->conic[1] = -cy * det_inv;
    g->conic[2] = cx * det_inv;
    g->log2op = log2f(op);
    const float ln2 = 0.69314718055f;
    g->power = fmaf(ln2, g->log2op, ln2 * 8.0f);
    const int ew = trunc_i(fmaf(1.414214f, sqrtf(cx * g->power), 1.0f));
    const int eh = trunc_i(fmaf(1.414214f, sqrtf(cz * g->power), 1.0f));
    g->xy[0] = ndc_to_pixel(ppx, W);
    g->xy[1] = ndc_to_pixel(ppy, H);
    g->rmin[0] = imin(gx, imax(0, trunc_i((g->xy[0] - (float)ew) / 16.0f)));
    g->rmin[1] = imin(gy, imax(0, trunc_i((g->xy[1] - (float)eh) / 16.0f)));
    g->rmax[0] = imin(gx, imax(0, trunc_i((g->xy[0] + (float)ew) / 16.0f) + 1));
    g->rmax[1] = imin(gy, imax(0, trunc_i((g->xy[1] + (float)eh) / 16.0f) + 1));
    const int area = (g->rmax[0] - g->rmin[0]) * (g->rmax[1] - g->rmin[1]);
    float n[3];
    splat_transform(view, proj, p, scales[2 * (size_t)idx], scales[2 * (size_t)idx + 1], mod,
                    rot + 4 * (size_t)idx, W, H, g->tu, g->tv, g->tw, n);
    const float cosv = -dot3_f(pvx, n[0], pvy, n[1], pvz, n[2]);
    if (cosv == 0.0f || area <= 0) return;
    const float sign = cosv > 0.0f ? 1.0f : -1.0f;
    for (int k = 0; k < 3; ++k) g->normal[k] = sign * n[k];
    if (area == 1) {
        g->write = 1;
        g->hits = (uint32_t)tile_hit(g->rmin[0], g->rmin[1], g->xy, g->conic, g->power);
    } else {
        for (int y = g->rmin[1]; y < g->rmax[1]; ++y)
            for (int x = g->rmin[0]; x < g->rmax[0]; ++x) g->hits += (uint32_t)tile_hit(x, y, g->xy, g->conic, g->power);
        g->write = g->hits > 0;
    }
    if (g->write) {
        if (use_sh) {
            sh_color(p, campos, shs + 48 * (size_t)idx, g->rgb);
        } else {
            for (int k = 0; k < 3; ++k) g->rgb[k] = colors[3 * (size_t)idx + k];
        }
    }
}

typedef struct {
    float cr, cg, cb, o0, o1, t, d, m1, m2, dist, median, nx, ny, nz;
} FgPixel;

/* pixel_shader (render.cu:77-136); rec = x,y,nx,ny,nz,op,r,g,b,spec,rough,tu3,tv3,tw3 */
static void fg_blend(FgPixel* s, float px, float py, const float* g) {
    const float kx = fmaf(px, g[17], -g[11]), ky = fmaf(px, g[18], -g[12]), kz = fmaf(px, g[19], -g[13]);
    const float lx = fmaf(py, g[17], -g[14]), ly = fmaf(py, g[18], -g[15]), lz = fmaf(py, g[19], -g[16]);
    const float pxv = diff2_f(ky, lz, kz, ly), pyv = diff2_f(kz, lx, kx, lz), pzv = diff2_f(kx, ly, ky, lx);
    const float sx = pxv / pzv, sy = pyv / pzv;
    const float rho3d = dot2_f(sx, sx, sy, sy);
    const float dx = g[0] - px, dy = g[1] - py;
    const float rho2d = 2.0f * fmaf(dy, dy, dx * dx);
    const float rho = fminf(rho3d, rho2d);
    const float depth = rho3d <= rho2d ? dot2_f(sx, g[17], sy, g[18]) + g[19] : g[19];
    const float alpha = fminf(0.99f, g[5] * expf(-0.5f * rho));
    const float w = alpha * s->t;
    s->cr = fmaf(g[6], w, s->cr);
    s->cg = fmaf(g[7], w, s->cg);
    s->cb = fmaf(g[8], w, s->cb);
    s->t = fmaf(-alpha, s->t, s->t);
    s->o0 = fmaf(g[9], w, s->o0);
    s->o1 = fmaf(g[10], w, s->o1);
    const float a = 1.0f - s->t;
    const float m = (100.0f / (100.0f - 0.2f)) * (1.0f - 0.2f / depth);
    const float mm = m * m;
    const float dd = fmaf(-(2.0f * m), s->m1, fmaf(mm, a, s->m2));
    s->dist = fmaf(dd, w, s->dist);
    s->m1 = fmaf(m, w, s->m1);
    s->m2 = fmaf(mm, w, s->m2);
    if (s->t > 0.5f) s->median = depth;
    s->d = fmaf(depth, w, s->d);
    s->nx = fmaf(g[2], w, s->nx);
    s->ny = fmaf(g[3], w, s->ny);
    s->nz = fmaf(g[4], w, s->nz);
}

static float encode_bg(float v) {
    float c = fmaxf(0.0f, v * 255.0f);
    c = fminf(c, 255.0f);
    return (float)(unsigned char)c;
}

/*
 * Full FlashGS forward. Outputs are channel-first like the C ABI. When
 * rec24 is non-NULL it receives the per-Gaussian debug state in the layout
 * xy2, normal_opacity4, rgb3, other2, tu3, tv3, tw3, conic_opacity4.
 * keys/values receive the sorted pairs when non-NULL and *pairs fits.
 * Only tile rows with ty % row_stride == 0 are binned and rendered (1 =
 * the whole frame; larger strides give a bounded sample for CPU timing).
 * stage_ms, when non-NULL, receives 5 doubles: the wall times (ms) of
 * preprocess, binning (pair emission, sort, ranges) and blending, the
 * number of pixel x Gaussian blend evaluations and the number of those that
 * changed the pixel (FlashGS blends on every evaluation, so both are equal).
 * Returns the number of pairs emitted, or -1 on allocation failure.
 */
API int64_t oracle_flashgs_forward(int P, int W, int H, const float* pos, const float* shs,
                                   const float* colors, int use_sh, const float* opac,
                                   const float* cov6, const float* scales, float mod,
                                   const float* rot, const float* spec, const float* rough,
                                   const float campos[3], const float rot9[9], float fx, float fy,
                                   float zfar, float znear, const float bg[3], float* out_color,
                                   float* out_other, float* out_depth, float* out_alpha,
                                   float* out_normal, float* out_median, float* out_dist,
                                   float* rec24, uint64_t* keys, uint32_t* values,
                                   int64_t pair_capacity, int32_t* ranges_out, int threads,
                                   int row_stride, double* stage_ms) {
    const double t0 = now_ms();
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    float view[16], proj[16];
    oracle_flashgs_camera(campos, rot9, W, H, fx, fy, zfar, znear, view, proj);
    const int gx = (W + 15) / 16, gy = (H + 15) / 16, tiles = gx * gy;
    FgGauss* gs = (FgGauss*)calloc((size_t)(P > 0 ? P : 1), sizeof(FgGauss));
    float* rec = (float*)calloc((size_t)(P > 0 ? P : 1) * 20, sizeof(float));
    if (gs == NULL || rec == NULL) {
        free(gs);
        free(rec);
        return -1;
    }
#pragma omp parallel for schedule(dynamic, 1024)
    for (int i = 0; i < P; ++i) {
        fg_preprocess_one(i, view, proj, campos, W, H, fx, fy, gx, gy, pos, shs, colors, use_sh,
                          opac, cov6, scales, mod, rot, &gs[i]);
        float* r = rec + 20 * (size_t)i;
        const FgGauss* g = &gs[i];
        if (g->write) {
            const float vals[20] = {g->xy[0], g->xy[1], g->normal[0], g->normal[1], g->normal[2], opac[i],
                                    g->rgb[0], g->rgb[1], g->rgb[2], spec[i], rough[i],
                                    g->tu[0], g->tu[1], g->tu[2], g->tv[0], g->tv[1], g->tv[2],
                                    g->tw[0], g->tw[1], g->tw[2]};
            memcpy(r, vals, sizeof(vals));
        }
        if (rec24 != NULL) {
            float* d = rec24 + 24 * (size_t)i;
            memset(d, 0, 24 * sizeof(float));
            if (g->write) {
                d[0] = r[0]; d[1] = r[1];
                d[2] = r[2]; d[3] = r[3]; d[4] = r[4]; d[5] = r[5];
                d[6] = r[6]; d[7] = r[7]; d[8] = r[8];
                d[9] = r[9]; d[10] = r[10];
                for (int k = 0; k < 9; ++k) d[11 + k] = r[11 + k];
                const float log2e = 1.4426950216293334961f;
                d[20] = (-0.5f * log2e) * g->conic[0];
                d[21] = -log2e * g->conic[1];
                d[22] = (-0.5f * log2e) * g->conic[2];
                d[23] = g->log2op;
            }
        }
    }
    if (row_stride < 1) row_stride = 1;
    const double t1 = now_ms();
    int64_t total = 0;
    for (int i = 0; i < P; ++i) total += gs[i].hits;
    Pair* pairs = (Pair*)malloc((size_t)(total > 0 ? total : 1) * sizeof(Pair));
    if (pairs == NULL) {
        free(gs);
        free(rec);
        return -1;
    }
    int64_t at = 0;
    for (int i = 0; i < P; ++i) {
        const FgGauss* g = &gs[i];
        if (g->hits == 0) continue;
        uint32_t depth_bits;
        memcpy(&depth_bits, &g->depth, 4);
        for (int y = g->rmin[1]; y < g->rmax[1]; ++y)
            for (int x = g->rmin[0]; x < g->rmax[0]; ++x)
                if (y % row_stride == 0 && tile_hit(x, y, g->xy, g->conic, g->power)) {
                    pairs[at].key = ((uint64_t)(y * gx + x) << 32) | depth_bits;
                    pairs[at].value = (uint32_t)i;
                    ++at;
                }
    }
    total = at;
    qsort(pairs, (size_t)total, sizeof(Pair), pair_less);
    int32_t* ranges = (int32_t*)calloc((size_t)tiles * 2, sizeof(int32_t));
    for (int64_t i = 0; i < total; ++i) {
        const uint32_t t = (uint32_t)(pairs[i].key >> 32);
        if (i == 0) ranges[2 * t] = 0;
        else {
            const uint32_t prev = (uint32_t)(pairs[i - 1].key >> 32);
            if (t != prev) {
                ranges[2 * prev + 1] = (int32_t)i;
                ranges[2 * t] = (int32_t)i;
            }
        }
        if (i == total - 1) ranges[2 * t + 1] = (int32_t)total;
    }
    if (keys != NULL && values != NULL && total <= pair_capacity) {
        for (int64_t i = 0; i < total; ++i) {
            keys[i] = pairs[i].key;
            values[i] = pairs[i].value;
        }
    }
    if (ranges_out != NULL) memcpy(ranges_out, ranges, (size_t)tiles * 2 * sizeof(int32_t));
    const double t2 = now_ms();
    const size_t plane = (size_t)W * H;
    int64_t evaluations = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : evaluations)
    for (int tile = 0; tile < tiles; ++tile) {
        const int tx = tile % gx, ty = tile / gx;
        if (ty % row_stride != 0) continue;
        const int start = ranges[2 * tile], end = ranges[2 * tile + 1];
        FgPixel px[256];
        for (int k = 0; k < 256; ++k) {
            memset(&px[k], 0, sizeof(FgPixel));
            px[k].t = 1.0f;
        }
        if (start < end) {
            /* Stop after the first Gaussian that leaves every pixel of the
             * tile (including pixels outside the image) with T < 1e-4
             * (render.cu:499-698). */
            for (int j = start; j < end; ++j) {
                const float* g = rec + 20 * (size_t)pairs[j].value;
                evaluations += 256;
                int done = 1;
                for (int k = 0; k < 256; ++k) {
                    fg_blend(&px[k], (float)(tx * 16 + (k & 15)), (float)(ty * 16 + (k >> 4)), g);
                    done = done && px[k].t < 0.0001f;
                }
                if (done) break;
            }
        }
        for (int k = 0; k < 256; ++k) {
            const int x = tx * 16 + (k & 15), y = ty * 16 + (k >> 4);
            if (x >= W || y >= H) continue;
            const size_t pid = (size_t)y * W + x;
            const FgPixel* s = &px[k];
            if (start >= end) {
                out_color[pid] = encode_bg(bg[0]);
                out_color[plane + pid] = encode_bg(bg[1]);
                out_color[2 * plane + pid] = encode_bg(bg[2]);
                out_other[pid] = out_other[plane + pid] = 0.0f;
                out_depth[pid] = out_alpha[pid] = 0.0f;
                out_normal[pid] = out_normal[plane + pid] = out_normal[2 * plane + pid] = 0.0f;
                out_median[pid] = out_dist[pid] = 0.0f;
                continue;
            }
            const float t = s->t < 0.0001f ? 0.0f : s->t;
            out_color[pid] = fmaf(t, bg[0], s->cr);
            out_color[plane + pid] = fmaf(t, bg[1], s->cg);
            out_color[2 * plane + pid] = fmaf(t, bg[2], s->cb);
            out_other[pid] = fmaf(t, bg[0], s->o0);
            out_other[plane + pid] = fmaf(t, bg[1], s->o1);
            out_depth[pid] = s->d;
            out_alpha[pid] = 1.0f - t;
            out_normal[pid] = s->nx;
            out_normal[plane + pid] = s->ny;
            out_normal[2 * plane + pid] = s->nz;
            out_median[pid] = s->median;
            out_dist[pid] = s->dist;
        }
    }
    if (stage_ms != NULL) {
        stage_ms[0] = t1 - t0;
        stage_ms[1] = t2 - t1;
        stage_ms[2] = now_ms() - t2;
        stage_ms[3] = (double)evaluations;
        stage_ms[4] = (double)evaluations;
    }
    free(ranges);
    free(pairs);
    free(rec);
    free(gs);
    return total;
}

/* --------------------------------------------------------------- standard */

typedef struct {
    float rec[20]; /* x,y,n3,op,c5,tu3,tv3,tw3 */
    float depth;
    int radius;
    int rmin[2], rmax[2];
    int valid;
} StGauss;

/* preprocessCUDA<5> (forward.cu:148-251) with in_frustum, compute_aabb, getRect. */
static void st_preprocess_one(int idx, const float* view, const float* proj, int W, int H, int gx,
                              int gy, const float* means, const float* colors5, const float* opac,
                              const float* scales, float mod, const float* rot, StGauss* g) {
    memset(g, 0, sizeof(*g));
    const float* p = means + 3 * (size_t)idx;
    const float pvx = affine_row(view, 0, p[0], p[1], p[2]);
    const float pvy = affine_row(view, 1, p[0], p[1], p[2]);
    const float pvz = affine_row(view, 2, p[0], p[1], p[2]);
    if (pvz <= 0.2f) return;
    float tu[3], tv[3], tw[3], n[3];
    splat_transform(view, proj, p, scales[2 * (size_t)idx], scales[2 * (size_t)idx + 1], mod,
                    rot + 4 * (size_t)idx, W, H, tu, tv, tw, n);
    const float cosv = -dot3_f(pvx, n[0], pvy, n[1], pvz, n[2]);
    if (cosv == 0.0f) return;
    const float sign = cosv > 0.0f ? 1.0f : -1.0f;
    /* contraction forms of the reference standard build: 9*Tw.y^2 fused onto
     * the rounded 9*Tw.x^2; the x pairs of the centre and the extent fuse
     * their second product, the y pairs their first */
    const float d = fmaf(-tw[2], tw[2], fmaf(9.0f, tw[1] * tw[1], 9.0f * (tw[0] * tw[0])));
    if (d == 0.0f) return;
    const float inv = 1.0f / d;
    const float fxv = inv * 9.0f, fyv = inv * 9.0f, fzv = -inv;
    const float px = fmaf(fzv, tu[2] * tw[2], fmaf(fyv, tu[1] * tw[1], fxv * (tu[0] * tw[0])));
    const float py = dot3_f(fxv, tv[0] * tw[0], fyv, tv[1] * tw[1], fzv, tv[2] * tw[2]);
    const float qx = fmaf(fzv, tu[2] * tu[2], fmaf(fyv, tu[1] * tu[1], fxv * (tu[0] * tu[0])));
    const float qy = dot3_f(fxv, tv[0] * tv[0], fyv, tv[1] * tv[1], fzv, tv[2] * tv[2]);
    const float h0x = fmaf(px, px, -qx), h0y = fmaf(py, py, -qy);
    const float hx = sqrtf(1e-4f < h0x ? h0x : 1e-4f), hy = sqrtf(1e-4f < h0y ? h0y : 1e-4f);
    const float radius = ceilf(fmaxf(fmaxf(hx, hy), 3.0f * 0.707106f));
    const float rad = (float)(int)radius;
    g->rmin[0] = imin(gx, imax(0, trunc_i((px - rad) / 16.0f)));
    g->rmin[1] = imin(gy, imax(0, trunc_i((py - rad) / 16.0f)));
    g->rmax[0] = imin(gx, imax(0, trunc_i((px + rad + 16.0f - 1.0f) / 16.0f)));
    g->rmax[1] = imin(gy, imax(0, trunc_i((py + rad + 16.0f - 1.0f) / 16.0f)));
    if ((g->rmax[0] - g->rmin[0]) * (g->rmax[1] - g->rmin[1]) == 0) return;
    g->valid = 1;
    g->depth = pvz;
    g->radius = (int)radius;
    float* r = g->rec;
    r[0] = px; r[1] = py;
    r[2] = sign * n[0]; r[3] = sign * n[1]; r[4] = sign * n[2];
    r[5] = opac[idx];
    for (int k = 0; k < 5; ++k) r[6 + k] = colors5[5 * (size_t)idx + k];
    for (int k = 0; k < 3; ++k) {
        r[11 + k] = tu[k];
        r[14 + k] = tv[k];
        r[17 + k] = tw[k];
    }
}

typedef struct {
    float c[5], t, d, m1, m2, dist, median, n[3];
    int done;
} StPixel;

/* One pixel, one Gaussian (forward.cu:345-421); returns the blend weight. */
static float st_blend(StPixel* s, float px, float py, const float* g) {
    if (s->done) return 0.0f;
    const float kx = fmaf(px, g[17], -g[11]), ky = fmaf(px, g[18], -g[12]), kz = fmaf(px, g[19], -g[13]);
    const float lx = fmaf(py, g[17], -g[14]), ly = fmaf(py, g[18], -g[15]), lz = fmaf(py, g[19], -g[16]);
    const float pzv = diff2_f(kx, ly, ky, lx);
    if (pzv == 0.0f) return 0.0f;
    const float pxv = diff2_f(ky, lz, kz, ly), pyv = diff2_f(kz, lx, kx, lz);
    const float sx = pxv / pzv, sy = pyv / pzv;
    const float rho3d = dot2_f(sx, sx, sy, sy);
    const float dx = g[0] - px, dy = g[1] - py;
    const float rho2d = 2.0f * fmaf(dy, dy, dx * dx);
    const float rho = fminf(rho3d, rho2d);
    const float depth = rho3d <= rho2d ? dot2_f(sx, g[17], sy, g[18]) + g[19] : g[19];
    if (depth < 0.2f) return 0.0f;
    const float power = -0.5f * rho;
    if (power > 0.0f) return 0.0f;
    const float alpha = fminf(0.99f, g[5] * expf(power));
    if (alpha < 1.0f / 255.0f) return 0.0f;
    const float test_t = s->t * (1.0f - alpha);
    if (test_t < 0.0001f) {
        s->done = 1;
        return 0.0f;
    }
    const float w = alpha * s->t;
    const float a = 1.0f - s->t;
    const float m = (100.0f / (100.0f - 0.2f)) * (1.0f - 0.2f / depth);
    const float mm = m * m;
    s->dist = fmaf(fmaf(-(2.0f * m), s->m1, fmaf(mm, a, s->m2)), w, s->dist);
    s->d = fmaf(depth, w, s->d);
    s->m1 = fmaf(m, w, s->m1);
    s->m2 = fmaf(mm, w, s->m2);
    if (s->t > 0.5f) s->median = depth;
    for (int k = 0; k < 3; ++k) s->n[k] = fmaf(g[2 + k], w, s->n[k]);
    for (int k = 0; k < 5; ++k) s->c[k] = fmaf(g[6 + k], w, s->c[k]);
    s->t = test_t;
    return w;
}

/* Full standard forward (full_rasterizer.cu:203-394); matrices column-major
 * as stored by the caller. row_stride samples tile rows as in
 * oracle_flashgs_forward. Returns the full-frame pair count or -1. */
API int64_t oracle_standard_forward(int P, const float* bg5, int W, int H, const float* means,
                                    const float* colors5, const float* opac, const float* scales,
                                    float mod, const float* rot, const float* view,
                                    const float* proj, float* out_color5, float* out_aux7,
                                    float* out_weight, int32_t* out_radii, int threads,
                                    int row_stride, double* stage_ms) {
    const double t0 = now_ms();
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    const size_t plane = (size_t)W * H;
    if (P == 0) {
        memset(out_color5, 0, 5 * plane * sizeof(float));
        memset(out_aux7, 0, 7 * plane * sizeof(float));
        return 0;
    }
    const int gx = (W + 15) / 16, gy = (H + 15) / 16, tiles = gx * gy;
    StGauss* gs = (StGauss*)calloc((size_t)P, sizeof(StGauss));
    if (gs == NULL) return -1;
#pragma omp parallel for schedule(dynamic, 1024)
    for (int i = 0; i < P; ++i) {
        st_preprocess_one(i, view, proj, W, H, gx, gy, means, colors5, opac, scales, mod, rot, &gs[i]);
        out_radii[i] = gs[i].valid ? gs[i].radius : 0;
        out_weight[i] = 0.0f;
    }
    if (row_stride < 1) row_stride = 1;
    const double t1 = now_ms();
    int64_t total = 0;
    for (int i = 0; i < P; ++i)
        if (gs[i].valid) total += (int64_t)(gs[i].rmax[0] - gs[i].rmin[0]) * (gs[i].rmax[1] - gs[i].rmin[1]);
    Pair* pairs = (Pair*)malloc((size_t)(total > 0 ? total : 1) * sizeof(Pair));
    if (pairs == NULL) {
        free(gs);
        return -1;
    }
    int64_t at = 0;
    for (int i = 0; i < P; ++i) {
        if (!gs[i].valid) continue;
        uint32_t depth_bits;
        memcpy(&depth_bits, &gs[i].depth, 4);
        for (int y = gs[i].rmin[1]; y < gs[i].rmax[1]; ++y) {
            if (y % row_stride != 0) continue;
            for (int x = gs[i].rmin[0]; x < gs[i].rmax[0]; ++x) {
                pairs[at].key = ((uint64_t)(y * gx + x) << 32) | depth_bits;
                pairs[at].value = (uint32_t)i;
                ++at;
            }
        }
    }
    const int64_t all_pairs = total;
    total = at;
    qsort(pairs, (size_t)total, sizeof(Pair), pair_less);
    int64_t* ranges = (int64_t*)calloc((size_t)tiles * 2, sizeof(int64_t));
    for (int64_t i = 0; i < total; ++i) {
        const uint32_t t = (uint32_t)(pairs[i].key >> 32);
        if (i == 0) ranges[2 * t] = 0;
        else {
            const uint32_t prev = (uint32_t)(pairs[i - 1].key >> 32);
            if (t != prev) {
                ranges[2 * prev + 1] = i;
                ranges[2 * t] = i;
            }
        }
        if (i == total - 1) ranges[2 * t + 1] = total;
    }
    const double t2 = now_ms();
    int64_t evaluations = 0, live = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : evaluations, live)
    for (int tile = 0; tile < tiles; ++tile) {
        const int tx = tile % gx, ty = tile / gx;
        if (ty % row_stride != 0) continue;
        StPixel px[256];
        for (int k = 0; k < 256; ++k) {
            memset(&px[k], 0, sizeof(StPixel));
            px[k].t = 1.0f;
            px[k].done = !(tx * 16 + (k & 15) < W && ty * 16 + (k >> 4) < H);
        }
        for (int64_t j = ranges[2 * tile]; j < ranges[2 * tile + 1]; ++j) {
            const StGauss* g = &gs[pairs[j].value];
            int all_done = 1;
            for (int k = 0; k < 256; ++k) {
                const int was_done = px[k].done;
                evaluations += was_done ? 0 : 1;
                const float w = st_blend(&px[k], (float)(tx * 16 + (k & 15)), (float)(ty * 16 + (k >> 4)), g->rec);
                live += (!was_done && (w != 0.0f || px[k].done)) ? 1 : 0;
                if (w != 0.0f) {
#pragma omp atomic
                    out_weight[pairs[j].value] += w;
                }
                all_done = all_done && px[k].done;
            }
            if (all_done) break;
        }
        for (int k = 0; k < 256; ++k) {
            const int x = tx * 16 + (k & 15), y = ty * 16 + (k >> 4);
            if (x >= W || y >= H) continue;
            const size_t pid = (size_t)y * W + x;
            const StPixel* s = &px[k];
            for (int c = 0; c < 5; ++c) out_color5[c * plane + pid] = fmaf(s->t, bg5[c], s->c[c]);
            out_aux7[pid] = s->d;
            out_aux7[plane + pid] = 1.0f - s->t;
            for (int c = 0; c < 3; ++c) out_aux7[(2 + c) * plane + pid] = s->n[c];
            out_aux7[5 * plane + pid] = s->median;
            out_aux7[6 * plane + pid] = s->dist;
        }
    }
    if (stage_ms != NULL) {
        stage_ms[0] = t1 - t0;
        stage_ms[1] = t2 - t1;
        stage_ms[2] = now_ms() - t2;
        stage_ms[3] = (double)evaluations;
        stage_ms[4] = (double)live;
    }
    free(ranges);
    free(pairs);
    free(gs);
    return all_pairs;
}

/* ---- checker of the standard backend's culling (test infrastructure) ----
 *
 * Restates the CUDA library's tile/quadrant culling (csrc/standard_math.cuh:
 * cull_shape, cull_tile_box, the chord spans, row hulls, row columns and
 * quadrant masks) with correctly rounded CPU arithmetic in place of the
 * GPU's approximate square roots, and checks it against the reference's
 * per-pixel arithmetic (forward.cu:345-393 as restated in st_blend): every
 * 8x8 quadrant of a Gaussian's reference rectangle holding a pixel whose
 * evaluation reaches alpha >= 1/255 must be emitted with its mask bit set.
 * out[0] = quadrants holding such a pixel, out[1] = those the culling misses,
 * out[2] = tiles emitted, out[3] = tiles of the reference rectangles. */
typedef struct { float mx, my, k, w0, hx, hy, yr, ihy, gx, gy, r2; int mode; } CullC;
enum { kCullEllipseC = 0, kCullNeverC = 1, kCullAlwaysC = 2 };

static CullC cull_c(float op, float x, float y, const float* tu, const float* tv, const float* tw) {
    CullC c;
    memset(&c, 0, sizeof c);
    c.gx = x;
    c.gy = y;
    if (!(op > 1.0f / 255.0f)) { c.mode = kCullAlwaysC; return c; }
    const float cwf = 1.02f * (2.0f * logf(255.0f * op)) + 0.05f;
    const double cw = (double)cwf * 1.0001;
    c.r2 = (float)(0.5 * cw * 1.0001);
    const double twx = tw[0], twy = tw[1], twz = tw[2];
    const double d = cw * (twx * twx + twy * twy) - twz * twz;
    c.mode = kCullNeverC;
    if (!(d < -1e-6 * twz * twz)) return c;
    const double fxy = cw / d, fz = -1.0 / d;
    const double mx = fxy * ((double)tu[0] * twx + (double)tu[1] * twy) + fz * (double)tu[2] * twz;
    const double my = fxy * ((double)tv[0] * twx + (double)tv[1] * twy) + fz * (double)tv[2] * twz;
    const double quu = fxy * ((double)tu[0] * tu[0] + (double)tu[1] * tu[1]) + fz * (double)tu[2] * tu[2];
    const double qvv = fxy * ((double)tv[0] * tv[0] + (double)tv[1] * tv[1]) + fz * (double)tv[2] * tv[2];
    const double quv = fxy * ((double)tu[0] * tv[0] + (double)tu[1] * tv[1]) + fz * (double)tu[2] * tv[2];
    const double sxx = mx * mx - quu, syy = my * my - qvv, sxy = mx * my - quv, det = sxx * syy - sxy * sxy;
    if (!(sxx > 0 && syy > 0 && det > 0) || !(fabs(mx) < 1e7 && fabs(my) < 1e7)) return c;
    const double s = 1.0003;
    c.mx = (float)mx; c.my = (float)my; c.k = (float)(sxy / syy); c.w0 = (float)(sqrt(det / syy) * s);
    c.hx = (float)(sqrt(sxx) * s); c.hy = (float)(sqrt(syy) * s); c.yr = (float)(sxy / sqrt(sxx) * s);
    c.ihy = (float)(1.0 / (sqrt(syy) * s));
    c.mode = kCullEllipseC;
    return c;
}

static void espan_c(const CullC* c, float ya, float yb, float* l, float* r) {
    const float y0 = fmaxf(ya - c->my, -c->hy), y1 = fminf(yb - c->my, c->hy);
    if (!(y0 <= y1)) { *l = 1.0f; *r = 0.0f; return; }
    const float t0 = fminf(fmaxf(y0 * c->ihy, -1.0f), 1.0f), t1 = fminf(fmaxf(y1 * c->ihy, -1.0f), 1.0f);
    const float h0 = c->w0 * sqrtf((1.0f - t0) * (1.0f + t0)), h1 = c->w0 * sqrtf((1.0f - t1) * (1.0f + t1));
    const float c0 = c->k * y0, c1 = c->k * y1;
    float xl = fminf(c0 - h0, c1 - h1), xr = fmaxf(c0 + h0, c1 + h1);
    if (y0 <= -c->yr && -c->yr <= y1) xl = fminf(xl, -c->hx);
    if (y0 <= c->yr && c->yr <= y1) xr = fmaxf(xr, c->hx);
    *l = c->mx + xl;
    *r = c->mx + xr;
}

static void dspan_c(const CullC* c, float ya, float yb, float* l, float* r) {
    const float dy = fmaxf(fmaxf(ya - c->gy, c->gy - yb), 0.0f);
    const float q = c->r2 - dy * dy;
    if (!(q >= 0.0f)) { *l = 1.0f; *r = 0.0f; return; }
    const float w = sqrtf(q);
    *l = c->gx - w;
    *r = c->gx + w;
}

static int meets_c(float l, float r, float x0, float x1) { return x0 <= r && x1 >= l && l <= r; }

static void hull_c(float al, float ar, float bl, float br, float* l, float* r) {
    const int a = al <= ar, b = bl <= br;
    *l = a && b ? fminf(al, bl) : (a ? al : (b ? bl : 1.0f));
    *r = a && b ? fmaxf(ar, br) : (a ? ar : (b ? br : 0.0f));
}

/* Emitted? and mask of tile (tx, ty) for an ellipse-mode shape. Tiles and
 * quadrants are widened by CULL_PAD pixels on each side (csrc kCullPad). */
#define CULL_PAD 0.25f
static unsigned tile_mask_c(const CullC* c, int tx, int ty) {
    float s[2][4];
    for (int qy = 0; qy < 2; ++qy) {
        const float y = (float)(ty * 16 + qy * 8);
        espan_c(c, y - CULL_PAD, y + (7.0f + CULL_PAD), &s[qy][0], &s[qy][1]);
        dspan_c(c, y - CULL_PAD, y + (7.0f + CULL_PAD), &s[qy][2], &s[qy][3]);
    }
    float el, er, dl, dr;
    hull_c(s[0][0], s[0][1], s[1][0], s[1][1], &el, &er);
    hull_c(s[0][2], s[0][3], s[1][2], s[1][3], &dl, &dr);
    const float x0 = (float)(tx * 16) - CULL_PAD, x1 = (float)(tx * 16) + (15.0f + CULL_PAD);
    if (!(meets_c(el, er, x0, x1) || meets_c(dl, dr, x0, x1))) return 0u;
    unsigned m = 0;
    for (int qy = 0; qy < 2; ++qy)
        for (int qx = 0; qx < 2; ++qx) {
            const float a = (float)(tx * 16 + qx * 8) - CULL_PAD, b = (float)(tx * 16 + qx * 8) + (7.0f + CULL_PAD);
            if (meets_c(s[qy][0], s[qy][1], a, b) || meets_c(s[qy][2], s[qy][3], a, b)) m |= 1u << (qy * 2 + qx);
        }
    return m ? m : 15u;
}

/* Does the evaluation of Gaussian record g at pixel (px, py) reach alpha >= 1/255? */
static int pixel_live_c(const float* g, float px, float py) {
    StPixel s;
    memset(&s, 0, sizeof s);
    s.t = 1.0f;
    return st_blend(&s, px, py, g) != 0.0f || s.done;
}

API int oracle_standard_cull_check(int P, int W, int H, const float* means, const float* opac,
                                   const float* scales, float mod, const float* rot,
                                   const float* view, const float* proj, int threads,
                                   int64_t* out) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    const int gx = (W + 15) / 16, gy = (H + 15) / 16;
    static const float zero5[5] = {0, 0, 0, 0, 0};
    int64_t live_q = 0, missed = 0, emitted = 0, rect_tiles = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : live_q, missed, emitted, rect_tiles)
    for (int i = 0; i < P; ++i) {
        StGauss g;
        st_preprocess_one(0, view, proj, W, H, gx, gy, means + 3 * (size_t)i, zero5, opac + i,
                          scales + 2 * (size_t)i, mod, rot + 4 * (size_t)i, &g);
        if (!g.valid) continue;
        const float* R = g.rec;
        const CullC c = cull_c(R[5], R[0], R[1], R + 11, R + 14, R + 17);
        int bx0 = 0, by0 = 0, bx1 = -1, by1 = -1;
        if (c.mode == kCullNeverC) {
            bx0 = by0 = -1000000;
            bx1 = by1 = 1000000;
        } else if (c.mode == kCullEllipseC) {
            const float rd = sqrtf(c.r2) + 1.0f, ex = c.hx + 1.0f, ey = c.hy + 1.0f;
            bx0 = (int)floorf(fmaxf(fminf(c.gx - rd, c.mx - ex), -1e6f) * (1.0f / 16.0f));
            by0 = (int)floorf(fmaxf(fminf(c.gy - rd, c.my - ey), -1e6f) * (1.0f / 16.0f));
            bx1 = (int)floorf(fminf(fmaxf(c.gx + rd, c.mx + ex), 1e6f) * (1.0f / 16.0f));
            by1 = (int)floorf(fminf(fmaxf(c.gy + rd, c.my + ey), 1e6f) * (1.0f / 16.0f));
        }
        for (int ty = g.rmin[1]; ty < g.rmax[1]; ++ty)
            for (int tx = g.rmin[0]; tx < g.rmax[0]; ++tx) {
                ++rect_tiles;
                const int in_box = tx >= bx0 && tx <= bx1 && ty >= by0 && ty <= by1;
                unsigned mask = 0;
                if (in_box) mask = c.mode == kCullNeverC ? 15u : tile_mask_c(&c, tx, ty);
                emitted += mask != 0u;
                for (int q = 0; q < 4; ++q) {
                    int live = 0;
                    for (int k = 0; k < 64 && !live; ++k) {
                        const int x = tx * 16 + (q & 1) * 8 + (k & 7), y = ty * 16 + (q >> 1) * 8 + (k >> 3);
                        if (x < W && y < H) live = pixel_live_c(R, (float)x, (float)y);
                    }
                    live_q += live;
                    missed += live && !(mask & (1u << q));
                }
            }
    }
    out[0] = live_q;
    out[1] = missed;
    out[2] = emitted;
    out[3] = rect_tiles;
    return 0;
}
