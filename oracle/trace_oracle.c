/*
 * CPU restatement of the HybridSplat reflection trace.
 *
 * TEST INFRASTRUCTURE ONLY. It is the oracle the GPU trace
 * (hybridsplat_jittor_render_b200/csrc/trace.cu) is compared with; the
 * product never links or calls it.
 *
 * It restates the reference OptiX programs (vendor/optix_tracer/forward.cu:
 * traceRay 219-405, tracePath 408-538, __raygen__ot 541-596, __anyhit__ot
 * 599-660; constants config.h:31-45, auxiliary.h:31-55; geometry
 * compute_transmat_uv 75-110, compute_transmat_xy 112-169) without a BVH:
 * every trace step tests every triangle of the scene (the watertight test of
 * Woop, Benthin and Wald, JCGT 2013), sorts the hits by (distance,
 * primitive) and keeps the 16 nearest, as the any-hit program's sorted
 * CHUNK_SIZE buffer does. The arithmetic is the GPU library's, operation by
 * operation (-ffp-contract=off, fmaf where it fuses); the reference's rsqrtf
 * is 1/sqrtf in both. Only expf differs (C library vs CUDA), so GPU and
 * oracle agree to a tolerance. No OptiX build exists here, so neither is
 * pinned against the reference's own trace ("parity unpinned").
 *
 * Built into oracle/libcpu_oracle.so by oracle/build_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define API __attribute__((visibility("default")))

#define CHUNK 16
#define DEPTH_INF 1e16f
#define MAX_CONTRIB 256
#define STEP_EPS 0.00001
#define START_OFFSET_F 0.06f
#define NEAR_N 0.2f
#define FAR_N 100.0f
#define T_THRESHOLD 0.0001f
#define MAX_TRACE_STEPS 4096 /* bound of the library's trace steps per segment */

typedef struct { float x, y, z; } V3;

static V3 v3(float x, float y, float z) { V3 r = {x, y, z}; return r; }
static float comp3(V3 v, int k) { return k == 0 ? v.x : (k == 1 ? v.y : v.z); }
static float dot3(V3 a, V3 b) { return fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)); }
static V3 normalize3(V3 v) {
    const float n = sqrtf(dot3(v, v));
    return v3(v.x / n, v.y / n, v.z / n);
}

typedef struct { int kx, ky, kz; float sx, sy, sz; } Shear;

static Shear ray_shear(V3 d) {
    const float ax = fabsf(d.x), ay = fabsf(d.y), az = fabsf(d.z);
    Shear r;
    r.kz = (ax > ay) ? (ax > az ? 0 : 2) : (ay > az ? 1 : 2);
    r.kx = r.kz == 2 ? 0 : r.kz + 1;
    r.ky = r.kx == 2 ? 0 : r.kx + 1;
    if (comp3(d, r.kz) < 0.0f) {
        const int t = r.kx;
        r.kx = r.ky;
        r.ky = t;
    }
    const float dz = comp3(d, r.kz);
    r.sx = comp3(d, r.kx) / dz;
    r.sy = comp3(d, r.ky) / dz;
    r.sz = 1.0f / dz;
    return r;
}

static float hit_triangle(V3 o, const Shear* r, V3 a, V3 b, V3 c) {
    const V3 A = v3(a.x - o.x, a.y - o.y, a.z - o.z);
    const V3 B = v3(b.x - o.x, b.y - o.y, b.z - o.z);
    const V3 C = v3(c.x - o.x, c.y - o.y, c.z - o.z);
    const float ax = comp3(A, r->kx) - r->sx * comp3(A, r->kz);
    const float ay = comp3(A, r->ky) - r->sy * comp3(A, r->kz);
    const float bx = comp3(B, r->kx) - r->sx * comp3(B, r->kz);
    const float by = comp3(B, r->ky) - r->sy * comp3(B, r->kz);
    const float cx = comp3(C, r->kx) - r->sx * comp3(C, r->kz);
    const float cy = comp3(C, r->ky) - r->sy * comp3(C, r->kz);
    float u = cx * by - cy * bx;
    float v = ax * cy - ay * cx;
    float w = bx * ay - by * ax;
    if (u == 0.0f || v == 0.0f || w == 0.0f) {
        u = (float)((double)cx * by - (double)cy * bx);
        v = (float)((double)ax * cy - (double)ay * cx);
        w = (float)((double)bx * ay - (double)by * ax);
    }
    if ((u < 0.0f || v < 0.0f || w < 0.0f) && (u > 0.0f || v > 0.0f || w > 0.0f)) return -1.0f;
    const float det = (u + v) + w;
    if (det == 0.0f) return -1.0f;
    const float az = r->sz * comp3(A, r->kz);
    const float bz = r->sz * comp3(B, r->kz);
    const float cz = r->sz * comp3(C, r->kz);
    const float t = ((u * az + v * bz) + w * cz) / det;
    return t >= 0.0f ? t : -1.0f;
}

static void rotation_rows_t(const float* q, V3 R[3]) {
    const float s = 1.0f / sqrtf(fmaf(q[2], q[2], fmaf(q[1], q[1], fmaf(q[0], q[0], q[3] * q[3]))));
    const float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    R[0] = v3(1.0f - 2.0f * fmaf(z, z, y * y), 2.0f * fmaf(w, z, x * y), 2.0f * fmaf(-w, y, x * z));
    R[1] = v3(2.0f * fmaf(-w, z, x * y), 1.0f - 2.0f * fmaf(z, z, x * x), 2.0f * fmaf(w, x, y * z));
    R[2] = v3(2.0f * fmaf(w, y, x * z), 2.0f * fmaf(-w, x, y * z), 1.0f - 2.0f * fmaf(y, y, x * x));
}

static V3 sh_color(int deg, const float* sh, V3 dir_orig) {
    static const float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
    static const float C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                                -1.0925484305920792f, 0.5462742152960396f};
    static const float C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                                0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                                -0.5900435899266435f};
    float res[3];
    for (int ch = 0; ch < 3; ++ch) res[ch] = C0 * sh[ch];
    const V3 d = normalize3(dir_orig);
    if (deg > 0) {
        const float x = d.x, y = d.y, z = d.z;
        const float c1y = C1 * y, c1z = C1 * z, c1x = C1 * x;
        for (int ch = 0; ch < 3; ++ch)
            res[ch] = fmaf(-c1x, sh[9 + ch], fmaf(c1z, sh[6 + ch], fmaf(-c1y, sh[3 + ch], res[ch])));
        if (deg > 1) {
            const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
            const float f4 = C2[0] * xy, f5 = C2[1] * yz, f6 = C2[2] * ((2.0f * zz - xx) - yy);
            const float f7 = C2[3] * xz, f8 = C2[4] * (xx - yy);
            for (int ch = 0; ch < 3; ++ch) {
                float t = fmaf(f4, sh[12 + ch], res[ch]);
                t = fmaf(f5, sh[15 + ch], t);
                t = fmaf(f6, sh[18 + ch], t);
                t = fmaf(f7, sh[21 + ch], t);
                res[ch] = fmaf(f8, sh[24 + ch], t);
            }
            if (deg > 2) {
                const float g9 = (C3[0] * y) * (3.0f * xx - yy);
                const float g10 = (C3[1] * xy) * z;
                const float g11 = (C3[2] * y) * ((4.0f * zz - xx) - yy);
                const float g12 = (C3[3] * z) * ((2.0f * zz - 3.0f * xx) - 3.0f * yy);
                const float g13 = (C3[4] * x) * ((4.0f * zz - xx) - yy);
                const float g14 = (C3[5] * z) * (xx - yy);
                const float g15 = (C3[6] * x) * (xx - 3.0f * yy);
                for (int ch = 0; ch < 3; ++ch) {
                    float t = fmaf(g9, sh[27 + ch], res[ch]);
                    t = fmaf(g10, sh[30 + ch], t);
                    t = fmaf(g11, sh[33 + ch], t);
                    t = fmaf(g12, sh[36 + ch], t);
                    t = fmaf(g13, sh[39 + ch], t);
                    t = fmaf(g14, sh[42 + ch], t);
                    res[ch] = fmaf(g15, sh[45 + ch], t);
                }
            }
        }
    }
    return v3(fmaxf(res[0] + 0.5f, 0.0f), fmaxf(res[1] + 0.5f, 0.0f), fmaxf(res[2] + 0.5f, 0.0f));
}

static float col4(const float m[4], float a0, float a1, float a2, float a3) {
    return fmaf(m[3], a3, fmaf(m[2], a2, fmaf(m[1], a1, m[0] * a0)));
}

static int transmat_xy(V3 p, const float* scale, float mod, const float* rot, const float* proj, int W, int H,
                       float cutoff, float* s2pz, float xy[2]) {
    V3 T[3];
    rotation_rows_t(rot, T);
    const V3 R[3] = {v3(T[0].x, T[1].x, T[2].x), v3(T[0].y, T[1].y, T[2].y), v3(T[0].z, T[1].z, T[2].z)};
    const float sx = mod * scale[0], sy = mod * scale[1];
    const V3 L[3] = {v3(R[0].x * sx, R[0].y * sy, R[0].z), v3(R[1].x * sx, R[1].y * sy, R[1].z),
                     v3(R[2].x * sx, R[2].y * sy, R[2].z)};
    const float s2w[4][3] = {{L[0].x, L[0].y, p.x}, {L[1].x, L[1].y, p.y}, {L[2].x, L[2].y, p.z}, {0.0f, 0.0f, 1.0f}};
    const float w2n[4][4] = {{proj[0], proj[4], proj[8], proj[12]}, {proj[1], proj[5], proj[9], proj[13]},
                             {proj[2], proj[6], proj[10], proj[14]}, {proj[3], proj[7], proj[11], proj[15]}};
    const float n2p[3][4] = {{(float)(W / 2.0), 0.0f, 0.0f, (float)((W - 1) / 2.0)},
                             {0.0f, (float)(H / 2.0), 0.0f, (float)((H - 1) / 2.0)},
                             {0.0f, 0.0f, 0.0f, 1.0f}};
    float P[3][4], S[3][3];
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 4; ++c) P[r][c] = col4(n2p[r], w2n[0][c], w2n[1][c], w2n[2][c], w2n[3][c]);
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) S[r][c] = col4(P[r], s2w[0][c], s2w[1][c], s2w[2][c], s2w[3][c]);
    *s2pz = S[2][2];
    const float c2 = cutoff * cutoff;
    const V3 t = v3(c2, c2, -1.0f);
    const float d = dot3(t, v3(S[2][0] * S[2][0], S[2][1] * S[2][1], S[2][2] * S[2][2]));
    if (d == 0.0f) return 0;
    const float f[3] = {t.x / d, t.y / d, t.z / d};
    xy[0] = ((f[0] * S[0][0]) * S[2][0] + (f[1] * S[0][1]) * S[2][1]) + (f[2] * S[0][2]) * S[2][2];
    xy[1] = ((f[0] * S[1][0]) * S[2][0] + (f[1] * S[1][1]) * S[2][1]) + (f[2] * S[1][2]) * S[2][2];
    return 1;
}

typedef struct {
    uint64_t rays;
    const float *bg, *means, *shs, *others, *opac, *scales, *rot, *proj, *campos;
    uint32_t coeffs;
    int degree, sff, max_depth;
    float mod, spec_thr;
    const float* tri_v;  /* [T][9] vertices, NaN for an invalid triangle */
    uint64_t tris;
} Scene;

typedef struct { float t; uint32_t p; } Hit;

static int hit_less(const void* a, const void* b) {
    const Hit *x = (const Hit*)a, *y = (const Hit*)b;
    if (x->t != y->t) return x->t < y->t ? -1 : 1;
    return x->p < y->p ? -1 : (x->p > y->p);
}

typedef struct { float c[3], d, a, dist, m1, m2, t, n[3], o[2]; V3 e; } Seg;

/* stats (optional, per ray): [0] trace steps, [1] hits found over all steps,
   [2] contributors, [3] hits shaded (not skipped as a repeat) */
static void trace_segment(const Scene* s, V3 o, V3 d, float min_depth, int depth_index, Seg* g, Hit* all,
                          uint32_t* stats) {
    const Shear shear = ray_shear(d);
    const V3 campos = v3(s->campos[0], s->campos[1], s->campos[2]);
    const float far_ratio = FAR_N / (FAR_N - NEAR_N);
    float t_prev = 1.0f, t_next = 1.0f, dpt = 0.0f, pdpt = 0.0f;
    int last = -1, contributors = 0;
    V3 ot = o;
    for (int step_count = 0; step_count < MAX_TRACE_STEPS; ++step_count) {
        uint64_t found = 0;
        for (uint64_t k = 0; k < s->tris; ++k) {
            const float* v = s->tri_v + 9 * k;
            const float t = hit_triangle(ot, &shear, v3(v[0], v[1], v[2]), v3(v[3], v[4], v[5]), v3(v[6], v[7], v[8]));
            if (t >= 0.0f && t < DEPTH_INF) {
                all[found].t = t;
                all[found].p = (uint32_t)k;
                ++found;
            }
        }
        qsort(all, found, sizeof(Hit), hit_less);
        const int n = found < CHUNK ? (int)found : CHUNK;
        if (stats) {
            stats[0] += 1;
            stats[1] += (uint32_t)found;
        }
        int stop = 0;
        for (int i = 0; i < n; ++i) {
            const int gi = (int)(all[i].p / 2u);
            if (gi == last) continue;
            dpt = (float)((double)(all[i].t + pdpt) + (pdpt == 0.0f ? 0.0 : STEP_EPS));
            if (stats) stats[3] += 1;
            if ((uint64_t)gi >= s->rays) continue;
            const V3 xyz = v3(fmaf(dpt, d.x, o.x), fmaf(dpt, d.y, o.y), fmaf(dpt, d.z, o.z));
            const float* q = s->rot + 4 * (uint64_t)gi;
            const V3 p = v3(s->means[3 * gi], s->means[3 * gi + 1], s->means[3 * gi + 2]);
            const float* sc = s->scales + 2 * (uint64_t)gi;
            V3 R[3];
            rotation_rows_t(q, R);
            const float tx = dot3(R[0], p), ty = dot3(R[1], p);
            const float u1 = dot3(R[0], xyz) + (-tx), v1 = dot3(R[1], xyz) + (-ty);
            const float uvx = u1 / sc[0], uvy = v1 / sc[1];
            const float rho3d = fmaf(uvy, uvy, uvx * uvx);
            V3 normal = R[2];
            const V3 dir = v3(p.x - campos.x, p.y - campos.y, p.z - campos.z);
            const float cosv = -dot3(dir, normal);
            if (cosv == 0.0f) continue;
            if (!(cosv > 0.0f)) normal = v3(-normal.x, -normal.y, -normal.z);
            float rho2d, cmd;
            if (depth_index == 0 && s->sff) {
                float s2pz = 0.0f, xy[2] = {0.0f, 0.0f};
                const int ok = transmat_xy(p, sc, s->mod, q, s->proj, 3, (int)s->rays, 3.0f, &s2pz, xy);
                rho2d = fmaf(xy[1], xy[1], xy[0] * xy[0]) * 2.0f;
                if (!ok && rho3d > rho2d) continue;
                cmd = rho3d <= rho2d ? dpt : s2pz;
            } else {
                rho2d = rho3d + 1.0f;
                cmd = dpt;
            }
            if (cmd < min_depth) continue;
            const float power = -0.5f * fminf(rho3d, rho2d);
            if (power > 0.0f) continue;
            const float alpha = fminf(0.99f, s->opac[gi] * expf(power));
            if (alpha < 1.0f / 255.0f) continue;
            t_next = t_prev * (1.0f - alpha);
            if (t_next < T_THRESHOLD) { stop = 1; break; }
            if (++contributors > MAX_CONTRIB) { stop = 1; break; }
            if (stats) stats[2] += 1;
            last = gi;
            const float w = alpha * t_prev;
            const V3 col = sh_color(s->degree, s->shs + (uint64_t)gi * s->coeffs * 3, d);
            g->c[0] = fmaf(w, col.x, g->c[0]);
            g->c[1] = fmaf(w, col.y, g->c[1]);
            g->c[2] = fmaf(w, col.z, g->c[2]);
            if (s->others) {
                g->o[0] = fmaf(w, s->others[2 * gi], g->o[0]);
                g->o[1] = fmaf(w, s->others[2 * gi + 1], g->o[1]);
            }
            const float aa = 1.0f - t_prev;
            const float m = far_ratio * (1.0f - NEAR_N / cmd);
            g->dist = fmaf(w, fmaf(-(2.0f * m), g->m1, fmaf(m * m, aa, g->m2)), g->dist);
            g->m1 = fmaf(w, m, g->m1);
            g->m2 = fmaf(w * m, m, g->m2);
            g->d = fmaf(w, cmd, g->d);
            g->n[0] = fmaf(w, normal.x, g->n[0]);
            g->n[1] = fmaf(w, normal.y, g->n[1]);
            g->n[2] = fmaf(w, normal.z, g->n[2]);
            t_prev = t_next;
        }
        if (stop || t_next < T_THRESHOLD || found < CHUNK || contributors > MAX_CONTRIB) break;
        pdpt = dpt;
        const float step = (float)((double)pdpt + STEP_EPS);
        ot = v3(fmaf(step, d.x, o.x), fmaf(step, d.y, o.y), fmaf(step, d.z, o.z));
    }
    for (int ch = 0; ch < 3; ++ch) g->c[ch] = fmaf(t_prev, s->bg[ch], g->c[ch]);
    g->a = 1.0f - t_prev;
    g->t = t_prev;
    g->e = v3(fmaf(g->d, d.x, o.x), fmaf(g->d, d.y, o.y), fmaf(g->d, d.z, o.z));
}

API int oracle_trace_f32(uint64_t rays, const float* ray_o, const float* ray_d, const float* bg, const float* means,
                         const float* shs, uint32_t coeffs, uint32_t degree, const float* others, const float* opac,
                         const float* scales, float mod, const float* rot, const float* proj, const float* campos,
                         const float* vertices, uint64_t vertex_count, const int32_t* triangles, uint64_t tri_count,
                         int start_from_first, int max_depth, float spec_thr, float* out_rgb, float* out_depth,
                         float* out_acc, float* out_normal, float* out_dist, float* out_aux, float* out_mid,
                         const int64_t* ray_ids, uint64_t ray_id_count, uint32_t* stats, int threads) {
    /* ray_ids (optional): trace only these rays (outputs of the others stay
       zero); the scene and the Gaussian arrays are complete either way. */
    float* tri_v = (float*)malloc(sizeof(float) * 9 * (tri_count ? tri_count : 1));
    if (!tri_v) return 1;
    for (uint64_t k = 0; k < tri_count; ++k) {
        for (int c = 0; c < 3; ++c) {
            const int32_t idx = triangles[3 * k + c];
            for (int a = 0; a < 3; ++a)
                tri_v[9 * k + 3 * c + a] = (idx < 0 || (uint64_t)idx >= vertex_count) ? NAN : vertices[3 * (uint64_t)idx + a];
        }
    }
    Scene s = {rays, bg, means, shs, others, opac, scales, rot, proj, campos, coeffs, (int)degree,
               start_from_first, max_depth, mod, spec_thr, tri_v, tri_count};
    memset(out_rgb, 0, sizeof(float) * 3 * rays);
    memset(out_depth, 0, sizeof(float) * rays);
    memset(out_acc, 0, sizeof(float) * rays);
    memset(out_normal, 0, sizeof(float) * 3 * rays);
    memset(out_dist, 0, sizeof(float) * rays);
    memset(out_aux, 0, sizeof(float) * 2 * rays);
    memset(out_mid, 0, sizeof(float) * 32 * rays);
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
    int failed = 0;
#pragma omp parallel
    {
        Hit* all = (Hit*)malloc(sizeof(Hit) * (tri_count ? tri_count : 1));
        if (!all) {
#pragma omp atomic write
            failed = 1;
        } else {
            const int64_t todo = ray_ids ? (int64_t)ray_id_count : (int64_t)rays;
#pragma omp for schedule(dynamic, 4)
            for (int64_t q = 0; q < todo; ++q) {
                const int64_t r = ray_ids ? ray_ids[q] : q;
                if (r < 0 || r >= (int64_t)rays) continue;
                V3 o = v3(ray_o[3 * r], ray_o[3 * r + 1], ray_o[3 * r + 2]);
                V3 d = v3(ray_d[3 * r], ray_d[3 * r + 1], ray_d[3 * r + 2]);
                float rgb[3] = {0.0f, 0.0f, 0.0f}, s_prod = 1.0f;
                for (int i = 0; i < max_depth + 1; ++i) {
                    Seg g;
                    memset(&g, 0, sizeof(g));
                    g.t = 1.0f;
                    const float min_depth = (i == 0 && start_from_first) ? NEAR_N : START_OFFSET_F;
                    trace_segment(&s, o, d, min_depth, i, &g, all, stats ? stats + 4 * r : NULL);
                    if (i == 0) {
                        out_depth[r] = g.d;
                        out_acc[r] = g.a;
                        for (int c = 0; c < 3; ++c) out_normal[3 * r + c] = g.n[c];
                        out_dist[r] = g.dist;
                        out_aux[2 * r] = g.o[0];
                        out_aux[2 * r + 1] = g.o[1];
                    }
                    const float f_this = i == max_depth ? 1.0f : 1.0f - g.o[0];
                    for (int c = 0; c < 3; ++c) rgb[c] = rgb[c] + (g.c[c] * f_this) * s_prod;
                    s_prod = s_prod * g.o[0];
                    float* m = out_mid + 32 * r + 16 * i;
                    m[0] = o.x; m[1] = o.y; m[2] = o.z; m[3] = d.x; m[4] = d.y; m[5] = d.z;
                    m[6] = g.d; m[7] = g.a; m[8] = g.n[0]; m[9] = g.n[1]; m[10] = g.n[2];
                    m[11] = g.o[0]; m[12] = g.o[1]; m[13] = g.c[0]; m[14] = g.c[1]; m[15] = g.c[2];
                    const V3 nn = v3(g.n[0], g.n[1], g.n[2]);
                    if (sqrtf(dot3(nn, nn)) == 0.0f || g.o[0] <= spec_thr) break;
                    const V3 nrm = normalize3(nn);
                    const float k = 2.0f * dot3(nrm, d);
                    d = v3(fmaf(-k, nrm.x, d.x), fmaf(-k, nrm.y, d.y), fmaf(-k, nrm.z, d.z));
                    o = v3(fmaf((float)STEP_EPS, d.x, g.e.x), fmaf((float)STEP_EPS, d.y, g.e.y),
                           fmaf((float)STEP_EPS, d.z, g.e.z));
                }
                for (int c = 0; c < 3; ++c) out_rgb[3 * r + c] = rgb[c];
            }
            free(all);
        }
    }
    free(tri_v);
    return failed;
}
