// 2DGS splat arithmetic shared by the FlashGS and standard backends.
//
// Both reference backends build the same 2DGS ray-splat transform from a
// quaternion, two scales and the projection (quat_to_rotmat, scale_to_mat,
// compute_transmat: vendor/flashgs/cuda_rasterizer/preprocess.cu:246-362 and
// vendor/standard_rasterizer/auxiliary.h:231-310 + forward.cu:75-115), with
// GLM products expanded in the vendored GLM's order
// (glm/detail/type_mat3x3.inl:486-519, type_mat4x3.inl:506-563).
//
// Rounding sites: every expression whose fused/unfused form the reference
// left to the compiler is a numbered site (Site). A Rounding policy `r` maps
// a site to the variant index of the fp.cuh helper that evaluates it. Each
// backend has its own pinned policy because the reference compiles the two
// backends with different optimisation flags.
#pragma once

#include "fp.cuh"

namespace hs {

enum Site : int {
    // projection and EWA covariance (FlashGS)
    S_PVIEW_PAIR = 0,  // p_view rows: m0*x + m4*y   (dot2)
    S_PVIEW_TAIL,      //   + m8*z                   (mad); + m12 is a plain add
    S_PHOM_PAIR,       // p_hom rows (projection), pair
    S_PHOM_TAIL,       //   tail
    S_WJ_TAIL,         // T = W*J: W2r*J[c][2] onto the rounded W0r*J00 / W1r*J11
    S_M1_PAIR,         // (T^T * Vrk) 3-term dots, pair
    S_M1_TAIL,         //   tail
    S_COV_PAIR,        // (T^T Vrk) * T 3-term dots, pair
    S_COV_TAIL,        //   tail
    S_DET,             // cov.x*cov.z - cov.y*cov.y   (diff2)
    S_POWER,           // ln2*8 + ln2*log2(opacity)   (mad)
    S_EXTENT,          // 1.414214*sqrt(cov*power) + 1
    // 2DGS transform (both backends)
    S_QN_PAIR,         // quaternion w*w + x*x
    S_QN_TAIL,         //   + y*y, + z*z
    S_R00,             // rotation entry [col 0][row 0]: 1 - 2(y*y + z*z)   (dot2)
    S_R01,             //   [0][1]: 2(x*y + w*z)                           (dot2)
    S_R02,             //   [0][2]: 2(x*z - w*y)                           (diff2)
    S_R10,             //   [1][0]: 2(x*y - w*z)                           (diff2)
    S_R11,             //   [1][1]: 1 - 2(x*x + z*z)                       (dot2)
    S_R12,             //   [1][2]: 2(y*z + w*x)                           (dot2)
    S_R20,             //   [2][0]: 2(x*z + w*y)                           (dot2)
    S_R21,             //   [2][1]: 2(y*z - w*x)                           (diff2)
    S_R22,             //   [2][2]: 1 - 2(x*x + y*y)                       (dot2)
    S_B0_PAIR,         // splat2world^T * world2ndc row 0 (L0 column), pair
    S_B0_TAIL,         //   third term
    S_B1_PAIR,         // row 1 (L1 column)
    S_B1_TAIL,
    S_B2_PAIR,         // row 2 (centre)
    S_B2_TAIL,
    S_TN_U,            // Tu = B0*W/2 + B3*(W-1)/2: fused tail
    S_TN_V,            // Tv = B1*H/2 + B3*(H-1)/2: fused tail
    S_NRM_PAIR,        // camera-space normal, pair
    S_NRM_TAIL,        //   tail
    S_COS_PAIR,        // p_view . normal, pair
    S_COS_TAIL,        //   tail
    // tile / ellipse test (FlashGS)
    S_EL_C,            // conic*dx*dx - w   (msub)
    S_EL_DELTA,        // b*b - 4a*c        (diff2)
    S_EL_T,            // (l-d)*2a + b      (mad)
    // degree-3 SH (FlashGS)
    S_SH_L2_PAIR,      // |p - campos|^2 pair
    S_SH_L2_TAIL,      //   tail
    S_SH_DC,           // C0*sh0 + 0.5
    S_SH_ACC,          // result +- s*sh accumulation steps
    S_SH_P6A,          // 2zz - xx        (0: rounded xx, 1: fused x*x)
    S_SH_P6B,          //   ... - yy      (0: fused y*y, 1: rounded yy)
    S_SH_P8,           // xx - yy         (diff2 on x,x,y,y)
    S_SH_P9,           // 3xx - yy        (diff2 on 3,xx,y,y)
    S_SH_P11A,         // 4zz - xx        (as P6A)
    S_SH_P11B,         //   ... - yy      (as P6B)
    S_SH_P12A,         // 2zz - 3xx       (diff2 on 2,zz,3,xx)
    S_SH_P12B,         //   ... - 3yy     (0: fused 3*yy, 1: rounded)
    S_SH_P15,          // xx - 3yy        (diff2 on x,x,3,yy)
    // screen-space bounding box (standard)
    S_AABB_D_PAIR,     // 9*Tw.x^2 + 9*Tw.y^2
    S_AABB_D_TAIL,     //   - Tw.z^2          (0: fused Tw.z*Tw.z, 1: rounded square)
    S_AABB_PX_PAIR,    // f . (Tu*Tw), pair (centre x)
    S_AABB_PY_PAIR,    // f . (Tv*Tw), pair (centre y)
    S_AABB_P_TAIL,     //   tail
    S_AABB_QX_PAIR,    // f . (Tu*Tu), pair (extent x)
    S_AABB_QY_PAIR,    // f . (Tv*Tv), pair (extent y)
    S_AABB_Q_TAIL,     //   tail
    S_AABB_H,          // p*p - q            (0: fused, 1: rounded square)
    // per-pixel blend (both backends)
    S_K,               // pix*Tw - Tu     (msub)
    S_CROSS,           // cross product components (diff2)
    S_RHO3,            // s.x*s.x + s.y*s.y
    S_RHO2,            // d.x*d.x + d.y*d.y
    S_DEPTH,           // s.x*Tw.x + s.y*Tw.y
    S_ACC,             // accumulator += value * w
    S_T,               // FlashGS T -= alpha*T   (0: fma(-alpha,T,T), 1: T - w)
    S_D1,              // m*m*A + M2
    S_D2,              //   ... - 2m*M1
    S_OUT,             // C + T*bg
    S_COUNT
};

// render.cu:7-10 and auxiliary.h:55-58
constexpr float kNear = 0.2f;
constexpr float kFar = 100.0f;

// transformPoint4x3 / transformPoint4x4 row i of a column-major matrix:
// m[i]*x + m[4+i]*y + m[8+i]*z + m[12+i]
template <class R>
__device__ __forceinline__ float affine_row(const R& r, int pair_site, int tail_site,
                                            const float* m, int i, float x, float y, float z) {
    return add(dot3(r(pair_site), r(tail_site), m[i], x, m[4 + i], y, m[8 + i], z), m[12 + i]);
}

// quat_to_rotmat + scale_to_mat + compute_transmat + the camera-space
// normal. rot = (x, y, z, w) of the glm::vec4 read from the [P,4] buffer;
// view/proj are column-major 4x4. Outputs T's three columns (tu, tv, tw)
// and view3x3 * R[:,2] (before the facing flip).
template <class R>
__device__ __forceinline__ void splat_transform(const R& r, const float* view, const float* proj,
                                                float3 p, float2 scale, float scale_modifier,
                                                float4 rot, int width, int height, float3& tu,
                                                float3& tv, float3& tw, float3& normal) {
    // s = rsqrt(w*w + x*x + y*y + z*z) in that order of the glm::vec4 fields.
    const float qn = mad(r(S_QN_TAIL), rot.z, rot.z,
                         mad(r(S_QN_TAIL), rot.y, rot.y,
                             dot2(r(S_QN_PAIR), rot.w, rot.w, rot.x, rot.x)));
    const float s = rsqrtf(qn);  // approximate reciprocal square root, as the reference
    const float qw = mul(rot.x, s), qx = mul(rot.y, s), qy = mul(rot.z, s), qz = mul(rot.w, s);
    float rm[3][3];  // rm[column][row]
    rm[0][0] = sub(1.0f, mul(2.0f, dot2(r(S_R00), qy, qy, qz, qz)));
    rm[0][1] = mul(2.0f, dot2(r(S_R01), qx, qy, qw, qz));
    rm[0][2] = mul(2.0f, diff2(r(S_R02), qx, qz, qw, qy));
    rm[1][0] = mul(2.0f, diff2(r(S_R10), qx, qy, qw, qz));
    rm[1][1] = sub(1.0f, mul(2.0f, dot2(r(S_R11), qx, qx, qz, qz)));
    rm[1][2] = mul(2.0f, dot2(r(S_R12), qy, qz, qw, qx));
    rm[2][0] = mul(2.0f, dot2(r(S_R20), qx, qz, qw, qy));
    rm[2][1] = mul(2.0f, diff2(r(S_R21), qy, qz, qw, qx));
    rm[2][2] = sub(1.0f, mul(2.0f, dot2(r(S_R22), qx, qx, qy, qy)));
    // L = R * diag(mod*sx, mod*sy, 1). GLM forms every product of the matrix
    // products below, including those with the structural zeros of S,
    // splat2world and ndc2pix. Such a product is a signed zero (NaN for an
    // infinite factor): it leaves a non-zero sum unchanged but decides the
    // sign of a zero one, so each is added here too (in any order: a sum of
    // zeros is -0 exactly when every term is).
    const float s0 = mul(scale_modifier, scale.x), s1 = mul(scale_modifier, scale.y);
    float zr[3][3];
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int i = 0; i < 3; ++i) zr[c][i] = mul(rm[c][i], 0.0f);
    float l0[3], l1[3], l2[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        l0[i] = add(add(mul(rm[0][i], s0), zr[1][i]), zr[2][i]);
        l1[i] = add(add(zr[0][i], mul(rm[1][i], s1)), zr[2][i]);
        l2[i] = add(add(zr[0][i], zr[1][i]), rm[2][i]);
    }
    // B = splat2world^T * world2ndc, world2ndc[c][k] = proj[4k + c]:
    // B[c][i] = A[0][i]*proj[c] + A[1][i]*proj[4+c] + A[2][i]*proj[8+c] + A[3][i]*proj[12+c]
    // with A[.][0] = L0, A[.][1] = L1, A[.][2] = p and A[3] = (0, 0, 1).
    float b[4][3];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float zp = mul(0.0f, proj[12 + c]);  // A[3][0] = A[3][1] = +0
        b[c][0] = add(dot3(r(S_B0_PAIR), r(S_B0_TAIL), l0[0], proj[c], l0[1], proj[4 + c], l0[2],
                           proj[8 + c]),
                      zp);
        b[c][1] = add(dot3(r(S_B1_PAIR), r(S_B1_TAIL), l1[0], proj[c], l1[1], proj[4 + c], l1[2],
                           proj[8 + c]),
                      zp);
        b[c][2] = add(dot3(r(S_B2_PAIR), r(S_B2_TAIL), p.x, proj[c], p.y, proj[4 + c], p.z,
                           proj[8 + c]),
                      proj[12 + c]);
    }
    // T = B * ndc2pix, ndc2pix columns (W/2,0,0,(W-1)/2), (0,H/2,0,(H-1)/2), (0,0,0,1).
    const float w2 = static_cast<float>(width) * 0.5f, wm = static_cast<float>(width - 1) * 0.5f;
    const float h2 = static_cast<float>(height) * 0.5f, hm = static_cast<float>(height - 1) * 0.5f;
    float zb[3][3];
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int i = 0; i < 3; ++i) zb[c][i] = mul(b[c][i], 0.0f);
    float t[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        t[0][i] = add(mad(r(S_TN_U), b[3][i], wm, mul(b[0][i], w2)), add(zb[1][i], zb[2][i]));
        t[1][i] = add(mad(r(S_TN_V), b[3][i], hm, mul(b[1][i], h2)), add(zb[0][i], zb[2][i]));
        t[2][i] = add(b[3][i], add(add(zb[0][i], zb[1][i]), zb[2][i]));
    }
    tu = make_float3(t[0][0], t[0][1], t[0][2]);
    tv = make_float3(t[1][0], t[1][1], t[1][2]);
    tw = make_float3(t[2][0], t[2][1], t[2][2]);
    // normal = view3x3 * L[2] (transformVec4x3).
    normal.x = dot3(r(S_NRM_PAIR), r(S_NRM_TAIL), view[0], l2[0], view[4], l2[1], view[8], l2[2]);
    normal.y = dot3(r(S_NRM_PAIR), r(S_NRM_TAIL), view[1], l2[0], view[5], l2[1], view[9], l2[2]);
    normal.z = dot3(r(S_NRM_PAIR), r(S_NRM_TAIL), view[2], l2[0], view[6], l2[1], view[10], l2[2]);
}

}  // namespace hs
