// Explicitly rounded FP32 arithmetic used by every kernel whose results must
// be bit-identical to the reference backend.
//
// The reference kernels are plain C++ expressions compiled by nvcc with
// --fmad=true, so the compiler decided where a product and a following
// add/sub became one fused multiply-add. Results are reproduced bit-exactly
// here by writing each such expression with explicit __fmul_rn / __fadd_rn /
// __fmaf_rn operations; the fused/unfused form of every expression is a
// "rounding site" with a small numbered choice, pinned by a Rounding policy
// (see flashgs_math.cuh). Explicit *_rn operations are never re-contracted
// by the compiler, whatever --fmad says.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hs {

__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float div(float a, float b) { return __fdiv_rn(a, b); }

// Approximate special-function unit instructions, the same PTX instructions
// the reference issues through inline asm (flashgs preprocess.cu:36-62).
__device__ __forceinline__ float approx_sqrt(float x) {
    float y;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float approx_rsqrt(float x) {
    float y;
    asm("rsqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float approx_lg2(float x) {
    float y;
    asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float ptx_max(float a, float b) {
    float d;
    asm("max.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// a*b + c with rounding choice: 0 fused, 1 product rounded first.
__device__ __forceinline__ float mad(int v, float a, float b, float c) {
    return v == 0 ? fma(a, b, c) : add(mul(a, b), c);
}
// a*b - c: 0 fma(a, b, -c), 1 product rounded first.
__device__ __forceinline__ float msub(int v, float a, float b, float c) {
    return v == 0 ? fma(a, b, -c) : sub(mul(a, b), c);
}
// x - a*b: 0 fma(-a, b, x), 1 product rounded first.
__device__ __forceinline__ float nmad(int v, float x, float a, float b) {
    return v == 0 ? fma(-a, b, x) : sub(x, mul(a, b));
}
// a*b + c*d: 0 fma(a, b, c*d), 1 fma(c, d, a*b), 2 both products rounded.
__device__ __forceinline__ float dot2(int v, float a, float b, float c, float d) {
    if (v == 0) return fma(a, b, mul(c, d));
    if (v == 1) return fma(c, d, mul(a, b));
    return add(mul(a, b), mul(c, d));
}
// a*b - c*d: 0 fma(a, b, -(c*d)), 1 fma(-c, d, a*b), 2 both rounded.
__device__ __forceinline__ float diff2(int v, float a, float b, float c, float d) {
    if (v == 0) return fma(a, b, -mul(c, d));
    if (v == 1) return fma(-c, d, mul(a, b));
    return sub(mul(a, b), mul(c, d));
}
// Packed pairs: the FP32x2 instructions of sm_100 (__ffma2_rn, __fmul2_rn,
// __fadd2_rn) round each component exactly as the scalar instruction does, so
// two independent evaluations of the same expression can issue as one
// instruction per operation. The helpers below mirror mad / msub / dot2 /
// diff2 with the same variant numbers; subtraction is addition of the
// negation, which IEEE arithmetic defines to be the same operation.
__device__ __forceinline__ float2 pair(float x) { return make_float2(x, x); }
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __fadd2_rn(a, neg2(b)); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mad_x2(int v, float2 a, float2 b, float2 c) {
    return v == 0 ? fma2(a, b, c) : add2(mul2(a, b), c);
}
__device__ __forceinline__ float2 nmad_x2(int v, float2 x, float2 a, float2 b) {
    return v == 0 ? fma2(neg2(a), b, x) : sub2(x, mul2(a, b));
}
__device__ __forceinline__ float2 msub_x2(int v, float2 a, float2 b, float2 c) {
    return v == 0 ? fma2(a, b, neg2(c)) : sub2(mul2(a, b), c);
}
__device__ __forceinline__ float2 dot2_x2(int v, float2 a, float2 b, float2 c, float2 d) {
    if (v == 0) return fma2(a, b, mul2(c, d));
    if (v == 1) return fma2(c, d, mul2(a, b));
    return add2(mul2(a, b), mul2(c, d));
}
__device__ __forceinline__ float2 diff2_x2(int v, float2 a, float2 b, float2 c, float2 d) {
    if (v == 0) return fma2(a, b, neg2(mul2(c, d)));
    if (v == 1) return fma2(neg2(c), d, mul2(a, b));
    return sub2(mul2(a, b), mul2(c, d));
}

// (a*b + c*d) + e*f: pair choice as dot2, tail 0 fused, 1 rounded.
__device__ __forceinline__ float dot3(int vp, int vt, float a, float b, float c, float d,
                                      float e, float f) {
    const float s = dot2(vp, a, b, c, d);
    return mad(vt, e, f, s);
}

}  // namespace hs
