// fmath.cuh -- the exponential of the decode path (softmax weights in the decode
// attentions and their split merges, SiLU in the SwiGLU kernels).
//
// A greedy transcript is bit-identical to the CPU restatement only if every f32
// operation of a decode step rounds the same way on both sides.  CUDA's expf and
// a C library's expf are both faithful but not identical, so the decode path uses
// this function instead, and the CPU restatement carries the same algorithm
// written in C.  Method: Cody & Waite argument reduction x = n ln2 + r with ln2
// split into a 16-bit head and a tail (fdlibm's float split), |r| <= ln2 / 2, then
// the degree-7 Taylor polynomial of e^r in Horner form with fused multiply-adds
// (truncation error r^8 / 8! < 6e-9, far below one f32 ulp), and the result
// scaled by 2^n through the exponent bits (two steps below 2^-126, so a
// subnormal result rounds once).  Accuracy: within 2 ulp of exp over the f32
// range; exp(-inf) = 0, exp(+inf) = inf, exp(NaN) = NaN.
#pragma once

#include <cuda_runtime.h>
#include <math.h>

namespace oasr {

static __device__ __forceinline__ float pow2i(int k) {  // 2^k for -126 <= k <= 127
    return __int_as_float((k + 127) << 23);
}

static __device__ __forceinline__ float exp_f32(float x) {
    if (!(x == x)) return x;                 // NaN
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;  // below half the smallest subnormal (and -inf)
    const float t = rintf(__fmul_rn(x, 1.44269502162933349609375f));  // n = rint(x log2 e)
    float r = __fmaf_rn(-t, 0.693145751953125f, x);                     // x - n ln2_hi (exact)
    r = __fmaf_rn(-t, 1.428606765330187045e-06f, r);                    // - n ln2_lo
    float p = 1.9841270113e-04f;                                        // 1/7!
    p = __fmaf_rn(p, r, 1.3888889225e-03f);                             // 1/6!
    p = __fmaf_rn(p, r, 8.3333337680e-03f);                             // 1/5!
    p = __fmaf_rn(p, r, 4.1666667908e-02f);                             // 1/4!
    p = __fmaf_rn(p, r, 1.6666667163e-01f);                             // 1/3!
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int n = (int)t;
    if (n > 127) return __fmul_rn(__fmul_rn(p, pow2i(127)), 2.0f);
    if (n < -126) return __fmul_rn(__fmul_rn(p, pow2i(n + 64)), pow2i(-64));
    return __fmul_rn(p, pow2i(n));
}

}  // namespace oasr
