// quant_warp.cuh -- warp-level activation quantizers shared by the kernels that emit the
// next mul_mat's input planes themselves (dgemv.cu's quantize prologue, the decode
// attention epilogues in fattn.cu).  Arithmetic as quantize_row_q8_K / quantize_row_q8_0
// (ggml's rounding) and as quant_act.cu.
#pragma once

#include "kernels.cuh"

namespace oasr {

// q8_K of one 256-chunk: lane holds elements 8*lane .. 8*lane+7 (first-max)
static __device__ __forceinline__ void q8k_chunk(const float (&v)[8], int8_t *qdst, float *ddst, int16_t *bdst,
                                                 int lane) {
    float amax = -1.0f, maxv = 0.0f;
    int idx = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (fabsf(v[i]) > amax) { amax = fabsf(v[i]); maxv = v[i]; idx = 8 * lane + i; }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, maxv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oa > amax || (oa == amax && oi < idx)) { amax = oa; maxv = ov; idx = oi; }
    }
    int q[8];
    float d = 0.0f;
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
        d = __frcp_rn(iscale);
    }
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += q[i];
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    uint2 pk;
    pk.x = (uint32_t)(uint8_t)q[0] | (uint32_t)(uint8_t)q[1] << 8 | (uint32_t)(uint8_t)q[2] << 16 |
           (uint32_t)(uint8_t)q[3] << 24;
    pk.y = (uint32_t)(uint8_t)q[4] | (uint32_t)(uint8_t)q[5] << 8 | (uint32_t)(uint8_t)q[6] << 16 |
           (uint32_t)(uint8_t)q[7] << 24;
    *reinterpret_cast<uint2 *>(qdst + 8 * lane) = pk;
    if ((lane & 1) == 0) bdst[lane >> 1] = (int16_t)sum;
    if (lane == 0) *ddst = d;
}

// q8_0 of a 256-chunk as eight 32-blocks: lane holds elements 8*lane .. 8*lane+7,
// block b = lane / 4 (4 lanes per block)
static __device__ __forceinline__ void q80_chunk(const float (&v)[8], int8_t *qdst, float *ddst, int lane) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    uint32_t p0 = 0, p1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        p0 |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[i], id)) << (8 * i);
        p1 |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[4 + i], id)) << (8 * i);
    }
    *reinterpret_cast<uint2 *>(qdst + 8 * lane) = make_uint2(p0, p1);
    if ((lane & 3) == 0) ddst[lane >> 2] = __half2float(__float2half_rn(d));
}

}  // namespace oasr
