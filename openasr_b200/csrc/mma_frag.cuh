// mma_frag.cuh -- decode-tile layout constants and mma.sync fragment helpers shared by
// the decode GEMV (mmv_tc.cu) and the fused decoder GEMV (dgemv.cu).
#pragma once

#include "kernels.cuh"

namespace oasr {

constexpr int TILE_ROWS = 16;
constexpr int Q4K_UNIT = 2368;
constexpr int Q80_UNIT = 1088;

static __device__ __forceinline__ void mma_s8_16832(int (&d)[4], int a0, int a1, int a2, int a3, int b0, int b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

static __device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                     uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

static __device__ __forceinline__ int ldg_nc_b32(const void *p) {
    int r;
    asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

static __device__ __forceinline__ int4 ldg_nc_v4(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

static __device__ __forceinline__ int byte_at(int w, int i) { return (w >> (8 * i)) & 0xFF; }

// two equal f16 values from a small non-negative integer
static __device__ __forceinline__ uint32_t dup_h2(int v) {
    const __half h = __int2half_rn(v);
    const uint16_t u = __half_as_ushort(h);
    return (uint32_t)u | ((uint32_t)u << 16);
}

static __device__ __forceinline__ uint32_t i16x2_to_h2(int packed) {
    const __half lo = __int2half_rn((int)(int16_t)(packed & 0xFFFF));
    const __half hi = __int2half_rn((int)(int16_t)((unsigned)packed >> 16));
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

struct Q4kUnit {
    int4 q[4];
    int4 sa, sb;   // rows g, g+8: sc[0..7] | m[0..7]
    int dda, ddb;  // rows g, g+8: fp16 d | fp16 dmin << 16
};

static __device__ __forceinline__ void load_q4k_unit(Q4kUnit &u, const uint8_t *p, int lane, int g) {
#pragma unroll
    for (int i = 0; i < 4; ++i) u.q[i] = ldg_stream(p + i * 512 + lane * 16);
    u.sa = ldg_nc_v4(p + 2048 + 16 * g);
    u.sb = ldg_nc_v4(p + 2048 + 16 * (g + 8));
    u.dda = ldg_nc_b32(p + 2304 + 4 * g);
    u.ddb = ldg_nc_b32(p + 2304 + 4 * (g + 8));
}


struct Q80Unit {
    int4 q[2];
    int dda, ddb;  // rows g, g+8: fp16 d of block 2p | block 2p+1 << 16
};

static __device__ __forceinline__ void load_q80_unit(Q80Unit &u, const uint8_t *p, int lane, int g) {
    u.q[0] = ldg_stream(p + lane * 16);
    u.q[1] = ldg_stream(p + 512 + lane * 16);
    u.dda = ldg_nc_b32(p + 1024 + 4 * g);
    u.ddb = ldg_nc_b32(p + 1024 + 4 * (g + 8));
}

// Activation loads for the B fragments: read-only global (L1) or shared memory.
template <bool SMEM>
static __device__ __forceinline__ int2 act_ld8(const int8_t *p) {
    if (SMEM) return *reinterpret_cast<const int2 *>(p);
    return __ldg(reinterpret_cast<const int2 *>(p));
}
template <bool SMEM>
static __device__ __forceinline__ int act_ld4(const int16_t *p) {
    if (SMEM) return *reinterpret_cast<const int *>(p);
    return __ldg(reinterpret_cast<const int *>(p));
}

// ---- canonical summation order ---------------------------------------------------------
// Every quantized mul_mat output is the sum of its per-block float terms in block order,
// starting from zero:  y = ((0 + t_0) + t_1) + ... + t_{nb-1}.  That is ggml's vec_dot
// loop order and the CPU restatement's, and the tensor-core GEMMs add their per-block
// tiles in the same order, so a result does not depend on the kernel, the warp count or
// the device.  The MMA cores below write each block's terms of a 16-row x 8-column tile to
// shared memory (TERM_FLOATS per block: [lane][4], one float4 per lane) and one warp then
// folds them in block order (fold_terms).  Terms of activation columns >= M are never read.
constexpr int TERM_FLOATS = 32 * 4;
constexpr int TERM_SEG_BLOCKS = 96;  // blocks of terms one segment holds (48 KB)

// One Q4_K unit (16 rows x super-block s) against the 8 activation rows:
//   arow = q8_K quants of activation row g (row base), brow = its 16-wide sums (row base),
//   da0 / da1 = the q8_K scales of activation rows 2t, 2t+1 for super-block s (0 past M).
// C layout: c[0] (row g, act 2t), c[1] (row g, act 2t+1), c[2] (row g+8, 2t), c[3] (row g+8, 2t+1).
// Writes the super-block's term (d_w*d_a)*isum - (dmin_w*d_a)*msum to tb[4 lane + e].
template <bool SMEM>
static __device__ __forceinline__ void q4k_unit_terms(float *tb, const Q4kUnit &u, int s, const int8_t *arow,
                                                      const int16_t *brow, float da0, float da1, int lane, int t) {
    int isum[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int2 blo = act_ld8<SMEM>(arow + 256 * s + 64 * i + 8 * t);
        const int2 bhi = act_ld8<SMEM>(arow + 256 * s + 64 * i + 32 + 8 * t);
        const int4 q = u.q[i];
        int dlo[4], dhi[4];
        // a0 = row g quants 8t..8t+3, a1 = row g+8, a2 = row g quants 8t+4..8t+7, a3 = row g+8
        mma_s8_16832(dlo, q.x & 0x0F0F0F0F, q.z & 0x0F0F0F0F, q.y & 0x0F0F0F0F, q.w & 0x0F0F0F0F, blo.x, blo.y);
        mma_s8_16832(dhi, (q.x >> 4) & 0x0F0F0F0F, (q.z >> 4) & 0x0F0F0F0F, (q.y >> 4) & 0x0F0F0F0F,
                     (q.w >> 4) & 0x0F0F0F0F, bhi.x, bhi.y);
        // sub-blocks 2i (low nibbles) and 2i+1 (high nibbles)
        const int wa = i < 2 ? u.sa.x : u.sa.y, wb = i < 2 ? u.sb.x : u.sb.y;
        const int sh = 2 * (i & 1);
        const int sca0 = byte_at(wa, sh), sca1 = byte_at(wa, sh + 1);
        const int scb0 = byte_at(wb, sh), scb1 = byte_at(wb, sh + 1);
        isum[0] += sca0 * dlo[0] + sca1 * dhi[0];
        isum[1] += sca0 * dlo[1] + sca1 * dhi[1];
        isum[2] += scb0 * dlo[2] + scb1 * dhi[2];
        isum[3] += scb0 * dlo[3] + scb1 * dhi[3];
    }
    // min term: k slots 2t, 2t+1 <-> 16-sums 2t, 2t+1 (sub-block t); slots 8+2t, 9+2t <-> sub-block 4+t
    const uint32_t b0 = i16x2_to_h2(act_ld4<SMEM>(brow + 16 * s + 2 * t));
    const uint32_t b1 = i16x2_to_h2(act_ld4<SMEM>(brow + 16 * s + 8 + 2 * t));
    float msum[4];
    mma_f16_16816(msum, dup_h2(byte_at(u.sa.z, t)), dup_h2(byte_at(u.sb.z, t)), dup_h2(byte_at(u.sa.w, t)),
                  dup_h2(byte_at(u.sb.w, t)), b0, b1);
    const float dwa = h2f((uint16_t)(u.dda & 0xFFFF)), dma = h2f((uint16_t)((unsigned)u.dda >> 16));
    const float dwb = h2f((uint16_t)(u.ddb & 0xFFFF)), dmb = h2f((uint16_t)((unsigned)u.ddb >> 16));
    float4 v;
    v.x = __fsub_rn(__fmul_rn(__fmul_rn(dwa, da0), (float)isum[0]), __fmul_rn(__fmul_rn(dma, da0), msum[0]));
    v.y = __fsub_rn(__fmul_rn(__fmul_rn(dwa, da1), (float)isum[1]), __fmul_rn(__fmul_rn(dma, da1), msum[1]));
    v.z = __fsub_rn(__fmul_rn(__fmul_rn(dwb, da0), (float)isum[2]), __fmul_rn(__fmul_rn(dmb, da0), msum[2]));
    v.w = __fsub_rn(__fmul_rn(__fmul_rn(dwb, da1), (float)isum[3]), __fmul_rn(__fmul_rn(dmb, da1), msum[3]));
    *reinterpret_cast<float4 *>(tb + 4 * lane) = v;
}

// One Q8_0 unit (16 rows x blocks 2p, 2p+1); ad0 / ad1 = q8_0 scale rows of activations 2t, 2t+1
// (null past M).  Writes block 2p's terms (float)isum * (d_w * d_a) to tb[4 lane + e] and block
// 2p+1's to tb[TERM_FLOATS + 4 lane + e].
template <bool SMEM>
static __device__ __forceinline__ void q80_unit_terms(float *tb, const Q80Unit &u, int p, const int8_t *arow,
                                                      const float *ad0, const float *ad1, int lane, int t) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int b = 2 * p + i;
        const int2 bb = act_ld8<SMEM>(arow + 32 * b + 8 * t);
        const int4 q = u.q[i];
        int d[4];
        mma_s8_16832(d, q.x, q.z, q.y, q.w, bb.x, bb.y);
        const float dwa = h2f((uint16_t)(i == 0 ? (u.dda & 0xFFFF) : ((unsigned)u.dda >> 16)));
        const float dwb = h2f((uint16_t)(i == 0 ? (u.ddb & 0xFFFF) : ((unsigned)u.ddb >> 16)));
        const float da0 = ad0 ? (SMEM ? ad0[b] : __ldg(ad0 + b)) : 0.0f;
        const float da1 = ad1 ? (SMEM ? ad1[b] : __ldg(ad1 + b)) : 0.0f;
        float4 v;
        v.x = __fmul_rn((float)d[0], __fmul_rn(dwa, da0));
        v.y = __fmul_rn((float)d[1], __fmul_rn(dwa, da1));
        v.z = __fmul_rn((float)d[2], __fmul_rn(dwb, da0));
        v.w = __fmul_rn((float)d[3], __fmul_rn(dwb, da1));
        *reinterpret_cast<float4 *>(tb + i * TERM_FLOATS + 4 * lane) = v;
    }
}

// acc[e] += t_b[4 lane + e] for b = 0 .. nblk-1, in that order
static __device__ __forceinline__ void fold_terms(float (&acc)[4], const float *terms, int nblk, int lane) {
#pragma unroll 4
    for (int b = 0; b < nblk; ++b) {
        const float4 v = *reinterpret_cast<const float4 *>(terms + b * TERM_FLOATS + 4 * lane);
        acc[0] = __fadd_rn(acc[0], v.x);
        acc[1] = __fadd_rn(acc[1], v.y);
        acc[2] = __fadd_rn(acc[2], v.z);
        acc[3] = __fadd_rn(acc[3], v.w);
    }
}

// Rounds of W units (round j holds units j W .. j W + W - 1, unit j W + w in warp w) are
// written to shared memory SEGJ rounds at a time; after the last round of a segment the CTA
// syncs and warp 0 folds the segment's blocks (units [u0, u1), BPU blocks each) into acc.
// Every warp must call it for the same rounds.
template <int W, int BPU, int SEGJ>
static __device__ __forceinline__ void segment_end(float (&acc)[4], const float *terms, int j, int nrounds,
                                                   int nunits, int warp, int lane) {
    if (j % SEGJ != SEGJ - 1 && j != nrounds - 1) return;
    const int u0 = (j - j % SEGJ) * W, u1 = min(nunits, (j + 1) * W);
    __syncthreads();
    if (warp == 0) fold_terms(acc, terms, (u1 - u0) * BPU, lane);
    __syncthreads();
}

// term slot of unit (round j, warp w) within its segment
template <int W, int BPU, int SEGJ>
static __device__ __forceinline__ float *term_slot(float *terms, int j, int warp) {
    return terms + ((j % SEGJ) * W + warp) * BPU * TERM_FLOATS;
}

// dynamic shared memory of one segment for `nunits` units
template <int W, int BPU, int SEGJ>
static inline size_t term_smem_bytes(int nunits) {
    const int rounds = (nunits + W - 1) / W;
    return (size_t)(rounds < SEGJ ? rounds : SEGJ) * W * BPU * TERM_FLOATS * sizeof(float);
}

}  // namespace oasr
