// mmv_tc.cu -- decode GEMV (M <= 8 activation rows) on the integer tensor-core path.
//
// The decode mul_mat nodes (GgmlCpuGraphBuilder::mul_mat, cpu_graph.rs:3616-3686)
// stream every weight byte once for at most 8 activation rows.  The dp4a GEMV
// (mmv.cu) spends ~4 instructions per weight byte at M = 8; here one
// mma.sync m16n8k32 (s8 x s8 -> s32) does the 16 x 32 x 8 block dot of one
// 16-row weight tile against all 8 activation rows, so a warp issues a few
// instructions per 16 x 32 weights.  The weights go HBM -> registers -> MMA
// with no shared-memory staging (the work is HBM-bound; tcgen05 would need the
// nibbles unpacked into shared memory or TMEM first).
//
// Weights are read from a "decode tile" copy built at upload (repack kernels
// below).  A tile is 16 weight rows; a unit is one tile x one Q4_K super-block
// (256 k) or one tile x one Q8_0 block pair (64 k), laid out so that each lane
// issues contiguous 16-byte loads that land directly in its MMA A fragment:
//   Q4_K unit (2368 B): qs 4 x 512 B (load i, lane L=(g,t): row g bytes
//     [32i+8t, +8) then row g+8 bytes [32i+8t, +8) of the raw 128-byte quant
//     field) | per row 8 unpacked 6-bit scales + 8 mins (16 B x 16 rows) |
//     per row fp16 d, dmin (4 B x 16 rows)
//   Q8_0 unit (1088 B): qs 2 x 512 B (load i = block 2p+i, lane (g,t): row g
//     bytes [8t, +8) then row g+8 bytes [8t, +8)) | per row fp16 d of both
//     blocks (4 B x 16 rows)
// The MMA k order inside a block is a permutation (lane t holds quants 8t..8t+7
// of the block); the activation B fragment is loaded with the same permutation,
// so every block dot is the exact integer ggml forms.  The per-block float
// terms are then formed exactly as in mmv.cu:
//   Q8_0: acc += (float)isum * (d_w * d_a)
//   Q4_K: acc += (d_w*d_a)*(float)isum - (dmin_w*d_a)*(float)msum
// with isum = sum_j sc_j * dot_j over the 8 sub-blocks (int32) and
// msum = sum_j m_j * bsum_j, the latter from one f16 MMA of the duplicated mins
// against the 16-wide activation sums (|bsum16| <= 2032, products and sums are
// integers below 2^24, so the f32 result is exact).
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

// One CTA per 16-row tile; warp w handles super-blocks w, w + W, ...; the W
// partial tiles are summed in shared memory in warp order.
template <int W>
__global__ void __launch_bounds__(W * 32) mmv_q4k_tc_kernel(const uint8_t *__restrict__ tiles, int nsb, int64_t N,
                                                            int M, const int8_t *__restrict__ aqs,
                                                            const float *__restrict__ ad,
                                                            const int16_t *__restrict__ abs16, int K,
                                                            float *__restrict__ y, int64_t y_ld) {
    __shared__ float red[W > 1 ? W : 1][32][4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *tile = tiles + (int64_t)blockIdx.x * nsb * Q4K_UNIT;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    // weights do not depend on the previous kernel: issue them before the wait
    griddep_launch_dependents();
    Q4kUnit cur, nxt;
    int s = warp;
    if (s < nsb) load_q4k_unit(cur, tile + (int64_t)s * Q4K_UNIT, lane, g);
    griddep_wait();

    const bool gv = g < M;                 // B-fragment activation row
    const int m0 = 2 * t, m1 = 2 * t + 1;  // C-fragment activation rows
    const int8_t *arow = aqs + (int64_t)(gv ? g : 0) * K;
    const int16_t *brow = abs16 + (int64_t)(gv ? g : 0) * (K / 16);
    for (; s < nsb; s += W) {
        const bool more = s + W < nsb;
        if (more) load_q4k_unit(nxt, tile + (int64_t)(s + W) * Q4K_UNIT, lane, g);
        int isum[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int2 blo = make_int2(0, 0), bhi = make_int2(0, 0);
            if (gv) {
                blo = __ldg(reinterpret_cast<const int2 *>(arow + 256 * s + 64 * i + 8 * t));
                bhi = __ldg(reinterpret_cast<const int2 *>(arow + 256 * s + 64 * i + 32 + 8 * t));
            }
            const int4 q = cur.q[i];
            int dlo[4], dhi[4];
            // a0 = row g quants 8t..8t+3, a1 = row g+8, a2 = row g quants 8t+4..8t+7, a3 = row g+8
            mma_s8_16832(dlo, q.x & 0x0F0F0F0F, q.z & 0x0F0F0F0F, q.y & 0x0F0F0F0F, q.w & 0x0F0F0F0F, blo.x, blo.y);
            mma_s8_16832(dhi, (q.x >> 4) & 0x0F0F0F0F, (q.z >> 4) & 0x0F0F0F0F, (q.y >> 4) & 0x0F0F0F0F,
                         (q.w >> 4) & 0x0F0F0F0F, bhi.x, bhi.y);
            // sub-blocks 2i (low nibbles) and 2i+1 (high nibbles)
            const int wa = i < 2 ? cur.sa.x : cur.sa.y, wb = i < 2 ? cur.sb.x : cur.sb.y;
            const int sh = 2 * (i & 1);
            const int sca0 = byte_at(wa, sh), sca1 = byte_at(wa, sh + 1);
            const int scb0 = byte_at(wb, sh), scb1 = byte_at(wb, sh + 1);
            isum[0] += sca0 * dlo[0] + sca1 * dhi[0];
            isum[1] += sca0 * dlo[1] + sca1 * dhi[1];
            isum[2] += scb0 * dlo[2] + scb1 * dhi[2];
            isum[3] += scb0 * dlo[3] + scb1 * dhi[3];
        }
        // min term: k slots 2t, 2t+1 <-> 16-sums 2t, 2t+1 (sub-block t); slots 8+2t, 9+2t <-> sub-block 4+t
        uint32_t b0 = 0, b1 = 0;
        if (gv) {
            b0 = i16x2_to_h2(__ldg(reinterpret_cast<const int *>(brow + 16 * s + 2 * t)));
            b1 = i16x2_to_h2(__ldg(reinterpret_cast<const int *>(brow + 16 * s + 8 + 2 * t)));
        }
        float msum[4];
        mma_f16_16816(msum, dup_h2(byte_at(cur.sa.z, t)), dup_h2(byte_at(cur.sb.z, t)), dup_h2(byte_at(cur.sa.w, t)),
                      dup_h2(byte_at(cur.sb.w, t)), b0, b1);
        const float da0 = m0 < M ? __ldg(ad + (int64_t)m0 * nsb + s) : 0.0f;
        const float da1 = m1 < M ? __ldg(ad + (int64_t)m1 * nsb + s) : 0.0f;
        const float dwa = h2f((uint16_t)(cur.dda & 0xFFFF)), dma = h2f((uint16_t)((unsigned)cur.dda >> 16));
        const float dwb = h2f((uint16_t)(cur.ddb & 0xFFFF)), dmb = h2f((uint16_t)((unsigned)cur.ddb >> 16));
        acc[0] += __fsub_rn(__fmul_rn(__fmul_rn(dwa, da0), (float)isum[0]), __fmul_rn(__fmul_rn(dma, da0), msum[0]));
        acc[1] += __fsub_rn(__fmul_rn(__fmul_rn(dwa, da1), (float)isum[1]), __fmul_rn(__fmul_rn(dma, da1), msum[1]));
        acc[2] += __fsub_rn(__fmul_rn(__fmul_rn(dwb, da0), (float)isum[2]), __fmul_rn(__fmul_rn(dmb, da0), msum[2]));
        acc[3] += __fsub_rn(__fmul_rn(__fmul_rn(dwb, da1), (float)isum[3]), __fmul_rn(__fmul_rn(dmb, da1), msum[3]));
        if (more) cur = nxt;
    }

    if (W > 1) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][lane][e] = acc[e];
        __syncthreads();
        if (warp != 0) return;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float v = red[0][lane][e];
            for (int w2 = 1; w2 < W; ++w2) v += red[w2][lane][e];
            acc[e] = v;
        }
    }
    const int64_t ra = (int64_t)blockIdx.x * TILE_ROWS + g, rb = ra + 8;
    if (m0 < M) {
        if (ra < N) y[(int64_t)m0 * y_ld + ra] = acc[0];
        if (rb < N) y[(int64_t)m0 * y_ld + rb] = acc[2];
    }
    if (m1 < M) {
        if (ra < N) y[(int64_t)m1 * y_ld + ra] = acc[1];
        if (rb < N) y[(int64_t)m1 * y_ld + rb] = acc[3];
    }
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

template <int W>
__global__ void __launch_bounds__(W * 32) mmv_q80_tc_kernel(const uint8_t *__restrict__ tiles, int npairs, int64_t N,
                                                            int M, const int8_t *__restrict__ aqs,
                                                            const float *__restrict__ ad, int K,
                                                            float *__restrict__ y, int64_t y_ld) {
    __shared__ float red[W > 1 ? W : 1][32][4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *tile = tiles + (int64_t)blockIdx.x * npairs * Q80_UNIT;
    const int nb = K / 32;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    griddep_launch_dependents();
    Q80Unit cur, nxt;
    int p = warp;
    if (p < npairs) load_q80_unit(cur, tile + (int64_t)p * Q80_UNIT, lane, g);
    griddep_wait();

    const bool gv = g < M;
    const int m0 = 2 * t, m1 = 2 * t + 1;
    const int8_t *arow = aqs + (int64_t)(gv ? g : 0) * K;
    const float *ad0 = ad + (int64_t)(m0 < M ? m0 : 0) * nb, *ad1 = ad + (int64_t)(m1 < M ? m1 : 0) * nb;
    for (; p < npairs; p += W) {
        const bool more = p + W < npairs;
        if (more) load_q80_unit(nxt, tile + (int64_t)(p + W) * Q80_UNIT, lane, g);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int b = 2 * p + i;
            int2 bb = make_int2(0, 0);
            if (gv) bb = __ldg(reinterpret_cast<const int2 *>(arow + 32 * b + 8 * t));
            const int4 q = cur.q[i];
            int d[4];
            mma_s8_16832(d, q.x, q.z, q.y, q.w, bb.x, bb.y);
            const float dwa = h2f((uint16_t)(i == 0 ? (cur.dda & 0xFFFF) : ((unsigned)cur.dda >> 16)));
            const float dwb = h2f((uint16_t)(i == 0 ? (cur.ddb & 0xFFFF) : ((unsigned)cur.ddb >> 16)));
            const float da0 = m0 < M ? __ldg(ad0 + b) : 0.0f;
            const float da1 = m1 < M ? __ldg(ad1 + b) : 0.0f;
            acc[0] += __fmul_rn((float)d[0], __fmul_rn(dwa, da0));
            acc[1] += __fmul_rn((float)d[1], __fmul_rn(dwa, da1));
            acc[2] += __fmul_rn((float)d[2], __fmul_rn(dwb, da0));
            acc[3] += __fmul_rn((float)d[3], __fmul_rn(dwb, da1));
        }
        if (more) cur = nxt;
    }

    if (W > 1) {
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][lane][e] = acc[e];
        __syncthreads();
        if (warp != 0) return;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float v = red[0][lane][e];
            for (int w2 = 1; w2 < W; ++w2) v += red[w2][lane][e];
            acc[e] = v;
        }
    }
    const int64_t ra = (int64_t)blockIdx.x * TILE_ROWS + g, rb = ra + 8;
    if (m0 < M) {
        if (ra < N) y[(int64_t)m0 * y_ld + ra] = acc[0];
        if (rb < N) y[(int64_t)m0 * y_ld + rb] = acc[2];
    }
    if (m1 < M) {
        if (ra < N) y[(int64_t)m1 * y_ld + ra] = acc[1];
        if (rb < N) y[(int64_t)m1 * y_ld + rb] = acc[3];
    }
}

// ---- decode-tile repack (runs once at upload) --------------------------------------------
// get_scale_min_k4 on the 12 packed bytes (layout: gguf/quants.py Q4_K.get_scale_min)
static __device__ __forceinline__ void unpack_scale_min(const uint8_t *s, int j, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// one warp per unit (tile T, super-block s); raw rows are 16-byte aligned ggml Q4_K blocks
__global__ void repack_q4k_tiles_kernel(const uint8_t *__restrict__ raw, int64_t N, int nsb, int64_t row_bytes,
                                        int64_t n_units, uint8_t *__restrict__ tiles) {
    const int lane = threadIdx.x & 31;
    const int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (unit >= n_units) return;
    const int64_t T = unit / nsb;
    const int s = (int)(unit - T * nsb);
    const int g = lane >> 2, t = lane & 3;
    uint8_t *u = tiles + unit * Q4K_UNIT;
    const int64_t ra = T * TILE_ROWS + g, rb = ra + 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint2 a = make_uint2(0, 0), b = make_uint2(0, 0);
        if (ra < N) a = *reinterpret_cast<const uint2 *>(raw + ra * row_bytes + (int64_t)s * 144 + 16 + 32 * i + 8 * t);
        if (rb < N) b = *reinterpret_cast<const uint2 *>(raw + rb * row_bytes + (int64_t)s * 144 + 16 + 32 * i + 8 * t);
        *reinterpret_cast<uint4 *>(u + i * 512 + lane * 16) = make_uint4(a.x, a.y, b.x, b.y);
    }
    if (lane < TILE_ROWS) {
        const int64_t r = T * TILE_ROWS + lane;
        uint8_t scm[16];
        uint32_t dd = 0;
        if (r < N) {
            const uint8_t *blk = raw + r * row_bytes + (int64_t)s * 144;
            for (int j = 0; j < 8; ++j) {
                int sc, m;
                unpack_scale_min(blk + 4, j, sc, m);
                scm[j] = (uint8_t)sc;
                scm[8 + j] = (uint8_t)m;
            }
            dd = *reinterpret_cast<const uint32_t *>(blk);
        } else {
            for (int j = 0; j < 16; ++j) scm[j] = 0;
        }
        uint4 v;
        memcpy(&v, scm, 16);
        *reinterpret_cast<uint4 *>(u + 2048 + 16 * lane) = v;
        *reinterpret_cast<uint32_t *>(u + 2304 + 4 * lane) = dd;
    }
}

// from the repacked Q8_0 planes: qs [N][K] int8, d [N][K/32] fp16
__global__ void repack_q80_tiles_kernel(const uint8_t *__restrict__ qs, const uint16_t *__restrict__ d, int64_t N,
                                        int K, int npairs, int64_t n_units, uint8_t *__restrict__ tiles) {
    const int lane = threadIdx.x & 31;
    const int64_t unit = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (unit >= n_units) return;
    const int64_t T = unit / npairs;
    const int p = (int)(unit - T * npairs);
    const int g = lane >> 2, t = lane & 3;
    uint8_t *u = tiles + unit * Q80_UNIT;
    const int64_t ra = T * TILE_ROWS + g, rb = ra + 8;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t k0 = (int64_t)(2 * p + i) * 32 + 8 * t;
        uint2 a = make_uint2(0, 0), b = make_uint2(0, 0);
        if (ra < N) a = *reinterpret_cast<const uint2 *>(qs + ra * K + k0);
        if (rb < N) b = *reinterpret_cast<const uint2 *>(qs + rb * K + k0);
        *reinterpret_cast<uint4 *>(u + i * 512 + lane * 16) = make_uint4(a.x, a.y, b.x, b.y);
    }
    if (lane < TILE_ROWS) {
        const int64_t r = T * TILE_ROWS + lane;
        uint32_t v = 0;
        if (r < N) v = (uint32_t)d[r * (K / 32) + 2 * p] | ((uint32_t)d[r * (K / 32) + 2 * p + 1] << 16);
        *reinterpret_cast<uint32_t *>(u + 1024 + 4 * lane) = v;
    }
}

bool mmv_tiles_supported(int type, int64_t K) {
    if (type == OASR_TYPE_Q4_K) return K % 256 == 0;
    if (type == OASR_TYPE_Q8_0) return K % 64 == 0;
    return false;
}

size_t mmv_tiles_bytes(int type, int64_t N, int64_t K, int64_t slices) {
    const int64_t ntiles = (N + TILE_ROWS - 1) / TILE_ROWS;
    if (type == OASR_TYPE_Q4_K) return (size_t)(slices * ntiles * (K / 256) * Q4K_UNIT);
    return (size_t)(slices * ntiles * (K / 64) * Q80_UNIT);
}

cudaError_t build_mmv_tiles(oasr_weight *w, cudaStream_t st) {
    const int64_t N = w->ne[1], K = w->ne[0], slices = w->ne[2] * w->ne[3];
    const int64_t ntiles = (N + TILE_ROWS - 1) / TILE_ROWS;
    const size_t per_slice = mmv_tiles_bytes(w->type, N, K, 1);
    for (int64_t sl = 0; sl < slices; ++sl) {
        uint8_t *dst = w->tiles + sl * per_slice;
        if (w->type == OASR_TYPE_Q4_K) {
            const int nsb = (int)(K / 256);
            const int64_t units = ntiles * nsb;
            repack_q4k_tiles_kernel<<<(unsigned)((units + 7) / 8), 256, 0, st>>>(
                w->qs + sl * N * w->qs_row_bytes, N, nsb, w->qs_row_bytes, units, dst);
        } else {
            const int npairs = (int)(K / 64);
            const int64_t units = ntiles * npairs;
            repack_q80_tiles_kernel<<<(unsigned)((units + 7) / 8), 256, 0, st>>>(
                w->qs + sl * N * w->qs_row_bytes, w->d + sl * N * w->d_row_elems, N, (int)K, npairs, units, dst);
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---- launcher -------------------------------------------------------------------------
// Warps per CTA: one per unit of a tile up to 8 (Q4_K: K <= 2048 gives one super-block
// per warp); larger K loops with the next unit's loads issued ahead.
template <int W>
static cudaError_t launch_q4k_w(oasr_backend *be, const uint8_t *tiles, int nsb, int64_t N, int M, const ActPlanes &a,
                                int K, float *y, int64_t y_ld) {
    const unsigned grid = (unsigned)((N + TILE_ROWS - 1) / TILE_ROWS);
    return launch_k(be, mmv_q4k_tc_kernel<W>, dim3(grid), dim3(W * 32), 0, tiles, nsb, N, M, (const int8_t *)a.qs,
                    (const float *)a.d, (const int16_t *)a.bs16, K, y, y_ld);
}

template <int W>
static cudaError_t launch_q80_w(oasr_backend *be, const uint8_t *tiles, int npairs, int64_t N, int M,
                                const ActPlanes &a, int K, float *y, int64_t y_ld) {
    const unsigned grid = (unsigned)((N + TILE_ROWS - 1) / TILE_ROWS);
    return launch_k(be, mmv_q80_tc_kernel<W>, dim3(grid), dim3(W * 32), 0, tiles, npairs, N, M, (const int8_t *)a.qs,
                    (const float *)a.d, K, y, y_ld);
}

int launch_mmv_tc(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int M, int K, float *y,
                  int64_t y_ld) {
    const int64_t N = w->ne[1];
    const uint8_t *tiles = w->tiles + slice * mmv_tiles_bytes(w->type, N, K, 1);
    cudaError_t e;
    if (w->type == OASR_TYPE_Q4_K) {
        const int nsb = K / 256;
        if (nsb <= 1) e = launch_q4k_w<1>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 2) e = launch_q4k_w<2>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 4) e = launch_q4k_w<4>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else if (nsb <= 5) e = launch_q4k_w<5>(be, tiles, nsb, N, M, a, K, y, y_ld);
        else e = launch_q4k_w<8>(be, tiles, nsb, N, M, a, K, y, y_ld);
    } else {
        const int npairs = K / 64;
        // long rows (e.g. the logits head) keep 4 warps per tile, each looping over ~5 units
        if (npairs <= 4) e = launch_q80_w<2>(be, tiles, npairs, N, M, a, K, y, y_ld);
        else e = launch_q80_w<4>(be, tiles, npairs, N, M, a, K, y, y_ld);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "mmv_tc launch", __LINE__);
    return oasr_internal_launch_check(be, "mmv_tc");
}

}  // namespace oasr
