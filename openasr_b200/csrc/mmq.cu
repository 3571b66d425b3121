// mmq.cu -- K2: quantized GEMM for M > 8 activation rows (encoder, prefill).
//
// Q4_K weights run on the 5th-generation tensor cores (tcgen05, accumulators
// in TMEM) with ggml's exact per-super-block arithmetic:
//   ggml CPU (vec_dot_q4_K_q8_K) forms, per 256-element super-block,
//     isum = sum_j sc_j * <q4_j, q8_j>          (integers)
//     msum = sum_j m_j * bsum32_j               (integers)
//     term = (d_w*d_a)*isum - (dmin_w*d_a)*msum (f32)
//   Here the 6-bit sub-scales are folded into the weight operand (sc*q <= 945,
//   exact in fp16) and the q8_K activations are fp16 integers, so one
//   tcgen05.mma.kind::f16 chain over the super-block yields isum exactly in
//   the f32 accumulator; a second K=16 MMA of the 16-wide activation sums
//   against the duplicated mins yields msum.  The epilogue forms `term` with
//   the same roundings as ggml and adds the super-blocks in order, so the
//   result equals the CPU oracle's bit for bit.
//
// CTA = 128 activation rows x 128 weight rows, 14 warps:
//   warp 0      TMA producer of the activation tiles (128 x 64 fp16, SW128)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-5   weight transform: raw Q4_K blocks -> fp16 sc*q in the SW128
//               K-major layout, plus the per-super-block min tiles
//   warps 6-13  epilogue: TMEM -> registers, per-super-block scaling
// TMEM: two accumulator sets (isum 128 cols + msum 128 cols) so the epilogue
// of super-block s overlaps the MMAs of s+1.  Every mbarrier wait is bounded.
//
// Q8_0 runs on tcgen05 kind::i8 (mmq_q80_tc_kernel below); Q4_0 still uses the
// K1 GEMV kernel over groups of 8 rows.
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace oasr {

namespace q4k {
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int STAGES = 3;
constexpr int WSTAGES = 3;       // raw Q4_K super-block ring
constexpr int TILE = 128 * 128;  // bytes of one 128-row x 128-byte operand tile
constexpr int WTILE = 128 * 144; // 128 weight rows x one raw super-block (18 KB)
constexpr int NTHREADS = 448;
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * TILE;
constexpr int OFF_AMIN = OFF_B + STAGES * TILE;
constexpr int OFF_BMIN = OFF_AMIN + 2 * TILE;
constexpr int OFF_W = OFF_BMIN + 2 * TILE;
constexpr int OFF_BAR = OFF_W + WSTAGES * WTILE;
constexpr int NBAR = 3 * STAGES + 9 + 2 * WSTAGES;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
}  // namespace q4k

static __device__ __forceinline__ int q4k_byte(const int4 &h, int i) {
    const int w = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (w >> (8 * (i & 3))) & 0xFF;
}
static __device__ __forceinline__ void q4k_scale_min(const int4 &h, int j, int &sc, int &m) {
    if (j < 4) {
        sc = q4k_byte(h, j) & 63;
        m = q4k_byte(h, j + 4) & 63;
    } else {
        sc = (q4k_byte(h, j + 4) & 0xF) | ((q4k_byte(h, j - 4) >> 6) << 4);
        m = (q4k_byte(h, j + 4) >> 4) | ((q4k_byte(h, j) >> 6) << 4);
    }
}

// two nibble-sized values -> fp16 pair: v | 0x6400 is the half 1024 + v (v < 1024), minus 1024
static __device__ __forceinline__ uint32_t u16x2_to_h2(uint32_t v2) {
    const uint32_t x = v2 | 0x64006400u;
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&x), __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
    return *reinterpret_cast<const uint32_t *>(&r);
}

// 8 consecutive K elements sc*nibble from 8 qs bytes (words w0, w1), low (sh=0) or high (sh=4) nibbles
static __device__ __forceinline__ int4 q4k_chunk_f16(uint32_t w0, uint32_t w1, int sh, uint32_t sc) {
    const uint32_t n0 = (w0 >> sh) & 0x0F0F0F0Fu, n1 = (w1 >> sh) & 0x0F0F0F0Fu;
    int4 r;
    r.x = (int)u16x2_to_h2(__byte_perm(n0, 0, 0x4140) * sc);
    r.y = (int)u16x2_to_h2(__byte_perm(n0, 0, 0x4342) * sc);
    r.z = (int)u16x2_to_h2(__byte_perm(n1, 0, 0x4140) * sc);
    r.w = (int)u16x2_to_h2(__byte_perm(n1, 0, 0x4342) * sc);
    return r;
}

__global__ void __launch_bounds__(448, 1)
    mmq_q4k_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                      int N, const __half *__restrict__ bs16h, const float *__restrict__ ad, int M, int K,
                      float *__restrict__ y, int64_t y_ld, int *err) {
    using namespace q4k;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + OFF_BAR);
    uint64_t *full_a = bars;
    uint64_t *full_b = bars + STAGES;
    uint64_t *empty = bars + 2 * STAGES;
    uint64_t *full_min = bars + 3 * STAGES;
    uint64_t *empty_min = full_min + 2;
    uint64_t *tmem_full = empty_min + 2;
    uint64_t *tmem_empty = tmem_full + 2;
    uint64_t *done = tmem_empty + 2;
    uint64_t *full_w = done + 1;
    uint64_t *empty_w = full_w + WSTAGES;
    uint32_t *tmem_slot = (uint32_t *)(smem + OFF_MISC);
    volatile int *abort_flag = (volatile int *)(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nkc = K / BK, nsb = K / 256;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full_a[i], 1);
            mbar_init(&full_b[i], 128);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full_min[i], 128);
            mbar_init(&empty_min[i], 1);
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], 256);
        }
        for (int i = 0; i < WSTAGES; ++i) {
            mbar_init(&full_w[i], 1);
            mbar_init(&empty_w[i], 128 + 256);  // transform + epilogue release a raw super-block
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // TMA producer: raw weight super-blocks (ring of WSTAGES) and activation tiles (ring of STAGES)
            int issued_a = 0, issued_w = 0;
            for (int kc = 0; kc < nkc; ++kc) {
                const int sb = kc >> 2;
                if ((kc & 3) == 0) {
                    const int wb = sb % WSTAGES;
                    if (!mbar_wait(&empty_w[wb], ((sb / WSTAGES) & 1) ^ 1, abort_flag, err)) break;
                    mbar_arrive_expect_tx(&full_w[wb], WTILE);
                    tma_load_2d(smem + OFF_W + wb * WTILE, &tmap_w, &full_w[wb], sb * 144, n0);
                    issued_w = sb + 1;
                }
                const int s = kc % STAGES;
                if (!mbar_wait(&empty[s], ((kc / STAGES) & 1) ^ 1, abort_flag, err)) break;
                mbar_arrive_expect_tx(&full_a[s], TILE);
                tma_load_2d(smem + OFF_A + s * TILE, &tmap_a, &full_a[s], kc * BK, m0);
                issued_a = kc + 1;
            }
            // no TMA write may still be in flight when the CTA exits
            for (int kc = max(0, issued_a - STAGES); kc < issued_a; ++kc) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&full_a[kc % STAGES], (kc / STAGES) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
            for (int sb = max(0, issued_w - WSTAGES); sb < issued_w; ++sb) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&full_w[sb % WSTAGES], (sb / WSTAGES) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
            bool ok = true;
            for (int sb = 0; sb < nsb && ok; ++sb) {
                const int ab = sb & 1;
                const uint32_t aph = (sb >> 1) & 1;
                if (!mbar_wait(&tmem_empty[ab], aph ^ 1, abort_flag, err)) break;
                tc_fence_after();
                const uint32_t d_isum = tmem + ab * 256, d_msum = tmem + ab * 256 + 128;
                for (int c = 0; c < 4 && ok; ++c) {
                    const int kc = sb * 4 + c, s = kc % STAGES;
                    const uint32_t ph = (kc / STAGES) & 1;
                    if (!mbar_wait(&full_a[s], ph, abort_flag, err) || !mbar_wait(&full_b[s], ph, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = sw128_desc(smem_u32(smem + OFF_A + s * TILE));
                    const uint64_t db = sw128_desc(smem_u32(smem + OFF_B + s * TILE));
#pragma unroll
                    for (int k = 0; k < 4; ++k)  // 4 x K=16 (32 bytes) inside the 128-byte swizzle row
                        umma_f16(d_isum, da + 2 * k, db + 2 * k, idesc, (c | k) != 0);
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                const int mb = sb & 1;
                if (!mbar_wait(&full_min[mb], (sb >> 1) & 1, abort_flag, err)) break;
                tc_fence_after();
                umma_f16(d_msum, sw128_desc(smem_u32(smem + OFF_AMIN + mb * TILE)),
                         sw128_desc(smem_u32(smem + OFF_BMIN + mb * TILE)), idesc, 0);
                umma_commit(&empty_min[mb]);
                umma_commit(&tmem_full[ab]);
            }
            // every MMA issued above completes before TMEM is released
            umma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0) && clock64() - t0 < (1LL << 31)) {
            }
        }
    } else if (warp < 6) {
        // ---- weight transform: one weight row (and one activation min row) per thread ----
        const int t = threadIdx.x - 64;
        const int m = m0 + t;
        const bool mv = m < M;
        // activation 16-wide sums of the next super-block, one super-block ahead
        int4 nb0 = make_int4(0, 0, 0, 0), nb1 = nb0;
        if (mv) {
            const __half *ap = bs16h + (int64_t)m * (K / 16);
            nb0 = *reinterpret_cast<const int4 *>(ap);
            nb1 = *reinterpret_cast<const int4 *>(ap + 8);
        }
        for (int kc = 0; kc < nkc; ++kc) {
            const int s = kc % STAGES, sb = kc >> 2, c = kc & 3, wb = sb % WSTAGES;
            if (c == 0 && !mbar_wait(&full_w[wb], (sb / WSTAGES) & 1, abort_flag, err)) break;
            if (!mbar_wait(&empty[s], ((kc / STAGES) & 1) ^ 1, abort_flag, err)) break;
            const uint8_t *wrow = smem + OFF_W + wb * WTILE + t * 144;  // rows past N are zero-filled by TMA
            const int4 hdr = *reinterpret_cast<const int4 *>(wrow);
            const int4 q0 = *reinterpret_cast<const int4 *>(wrow + 16 + 32 * c);
            const int4 q1 = *reinterpret_cast<const int4 *>(wrow + 32 + 32 * c);
            int sc0, mn0, sc1, mn1;
            q4k_scale_min(hdr, 2 * c, sc0, mn0);
            q4k_scale_min(hdr, 2 * c + 1, sc1, mn1);
            uint8_t *bt = smem + OFF_B + s * TILE;
            // chunk j = K elements 8j..8j+7 of this 64-wide slice: j < 4 low nibbles of
            // qs bytes 8j..8j+7 (sub-block 2c), j >= 4 high nibbles (sub-block 2c+1)
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 0)) = q4k_chunk_f16(q0.x, q0.y, 0, sc0);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 1)) = q4k_chunk_f16(q0.z, q0.w, 0, sc0);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 2)) = q4k_chunk_f16(q1.x, q1.y, 0, sc0);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 3)) = q4k_chunk_f16(q1.z, q1.w, 0, sc0);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 4)) = q4k_chunk_f16(q0.x, q0.y, 4, sc1);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 5)) = q4k_chunk_f16(q0.z, q0.w, 4, sc1);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 6)) = q4k_chunk_f16(q1.x, q1.y, 4, sc1);
            *reinterpret_cast<int4 *>(bt + sw128_off(t, 7)) = q4k_chunk_f16(q1.z, q1.w, 4, sc1);
            if (c == 0) {
                const int mb = sb & 1;
                if (!mbar_wait(&empty_min[mb], ((sb >> 1) & 1) ^ 1, abort_flag, err)) break;
                int mn[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    int scj;
                    q4k_scale_min(hdr, j, scj, mn[j]);
                }
                __half2 hb[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) hb[j] = __halves2half2(__int2half_rn(mn[j]), __int2half_rn(mn[j]));
                uint8_t *bm = smem + OFF_BMIN + mb * TILE;
                *reinterpret_cast<int4 *>(bm + sw128_off(t, 0)) = *reinterpret_cast<int4 *>(&hb[0]);
                *reinterpret_cast<int4 *>(bm + sw128_off(t, 1)) = *reinterpret_cast<int4 *>(&hb[4]);
                uint8_t *am = smem + OFF_AMIN + mb * TILE;
                *reinterpret_cast<int4 *>(am + sw128_off(t, 0)) = nb0;
                *reinterpret_cast<int4 *>(am + sw128_off(t, 1)) = nb1;
                if (mv && sb + 1 < nsb) {
                    const __half *ap = bs16h + (int64_t)m * (K / 16) + (sb + 1) * 16;
                    nb0 = *reinterpret_cast<const int4 *>(ap);
                    nb1 = *reinterpret_cast<const int4 *>(ap + 8);
                }
                fence_proxy_async_smem();
                mbar_arrive(&full_min[mb]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&full_b[s]);
            if (c == 3) mbar_arrive(&empty_w[wb]);
        }
    } else {
        // ---- epilogue ----
        const int e = warp - 6, q = warp & 3, hcol = e >> 2;
        const int row = m0 + 32 * q + lane;
        const bool rv = row < M;
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
        float da_next = rv ? __ldg(ad + (int64_t)row * nsb) : 0.0f;
        for (int sb = 0; sb < nsb; ++sb) {
            const int ab = sb & 1, wb = sb % WSTAGES;
            const float da = da_next;
            if (rv && sb + 1 < nsb) da_next = __ldg(ad + (int64_t)row * nsb + sb + 1);
            if (!mbar_wait(&tmem_full[ab], (sb >> 1) & 1, abort_flag, err)) break;
            // the raw super-block stays in its slot until this epilogue releases it, so its
            // phase is still the one to observe (makes the TMA bytes visible to these threads)
            if (!mbar_wait(&full_w[wb], (sb / WSTAGES) & 1, abort_flag, err)) break;
            tc_fence_after();
            const uint8_t *wsc = smem + OFF_W + wb * WTILE + 64 * hcol * 144;  // d, dmin of each weight row
            const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * 256 + 64 * hcol);
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) {
                uint32_t ri[16], rm[16];
                tmem_ld16(tb + 16 * cb, ri);
                tmem_ld16(tb + 128 + 16 * cb, rm);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t dd = *reinterpret_cast<const uint32_t *>(wsc + (16 * cb + i) * 144);
                    const float d = __fmul_rn(h2f((uint16_t)(dd & 0xFFFF)), da);
                    const float dm = __fmul_rn(h2f((uint16_t)(dd >> 16)), da);
                    acc[16 * cb + i] += __fsub_rn(__fmul_rn(d, __uint_as_float(ri[i])), __fmul_rn(dm, __uint_as_float(rm[i])));
                }
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[ab]);
            mbar_arrive(&empty_w[wb]);
        }
        if (rv) {
            float *yr = y + (int64_t)row * y_ld + n0 + 64 * hcol;
            if (n0 + 64 * hcol + 64 <= N && (((uintptr_t)yr) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4 *>(yr + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (n0 + 64 * hcol + i < N) yr[i] = acc[i];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---- Q8_0: tcgen05 kind::i8 -------------------------------------------------------------------
// ggml CPU (vec_dot_q8_0_q8_0) forms, per 32-element block b, the integer dot isum_b
// and adds (float)isum_b * (d_w,b * d_a,b) to an f32 sum in block order.  One
// tcgen05.mma.kind::i8 (K = 32 bytes = one block) writes isum_b for a 128 x 128 tile
// into its own TMEM buffer (four buffers rotate); sixteen epilogue warps read each
// buffer as soon as its MMA commits and apply that block's term with ggml's roundings,
// so the result equals the CPU oracle bit for bit.  Per stage TMA brings 128 K of
// activations and of weights (int8, 128B swizzle) and the 4 blocks' weight scales
// (f32, block-major copy made at upload).
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer, 2-17 epilogue (warp w reads
// TMEM lane quarter w % 4, 32 of the 128 columns).
namespace q80 {
constexpr int BM = 128, BN = 128, BK = 128;  // BK bytes = 4 blocks per stage
constexpr int STAGES = 4;
constexpr int TILE = 128 * 128;
constexpr int DWTILE = 4 * BN * 4;           // 4 blocks x 128 weight rows, f32
constexpr int STAGE_BYTES = 2 * TILE + DWTILE;
constexpr int NTHREADS = 576;
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * TILE;
constexpr int OFF_DW = OFF_B + STAGES * TILE;
constexpr int OFF_BAR = OFF_DW + STAGES * DWTILE;
constexpr int NBAR = 2 * STAGES + 8 + 1;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
}  // namespace q80

__global__ void __launch_bounds__(576, 1)
    mmq_q80_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_dw, int N, const float *__restrict__ ad, int M, int K,
                      float *__restrict__ y, int64_t y_ld, int *err) {
    using namespace q80;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + OFF_BAR);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *tmem_full = bars + 2 * STAGES;
    uint64_t *tmem_empty = tmem_full + 4;
    uint64_t *done = tmem_empty + 4;
    uint32_t *tmem_slot = (uint32_t *)(smem + OFF_MISC);
    volatile int *abort_flag = (volatile int *)(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nkc = K / BK, nb = K / 32;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1 + 16);  // MMA commit + every epilogue warp (weight scales read)
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], 16);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int kc = 0; kc < nkc; ++kc) {
                const int s = kc % STAGES;
                if (!mbar_wait(&empty[s], ((kc / STAGES) & 1) ^ 1, abort_flag, err)) break;
                mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                tma_load_2d(smem + OFF_A + s * TILE, &tmap_a, &full[s], kc * BK, m0);
                tma_load_2d(smem + OFF_B + s * TILE, &tmap_w, &full[s], kc * BK, n0);
                tma_load_2d(smem + OFF_DW + s * DWTILE, &tmap_dw, &full[s], n0, kc * 4);
                issued = kc + 1;
            }
            // no TMA write may still be in flight when the CTA exits
            for (int kc = max(0, issued - STAGES); kc < issued; ++kc) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&full[kc % STAGES], (kc / STAGES) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_s8_s32(BM, BN);
            bool ok = true;
            for (int kc = 0; kc < nkc && ok; ++kc) {
                const int s = kc % STAGES;
                if (!mbar_wait(&full[s], (kc / STAGES) & 1, abort_flag, err)) break;
                tc_fence_after();
                const uint64_t da = sw128_desc(smem_u32(smem + OFF_A + s * TILE));
                const uint64_t db = sw128_desc(smem_u32(smem + OFF_B + s * TILE));
                for (int j = 0; j < 4; ++j) {  // block 4kc + j -> TMEM buffer j
                    if (!mbar_wait(&tmem_empty[j], (kc & 1) ^ 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    umma_i8(tmem + 128 * j, da + 2 * j, db + 2 * j, idesc, 0);
                    umma_commit(&tmem_full[j]);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0) && clock64() - t0 < (1LL << 31)) {
            }
        }
    } else {
        // ---- epilogue: row m0 + 32q + lane, columns n0 + 32c .. +31 ----
        const int q = warp & 3, c = (warp - 2) >> 2;
        const int row = m0 + 32 * q + lane;
        const bool rv = row < M;
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
        const float *adr = ad + (int64_t)(rv ? row : 0) * nb;
        float4 da_next = rv ? *reinterpret_cast<const float4 *>(adr) : make_float4(0, 0, 0, 0);
        for (int kc = 0; kc < nkc; ++kc) {
            const int s = kc % STAGES;
            const float4 da4 = da_next;
            if (rv && kc + 1 < nkc) da_next = *reinterpret_cast<const float4 *>(adr + 4 * (kc + 1));
            // observe the stage's TMA completion: makes the weight-scale tile visible here
            if (!mbar_wait(&full[s], (kc / STAGES) & 1, abort_flag, err)) break;
            bool ok = true;
            for (int j = 0; j < 4; ++j) {
                if (!mbar_wait(&tmem_full[j], kc & 1, abort_flag, err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float da = j == 0 ? da4.x : (j == 1 ? da4.y : (j == 2 ? da4.z : da4.w));
                const float *dw = reinterpret_cast<const float *>(smem + OFF_DW + s * DWTILE) + j * BN + 32 * c;
                const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(128 * j + 32 * c);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t r[16];
                    tmem_ld16(tb + 16 * h, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; i += 4) {
                        const float4 w4 = *reinterpret_cast<const float4 *>(dw + 16 * h + i);
                        const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float dd = __fmul_rn(wv[u], da);
                            acc[16 * h + i + u] = __fadd_rn(acc[16 * h + i + u],
                                                            __fmul_rn((float)(int)r[i + u], dd));
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tmem_empty[j]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (!ok) break;
        }
        if (rv) {
            float *yr = y + (int64_t)row * y_ld + n0 + 32 * c;
            if (n0 + 32 * c + 32 <= N && (((uintptr_t)yr) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4 *>(yr + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (n0 + 32 * c + i < N) yr[i] = acc[i];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// block-major f32 copy of the Q8_0 scale plane: dT[slice][b][n] = d[slice][n][b]
__global__ void q80_scales_t_kernel(const uint16_t *__restrict__ d, int64_t N, int nb, int64_t total,
                                    float *__restrict__ dT) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i % N, t = i / N;
        const int64_t b = t % nb, sl = t / nb;
        dT[i] = h2f(d[(sl * N + n) * nb + b]);
    }
}

cudaError_t build_q80_scales_t(oasr_weight *w, cudaStream_t st) {
    const int64_t N = w->ne[1], nb = w->ne[0] / 32, slices = w->ne[2] * w->ne[3];
    const int64_t total = slices * nb * N;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 65535);
    q80_scales_t_kernel<<<grid, 256, 0, st>>>(w->d, N, (int)nb, total, w->dT);
    return cudaGetLastError();
}

// Q4_0 runs on the same kernel: ggml's Q4_0 x q8_0 block dot is the integer dot of the
// nibbles minus 8 with the q8_0 quants, scaled like Q8_0's ((float)isum * (d_w * d_a)), so
// the nibbles expanded to int8 at upload are a Q8_0 quant plane with the same scales
bool mmq_q80_tc_supported(int type, int64_t N, int64_t K) {
    return (type == OASR_TYPE_Q8_0 || type == OASR_TYPE_Q4_0) && K % q80::BK == 0 && N % 4 == 0;
}

// Q4_0 nibble plane [rows][K/2] (ggml order: byte j of a block holds elements j and j + 16
// in its low and high nibble) -> int8 (q - 8) [rows][K]; one thread per block
__global__ void q40_expand_kernel(const uint8_t *qs, int64_t nblocks, int64_t nb, int64_t qs_row, int8_t *q8) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nblocks; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nb, b = i - r * nb;
        const uint8_t *src = qs + r * qs_row + b * 16;
        int8_t *dst = q8 + (r * nb + b) * 32;
        for (int j = 0; j < 16; ++j) {
            const int v = src[j];
            dst[j] = (int8_t)((v & 0xF) - 8);
            dst[j + 16] = (int8_t)((v >> 4) - 8);
        }
    }
}

cudaError_t build_q40_expanded(oasr_weight *w, cudaStream_t st) {
    const int64_t nb = w->ne[0] / 32, rows = w->ne[1] * w->ne[2] * w->ne[3], nblocks = rows * nb;
    const unsigned grid = (unsigned)std::min<int64_t>((nblocks + 255) / 256, 65535);
    q40_expand_kernel<<<grid, 256, 0, st>>>(w->qs, nblocks, nb, w->qs_row_bytes, w->qs8);
    return cudaGetLastError();
}

// ---- host side ----------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

static int encode_2d(oasr_backend *be, CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner,
                     uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    auto enc = tensor_map_encoder();
    if (!enc) return oasr_internal_fail(be, OASR_STATUS_FAILED, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return oasr_internal_fail(be, OASR_STATUS_FAILED, "cuTensorMapEncodeTiled failed");
    return OASR_STATUS_SUCCESS;
}

static int launch_q4k_tc(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
                         float *y, int64_t y_ld) {
    const int64_t N = w->ne[1];
    CUtensorMap map_a, map_w;
    // activations: fp16 [M][K], 128 rows x 64 elements (128 B) per box, 128B swizzle
    int st = encode_2d(be, &map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.qs16, K, M, (uint64_t)K * 2, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // raw Q4_K rows: bytes [N][K/256*144], 128 rows x one 144-byte super-block per box
    st = encode_2d(be, &map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs + slice * N * w->qs_row_bytes, w->qs_row_bytes, N,
                   w->qs_row_bytes, 144, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    static std::atomic<bool> attr_set{false};  // idempotent set-up; concurrent first calls set the same attribute
    if (!attr_set) {
        cudaFuncSetAttribute(mmq_q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, q4k::SMEM_BYTES);
        attr_set = true;
    }
    dim3 grid((unsigned)((N + q4k::BN - 1) / q4k::BN), (unsigned)((M + q4k::BM - 1) / q4k::BM));
    mmq_q4k_tc_kernel<<<grid, q4k::NTHREADS, q4k::SMEM_BYTES, be->stream>>>(map_a, map_w, (int)N, a.bs16h, a.d,
                                                                            (int)M, K, y, y_ld, be->err_word);
    return oasr_internal_launch_check(be, "mmq_q4k_tc");
}

static int launch_q80_tc(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
                         float *y, int64_t y_ld) {
    const int64_t N = w->ne[1];
    CUtensorMap map_a, map_w, map_dw;
    // activations and weights: int8 [rows][K], 128 rows x 128 bytes per box, 128B swizzle
    int st = encode_2d(be, &map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.qs, K, M, (uint64_t)K, 128, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // Q8_0: the quant plane; Q4_0: its int8 expansion (rows of K bytes)
    const bool q40 = w->type == OASR_TYPE_Q4_0;
    const uint8_t *wq = q40 ? (const uint8_t *)w->qs8 : w->qs;
    const int64_t wrow = q40 ? (int64_t)K : w->qs_row_bytes;
    st = encode_2d(be, &map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq + slice * N * wrow, K, N, (uint64_t)wrow, 128, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // weight scales, block-major f32 [K/32][N]: 128 weight rows x 4 blocks per box
    st = encode_2d(be, &map_dw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w->dT + slice * (int64_t)(K / 32) * N, N, K / 32,
                   (uint64_t)N * 4, 128, 4, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    static std::atomic<bool> attr_set{false};  // idempotent set-up; concurrent first calls set the same attribute
    if (!attr_set) {
        cudaFuncSetAttribute(mmq_q80_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, q80::SMEM_BYTES);
        attr_set = true;
    }
    dim3 grid((unsigned)((N + q80::BN - 1) / q80::BN), (unsigned)((M + q80::BM - 1) / q80::BM));
    mmq_q80_tc_kernel<<<grid, q80::NTHREADS, q80::SMEM_BYTES, be->stream>>>(map_a, map_w, map_dw, (int)N, a.d, (int)M,
                                                                            K, y, y_ld, be->err_word);
    return oasr_internal_launch_check(be, "mmq_q80_tc");
}

int launch_mmq(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
               float *y, int64_t y_ld) {
    const bool k_family = w->type == OASR_TYPE_Q4_K;
    if (k_family && a.qs16 && a.bs16h) return launch_q4k_tc(be, w, slice, a, M, K, y, y_ld);
    if (w->dT && (w->type == OASR_TYPE_Q8_0 || w->qs8) && (y_ld & 3) == 0)
        return launch_q80_tc(be, w, slice, a, M, K, y, y_ld);
    const int family = k_family ? FAMILY_Q8_K : FAMILY_Q8_0;
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        const int mc = (int)std::min<int64_t>(8, M - m0);
        int st = launch_mmv_quant(be, w, slice, act_planes_offset(a, family, m0, K), mc, K, y + m0 * y_ld, y_ld);
        if (st) return st;
    }
    return OASR_STATUS_SUCCESS;
}

}  // namespace oasr
