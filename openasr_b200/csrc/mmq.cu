// mmq.cu -- K2: quantized GEMM for M > 8 activation rows (encoder, prefill).
//
// Q4_K weights run on the 5th-generation tensor cores (tcgen05, accumulators
// in TMEM) with ggml's exact per-super-block arithmetic:
//   ggml CPU (vec_dot_q4_K_q8_K) forms, per 256-element super-block,
//     isum = sum_j sc_j * <q4_j, q8_j>          (integers)
//     msum = sum_j m_j * bsum32_j               (integers)
//     term = (d_w*d_a)*isum - (dmin_w*d_a)*msum (f32)
//   At upload the 6-bit sub-scales are folded into the weight (sc*q <= 945, an
//   fp16 integer) once, so the B operand is a plain fp16 matrix streamed by TMA;
//   the q8_K activations are fp16 integers too.  tcgen05.mma.kind::f16 adds the
//   products in f32, exact while every partial sum stays below 2^24 -- so each
//   super-block accumulates as two 128-element halves in separate TMEM columns
//   (|half| <= 128*945*127 = 15,361,920 < 2^24) and the epilogue's f32 add of
//   the two exact halves is ggml's (float)isum (IEEE addition rounds the exact
//   sum once).  msum is 8 products per output (|msum| <= 8*63*4064 < 2^24), done
//   on the CUDA cores in integers: the activation's 32-quant sums split into a
//   6-bit low byte and a signed high byte, 4 dp4a against the mins bytes, and the
//   exact integer turned into a float by adding it to the bits of 1.5 * 2^23.  The epilogue forms `term` with ggml's
//   roundings and adds the super-blocks in order, so the result equals the CPU
//   oracle bit for bit for all inputs, the adversarial ones (all sub-scales 63,
//   quants 15, activations +-127) included.
//
// CTA = 128 activation rows x 128 weight rows, 18 warps:
//   warp 0      TMA producer: activation and weight tiles (128 x 64 fp16, SW128),
//               and per super-block the tile's weight metadata (d, dmin, 8 mins)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-17  epilogue: warp w reads TMEM lane quarter w % 4, 32 of the columns
// TMEM: two sets of (low half 128 cols + high half 128 cols) so the epilogue of
// super-block s overlaps the MMAs of s+1.  Every mbarrier wait is bounded.
//
// Q8_0 runs on tcgen05 kind::i8 (mmq_q80_tc_kernel below), Q4_0 on the same
// kernel over its quants expanded to int8.
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace oasr {

namespace q4k {
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;               // fp16 elements per stage = one 128-byte swizzle row
constexpr int STAGES = 5;
constexpr int TILE = 128 * 128;      // bytes of one 128-row x 128-byte operand tile
constexpr int META_COL = 4;          // 32-bit words per weight row: d, dmin (f32), mins 0-3, 4-7 (bytes)
constexpr int META = BN * META_COL * 4;  // one tile's metadata of one super-block: 2048 B
constexpr int MSTAGES = 2;
constexpr int NEPI = 16;
constexpr int NTHREADS = (2 + NEPI) * 32;
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * TILE;
constexpr int OFF_META = OFF_B + STAGES * TILE;
// per epilogue thread, two slots of its row's d_a and 16-wide sums of one super-block,
// copied one super-block ahead with cp.async
constexpr int OFF_ROWBS = OFF_META + MSTAGES * META;          // [2][NEPI * 32][32 B]
constexpr int OFF_ROWD = OFF_ROWBS + 2 * NEPI * 32 * 32;      // [2][NEPI * 32] f32
constexpr int OFF_REC = OFF_ROWD + 2 * NEPI * 32 * 4;         // [NEPI][32 rows][8 words] row records
constexpr int OFF_BAR = OFF_REC + NEPI * 32 * 32;
constexpr int NBAR = 2 * STAGES + 2 * MSTAGES + 4 + 1;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(META % 16 == 0, "bulk copies move multiples of 16 bytes");
}  // namespace q4k

static __device__ __forceinline__ int q4k_byte(const uint8_t *h, int i) { return h[4 + i]; }
static __device__ __forceinline__ void q4k_scale_min(const uint8_t *h, int j, int &sc, int &m) {
    if (j < 4) {
        sc = q4k_byte(h, j) & 63;
        m = q4k_byte(h, j + 4) & 63;
    } else {
        sc = (q4k_byte(h, j + 4) & 0xF) | ((q4k_byte(h, j - 4) >> 6) << 4);
        m = (q4k_byte(h, j + 4) >> 4) | ((q4k_byte(h, j) >> 6) << 4);
    }
}


__global__ void __launch_bounds__(q4k::NTHREADS, 1)
    mmq_q4k_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                      const float *__restrict__ meta, int64_t meta_sb_stride, const __half *__restrict__ bs16h,
                      const float *__restrict__ ad, int M, int K, int N, float *__restrict__ y, int64_t y_ld,
                      const float *__restrict__ bias, int *err) {
    using namespace q4k;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + OFF_BAR);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *meta_full = bars + 2 * STAGES;
    uint64_t *meta_empty = meta_full + MSTAGES;
    uint64_t *tmem_full = meta_empty + MSTAGES;
    uint64_t *tmem_empty = tmem_full + 2;
    uint64_t *done = tmem_empty + 2;
    uint32_t *tmem_slot = (uint32_t *)(smem + OFF_MISC);
    volatile int *abort_flag = (volatile int *)(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nkc = K / BK, nsb = K / 256;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < MSTAGES; ++i) {
            mbar_init(&meta_full[i], 1);
            mbar_init(&meta_empty[i], NEPI);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], NEPI);
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
            // TMA producer: operand tiles (ring of STAGES) and super-block metadata (ring of MSTAGES)
            int issued = 0, issued_meta = 0;
            for (int kc = 0; kc < nkc; ++kc) {
                const int sb = kc >> 2;
                if ((kc & 3) == 0) {
                    const int mb = sb % MSTAGES;
                    if (!mbar_wait(&meta_empty[mb], ((sb / MSTAGES) & 1) ^ 1, abort_flag, err)) break;
                    fence_proxy_async_smem();  // the epilogue's reads of this slot before the refill
                    mbar_arrive_expect_tx(&meta_full[mb], META);
                    bulk_load(smem + OFF_META + mb * META, meta + sb * meta_sb_stride + (int64_t)n0 * META_COL,
                              META, &meta_full[mb]);
                    issued_meta = sb + 1;
                }
                const int s = kc % STAGES;
                if (!mbar_wait(&empty[s], ((kc / STAGES) & 1) ^ 1, abort_flag, err)) break;
                mbar_arrive_expect_tx(&full[s], 2 * TILE);
                tma_load_2d(smem + OFF_A + s * TILE, &tmap_a, &full[s], kc * BK, m0);
                tma_load_2d(smem + OFF_B + s * TILE, &tmap_w, &full[s], kc * BK, n0);
                issued = kc + 1;
            }
            // no TMA write may still be in flight when the CTA exits
            for (int kc = max(0, issued - STAGES); kc < issued; ++kc) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&full[kc % STAGES], (kc / STAGES) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
            for (int sb = max(0, issued_meta - MSTAGES); sb < issued_meta; ++sb) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&meta_full[sb % MSTAGES], (sb / MSTAGES) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
            bool ok = true;
            for (int sb = 0; sb < nsb && ok; ++sb) {
                const int ab = sb & 1;
                if (!mbar_wait(&tmem_empty[ab], ((sb >> 1) & 1) ^ 1, abort_flag, err)) break;
                tc_fence_after();
                for (int c = 0; c < 4 && ok; ++c) {
                    const int kc = sb * 4 + c, s = kc % STAGES;
                    if (!mbar_wait(&full[s], (kc / STAGES) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = sw128_desc(smem_u32(smem + OFF_A + s * TILE));
                    const uint64_t db = sw128_desc(smem_u32(smem + OFF_B + s * TILE));
                    // chunks 0-1 (K 0..127 of the super-block) -> low half, 2-3 -> high half
                    const uint32_t d_acc = tmem + ab * 256 + (c >> 1) * 128;
#pragma unroll
                    for (int k = 0; k < 4; ++k)  // 4 x K=16 (32 bytes) inside the 128-byte swizzle row
                        umma_f16(d_acc, da + 2 * k, db + 2 * k, idesc, (c & 1) | k);
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&tmem_full[ab]);
            }
            // every MMA issued above completes before TMEM is released
            umma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0) && clock64() - t0 < (1LL << 31)) {
            }
        }
    } else {
        // ---- epilogue: warp w reads TMEM lane quarter w % 4 (32 rows), 32 weight columns ----
        // TMEM is read in the 16x256b shape: a thread holds 2 rows x 2 columns of each 16-lane
        // x 8-column block, so each column's metadata serves 4 of its outputs.  Lane l builds
        // the record of row 32q + l (d_a and the sub-block sums) for the whole warp.
        const int e = warp - 2, q = warp & 3, cg = e >> 2;
        const int row = m0 + 32 * q + lane;
        const bool rv = row < M;
        const int r4 = lane >> 2, c2 = 2 * (lane & 3);
        float acc[2][4][2][2];  // [16-row half][8-column group][row r4, r4 + 8][column c2, c2 + 1]
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int i = 0; i < 2; ++i) acc[h][k][i][0] = acc[h][k][i][1] = 0.0f;
        uint8_t *rbs = smem + OFF_ROWBS + (e * 32 + lane) * 32;  // slot stride NEPI * 32 * 32
        float *rd = reinterpret_cast<float *>(smem + OFF_ROWD) + e * 32 + lane;  // slot stride NEPI * 32
        uint32_t *rec = reinterpret_cast<uint32_t *>(smem + OFF_REC) + e * 32 * 8;  // this warp's rows
        auto fetch_row = [&](int sb) {  // this row's d_a and 16-wide sums of super-block sb
            if (rv) {
                const int sl = sb & 1;
                const __half *bp = bs16h + (int64_t)row * (K / 16) + sb * 16;
                cp_async16(rbs + sl * NEPI * 32 * 32, bp);
                cp_async16(rbs + sl * NEPI * 32 * 32 + 16, bp + 8);
                cp_async4(rd + sl * NEPI * 32, ad + (int64_t)row * nsb + sb);
            }
            cp_async_commit();
        };
        fetch_row(0);
        for (int sb = 0; sb < nsb; ++sb) {
            const int ab = sb & 1, mb = sb % MSTAGES;
            if (sb + 1 < nsb) fetch_row(sb + 1);
            else cp_async_commit();
            cp_async_wait1();  // super-block sb's row data has landed
            {
                // the row's sums of the 32 quants of each sub-block (exact integers, |.| <= 4064)
                // as b = 64 * bh + bl with bl in [0, 63] and bh in [-64, 63], 4 per word
                uint32_t bl0 = 0, bl1 = 0, bh0 = 0, bh1 = 0;
                const __half2 *hb = reinterpret_cast<const __half2 *>(rbs + (sb & 1) * NEPI * 32 * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float2 v = __half22float2(hb[j]);
                    const int b = __float_as_int(__fadd_rn(__fadd_rn(v.x, v.y), 12582912.0f)) - 0x4B400000;
                    const uint32_t lo6 = (uint32_t)(b & 63), hi8 = (uint32_t)(b >> 6) & 0xFFu;
                    if (j < 4) {
                        bl0 |= lo6 << (8 * j);
                        bh0 |= hi8 << (8 * j);
                    } else {
                        bl1 |= lo6 << (8 * (j - 4));
                        bh1 |= hi8 << (8 * (j - 4));
                    }
                }
                *reinterpret_cast<uint4 *>(rec + lane * 8) = make_uint4(__float_as_uint(rd[(sb & 1) * NEPI * 32]), bl0, bl1, bh0);
                rec[lane * 8 + 4] = bh1;
            }
            __syncwarp();
            if (!mbar_wait(&tmem_full[ab], (sb >> 1) & 1, abort_flag, err)) break;
            if (!mbar_wait(&meta_full[mb], (sb / MSTAGES) & 1, abort_flag, err)) break;
            tc_fence_after();
            const uint4 *mt = reinterpret_cast<const uint4 *>(smem + OFF_META + mb * META) + 32 * cg;
            const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * 256 + 32 * cg);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                // records of rows 16h + r4 and 16h + r4 + 8: d_a, bl0, bl1, bh0 | bh1
                uint4 ra[2];
                uint32_t rh[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    ra[i] = *reinterpret_cast<const uint4 *>(rec + (16 * h + r4 + 8 * i) * 8);
                    rh[i] = rec[(16 * h + r4 + 8 * i) * 8 + 4];
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    uint32_t lo[4], hi[4];
                    tmem_ld16x256(tb + ((uint32_t)(16 * h) << 16) + 8 * k, lo);
                    tmem_ld16x256(tb + ((uint32_t)(16 * h) << 16) + 128 + 8 * k, hi);
                    const uint4 mw[2] = {mt[8 * k + c2], mt[8 * k + c2 + 1]};  // d, dmin, mins 0-3, mins 4-7
                    tmem_ld_wait(lo, hi);
#pragma unroll
                    for (int i = 0; i < 2; ++i)
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
                            // (float)isum: the f32 sum of the two exact halves rounds the exact sum once
                            const float isum = __fadd_rn(__uint_as_float(lo[2 * i + j]), __uint_as_float(hi[2 * i + j]));
                            // msum + the bits of 1.5 * 2^23, then as a float minus 1.5 * 2^23: exact
                            const int ml = __dp4a((int)mw[j].w, (int)ra[i].z, __dp4a((int)mw[j].z, (int)ra[i].y, 0x4B400000));
                            const int mh = __dp4a((int)mw[j].w, (int)rh[i], __dp4a((int)mw[j].z, (int)ra[i].w, 0));
                            const float ms = __fsub_rn(__int_as_float(ml + 64 * mh), 12582912.0f);
                            // ggml's term with its roundings; the scalar _rn intrinsics are never
                            // contracted into a fused multiply-add
                            const float da = __uint_as_float(ra[i].x);
                            const float d = __fmul_rn(__uint_as_float(mw[j].x), da);
                            const float dm = __fmul_rn(__uint_as_float(mw[j].y), da);
                            acc[h][k][i][j] = __fadd_rn(acc[h][k][i][j], __fsub_rn(__fmul_rn(d, isum), __fmul_rn(dm, ms)));
                        }
                }
            }
            // the metadata slot was read here (generic proxy) and is refilled by a bulk copy
            // (async proxy): a proxy fence orders the reads before that write (without it, 1
            // launch in ~500 computed a fragment from the next super-block's metadata)
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tmem_empty[ab]);
                mbar_arrive(&meta_empty[mb]);
            }
        }
        cp_async_wait0();  // no row copy in flight past this point (also after an abort)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int rr = m0 + 32 * q + 16 * h + r4 + 8 * i;
                if (rr >= M) continue;
                float *yr = y + (int64_t)rr * y_ld + n0 + 32 * cg + c2;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int col = n0 + 32 * cg + 8 * k + c2;
                    // the optional bias is ggml's separate add of the mul_mat result (one f32 add)
                    float v0 = acc[h][k][i][0], v1 = acc[h][k][i][1];
                    if (bias) {
                        if (col < N) v0 = __fadd_rn(v0, bias[col]);
                        if (col + 1 < N) v1 = __fadd_rn(v1, bias[col + 1]);
                    }
                    if (col + 1 < N && (((uintptr_t)(yr + 8 * k)) & 7) == 0) {
                        *reinterpret_cast<float2 *>(yr + 8 * k) = make_float2(v0, v1);
                    } else {
                        if (col < N) yr[8 * k] = v0;
                        if (col + 1 < N) yr[8 * k + 1] = v1;
                    }
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

// ---- Q4_K operand build (upload) ----------------------------------------------------------------
// raw Q4_K rows [slices][N][K/256 x 144 B] ->
//   h16  [slices][N][K] fp16: sc_j * q (element order of ggml's dequantize_row_q4_K:
//        64-element chunk c holds the low nibbles of qs[32c..32c+31] (sub-block 2c)
//        then their high nibbles (sub-block 2c+1))
//   meta [slices][K/256][Np][4] words per weight row: d, dmin (f32), mins m_0..m_3 and
//        m_4..m_7 (one byte each); rows >= N zero; Np = N rounded up to 128
// One thread per (row, super-block).
__global__ void q4k_operand_kernel(const uint8_t *__restrict__ qs, int64_t row_bytes, int64_t N, int nsb, int64_t Np,
                                   int64_t total, __half *__restrict__ h16, float *__restrict__ meta) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nsb;  // row over all slices
        const int sb = (int)(i - r * nsb);
        const int64_t sl = r / N, n = r - sl * N;
        const uint8_t *blk = qs + r * row_bytes + (int64_t)sb * 144;
        int sc[8], mn[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q4k_scale_min(blk, j, sc[j], mn[j]);
        __half *dst = h16 + r * ((int64_t)nsb * 256) + (int64_t)sb * 256;
        for (int c = 0; c < 4; ++c)
            for (int l = 0; l < 32; ++l) {
                const int v = blk[16 + 32 * c + l];
                dst[64 * c + l] = __int2half_rn(sc[2 * c] * (v & 0xF));
                dst[64 * c + 32 + l] = __int2half_rn(sc[2 * c + 1] * (v >> 4));
            }
        float *mp = meta + ((sl * nsb + sb) * Np + n) * 4;
        mp[0] = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        mp[1] = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
        uint32_t *mw = reinterpret_cast<uint32_t *>(mp);
        mw[2] = (uint32_t)mn[0] | ((uint32_t)mn[1] << 8) | ((uint32_t)mn[2] << 16) | ((uint32_t)mn[3] << 24);
        mw[3] = (uint32_t)mn[4] | ((uint32_t)mn[5] << 8) | ((uint32_t)mn[6] << 16) | ((uint32_t)mn[7] << 24);
    }
}

bool mmq_q4k_tc_supported(int type, int64_t K) { return type == OASR_TYPE_Q4_K && K % 256 == 0; }

size_t q4k_operand_bytes(int64_t N, int64_t K, int64_t slices, size_t *meta_bytes) {
    const int64_t Np = (N + 127) / 128 * 128;
    *meta_bytes = (size_t)(slices * (K / 256) * Np * 4) * sizeof(float);
    return (size_t)(slices * N * K) * 2;
}

cudaError_t build_q4k_operand(oasr_weight *w, cudaStream_t st) {
    const int64_t N = w->ne[1], K = w->ne[0], slices = w->ne[2] * w->ne[3];
    const int64_t Np = (N + 127) / 128 * 128, nsb = K / 256, total = slices * N * nsb;
    size_t mb = 0;
    q4k_operand_bytes(N, K, slices, &mb);
    cudaError_t e = cudaMemsetAsync(w->k_meta, 0, mb, st);  // pad rows: zero metadata
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 65535);
    q4k_operand_kernel<<<grid, 256, 0, st>>>(w->qs, w->qs_row_bytes, N, (int)nsb, Np, total, w->h16, w->k_meta);
    return cudaGetLastError();
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
                fence_proxy_async_smem();  // the epilogue's reads of the stage's scales before the refill
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
                    tmem_ld_wait(r);
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
            // the stage's weight scales were read here (generic proxy); the stage is refilled by
            // TMA (async proxy): a proxy fence orders the reads before that write
            fence_proxy_async_smem();
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
                         float *y, int64_t y_ld, const float *bias) {
    const int64_t N = w->ne[1], Np = (N + 127) / 128 * 128;
    CUtensorMap map_a, map_w;
    // activations: fp16 [M][K], 128 rows x 64 elements (128 B) per box, 128B swizzle
    int st = encode_2d(be, &map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.qs16, K, M, (uint64_t)K * 2, 64, 128,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // weights: the fp16 sc*q operand [N][K], same box
    st = encode_2d(be, &map_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w->h16 + slice * N * K, K, N, (uint64_t)K * 2, 64, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    static std::atomic<bool> attr_set{false};  // idempotent set-up; concurrent first calls set the same attribute
    if (!attr_set) {
        cudaFuncSetAttribute(mmq_q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, q4k::SMEM_BYTES);
        attr_set = true;
    }
    const int64_t meta_sb = Np * q4k::META_COL;
    const float *meta = w->k_meta + slice * (K / 256) * meta_sb;
    dim3 grid((unsigned)((N + q4k::BN - 1) / q4k::BN), (unsigned)((M + q4k::BM - 1) / q4k::BM));
    mmq_q4k_tc_kernel<<<grid, q4k::NTHREADS, q4k::SMEM_BYTES, be->stream>>>(map_a, map_w, meta, meta_sb, a.bs16h, a.d,
                                                                            (int)M, K, (int)N, y, y_ld, bias, be->err_word);
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

bool mmq_fuses_bias(const oasr_weight *w, const ActPlanes &a) {
    return w->type == OASR_TYPE_Q4_K && w->h16 && a.qs16 && a.bs16h;
}

int launch_mmq(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
               float *y, int64_t y_ld, const float *bias) {
    const bool k_family = w->type == OASR_TYPE_Q4_K;
    if (mmq_fuses_bias(w, a)) return launch_q4k_tc(be, w, slice, a, M, K, y, y_ld, bias);
    if (bias) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mmq: bias epilogue needs the Q4_K tensor-core path");
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
