// gemm_f16.cu -- fp16 x fp16 -> f32 GEMM on the tcgen05 tensor cores:
//   Y[m][n] = epilogue( sum_k A[m][k] * B[n][k] )
// A [M][K] and B [N][K] fp16 row-major (K contiguous, K % 64 == 0), both fed by
// TMA in the 128-byte swizzle layout; one f32 accumulator in TMEM per CTA.
// Products of two halves are exact in f32, so this is ggml's F16 vec_dot
// (fp16 operands, f32 accumulation) on tensor cores.  Used for F16-weight
// mul_mat with more than 8 rows and for the Whisper conv stem (im2col rows),
// where the optional epilogue adds a bias and applies ggml's tabulated GELU.
//
// CTA = 128 rows of A x 128 rows of B, 6 warps: warp 0 TMA producer, warp 1
// TMEM allocator + MMA issuer, warps 2-5 epilogue.  3-stage smem ring (96 KB)
// and 128 TMEM columns, so two CTAs share an SM.  Every wait is bounded.
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace oasr {

namespace gf16 {
constexpr int BM = 128, BN = 128, BK = 64, STAGES = 3;
constexpr int TILE = 128 * 128;
constexpr int OFF_A = 0;
constexpr int OFF_B = STAGES * TILE;
constexpr int OFF_BAR = 2 * STAGES * TILE;
constexpr int NBAR = 2 * STAGES + 2;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
constexpr int NTHREADS = 192;
}  // namespace gf16

__global__ void __launch_bounds__(192, 2)
    gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int M, int N,
                       int K, float *__restrict__ y, int64_t y_ld, const float *__restrict__ bias,
                       const uint16_t *__restrict__ gelu_table, int *err) {
    using namespace gf16;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + OFF_BAR);
    uint64_t *full = bars, *empty = bars + STAGES, *acc_full = bars + 2 * STAGES, *done = acc_full + 1;
    uint32_t *tmem_slot = (uint32_t *)(smem + OFF_MISC);
    volatile int *abort_flag = (volatile int *)(smem + OFF_MISC + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nkc = K / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 128);
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
                mbar_arrive_expect_tx(&full[s], 2 * TILE);
                tma_load_2d(smem + OFF_A + s * TILE, &tm_a, &full[s], kc * BK, m0);
                tma_load_2d(smem + OFF_B + s * TILE, &tm_b, &full[s], kc * BK, n0);
                issued = kc + 1;
            }
            for (int kc = max(0, issued - STAGES); kc < issued; ++kc) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&full[kc % STAGES], (kc / STAGES) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
            for (int kc = 0; kc < nkc; ++kc) {
                const int s = kc % STAGES;
                if (!mbar_wait(&full[s], (kc / STAGES) & 1, abort_flag, err)) break;
                tc_fence_after();
                const uint64_t da = sw128_desc(smem_u32(smem + OFF_A + s * TILE));
                const uint64_t db = sw128_desc(smem_u32(smem + OFF_B + s * TILE));
#pragma unroll
                for (int k = 0; k < 4; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (kc | k) != 0);
                umma_commit(&empty[s]);
            }
            umma_commit(acc_full);
            umma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0) && clock64() - t0 < (1LL << 31)) {
            }
        }
    } else {
        const int q = warp & 3;
        const int row = m0 + 32 * q + lane;
        if (mbar_wait(acc_full, 0, abort_flag, err)) {
            tc_fence_after();
            const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tmem_ld16(tb + 16 * c, v);
                tmem_ld_wait(v);
                if (row < M) {
                    float *yr = y + (int64_t)row * y_ld + n0 + 16 * c;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int n = n0 + 16 * c + i;
                        if (n >= N) break;
                        float r = __uint_as_float(v[i]);
                        if (bias) r = __fadd_rn(r, bias[n]);
                        if (gelu_table) {
                            if (r <= -10.0f) r = 0.0f;
                            else if (r < 10.0f) r = h2f(gelu_table[__half_as_ushort(__float2half_rn(r))]);
                        }
                        yr[i] = r;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

static PFN_cuTensorMapEncodeTiled_v12000 gf16_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// A [M][lda] and B [N][ldb] fp16 (lda, ldb in elements, multiples of 8), K % 64 == 0
int launch_gemm_f16(oasr_backend *be, const __half *A, int64_t lda, const __half *B, int64_t ldb, int M, int N, int K,
                    float *y, int64_t y_ld, const float *bias, bool gelu) {
    if (K % 64 || lda % 8 || ldb % 8 || ((uintptr_t)A & 15) || ((uintptr_t)B & 15))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "gemm_f16: K must be a multiple of 64, rows 16-byte aligned");
    auto enc = gf16_encoder();
    if (!enc) return oasr_internal_fail(be, OASR_STATUS_FAILED, "cuTensorMapEncodeTiled unavailable");
    CUtensorMap ma, mb;
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    const cuuint64_t da[2] = {(cuuint64_t)K, (cuuint64_t)M}, sa[1] = {(cuuint64_t)lda * 2};
    const cuuint64_t db[2] = {(cuuint64_t)K, (cuuint64_t)N}, sb[1] = {(cuuint64_t)ldb * 2};
    if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(A), da, sa, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(B), db, sb, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "gemm_f16: tensor map encoding failed");
    static std::atomic<bool> attr_set{false};  // idempotent set-up; concurrent first calls set the same attribute
    if (!attr_set) {
        cudaFuncSetAttribute(gemm_f16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gf16::SMEM_BYTES);
        attr_set = true;
    }
    dim3 grid((unsigned)((N + gf16::BN - 1) / gf16::BN), (unsigned)((M + gf16::BM - 1) / gf16::BM));
    gemm_f16_tc_kernel<<<grid, gf16::NTHREADS, gf16::SMEM_BYTES, be->stream>>>(
        ma, mb, M, N, K, y, y_ld, bias, gelu ? be->gelu_table : nullptr, be->err_word);
    return oasr_internal_launch_check(be, "gemm_f16_tc");
}

}  // namespace oasr
