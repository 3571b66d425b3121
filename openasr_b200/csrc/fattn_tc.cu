// fattn_tc.cu -- K4: tiled flash attention on the tcgen05 tensor cores for long
// query blocks: the Whisper encoder's self-attention (n_q = n_kv = 1500, head_dim
// 64, no mask) and the Qwen decoder's causal prompt pass (head_dim 128, GQA).
//
// Semantics (cpu_graph.rs:4144-4220; call sites ggml_executor.rs:1650-1695 and
// nn/decoder.rs:2040-2064):
//   O[:, h, i, s] = softmax(scale * Q[:, i, h, s] . K[:, :, h/G, s] + mask) V
// where the only mask taken here is the causal one (key j visible to query i when
// j <= i + n_kv - n_q, build_causal_mask_f16_bits, nn/decoder.rs:766-790).
// Q, K and V are rounded to fp16 (the operand type of the tensor-core MMA;
// ggml's CUDA backend makes the same conversion for f32 K/V), S = Q K^T and
// O = P V accumulate in f32 in TMEM, P is rounded to fp16, and the softmax runs
// in f32 with online rescaling.
//
// A pre-pass writes Q and K as fp16 [S*H][n][D] rows and V transposed as
// fp16 [S*H_kv][D][n_pad] so that every MMA operand is a K-major tile of 64-element
// (128-byte) rows in the 128-byte swizzle layout fetched by TMA:
//   MMA1  S(128 q x 128 keys) = Q tile (128 x D) . K tile (128 keys x D)^T
//   MMA2  Ot(128 q x D dims)  = P tile (128 x 128 keys) . Vt tile (D dims x 128 keys)^T
// CTA = one 128-query tile of one head, 6 warps:
//   warps 0-3  softmax (one query row per thread) + output accumulation in registers
//   warp 4     TMA producer (Q once, then K / Vt tiles through a 2-slot ring)
//   warp 5     TMEM allocator (256 columns) + single-thread MMA issuer
// D = 64: two CTAs share an SM (112 KB shared memory each), so one CTA's softmax
// overlaps the other's MMAs; D = 128: one CTA per SM (192 KB).  Causal tiles wholly
// above the diagonal are skipped.  Every mbarrier wait is bounded.
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace oasr {

template <int D_>
struct FaTc {
    static constexpr int D = D_;
    static constexpr int BQ = 128, BKV = 128;
    static constexpr int SUB = 128 * 128;                // one 64-element-wide swizzled sub-tile of 128 rows
    static constexpr int QTILE = (D / 64) * SUB;        // 128 q x D
    static constexpr int KTILE = (D / 64) * SUB;        // 128 keys x D
    static constexpr int VTILE = D * 128;               // D dims x 64 keys
    static constexpr int SLOT = KTILE + 2 * VTILE;      // K tile + two Vt half-tiles
    static constexpr int PTILE = BQ * 128;              // 128 q x 64 keys
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_KV = OFF_Q + QTILE;
    static constexpr int OFF_P = OFF_KV + 2 * SLOT;
    static constexpr int OFF_BAR = OFF_P + 2 * PTILE;
    static constexpr int NBAR = 10;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int SMEM_BYTES = OFF_MISC + 16;
    static constexpr int CTAS_PER_SM = D == 64 ? 2 : 1;
    static constexpr int NTHREADS = 192;
    // D = 64: two CTAs per SM, <= (228 KB - 2 x 1 KB reserved) / 2; D = 128: one CTA, <= 227 KB
    static_assert(SMEM_BYTES <= (D == 64 ? 115712 : 232448), "shared memory per CTA");
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
};

// ---- pre-pass: q, k -> fp16 rows [S*H][n][D]; v -> fp16 [S*Hkv][D][n_pad] ------------
// CTA = 64 positions of one row block hs =
// s * H + h; each thread moves 16-byte chunks (4 f32 or 8 f16 values).  Rows go out as
// f16 [hs][n][D]; with TR they are transposed through shared memory into
// [hs][D][n_pad] (128-byte row pieces per store) and positions n..n_pad-1 are written
// as zeros.  Values round to fp16 with round-to-nearest-even (f16 inputs pass unchanged).
template <bool F16IN, int D, bool TR>
__global__ void __launch_bounds__(256) fa_prep_tile_kernel(const char *src, int64_t nb1, int64_t nb2, int64_t nb3, int n,
                                                           int H, __half *dst, int n_pad) {
    constexpr int TP = 64;               // positions per tile
    constexpr int EPC = F16IN ? 8 : 4;   // values per 16-byte chunk
    constexpr int CPR = D / EPC;         // chunks per row
    constexpr int LD = TP + 8;           // shared row pitch in halves (144 bytes: 16-byte aligned)
    __shared__ __align__(16) __half tile[TR ? D : 1][LD];
    const int p0 = blockIdx.x * TP;
    const int hs = blockIdx.y;
    const int h = hs % H, s = hs / H;
    const char *base = src + (int64_t)h * nb2 + (int64_t)s * nb3;
    for (int c = threadIdx.x; c < TP * CPR; c += 256) {
        const int pr = c / CPR, ch = c % CPR;
        const int p = p0 + pr;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (p < n) raw = *reinterpret_cast<const uint4 *>(base + (int64_t)p * nb1 + ch * 16);
        if (F16IN) {
            if (TR) {
                const __half *hv = reinterpret_cast<const __half *>(&raw);
#pragma unroll
                for (int j = 0; j < 8; ++j) tile[ch * 8 + j][pr] = hv[j];
            } else if (p < n) {
                *reinterpret_cast<uint4 *>(dst + ((int64_t)hs * n + p) * D + ch * 8) = raw;
            }
        } else {
            const float *fv = reinterpret_cast<const float *>(&raw);
            const __half2 h01 = __halves2half2(__float2half_rn(fv[0]), __float2half_rn(fv[1]));
            const __half2 h23 = __halves2half2(__float2half_rn(fv[2]), __float2half_rn(fv[3]));
            if (TR) {
                tile[ch * 4 + 0][pr] = __low2half(h01);
                tile[ch * 4 + 1][pr] = __high2half(h01);
                tile[ch * 4 + 2][pr] = __low2half(h23);
                tile[ch * 4 + 3][pr] = __high2half(h23);
            } else if (p < n) {
                uint2 pk;
                pk.x = *reinterpret_cast<const uint32_t *>(&h01);
                pk.y = *reinterpret_cast<const uint32_t *>(&h23);
                *reinterpret_cast<uint2 *>(dst + ((int64_t)hs * n + p) * D + ch * 4) = pk;
            }
        }
    }
    if (TR) {
        __syncthreads();
        for (int c = threadIdx.x; c < D * (TP / 8); c += 256) {
            const int d = c / (TP / 8), pc = c % (TP / 8);
            const int p = p0 + pc * 8;
            if (p >= n_pad) continue;  // n_pad is a multiple of 8: chunks are wholly in or out
            *reinterpret_cast<uint4 *>(dst + ((int64_t)hs * D + d) * n_pad + p) =
                *reinterpret_cast<const uint4 *>(&tile[d][pc * 8]);
        }
    }
}

// one pre-pass operand through the tiled kernel (D 64 or 128; data and byte strides
// multiples of 16; S * H <= 65535)
template <bool F16IN>
static void fa_prep_tiled(oasr_backend *be, const oasr_tensor *t, int n, int H, int S, int D, __half *dst, bool tr,
                          int n_pad) {
    const int rows = tr ? n_pad : n;
    const dim3 grid((unsigned)((rows + 63) / 64), (unsigned)(S * H));
    const char *src = (const char *)t->data;
#define FA_PREP_TILE(DD, TRV)                                                                                       \
    fa_prep_tile_kernel<F16IN, DD, TRV><<<grid, 256, 0, be->stream>>>(src, t->nb[1], t->nb[2], t->nb[3], n, H, dst, \
                                                                      n_pad)
    if (D == 64) { if (tr) FA_PREP_TILE(64, true); else FA_PREP_TILE(64, false); }
    else { if (tr) FA_PREP_TILE(128, true); else FA_PREP_TILE(128, false); }
#undef FA_PREP_TILE
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(192, FaTc<D>::CTAS_PER_SM)
    fattn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_vt, int NQ, int NKV, int H, int HKV, float scale_log2,
                    char *dst, int64_t d_nb1, int64_t d_nb2, int64_t d_nb3, int *err) {
    using C = FaTc<D>;
    constexpr int BQ = C::BQ, BKV = C::BKV, NSUB = D / 64;
    extern __shared__ __align__(1024) uint8_t smem_fa[];
    uint8_t *smem = smem_fa;
    // the 128-byte swizzle tiles need a 1024-byte aligned base; refuse (no waits, no TMEM) otherwise
    if (smem_u32(smem) & 1023u) {
        if (threadIdx.x == 0) atomicOr(err, ERR_BAD_SHAPE);
        return;
    }
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *q_full = bars + 0;
    uint64_t *kv_full = bars + 1;   // [2]
    uint64_t *kv_empty = bars + 3;  // [2]
    uint64_t *s_full = bars + 5;
    uint64_t *p_full = bars + 6;
    uint64_t *o_full = bars + 7;
    uint64_t *done = bars + 8;
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_MISC);
    volatile int *abort_flag = (volatile int *)(smem + C::OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x;       // query tile
    const int hs = blockIdx.y;       // s * H + h
    const int h = hs % H, s = hs / H;
    const int G = H / HKV;
    const int hks = s * HKV + h / G;  // kv row block
    const int q0 = qt * BQ;
    const int qoff = NKV - NQ;        // causal: query i sits at key position i + qoff
    int ntiles = (NKV + BKV - 1) / BKV;
    if (CAUSAL) ntiles = min(ntiles, (q0 + BQ - 1 + qoff) / BKV + 1);  // later tiles are wholly masked

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(p_full, 128);
        mbar_init(o_full, 1);
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 5) tmem_alloc(tmem_slot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // S: cols [0,128), Ot: cols [128,128+D)

    if (warp == 4) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, C::QTILE);
#pragma unroll
            for (int u = 0; u < NSUB; ++u) tma_load_2d(smem + C::OFF_Q + u * C::SUB, &tm_q, q_full, 64 * u, hs * NQ + q0);
            int issued = 0;
            for (int j = 0; j < ntiles; ++j) {
                const int b = j & 1;
                if (!mbar_wait(&kv_empty[b], ((j >> 1) & 1) ^ 1, abort_flag, err)) break;
                uint8_t *slot = smem + C::OFF_KV + b * C::SLOT;
                mbar_arrive_expect_tx(&kv_full[b], C::SLOT);
#pragma unroll
                for (int u = 0; u < NSUB; ++u)
                    tma_load_2d(slot + u * C::SUB, &tm_k, &kv_full[b], 64 * u, hks * NKV + j * BKV);
                tma_load_2d(slot + C::KTILE, &tm_vt, &kv_full[b], j * BKV, hks * D);
                tma_load_2d(slot + C::KTILE + C::VTILE, &tm_vt, &kv_full[b], j * BKV + 64, hks * D);
                issued = j + 1;
            }
            for (int j = max(0, issued - 2); j < issued; ++j) {
                const long long t0 = clock64();
                while (!mbar_try_wait(&kv_full[j & 1], (j >> 1) & 1) && clock64() - t0 < (1LL << 31)) {
                }
            }
            const long long t0 = clock64();
            while (!mbar_try_wait(q_full, 0) && clock64() - t0 < (1LL << 31)) {
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            constexpr uint32_t id1 = idesc_f16_f32(BQ, BKV);
            constexpr uint32_t id2 = idesc_f16_f32(BQ, D);
            const uint32_t t_s = tmem, t_o = tmem + 128;
            bool ok = mbar_wait(q_full, 0, abort_flag, err);
            for (int j = 0; j < ntiles && ok; ++j) {
                const int b = j & 1;
                uint8_t *slot = smem + C::OFF_KV + b * C::SLOT;
                if (!mbar_wait(&kv_full[b], (j >> 1) & 1, abort_flag, err)) break;
                // S may be overwritten once the softmax of tile j-1 has read it (p_full of j-1)
                if (j > 0 && !mbar_wait(p_full, (j - 1) & 1, abort_flag, err)) break;
                tc_fence_after();
                // 16 dims per MMA: 4 steps inside each 64-dim swizzled sub-tile
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint64_t dq = sw128_desc(smem_u32(smem + C::OFF_Q + (k >> 2) * C::SUB)) + 2 * (k & 3);
                    const uint64_t dk = sw128_desc(smem_u32(slot + (k >> 2) * C::SUB)) + 2 * (k & 3);
                    umma_f16(t_s, dq, dk, id1, k != 0);
                }
                umma_commit(s_full);
                // O_tile = P . Vt^T once the softmax has written P for this tile
                if (!mbar_wait(p_full, j & 1, abort_flag, err)) break;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint64_t dp = sw128_desc(smem_u32(smem + C::OFF_P + (k >> 2) * C::PTILE)) + 2 * (k & 3);
                    const uint64_t dv = sw128_desc(smem_u32(slot + C::KTILE + (k >> 2) * C::VTILE)) + 2 * (k & 3);
                    umma_f16(t_o, dp, dv, id2, k != 0);
                }
                umma_commit(&kv_empty[b]);
                umma_commit(o_full);
            }
            umma_commit(done);
            const long long t0 = clock64();
            while (!mbar_try_wait(done, 0) && clock64() - t0 < (1LL << 31)) {
            }
        }
    } else {
        // ---- softmax warpgroup: thread = query row q0 + 32*warp + lane ----
        const int r = 32 * warp + lane;
        const int qpos = q0 + r + qoff;  // last key position this row may see (causal)
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        float m = -INFINITY, l = 0.0f;
        float o[D];
#pragma unroll
        for (int i = 0; i < D; ++i) o[i] = 0.0f;
        for (int j = 0; j < ntiles; ++j) {
            if (!mbar_wait(s_full, j & 1, abort_flag, err)) break;
            tc_fence_after();
            // keys j*BKV + c visible to this row: c < lim
            int lim = min(BKV, NKV - j * BKV);
            if (CAUSAL) lim = min(lim, qpos - j * BKV + 1);
            // pass 1: row max of this tile
            float tmax = -INFINITY;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tmem_ld16(trow + 16 * c, v);
                tmem_ld_wait(v);
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (16 * c + i < lim) tmax = fmaxf(tmax, __uint_as_float(v[i]) * scale_log2);
            }
            const float mnew = fmaxf(m, tmax);
            // m = -inf on the first tile -> 0; a row with nothing visible yet keeps o = 0
            const float alpha = mnew == -INFINITY ? 1.0f : exp2f(m - mnew);
            // pass 2: p = 2^(s*scale*log2e - mnew), row sum, P (fp16) into the swizzled A tiles
            float tsum = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tmem_ld16(trow + 16 * c, v);
                tmem_ld_wait(v);
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const float p0 = 16 * c + i < lim ? exp2f(__uint_as_float(v[i]) * scale_log2 - mnew) : 0.0f;
                    const float p1 = 16 * c + i + 1 < lim ? exp2f(__uint_as_float(v[i + 1]) * scale_log2 - mnew) : 0.0f;
                    tsum += p0 + p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[i / 2] = *reinterpret_cast<const uint32_t *>(&hp);
                }
                // keys 16c..16c+15 = two 16-byte chunks of the 64-key tile c/4
                uint8_t *pt = smem + C::OFF_P + (c >> 2) * C::PTILE;
                const int ch = (c & 3) * 2;
                *reinterpret_cast<int4 *>(pt + sw128_off(r, ch)) = make_int4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<int4 *>(pt + sw128_off(r, ch + 1)) = make_int4(pk[4], pk[5], pk[6], pk[7]);
            }
            l = l * alpha + tsum;
            m = mnew;
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(p_full);
            // O = alpha * O + P V (tile)
            if (!mbar_wait(o_full, j & 1, abort_flag, err)) break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 16; ++c) {
                uint32_t v[16];
                tmem_ld16(trow + 128 + 16 * c, v);
                tmem_ld_wait(v);
#pragma unroll
                for (int i = 0; i < 16; ++i) o[16 * c + i] = fmaf(o[16 * c + i], alpha, __uint_as_float(v[i]));
            }
            tc_fence_before();
        }
        const int qi = q0 + r;
        if (qi < NQ) {
            const float inv = l == 0.0f ? 0.0f : 1.0f / l;
            float *out = reinterpret_cast<float *>(dst + h * d_nb1 + qi * d_nb2 + s * d_nb3);
#pragma unroll
            for (int i = 0; i < D; i += 4)
                *reinterpret_cast<float4 *>(out + i) = make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

static PFN_cuTensorMapEncodeTiled_v12000 fa_encoder() {
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

static bool encode_f16_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows, uint32_t box_inner,
                          uint32_t box_rows) {
    auto enc = fa_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool flash_attn_tc_eligible(const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *mask,
                            const oasr_tensor *dst) {
    // the public entry point routes the encoder shape here (head_dim 64, no mask); the causal
    // head_dim-128 form is taken by the Qwen prompt pass directly
    return q->ne[0] == 64 && k->ne[0] == 64 && q->ne[1] >= 64 && k->ne[1] >= 64 && mask == nullptr &&
           dst->nb[1] % 16 == 0 && dst->nb[2] % 16 == 0 && dst->nb[3] % 16 == 0 && ((uintptr_t)dst->data & 15) == 0;
}

template <int D, bool CAUSAL>
static cudaError_t launch_fa_tc(oasr_backend *be, dim3 grid, const CUtensorMap &mq, const CUtensorMap &mk,
                                const CUtensorMap &mv, int NQ, int NKV, int H, int HKV, float scale_log2,
                                const oasr_tensor *dst) {
    using C = FaTc<D>;
    static std::atomic<bool> attr_set{false};  // per instantiation, same for every device of this build
    if (!attr_set) {
        const cudaError_t e =
            cudaFuncSetAttribute(fattn_tc_kernel<D, CAUSAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    fattn_tc_kernel<D, CAUSAL><<<grid, C::NTHREADS, C::SMEM_BYTES, be->stream>>>(
        mq, mk, mv, NQ, NKV, H, HKV, scale_log2, (char *)dst->data, dst->nb[1], dst->nb[2], dst->nb[3], be->err_word);
    return cudaGetLastError();
}

int launch_flash_attn_tc(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                         float scale, oasr_tensor *dst, bool causal) {
    const int D = (int)q->ne[0];
    const int NQ = (int)q->ne[1], H = (int)q->ne[2], S = (int)q->ne[3];
    const int NKV = (int)k->ne[1], HKV = (int)k->ne[2];
    if ((D != 64 && D != 128) || (causal && NKV < NQ))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_tc: head_dim 64 or 128; causal needs n_kv >= n_q");
    const int n_pad = (NKV + 7) & ~7;
    const size_t q_bytes = align256((size_t)S * H * NQ * D * 2);
    const size_t k_bytes = align256((size_t)S * HKV * NKV * D * 2);
    const size_t v_bytes = align256((size_t)S * HKV * D * n_pad * 2);
    int st = 0;
    uint8_t *scr = (uint8_t *)oasr_internal_scratch(be, q_bytes + k_bytes + v_bytes, &st);
    if (st) return st;
    __half *q16 = (__half *)scr, *k16 = (__half *)(scr + q_bytes), *vt16 = (__half *)(scr + q_bytes + k_bytes);
    const bool f16k = k->type == OASR_TYPE_F16;
    // the pre-pass moves 16-byte chunks: every caller's views (flash_attn_ext's and
    // flash_attn_causal's validated inputs, the model drivers' buffers) are 16-byte aligned
    const bool aligned = ((uintptr_t)q->data & 15) == 0 && q->nb[1] % 16 == 0 && q->nb[2] % 16 == 0 &&
                         q->nb[3] % 16 == 0 && ((uintptr_t)k->data & 15) == 0 && k->nb[1] % 16 == 0 &&
                         k->nb[2] % 16 == 0 && k->nb[3] % 16 == 0 && ((uintptr_t)v->data & 15) == 0 &&
                         v->nb[1] % 16 == 0 && v->nb[2] % 16 == 0 && v->nb[3] % 16 == 0;
    if (!aligned || (int64_t)S * H > 65535)
        return oasr_internal_fail(be, OASR_STATUS_FAILED,
                                  "flash_attn_tc: q/k/v rows must be 16-byte aligned and S * H <= 65535");
    fa_prep_tiled<false>(be, q, NQ, H, S, D, q16, false, 0);
    if (f16k) {
        fa_prep_tiled<true>(be, k, NKV, HKV, S, D, k16, false, 0);
        fa_prep_tiled<true>(be, v, NKV, HKV, S, D, vt16, true, n_pad);
    } else {
        fa_prep_tiled<false>(be, k, NKV, HKV, S, D, k16, false, 0);
        fa_prep_tiled<false>(be, v, NKV, HKV, S, D, vt16, true, n_pad);
    }
    st = oasr_internal_launch_check(be, "fa_prep");
    if (st) return st;
    // 64-element (128-byte) boxes: Q / K tiles of 128 rows, Vt half-tiles of D rows x 64 keys
    CUtensorMap mq, mk, mv;
    if (!encode_f16_2d(&mq, q16, (uint64_t)D, (uint64_t)S * H * NQ, 64, 128) ||
        !encode_f16_2d(&mk, k16, (uint64_t)D, (uint64_t)S * HKV * NKV, 64, 128) ||
        !encode_f16_2d(&mv, vt16, (uint64_t)n_pad, (uint64_t)S * HKV * D, 64, (uint32_t)D))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_tc: tensor map encoding failed");
    dim3 grid((unsigned)((NQ + 127) / 128), (unsigned)(S * H));
    const float scale_log2 = scale * 1.4426950408889634f;
    cudaError_t e;
    if (D == 64) e = causal ? launch_fa_tc<64, true>(be, grid, mq, mk, mv, NQ, NKV, H, HKV, scale_log2, dst)
                            : launch_fa_tc<64, false>(be, grid, mq, mk, mv, NQ, NKV, H, HKV, scale_log2, dst);
    else e = causal ? launch_fa_tc<128, true>(be, grid, mq, mk, mv, NQ, NKV, H, HKV, scale_log2, dst)
                    : launch_fa_tc<128, false>(be, grid, mq, mk, mv, NQ, NKV, H, HKV, scale_log2, dst);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "fattn_tc launch", __LINE__);
    return oasr_internal_launch_check(be, "fattn_tc");
}

}  // namespace oasr
