// dgemv.cu -- the decoder step's GEMVs with their neighbours fused in.
//
// A decoder layer (ggml_decoder_graph.rs:2840-3010) runs, per step and for up
// to 8 utterances, LN -> QKV -> self-attention -> out -> residual -> LN ->
// cross-q -> cross-attention -> out -> residual -> LN -> fc1 -> GELU -> fc2 ->
// residual.  Every linear needs its input quantized to the weight's vec_dot
// type first (q8_K for Q4_K, q8_0 for Q8_0).  The GEMVs here (the MMA core of
// mmv_tc.cu over decode tiles) absorb the two neighbours that need no row-wide
// reduction across CTAs:
//   prologue PRO_QUANT  the attention output rows (8 x d f32) are quantized by
//                       every CTA into shared memory, all loads issued first
//   epilogue EPI_QKV    q + b_q -> f32; k, v + b_v -> f16 self-KV cache row *pos
// (the row-wide LayerNorm and the GELU + quantize stay separate chunk-parallel
// kernels in elementwise.cu: a single-CTA tail for them measured slower than a
// kernel boundary).  Arithmetic as quantize_q8_* and qkv_split_kv_write.
#include "mma_frag.cuh"
#include "model.cuh"
#include "quant_warp.cuh"

namespace oasr {

enum { PRO_PLANES = 0, PRO_QUANT = 1 };
enum { EPI_STORE = 0, EPI_QKV = 1 };

constexpr int DG_WARPS = 8;
constexpr int DG_ROWS = 8;         // activation rows (rows >= M are zero / never stored)
constexpr int DG_MAX_CHUNKS = 8;   // 256-chunks a warp loads before quantizing (PRO_QUANT)
constexpr int DG_SMEM_MAX = 200 << 10;

struct DgemvArgs {
    const uint8_t *tiles;
    int units;  // super-blocks (Q4_K) or block pairs (Q8_0) per row
    int terms_bytes;  // shared memory of one segment of block terms
    int64_t N;
    int K, M;
    // PRO_PLANES: quantized activations (family of the weight)
    ActPlanes in;
    // PRO_QUANT: f32 rows [M][K]
    const float *h;
    // EPI_STORE output rows [M][y_ld]
    float *y;
    int64_t y_ld;
    // EPI_QKV
    const float *bias3;
    float *q_out;
    __half *kc, *vc;
    int64_t cache_seq_stride;
    const int *pos;  // EPI_QKV: cache row of each activation row [M]
    int max_pos, d;
    int *err;
};

static __device__ __forceinline__ void ld8(const float *p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(p);
    const float4 b = *reinterpret_cast<const float4 *>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// ---- PRO_QUANT: f32 rows -> shared q8 planes ----------------------------------------------------
struct DgSmem {
    int8_t *aq;     // [8][K + 32]
    float *ad;      // [8][nd]
    int16_t *ab;    // [8][K / 16] (q8_K)
    float *terms;   // one segment of block terms (mma_frag.cuh)
    int aq_ld, nd;
};

// block terms per unit (Q4_K: one super-block; Q8_0: a block pair) and rounds per segment
template <int FAM>
struct DgTerms {
    static constexpr int BPU = FAM == FAMILY_Q8_K ? 1 : 2;
    static constexpr int SEGJ = TERM_SEG_BLOCKS / (DG_WARPS * BPU);
};

static inline size_t dg_terms_bytes(int fam, int units) {
    return fam == FAMILY_Q8_K ? term_smem_bytes<DG_WARPS, 1, DgTerms<FAMILY_Q8_K>::SEGJ>(units)
                              : term_smem_bytes<DG_WARPS, 2, DgTerms<FAMILY_Q8_0>::SEGJ>(units);
}

static __host__ __device__ inline size_t dg_align16(size_t x) { return (x + 15) & ~(size_t)15; }

static inline size_t dg_smem_bytes(int fam, int pro, int K) {
    size_t b = dg_align16(dg_terms_bytes(fam, fam == FAMILY_Q8_K ? K / 256 : K / 64));
    if (pro == PRO_QUANT) {
        const int nd = fam == FAMILY_Q8_K ? K / 256 : K / 32;
        b += dg_align16((size_t)DG_ROWS * (K + 32)) + dg_align16((size_t)DG_ROWS * nd * 4);
        if (fam == FAMILY_Q8_K) b += dg_align16((size_t)DG_ROWS * (K / 16) * 2);
    }
    return b;
}

// terms first (their size is the launch's: rounds of the segment), the planes after them
static __device__ inline DgSmem dg_carve(char *base, int fam, int pro, int K, size_t terms_bytes) {
    DgSmem s;
    s.terms = (float *)base;
    size_t off = terms_bytes;
    s.aq_ld = K + 32;
    s.nd = fam == FAMILY_Q8_K ? K / 256 : K / 32;
    s.aq = nullptr;
    s.ad = nullptr;
    s.ab = nullptr;
    if (pro == PRO_QUANT) {
        s.aq = (int8_t *)(base + off);
        off += dg_align16((size_t)DG_ROWS * s.aq_ld);
        s.ad = (float *)(base + off);
        off += dg_align16((size_t)DG_ROWS * s.nd * 4);
        if (fam == FAMILY_Q8_K) s.ab = (int16_t *)(base + off);
    }
    return s;
}

// units (row m, 256-chunk c) spread over the 8 warps; every load of a batch is issued
// before any arithmetic.  Rows >= M are zero.
template <int FAM>
static __device__ void pro_quant(const DgemvArgs &a, const DgSmem &sm, int warp, int lane) {
    const int nch = a.K / 256, total = DG_ROWS * nch;
    for (int base = 0; base < total; base += DG_WARPS * DG_MAX_CHUNKS) {
        float v[DG_MAX_CHUNKS][8];
#pragma unroll
        for (int j = 0; j < DG_MAX_CHUNKS; ++j) {
            const int u = base + warp + DG_WARPS * j;
            const int m = u / nch, c = u - m * nch;
            if (u < total && m < a.M) {
                ld8(a.h + (int64_t)m * a.K + 256 * c + 8 * lane, v[j]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[j][i] = 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < DG_MAX_CHUNKS; ++j) {
            const int u = base + warp + DG_WARPS * j;
            if (u >= total) continue;
            const int m = u / nch, c = u - m * nch;
            int8_t *q = sm.aq + m * sm.aq_ld + 256 * c;
            if (FAM == FAMILY_Q8_K) q8k_chunk(v[j], q, sm.ad + m * sm.nd + c, sm.ab + m * (a.K / 16) + 16 * c, lane);
            else q80_chunk(v[j], q, sm.ad + m * sm.nd + 8 * c, lane);
        }
    }
}

// ---- the kernel -------------------------------------------------------------------------------
// UPW > 0: warp w takes units w, w + 8, ... (UPW of them), all loaded before the wait;
// UPW = 0: looping form with one unit in flight ahead of the one in use.
template <int FAM, int PRO, int EPI, int UPW>
__global__ void __launch_bounds__(DG_WARPS * 32, 2) dgemv_kernel(DgemvArgs a) {
    extern __shared__ __align__(16) char dg_smem[];
    constexpr int BPU = DgTerms<FAM>::BPU, SEGJ = DgTerms<FAM>::SEGJ;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const DgSmem sm = dg_carve(dg_smem, FAM, PRO, a.K, a.terms_bytes);
    constexpr int UNIT = FAM == FAMILY_Q8_K ? Q4K_UNIT : Q80_UNIT;
    const uint8_t *tile = a.tiles + (int64_t)blockIdx.x * a.units * UNIT;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    // weights first (they do not depend on the previous kernel)
    griddep_launch_dependents();
    constexpr int NU = UPW > 0 ? UPW : 1;
    Q4kUnit ck[FAM == FAMILY_Q8_K ? NU : 1], nk;
    Q80Unit c8[FAM == FAMILY_Q8_K ? 1 : NU], n8;
    if (UPW > 0) {
#pragma unroll
        for (int j = 0; j < NU; ++j) {
            const int uj = warp + j * DG_WARPS;
            if (uj < a.units) {
                if (FAM == FAMILY_Q8_K) load_q4k_unit(ck[j], tile + (int64_t)uj * UNIT, lane, g);
                else load_q80_unit(c8[j], tile + (int64_t)uj * UNIT, lane, g);
            }
        }
    } else {
        // the whole tile streams toward L2 while the first units load into registers
        if (threadIdx.x == 0) prefetch_l2_bulk(tile, (uint32_t)a.units * UNIT);
        if (warp < a.units) {
            if (FAM == FAMILY_Q8_K) load_q4k_unit(ck[0], tile + (int64_t)warp * UNIT, lane, g);
            else load_q80_unit(c8[0], tile + (int64_t)warp * UNIT, lane, g);
        }
    }
    griddep_wait();

    const int m0 = 2 * t, m1 = 2 * t + 1;
    const int8_t *arow;
    const int16_t *brow = nullptr;
    const float *adrow0, *adrow1;  // activation scale rows of C columns 2t, 2t+1 (null past M)
    constexpr bool SM = PRO == PRO_QUANT;
    if (SM) {
        pro_quant<FAM>(a, sm, warp, lane);
        __syncthreads();
        arow = sm.aq + g * sm.aq_ld;
        if (FAM == FAMILY_Q8_K) brow = sm.ab + g * (a.K / 16);
        adrow0 = sm.ad + m0 * sm.nd;
        adrow1 = sm.ad + m1 * sm.nd;
    } else {
        const int gr = g < a.M ? g : 0;
        arow = a.in.qs + (int64_t)gr * a.K;
        if (FAM == FAMILY_Q8_K) brow = a.in.bs16 + (int64_t)gr * (a.K / 16);
        const int nd = FAM == FAMILY_Q8_K ? a.K / 256 : a.K / 32;
        adrow0 = m0 < a.M ? a.in.d + (int64_t)m0 * nd : nullptr;
        adrow1 = m1 < a.M ? a.in.d + (int64_t)m1 * nd : nullptr;
    }
    // one unit's block terms into its segment slot
    auto terms_of = [&](int j, int uj, const Q4kUnit &qk, const Q80Unit &q8) {
        float *slot = term_slot<DG_WARPS, BPU, SEGJ>(sm.terms, j, warp);
        if (FAM == FAMILY_Q8_K) {
            const float da0 = adrow0 ? (SM ? adrow0[uj] : __ldg(adrow0 + uj)) : 0.0f;
            const float da1 = adrow1 ? (SM ? adrow1[uj] : __ldg(adrow1 + uj)) : 0.0f;
            q4k_unit_terms<SM>(slot, qk, uj, arow, brow, da0, da1, lane, t);
        } else {
            q80_unit_terms<SM>(slot, q8, uj, arow, adrow0, adrow1, lane, t);
        }
    };
    const int nrounds = (a.units + DG_WARPS - 1) / DG_WARPS;
    if (UPW > 0) {
#pragma unroll
        for (int j = 0; j < NU; ++j) {
            if (j >= nrounds) break;  // CTA-uniform
            const int uj = warp + j * DG_WARPS;
            if (uj < a.units) terms_of(j, uj, ck[FAM == FAMILY_Q8_K ? j : 0], c8[FAM == FAMILY_Q8_K ? 0 : j]);
            segment_end<DG_WARPS, BPU, SEGJ>(acc, sm.terms, j, nrounds, a.units, warp, lane);
        }
    } else {
        for (int j = 0; j < nrounds; ++j) {
            const int u = j * DG_WARPS + warp;
            if (u < a.units) {
                const bool more = u + DG_WARPS < a.units;
                if (FAM == FAMILY_Q8_K) {
                    if (more) load_q4k_unit(nk, tile + (int64_t)(u + DG_WARPS) * UNIT, lane, g);
                    terms_of(j, u, ck[0], c8[0]);
                    if (more) ck[0] = nk;
                } else {
                    if (more) load_q80_unit(n8, tile + (int64_t)(u + DG_WARPS) * UNIT, lane, g);
                    terms_of(j, u, ck[0], c8[0]);
                    if (more) c8[0] = n8;
                }
            }
            segment_end<DG_WARPS, BPU, SEGJ>(acc, sm.terms, j, nrounds, a.units, warp, lane);
        }
    }
    if (warp != 0) return;

    const int64_t ra = (int64_t)blockIdx.x * TILE_ROWS + g, rb = ra + 8;
    {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int64_t n = (e < 2) ? ra : rb;
            const int m = (e & 1) ? m1 : m0;
            if (n >= a.N || m >= a.M) continue;
            if (EPI == EPI_QKV) {
                const int pos = a.pos[m];
                const float v = a.bias3 ? __fadd_rn(acc[e], a.bias3[n]) : acc[e];
                if (n < a.d) {
                    a.q_out[(int64_t)m * a.d + n] = v;
                } else if (pos < 0 || pos >= a.max_pos) {
                    atomicOr(a.err, ERR_BAD_INDEX);
                } else {
                    __half *cache = n < 2 * a.d ? a.kc : a.vc;
                    const int64_t col = n < 2 * a.d ? n - a.d : n - 2 * a.d;
                    cache[(int64_t)m * a.cache_seq_stride + (int64_t)pos * a.d + col] = __float2half_rn(v);
                }
            } else {
                a.y[(int64_t)m * a.y_ld + n] = acc[e];
            }
        }
    }
}

// ---- host side ----------------------------------------------------------------------------------
template <int FAM, int PRO, int EPI>
static cudaError_t dg_set_attr() {
    cudaError_t e = cudaSuccess;
    // the instantiations dg_launch can pick (Q4_K units hold 26 registers: one per warp at most)
    if constexpr (FAM == FAMILY_Q8_K) {
        for (auto fn : {dgemv_kernel<FAM, PRO, EPI, 0>, dgemv_kernel<FAM, PRO, EPI, 1>})
            if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, DG_SMEM_MAX);
    } else {
        for (auto fn : {dgemv_kernel<FAM, PRO, EPI, 0>, dgemv_kernel<FAM, PRO, EPI, 1>, dgemv_kernel<FAM, PRO, EPI, 2>,
                        dgemv_kernel<FAM, PRO, EPI, 4>})
            if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, DG_SMEM_MAX);
    }
    return e;
}

template <int FAM>
static cudaError_t dg_set_attr_fam() {
    cudaError_t e = dg_set_attr<FAM, PRO_PLANES, EPI_STORE>();
    if (e == cudaSuccess) e = dg_set_attr<FAM, PRO_PLANES, EPI_QKV>();
    if (e == cudaSuccess) e = dg_set_attr<FAM, PRO_QUANT, EPI_STORE>();
    return e;
}

static std::atomic<bool> g_dg_configured[64];  // per device: attributes raised (first call may race)

// Raise the dynamic shared memory limit of every instantiation once per device
// (model load calls this, outside any stream capture).
int dgemv_configure(oasr_backend *be) {
    if (be->device < 0 || be->device >= 64) return oasr_internal_fail(be, OASR_STATUS_FAILED, "dgemv: device ordinal");
    if (g_dg_configured[be->device].load(std::memory_order_acquire)) return OASR_STATUS_SUCCESS;
    OASR_CUDA_TRY(be, dg_set_attr_fam<FAMILY_Q8_K>());
    OASR_CUDA_TRY(be, dg_set_attr_fam<FAMILY_Q8_0>());
    g_dg_configured[be->device].store(true, std::memory_order_release);  // idempotent: racing callers set the same attributes
    return OASR_STATUS_SUCCESS;
}

template <int FAM, int PRO, int EPI>
static int dg_launch(oasr_backend *be, const DgemvArgs &a0) {
    if (be->device < 0 || be->device >= 64 || !g_dg_configured[be->device].load(std::memory_order_acquire))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "dgemv: dgemv_configure was not called on this device");
    DgemvArgs a = a0;
    a.terms_bytes = (int)dg_align16(dg_terms_bytes(FAM, a.units));
    const size_t smem = dg_smem_bytes(FAM, PRO, a.K);
    const unsigned grid = (unsigned)((a.N + TILE_ROWS - 1) / TILE_ROWS);
    // all of a warp's units in flight at once, up to 4 (Q8_0) or 1 (Q4_K) per warp, else looping
    const int upw = (a.units + DG_WARPS - 1) / DG_WARPS;
    cudaError_t e;
    if (upw <= 1) {
        e = launch_k(be, dgemv_kernel<FAM, PRO, EPI, 1>, dim3(grid), dim3(DG_WARPS * 32), smem, a);
    } else if constexpr (FAM == FAMILY_Q8_K) {
        e = launch_k(be, dgemv_kernel<FAM, PRO, EPI, 0>, dim3(grid), dim3(DG_WARPS * 32), smem, a);
    } else {
        if (upw <= 2) e = launch_k(be, dgemv_kernel<FAM, PRO, EPI, 2>, dim3(grid), dim3(DG_WARPS * 32), smem, a);
        else if (upw <= 4) e = launch_k(be, dgemv_kernel<FAM, PRO, EPI, 4>, dim3(grid), dim3(DG_WARPS * 32), smem, a);
        else e = launch_k(be, dgemv_kernel<FAM, PRO, EPI, 0>, dim3(grid), dim3(DG_WARPS * 32), smem, a);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "dgemv launch", __LINE__);
    return oasr_internal_launch_check(be, "dgemv");
}

template <int PRO, int EPI>
static int dg_dispatch(oasr_backend *be, const oasr_weight *w, const DgemvArgs &a) {
    if (w->type == OASR_TYPE_Q4_K) return dg_launch<FAMILY_Q8_K, PRO, EPI>(be, a);
    return dg_launch<FAMILY_Q8_0, PRO, EPI>(be, a);
}

bool dgemv_supported(const oasr_weight *w, bool quant_prologue) {
    if (!w || !w->tiles || (w->type != OASR_TYPE_Q4_K && w->type != OASR_TYPE_Q8_0) || w->ne[0] % 256) return false;
    const int fam = w->type == OASR_TYPE_Q4_K ? FAMILY_Q8_K : FAMILY_Q8_0;
    return dg_smem_bytes(fam, quant_prologue ? PRO_QUANT : PRO_PLANES, (int)w->ne[0]) <= DG_SMEM_MAX;
}

static DgemvArgs dg_base(const oasr_weight *w, int M) {
    DgemvArgs a = {};
    a.tiles = w->tiles;
    a.K = (int)w->ne[0];
    a.N = w->ne[1];
    a.M = M;
    a.units = w->type == OASR_TYPE_Q4_K ? a.K / 256 : a.K / 64;
    return a;
}

int launch_dgemv(oasr_backend *be, const oasr_weight *w, const ActPlanes &in, int M, float *y, int64_t y_ld) {
    DgemvArgs a = dg_base(w, M);
    a.in = in;
    a.y = y;
    a.y_ld = y_ld;
    return dg_dispatch<PRO_PLANES, EPI_STORE>(be, w, a);
}

int launch_dgemv_qkv(oasr_backend *be, const oasr_weight *w, const ActPlanes &in, int M, const float *bias3, int d,
                     float *q_out, __half *kc, __half *vc, int64_t cache_seq_stride, const int *pos_dev, int max_pos) {
    DgemvArgs a = dg_base(w, M);
    a.in = in;
    a.bias3 = bias3;
    a.d = d;
    a.q_out = q_out;
    a.kc = kc;
    a.vc = vc;
    a.cache_seq_stride = cache_seq_stride;
    a.pos = pos_dev;
    a.max_pos = max_pos;
    a.err = be->err_word;
    return dg_dispatch<PRO_PLANES, EPI_QKV>(be, w, a);
}

int launch_dgemv_quant(oasr_backend *be, const oasr_weight *w, const float *h, int M, float *y, int64_t y_ld) {
    DgemvArgs a = dg_base(w, M);
    a.h = h;
    a.y = y;
    a.y_ld = y_ld;
    return dg_dispatch<PRO_QUANT, EPI_STORE>(be, w, a);
}

}  // namespace oasr
