// fattn.cu -- K3: split-K flash attention over the f16 KV cache.
//
// Implements GGML_OP_FLASH_ATTN_EXT as built by
// GgmlCpuGraphBuilder::flash_attn_ext_with_precision (cpu_graph.rs:4144-4220):
//   O[:, h, iq, s] = softmax(scale * Q[:, iq, h, s] . K[:, :, h/G, s] + mask[:, iq]) V
// with GQA by integer division of the head index (q.ne2 % k.ne2 == 0,
// cpu_graph.rs:7476-7504), mask rows broadcast over ne2/ne3 (:7506-7519),
// positions whose mask is -inf skipped, and the output permuted to
// [D, H, n_q, S].  Q is rounded to K's type first (ggml converts Q to the
// vec_dot type of K), the Q.K products of two halves are exact in f32, and the
// softmax and V accumulation run in f32.
//
// Grid: (kv-head x seq x query-tile, split).  Each CTA streams a contiguous
// range of KV positions once with 16-byte loads (8 halves per lane, D/8 lanes
// per position, 32/(D/8) positions per warp step) for all query rows that
// share the kv head, keeps per-lane-group online-softmax state, merges it
// across lane groups and warps, and then either writes the output (one split)
// or its (max, sum, acc) partial; the last CTA of a group (atomic ticket, no
// waiting) merges the partials and resets the ticket.
#include <float.h>

#include <mutex>
#include <string>
#include <type_traits>

#include "kernels.cuh"
#include "fmath.cuh"
#include "quant_warp.cuh"

namespace oasr {

struct FaArgs {
    const char *q, *k, *v, *mask;
    char *dst;
    int64_t q_nb1, q_nb2, q_nb3;
    int64_t k_nb1, k_nb2, k_nb3;
    int64_t v_nb1, v_nb2, v_nb3;
    int64_t m_nb0, m_nb1, m_nb2, m_nb3;
    int64_t m_ne2, m_ne3;
    int64_t d_nb1, d_nb2, d_nb3;
    int NQ, H, HKV, S, NKV;
    int G;          // H / HKV
    int QG;         // G * NQ query rows per kv head
    int n_qtiles;   // ceil(QG / QT)
    int n_splits;
    int kv_per_split;
    float scale;
    float *partials;          // [rows][n_splits][D + 2]
    unsigned int *counters;   // one ticket per (kv head, seq, q tile)
    const float *q_bias;      // optional [H*D] added to q before the fp16 rounding
    const int *nkv_dev;       // optional device-side KV length of each sequence ([S], <= NKV), for
                              // graph-captured decode; the decode kernels may read it before their PDL
                              // wait, so no launch they can overlap writes it (the model drivers
                              // advance it between steps)
    // optional (GQA and 4-head decode kernels): the output rows [S][H * D] quantized to
    // activation planes instead of written as f32 -- the next mul_mat's input: quants oq
    // [S][H * D], scales od ([S][H * D / 32] q8_0, [S][H * D / 256] q8_K) and, for q8_K,
    // 16-wide sums obs [S][H * D / 16]
    int8_t *oq;
    float *od;
    int16_t *obs;
    int oq_family;
    // 4-head and GQA kernels, K/V rows that no launch this one can overlap under programmatic
    // dependent launch writes are loaded before the wait on the predecessor:
    // KV_STATIC_ALL every row (the cross-attention's encoder K/V); KV_STATIC_OLD every
    // row but the newest live one (self-attention: the predecessor writes row nkv_dev[s] - 1;
    // nkv_dev itself must not be written by an overlapping launch)
    int kv_static;
};

// One output element per thread of a full warp, 32 consecutive dims of one head per warp:
// quantize_row_q8_0 of the warp's block (d = amax / 127, q = round(v / d), d stored f16)
static __device__ __forceinline__ void store_q8_0_warp(float v, int8_t *q, float *d_slot, int lane) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    *q = (int8_t)(int)roundf(__fmul_rn(v, id));
    if (lane == 0) *d_slot = __half2float(__float2half_rn(d));
}

template <bool F16>
static __device__ __forceinline__ void load8(const char *p, float (&out)[8]) {
    if (F16) {
        const int4 r = *reinterpret_cast<const int4 *>(p);
        const __half2 *h = reinterpret_cast<const __half2 *>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    } else {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        const float4 b = *reinterpret_cast<const float4 *>(p + 16);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    }
}

// Copy n floats that other CTAs wrote (read through L2) into shared memory, 128
// threads, eight independent loads in flight per thread.
static __device__ __forceinline__ void stage_l2(float *dst, const float *src, int n) {
    for (int i0 = threadIdx.x; i0 < n; i0 += 8 * 128) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + j * 128;
            v[j] = i < n ? __ldcg(src + i) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + j * 128;
            if (i < n) dst[i] = v[j];
        }
    }
}

// Merge factors of the 4 warps of a CTA for row t (called by one thread per row):
// M = max_w m_w, f_w = m_w == -inf ? 0 : e^(m_w - M), L = sum_w l_w f_w (products fused, in
// warp order).  Each output element then adds its warps' accumulators with the same f_w, in
// the same order -- one set of exps per row instead of one per element.
template <int R>
static __device__ __forceinline__ void warp_merge_factors(const float (&m)[4][R], const float (&l)[4][R], int t,
                                                          float (&f)[4][R], float (&L)[R], float (&M)[R]) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, m[w][t]);
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const float fw = m[w][t] == -INFINITY ? 0.0f : exp_f32(__fsub_rn(m[w][t], mx));
        f[w][t] = fw;
        sum = __fmaf_rn(l[w][t], fw, sum);
    }
    L[t] = sum;
    M[t] = mx;
}

// The same for the n split partials of one row (pp = [split][D + 2]: acc[D], m, l), in split order.
static __device__ __forceinline__ void split_merge_factors(const float *pp, int n, int D, float *f, float *L) {
    float mx = -INFINITY;
    for (int sp = 0; sp < n; ++sp) mx = fmaxf(mx, pp[sp * (D + 2) + D]);
    float sum = 0.0f;
    for (int sp = 0; sp < n; ++sp) {
        const float m = pp[sp * (D + 2) + D];
        const float fs = m == -INFINITY ? 0.0f : exp_f32(__fsub_rn(m, mx));
        f[sp] = fs;
        sum = __fmaf_rn(pp[sp * (D + 2) + D + 1], fs, sum);
    }
    *L = sum;
}

constexpr int FA_HEADS_U = 8;            // KV positions per warp load batch (double buffered)
constexpr int FA_HEADS_MAX_SPLITS = 16;  // most KV splits of one query row (partials staged by the merging CTA)
constexpr int FA_GQA_U = 2;              // KV positions per lane group and load batch (double buffered)
constexpr int FA_SPLITS_HEADS = 7;       // KV splits of the 4-head decode kernel
constexpr int FA_HEADS_SPLIT_MIN = 513;  // shorter caches run unsplit (4-head kernel)
constexpr int FA_SPLITS_GQA = 4;         // KV splits of the GQA decode kernel

template <int D, int QT, bool F16>
__global__ void __launch_bounds__(128) fattn_split_kernel(FaArgs a) {
    griddep_launch_dependents();
    if (threadIdx.x == 0 && a.nkv_dev && a.k_nb1 == D * (F16 ? 2 : 4) && a.v_nb1 == a.k_nb1) {
        // decode over a cache whose rows of one head are contiguous: stream this CTA's K/V
        // rows toward L2 before the wait.  Only a hint (the range is recomputed below); the
        // KV length is set between steps, not by the predecessor kernel.
        const int g = blockIdx.x / a.n_qtiles, hk0 = g % a.HKV, s0 = g / a.HKV;
        const int nkv = min(a.nkv_dev[s0], a.NKV), per = (nkv + a.n_splits - 1) / a.n_splits;
        const int p0 = blockIdx.y * per, p1 = min(nkv, p0 + per);
        if (p1 > p0) {
            prefetch_l2_bulk(a.k + hk0 * a.k_nb2 + s0 * a.k_nb3 + (int64_t)p0 * a.k_nb1, (uint32_t)((p1 - p0) * a.k_nb1));
            prefetch_l2_bulk(a.v + hk0 * a.v_nb2 + s0 * a.v_nb3 + (int64_t)p0 * a.v_nb1, (uint32_t)((p1 - p0) * a.v_nb1));
        }
    }
    griddep_wait();
    constexpr int LPP = D / 8;        // lanes per KV position
    constexpr int PPW = 32 / LPP;     // positions per warp step
    constexpr int ES = F16 ? 2 : 4;   // element size
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = lane / LPP, sl = lane % LPP;  // position group in warp, lane in group
    const int split = blockIdx.y;
    int gid = blockIdx.x;
    const int qt = gid % a.n_qtiles;
    gid /= a.n_qtiles;
    const int hk = gid % a.HKV;
    const int s = gid / a.HKV;

    // query rows of this tile
    int qh[QT], qi[QT];
    bool qvalid[QT];
    float qv[QT][8];
#pragma unroll
    for (int t = 0; t < QT; ++t) {
        const int r = qt * QT + t;
        qvalid[t] = r < a.QG;
        const int rr = qvalid[t] ? r : 0;
        qh[t] = hk * a.G + rr / a.NQ;
        qi[t] = rr % a.NQ;
        const float *qp = reinterpret_cast<const float *>(a.q + qi[t] * a.q_nb1 + qh[t] * a.q_nb2 + s * a.q_nb3) + sl * 8;
        const float *qb = a.q_bias ? a.q_bias + qh[t] * D + sl * 8 : nullptr;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float x = qvalid[t] ? qp[e] : 0.0f;
            if (qb) x = __fadd_rn(x, qb[e]);
            qv[t][e] = F16 ? __half2float(__float2half_rn(x)) : x;
        }
    }
    const char *mrow[QT];
#pragma unroll
    for (int t = 0; t < QT; ++t)
        mrow[t] = a.mask ? a.mask + qi[t] * a.m_nb1 + (qh[t] % a.m_ne2) * a.m_nb2 + (s % a.m_ne3) * a.m_nb3 : nullptr;

    float mx[QT], sm[QT], acc[QT][8];
#pragma unroll
    for (int t = 0; t < QT; ++t) {
        mx[t] = -INFINITY;
        sm[t] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[t][e] = 0.0f;
    }

    // with a device-side KV length the splits share the live positions evenly
    const int nkv = a.nkv_dev ? min(a.nkv_dev[s], a.NKV) : a.NKV;
    const int per = a.nkv_dev ? (nkv + a.n_splits - 1) / a.n_splits : a.kv_per_split;
    const int kv0 = split * per;
    const int kv1 = min(nkv, kv0 + per);
    const char *kbase = a.k + hk * a.k_nb2 + s * a.k_nb3 + sl * 8 * ES;
    const char *vbase = a.v + hk * a.v_nb2 + s * a.v_nb3 + sl * 8 * ES;
    // U warp-steps of K/V rows are loaded before any is consumed so that each
    // lane keeps U x 2 16-byte (f16) loads in flight
    constexpr int U = 4;
    constexpr int RW = F16 ? 1 : 2;  // int4 words per lane per row
    for (int pb = kv0 + warp * PPW; pb < kv1; pb += 4 * PPW * U) {
        int4 kraw[U][RW], vraw[U][RW];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int p = pb + u * 4 * PPW + grp;
            if (p < kv1) {
#pragma unroll
                for (int r = 0; r < RW; ++r) {
                    kraw[u][r] = *reinterpret_cast<const int4 *>(kbase + (int64_t)p * a.k_nb1 + 16 * r);
                    vraw[u][r] = *reinterpret_cast<const int4 *>(vbase + (int64_t)p * a.v_nb1 + 16 * r);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
        const int p = pb + u * 4 * PPW + grp;
        const bool pv = p < kv1;
        float kf[8], vf[8];
        if (pv) {
            load8<F16>(reinterpret_cast<const char *>(kraw[u]), kf);
            load8<F16>(reinterpret_cast<const char *>(vraw[u]), vf);
        }
#pragma unroll
        for (int t = 0; t < QT; ++t) {
            float d = 0.0f;
            if (pv) {
#pragma unroll
                for (int e = 0; e < 8; ++e) d = __fmaf_rn(qv[t][e], kf[e], d);
            }
#pragma unroll
            for (int o = LPP / 2; o > 0; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, o));
            if (!pv || !qvalid[t]) continue;
            float sc = __fmul_rn(d, a.scale);
            if (mrow[t]) {
                const float mv = __half2float(*reinterpret_cast<const __half *>(mrow[t] + (int64_t)p * a.m_nb0));
                if (mv == -INFINITY) continue;
                sc = __fadd_rn(sc, mv);
            }
            const float mnew = fmaxf(mx[t], sc);
            const float corr = exp_f32(__fsub_rn(mx[t], mnew));  // mx = -inf -> 0
            const float w = exp_f32(__fsub_rn(sc, mnew));
            sm[t] = __fmaf_rn(sm[t], corr, w);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[t][e] = __fmaf_rn(w, vf[e], __fmul_rn(acc[t][e], corr));
            mx[t] = mnew;
        }
        }
    }

    // merge the PPW position groups of each warp (same sl, different grp)
#pragma unroll
    for (int t = 0; t < QT; ++t) {
#pragma unroll
        for (int o = LPP; o < 32; o <<= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, mx[t], o);
            const float os = __shfl_xor_sync(0xffffffffu, sm[t], o);
            const float nm = fmaxf(mx[t], om);
            const float f0 = mx[t] == -INFINITY ? 0.0f : exp_f32(__fsub_rn(mx[t], nm));
            const float f1 = om == -INFINITY ? 0.0f : exp_f32(__fsub_rn(om, nm));
            sm[t] = __fmaf_rn(os, f1, __fmul_rn(sm[t], f0));
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float oa = __shfl_xor_sync(0xffffffffu, acc[t][e], o);
                acc[t][e] = __fmaf_rn(oa, f1, __fmul_rn(acc[t][e], f0));
            }
            mx[t] = nm;
        }
    }
    // merge the 4 warps through shared memory
    __shared__ float s_m[4][QT], s_s[4][QT];
    __shared__ float s_acc[4][QT][D];
    if (grp == 0) {
#pragma unroll
        for (int t = 0; t < QT; ++t) {
#pragma unroll
            for (int e = 0; e < 8; ++e) s_acc[warp][t][sl * 8 + e] = acc[t][e];
            if (sl == 0) {
                s_m[warp][t] = mx[t];
                s_s[warp][t] = sm[t];
            }
        }
    }
    __syncthreads();
    // the 4 warps' merge factors of each query row, once per row (warp_merge_factors)
    __shared__ float s_f[4][QT], s_L[QT], s_M[QT];
    if (threadIdx.x < QT) warp_merge_factors<QT>(s_m, s_s, threadIdx.x, s_f, s_L, s_M);
    __syncthreads();
    // thread layout for the epilogue: QT*D outputs over 128 threads
    for (int o = threadIdx.x; o < QT * D; o += 128) {
        const int t = o / D, e = o % D;
        const float M = s_M[t], L = s_L[t];
        float A = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) A = __fmaf_rn(s_acc[w][t][e], s_f[w][t], A);
        const int r = qt * QT + t;
        if (r >= a.QG) continue;
        const int h = hk * a.G + r / a.NQ, iq = r % a.NQ;
        if (a.n_splits == 1) {
            float *out = reinterpret_cast<float *>(a.dst + h * a.d_nb1 + iq * a.d_nb2 + s * a.d_nb3);
            out[e] = L == 0.0f ? 0.0f : __fdiv_rn(A, L);
        } else {
            const int64_t row = ((int64_t)s * a.H + h) * a.NQ + iq;
            float *pp = a.partials + (row * a.n_splits + split) * (D + 2);
            pp[e] = A;
            if (e == 0) {
                pp[D] = M;
                pp[D + 1] = L;
            }
        }
    }
    if (a.n_splits == 1) return;

    // last CTA of this (kv head, seq, q tile) merges the split partials, one query row at
    // a time: the row's [split][D + 2] partials are staged in shared memory first
    if (!cta_last_arrival(a.counters + blockIdx.x, (unsigned)a.n_splits)) return;
    __shared__ float s_part[FA_HEADS_MAX_SPLITS * (D + 2)];
    for (int t = 0; t < QT; ++t) {
        const int r = qt * QT + t;
        if (r >= a.QG) break;  // CTA-uniform
        const int h = hk * a.G + r / a.NQ, iq = r % a.NQ;
        const int64_t row = ((int64_t)s * a.H + h) * a.NQ + iq;
        if (t > 0) __syncthreads();
        stage_l2(s_part, a.partials + row * a.n_splits * (D + 2), a.n_splits * (D + 2));
        __syncthreads();
        __shared__ float s_fs[FA_HEADS_MAX_SPLITS], s_Ls;
        if (threadIdx.x == 0) split_merge_factors(s_part, a.n_splits, D, s_fs, &s_Ls);
        __syncthreads();
        for (int e = threadIdx.x; e < D; e += 128) {
            const float L = s_Ls;
            float A = 0.0f;
            for (int sp = 0; sp < a.n_splits; ++sp) A = __fmaf_rn(s_part[sp * (D + 2) + e], s_fs[sp], A);
            float *out = reinterpret_cast<float *>(a.dst + h * a.d_nb1 + iq * a.d_nb2 + s * a.d_nb3);
            out[e] = L == 0.0f ? 0.0f : __fdiv_rn(A, L);
        }
    }
}

// The 4 heads' 256 outputs of a 4-head decode CTA (staged in s_out) are one 256-element
// chunk of the output row: warp 0 quantizes it into the next mul_mat's activation planes
// (q8_K: one super-block; q8_0: eight blocks).
static __device__ void heads_quantize_out(const FaArgs &a, const float *s_out, int s, int hg, int warp, int lane) {
    __syncthreads();
    if (warp != 0) return;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = s_out[8 * lane + i];
    const int64_t K = (int64_t)a.H * 64;
    int8_t *q = a.oq + s * K + 256 * hg;
    if (a.oq_family == FAMILY_Q8_K) q8k_chunk(v, q, a.od + s * (K / 256) + hg, a.obs + s * (K / 16) + 16 * hg, lane);
    else q80_chunk(v, q, a.od + s * (K / 32) + 8 * hg, lane);
}

// d plus the 8 products q_i k_i of two f16 octets as fused multiply-adds in element order
// (i = 0..7; element 2j is the low half of word j).  fma.rn.f32.f16 takes f16 operands,
// converts them to f32 exactly and rounds a * b + c once: each step is the value of
// __fmaf_rn(float(q_i), float(k_i), d), without separate conversions of the operands.
static __device__ __forceinline__ float dot8_f16(const int4 &q, const int4 &k, float d) {
    asm("{\n\t.reg .f16 q0, q1, q2, q3, q4, q5, q6, q7, k0, k1, k2, k3, k4, k5, k6, k7;\n\t"
        "mov.b32 {q0, q1}, %1;\n\tmov.b32 {q2, q3}, %2;\n\tmov.b32 {q4, q5}, %3;\n\tmov.b32 {q6, q7}, %4;\n\t"
        "mov.b32 {k0, k1}, %5;\n\tmov.b32 {k2, k3}, %6;\n\tmov.b32 {k4, k5}, %7;\n\tmov.b32 {k6, k7}, %8;\n\t"
        "fma.rn.f32.f16 %0, q0, k0, %0;\n\tfma.rn.f32.f16 %0, q1, k1, %0;\n\t"
        "fma.rn.f32.f16 %0, q2, k2, %0;\n\tfma.rn.f32.f16 %0, q3, k3, %0;\n\t"
        "fma.rn.f32.f16 %0, q4, k4, %0;\n\tfma.rn.f32.f16 %0, q5, k5, %0;\n\t"
        "fma.rn.f32.f16 %0, q6, k6, %0;\n\tfma.rn.f32.f16 %0, q7, k7, %0;\n\t}"
        : "+f"(d)
        : "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w), "r"(k.x), "r"(k.y), "r"(k.z), "r"(k.w));
    return d;
}

// 8 floats rounded to f16 and packed as the octet dot8_f16 takes
static __device__ __forceinline__ int4 pack8_f16(const float (&x)[8]) {
    int4 r;
    uint32_t *w = reinterpret_cast<uint32_t *>(&r);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(x[2 * j], x[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t *>(&h);
    }
    return r;
}

// One batch of a 4-head decode warp: U positions pb + 4u (u < U) of this lane group's
// head, K / V as 16-byte pieces (8 dims) per lane; positions >= kv1 carry zero rows and
// weight 0.  The U scores are independent: compute them all, then fold the block into the
// running softmax state with one rescale (a block-wise online softmax).  With U = 8 the
// 8 lanes of a head finish the 8 dot products as a transpose-reduce: at each butterfly
// level a lane keeps half of its partial sums and adds the partner's half, so lane sl
// ends with the whole dot of position sl (the same pairs added in the same order as a
// per-position butterfly: bit-identical scores), takes one exp instead of 8, and the
// weights are gathered back by shuffles.
template <int U>
static __device__ __forceinline__ void heads_consume(int pb, int kv1, float scale, int lane, int sl,
                                                     const int4 (&kr)[U], const int4 (&vr)[U], const int4 &qh,
                                                     float &mx, float &sm, float (&acc)[8]) {
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) sc[u] = dot8_f16(qh, kr[u], 0.0f);
    float wv[U];
    float mnew;
    if constexpr (U == 8) {
        const bool b4 = sl & 4, b2 = sl & 2, b1 = sl & 1;
        float r4[4], r2[2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float keep = b4 ? sc[j + 4] : sc[j], send = b4 ? sc[j] : sc[j + 4];
            r4[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float keep = b2 ? r4[j + 2] : r4[j], send = b2 ? r4[j] : r4[j + 2];
            r2[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 2));
        }
        const float keep = b1 ? r2[1] : r2[0], send = b1 ? r2[0] : r2[1];
        const float dot = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 1));  // position pb + 4 sl
        const float s1 = pb + 4 * sl < kv1 ? __fmul_rn(dot, scale) : -INFINITY;
        float mb = s1;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        mnew = fmaxf(mx, mb);                           // finite: position pb is valid
        const float w1 = exp_f32(__fsub_rn(s1, mnew));  // invalid positions: exp(-inf) = 0
#pragma unroll
        for (int u = 0; u < U; ++u) wv[u] = __shfl_sync(0xffffffffu, w1, (lane & ~7) | u);
    } else {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float d = sc[u];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, o));
            sc[u] = pb + 4 * u < kv1 ? __fmul_rn(d, scale) : -INFINITY;
        }
        float mb = sc[0];
#pragma unroll
        for (int u = 1; u < U; ++u) mb = fmaxf(mb, sc[u]);
        mnew = fmaxf(mx, mb);
#pragma unroll
        for (int u = 0; u < U; ++u) wv[u] = exp_f32(__fsub_rn(sc[u], mnew));
    }
    const float corr = exp_f32(__fsub_rn(mx, mnew));  // mx = -inf -> 0
    sm = __fmul_rn(sm, corr);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = __fmul_rn(acc[e], corr);
#pragma unroll
    for (int u = 0; u < U; ++u) {
        float vf[8];
        load8<true>(reinterpret_cast<const char *>(&vr[u]), vf);
        sm = __fadd_rn(sm, wv[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(wv[u], vf[e], acc[e]);
    }
    mx = mnew;
}

// The end of a 4-head decode CTA (warps 0-3 hold the online-softmax state of their
// positions; any further warps of the CTA take part in the barriers only): merge the 4
// warps through shared memory in warp order, then either write the outputs (one split) or
// the (acc, m, l) partial, and in the last-arriving CTA of the (sequence, head group) merge
// the splits in split order.  `scratch` holds 4 * FA_HEADS_MAX_SPLITS * 66 floats.
static __device__ __forceinline__ void heads_finish(const FaArgs &a, const float (&acc)[8], float mx, float sm, int s,
                                                    int hg, int split, int warp, int hl, int sl, int lane,
                                                    float *scratch) {
    constexpr int D = 64;
    const bool worker = threadIdx.x < 128;
    __shared__ float s_out[4 * D];  // the 4 heads' outputs when they leave as activation planes
    __shared__ float s_m[4][4], s_s[4][4];
    float(*s_acc)[4][D] = reinterpret_cast<float(*)[4][D]>(scratch);  // [warp][head][D]
    if (worker) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s_acc[warp][hl][sl * 8 + e] = acc[e];
        if (sl == 0) {
            s_m[warp][hl] = mx;
            s_s[warp][hl] = sm;
        }
    }
    __shared__ float s_f[4][4], s_L[4], s_M[4];
    __syncthreads();
    if (threadIdx.x < 4) warp_merge_factors<4>(s_m, s_s, threadIdx.x, s_f, s_L, s_M);
    __syncthreads();
    if (worker)
        for (int o = threadIdx.x; o < 4 * D; o += 128) {
            const int t = o / D, e = o % D;
            const float M = s_M[t], L = s_L[t];
            float A = 0.0f;
#pragma unroll
            for (int w = 0; w < 4; ++w) A = __fmaf_rn(s_acc[w][t][e], s_f[w][t], A);
            const int hh = 4 * hg + t;
            if (a.n_splits == 1) {
                const float val = L == 0.0f ? 0.0f : __fdiv_rn(A, L);
                if (a.oq) s_out[t * D + e] = val;
                else reinterpret_cast<float *>(a.dst + hh * a.d_nb1 + s * a.d_nb3)[e] = val;
            } else {
                const int64_t row = (int64_t)s * a.H + hh;
                float *pp = a.partials + (row * a.n_splits + split) * (D + 2);
                pp[e] = A;
                if (e == 0) {
                    pp[D] = M;
                    pp[D + 1] = L;
                }
            }
        }
    if (a.n_splits == 1) {
        if (a.oq) heads_quantize_out(a, s_out, s, hg, warp, lane);
        return;
    }
    if (!cta_last_arrival(a.counters + blockIdx.x, (unsigned)a.n_splits)) return;
    // the 4 heads' partials are contiguous ([head][split][D + 2]): stage them in shared
    // memory with every load in flight, then merge in split order
    float *s_part = scratch;  // the warps' accumulators are merged already
    const int nP = 4 * a.n_splits * (D + 2);
    const float *pbase = a.partials + ((int64_t)s * a.H + 4 * hg) * a.n_splits * (D + 2);
    __syncthreads();
    if (worker) stage_l2(s_part, pbase, nP);
    __syncthreads();
    __shared__ float s_fs[4][FA_HEADS_MAX_SPLITS], s_Ls[4];
    if (threadIdx.x < 4)
        split_merge_factors(s_part + threadIdx.x * a.n_splits * (D + 2), a.n_splits, D, s_fs[threadIdx.x],
                            &s_Ls[threadIdx.x]);
    __syncthreads();
    if (worker)
        for (int o = threadIdx.x; o < 4 * D; o += 128) {
            const int t = o / D, e = o % D;
            const float *pp = s_part + t * a.n_splits * (D + 2);
            const float L = s_Ls[t];
            float A = 0.0f;
            for (int sp = 0; sp < a.n_splits; ++sp) A = __fmaf_rn(pp[sp * (D + 2) + e], s_fs[t][sp], A);
            const float val = L == 0.0f ? 0.0f : __fdiv_rn(A, L);
            if (a.oq) s_out[t * D + e] = val;
            else reinterpret_cast<float *>(a.dst + (4 * hg + t) * a.d_nb1 + s * a.d_nb3)[e] = val;
        }
    if (a.oq) heads_quantize_out(a, s_out, s, hg, warp, lane);
}

// Decode attention with one query per (sequence, head) over f16 K/V whose heads lie
// contiguously in a KV row (the Whisper decoder's self- and cross-attention caches):
// a CTA takes 4 heads of one sequence and a range of KV positions, and every warp
// reads, per position, the 4 heads' 512 contiguous bytes of K and of V (8 lanes per
// head, 16 bytes per lane) with U positions of loads in flight, so the cache streams
// in long sequential runs.  Arithmetic as fattn_split_kernel<64, 1, true>: q rounded
// to f16, fmaf dot over 8 dims then the 8-lane shuffle tree, exp online softmax; the
// splits merge in the last-arriving CTA of each (sequence, head group).
template <int U>
__global__ void __launch_bounds__(128, 2) fattn_heads_kernel(FaArgs a) {
    constexpr int D = 64;
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hl = lane >> 3, sl = lane & 7;
    const int HG = a.H / 4;
    const int hg = blockIdx.x % HG, s = blockIdx.x / HG, split = blockIdx.y;
    const int h = 4 * hg + hl;
    const char *kb = a.k + h * a.k_nb2 + s * a.k_nb3 + sl * 16;
    const char *vb = a.v + h * a.v_nb2 + s * a.v_nb3 + sl * 16;

    float qv[8];
    int4 qh;  // qv as f16 octet
    float mx = -INFINITY, sm = 0.0f, acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    // with a device-side KV length the splits share the live positions evenly
    int kv0 = 0, kv1 = 0;
    auto range = [&]() {
        const int nkv = a.nkv_dev ? min(a.nkv_dev[s], a.NKV) : a.NKV;
        const int per = a.nkv_dev ? (nkv + a.n_splits - 1) / a.n_splits : a.kv_per_split;
        kv0 = split * per;
        kv1 = min(nkv, kv0 + per);
    };
    // register double buffering: the loads of the next U positions are in flight while
    // the current U are consumed
    auto load = [&](int pb, int4 (&kr)[U], int4 (&vr)[U]) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int p = pb + 4 * u;
            if (p < kv1) {
                kr[u] = *reinterpret_cast<const int4 *>(kb + (int64_t)p * a.k_nb1);
                vr[u] = *reinterpret_cast<const int4 *>(vb + (int64_t)p * a.v_nb1);
            } else {
                kr[u] = vr[u] = make_int4(0, 0, 0, 0);  // weight 0 below; keep 0 * v finite
            }
        }
    };
    auto consume = [&](int pb, const int4 (&kr)[U], const int4 (&vr)[U]) {
        heads_consume<U>(pb, kv1, a.scale, lane, sl, kr, vr, qh, mx, sm, acc);
    };

    int4 kA[U], vA[U], kB[U], vB[U];
    bool a_loaded = false, b_loaded = false;  // the first / second batch is already in flight
    const bool early = a.kv_static != KV_STATIC_NONE;
    if (early) {
        range();
        // rows below `lim` are final before the predecessor runs
        const int lim = a.kv_static == KV_STATIC_ALL ? kv1 : min(kv1, (a.nkv_dev ? a.nkv_dev[s] : a.NKV) - 1);
        const int p0 = kv0 + warp, p1 = p0 + 4 * U;
        if (p0 < kv1 && min(p0 + 4 * (U - 1), kv1 - 1) < lim) {
            load(p0, kA, vA);
            a_loaded = true;
            if (p1 < kv1 && min(p1 + 4 * (U - 1), kv1 - 1) < lim) {
                load(p1, kB, vB);
                b_loaded = true;
            }
        }
    }
    griddep_wait();
    {
        const float *qp = reinterpret_cast<const float *>(a.q + h * a.q_nb2 + s * a.q_nb3) + sl * 8;
        const float *qb = a.q_bias ? a.q_bias + h * D + sl * 8 : nullptr;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float x = qp[e];
            if (qb) x = __fadd_rn(x, qb[e]);
            qv[e] = __half2float(__float2half_rn(x));
        }
        qh = pack8_f16(qv);
    }
    if (!early) range();
    int pb = kv0 + warp;
    if (!a_loaded && pb < kv1) load(pb, kA, vA);
    while (pb < kv1) {
        int pn = pb + 4 * U;
        if (pn < kv1 && !b_loaded) load(pn, kB, vB);
        b_loaded = false;
        consume(pb, kA, vA);
        pb = pn;
        if (pb >= kv1) break;
        pn = pb + 4 * U;
        if (pn < kv1) load(pn, kA, vA);
        consume(pb, kB, vB);
        pb = pn;
    }

    __shared__ __align__(16) float s_scratch[4 * FA_HEADS_MAX_SPLITS * (D + 2)];
    heads_finish(a, acc, mx, sm, s, hg, split, warp, hl, sl, lane, s_scratch);
}

// Decode attention with grouped queries over head-major f16 caches (the Qwen decoder:
// [seq][kv head][pos][128], one kv head's positions in contiguous 256-byte rows): a CTA
// takes one (sequence, kv head), its G query heads and a range of positions.  Eight lanes
// share a position (16 dims = two 16-byte loads of K and of V per lane), so a warp covers
// four positions per step and all G heads reuse every K/V load; two batches of U
// positions per lane group are in flight in registers, and each batch is folded into the
// running softmax with one rescale per head.  Arithmetic as fattn_split_kernel<128, G,
// true>: q rounded to f16, fmaf dot over 16 dims then the 8-lane shuffle tree, exp online
// softmax; the splits merge in order in the last-arriving CTA of each (sequence, kv head).
template <int G, int U>
__global__ void __launch_bounds__(128) fattn_gqa_kernel(FaArgs a) {
    constexpr int D = 128;
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = lane >> 3, sl = lane & 7;  // position group in the warp, lane in the group
    const int hk = blockIdx.x % a.HKV, s = blockIdx.x / a.HKV, split = blockIdx.y;
    const char *kb = a.k + hk * a.k_nb2 + s * a.k_nb3 + sl * 32;
    const char *vb = a.v + hk * a.v_nb2 + s * a.v_nb3 + sl * 32;
    if (threadIdx.x == 0 && a.nkv_dev) {
        // stream this CTA's K/V rows toward L2 before the wait (a hint; the range is
        // recomputed below, and the KV length is set between steps)
        const int nk = min(a.nkv_dev[s], a.NKV), pp = (nk + a.n_splits - 1) / a.n_splits;
        const int p0 = split * pp, p1 = min(nk, p0 + pp);
        if (p1 > p0) {
            prefetch_l2_bulk(a.k + hk * a.k_nb2 + s * a.k_nb3 + (int64_t)p0 * a.k_nb1, (uint32_t)((p1 - p0) * a.k_nb1));
            prefetch_l2_bulk(a.v + hk * a.v_nb2 + s * a.v_nb3 + (int64_t)p0 * a.v_nb1, (uint32_t)((p1 - p0) * a.v_nb1));
        }
    }

    int4 qh[G][2];  // the G query rows' 16 dims of this lane, rounded to f16
    float mx_own = -INFINITY, sm[G], acc[G][16];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        sm[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[g][e] = 0.0f;
    }

    // the KV length is final before the launch (set between steps)
    const int nkv = a.nkv_dev ? min(a.nkv_dev[s], a.NKV) : a.NKV;
    const int per = a.nkv_dev ? (nkv + a.n_splits - 1) / a.n_splits : a.kv_per_split;
    const int kv0 = split * per;
    const int kv1 = min(nkv, kv0 + per);
    // positions of lane group (warp, grp) in a batch: pb + 16 u (pb = first position of
    // the batch for this group); a CTA batch covers 16 U positions
    constexpr int STEP = 16 * U;
    auto load = [&](int pb, int4 (&kr)[U][2], int4 (&vr)[U][2]) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int p = pb + 16 * u;
            if (p < kv1) {
                const int4 *kp = reinterpret_cast<const int4 *>(kb + (int64_t)p * a.k_nb1);
                const int4 *vp = reinterpret_cast<const int4 *>(vb + (int64_t)p * a.v_nb1);
                kr[u][0] = kp[0];
                kr[u][1] = kp[1];
                vr[u][0] = vp[0];
                vr[u][1] = vp[1];
            } else {
                kr[u][0] = kr[u][1] = vr[u][0] = vr[u][1] = make_int4(0, 0, 0, 0);  // weight 0 below
            }
        }
    };
    // One batch: the G x U partial dots of a lane (head g, position pb + 16 u at index
    // g U + u) are finished by a transpose-reduce over the group's 8 lanes -- at each
    // butterfly level a lane keeps half of its partial sums and adds the partner's half
    // (the pairs of a per-position butterfly, added in the same order: bit-identical
    // scores) -- so lane sl ends with the whole dot of index sl >> (3 - T) and takes
    // the batch's exps for that index and its head; the weights and rescale factors
    // are gathered back by shuffles.  The running maximum of head g lives on the lanes
    // that finish its dots (mx_own); a factor of exactly 1 leaves the state as it is.
    static_assert(U == 2, "the transposed batch holds two positions per lane group");
    constexpr int NV = G * U, T = NV == 8 ? 3 : NV == 4 ? 2 : 1;
    const int gbase = lane & ~7;
    auto consume = [&](int pb, const int4 (&kr)[U][2], const int4 (&vr)[U][2]) {
        float v[NV];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int g = 0; g < G; ++g) v[g * U + u] = dot8_f16(qh[g][1], kr[u][1], dot8_f16(qh[g][0], kr[u][0], 0.0f));
        int idx = 0;
        auto level = [&](auto n_c, int bit) {  // keep n of 2n partial sums
            constexpr int n = decltype(n_c)::value;
            const bool b = sl & bit;
#pragma unroll
            for (int j = 0; j < n; ++j) {
                const float keep = b ? v[j + n] : v[j], send = b ? v[j] : v[j + n];
                v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, bit));
            }
            idx += b ? n : 0;
        };
        level(std::integral_constant<int, NV / 2>{}, 4);
        if constexpr (T >= 2) level(std::integral_constant<int, NV / 4>{}, 2);
        else v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], 2));
        if constexpr (T >= 3) level(std::integral_constant<int, 1>{}, 1);
        else v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], 1));
        const float s1 = pb + 16 * (idx % U) < kv1 ? __fmul_rn(v[0], a.scale) : -INFINITY;
        const float mb = fmaxf(s1, __shfl_xor_sync(0xffffffffu, s1, 8 >> T));  // the other position
        const float mnew = fmaxf(mx_own, mb);
        const float c1 = mnew == -INFINITY ? 1.0f : exp_f32(__fsub_rn(mx_own, mnew));  // mx = -inf -> 0
        const float e1 = exp_f32(__fsub_rn(s1, mnew));
        const float w1 = s1 == -INFINITY ? -1.0f : e1;  // -1: no weight (invisible position)
        mx_own = mnew;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float corr = __shfl_sync(0xffffffffu, c1, gbase | ((g * U) << (3 - T)));
            if (corr != 1.0f) {
                sm[g] = __fmul_rn(sm[g], corr);
#pragma unroll
                for (int e = 0; e < 16; ++e) acc[g][e] = __fmul_rn(acc[g][e], corr);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float vf[16];
            load8<true>(reinterpret_cast<const char *>(&vr[u][0]), *reinterpret_cast<float(*)[8]>(&vf[0]));
            load8<true>(reinterpret_cast<const char *>(&vr[u][1]), *reinterpret_cast<float(*)[8]>(&vf[8]));
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float w = __shfl_sync(0xffffffffu, w1, gbase | ((g * U + u) << (3 - T)));
                if (w < 0.0f) continue;
                sm[g] = __fadd_rn(sm[g], w);
#pragma unroll
                for (int e = 0; e < 16; ++e) acc[g][e] = __fmaf_rn(w, vf[e], acc[g][e]);
            }
        }
    };
    int4 kA[U][2], vA[U][2], kB[U][2], vB[U][2];
    // warp-uniform loop bounds: every lane runs the same iterations (the shuffles need
    // all 32); positions past kv1 carry weight 0
    const int wbase = kv0 + 4 * warp;  // the warp's first position of a batch (group 0)
    // rows that no overlapping launch writes: the warp's first two batches load before the
    // wait on the predecessor when every live row of the batch is below `lim`
    bool a_loaded = false, b_loaded = false;
    if (a.kv_static != KV_STATIC_NONE) {
        const int lim = a.kv_static == KV_STATIC_ALL ? kv1 : min(kv1, nkv - 1);
        auto batch_static = [&](int p) { return p < kv1 && min(p + 3 + 16 * (U - 1), kv1 - 1) < lim; };
        if (batch_static(wbase)) {
            load(wbase + grp, kA, vA);
            a_loaded = true;
            if (batch_static(wbase + STEP)) {
                load(wbase + STEP + grp, kB, vB);
                b_loaded = true;
            }
        }
    }
    griddep_wait();
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float *qp = reinterpret_cast<const float *>(a.q + (hk * G + g) * a.q_nb2 + s * a.q_nb3) + sl * 16;
        float x[16];
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
            const float4 f = *reinterpret_cast<const float4 *>(qp + e);
            x[e] = f.x;
            x[e + 1] = f.y;
            x[e + 2] = f.z;
            x[e + 3] = f.w;
        }
        qh[g][0] = pack8_f16(*reinterpret_cast<const float(*)[8]>(&x[0]));
        qh[g][1] = pack8_f16(*reinterpret_cast<const float(*)[8]>(&x[8]));
    }
    int pb = wbase;
    if (!a_loaded && pb < kv1) load(pb + grp, kA, vA);
    while (pb < kv1) {
        int pn = pb + STEP;
        if (pn < kv1 && !b_loaded) load(pn + grp, kB, vB);
        b_loaded = false;
        consume(pb + grp, kA, vA);
        pb = pn;
        if (pb >= kv1) break;
        pn = pb + STEP;
        if (pn < kv1) load(pn + grp, kA, vA);
        consume(pb + grp, kB, vB);
        pb = pn;
    }

    // merge the warp's 4 position groups (same dims, different positions); head g's
    // running maximum from the lanes that kept it
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = __shfl_sync(0xffffffffu, mx_own, gbase | ((g * U) << (3 - T)));
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int o = 8; o < 32; o <<= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, mx[g], o);
            const float os = __shfl_xor_sync(0xffffffffu, sm[g], o);
            const float nm = fmaxf(mx[g], om);
            const float f0 = mx[g] == -INFINITY ? 0.0f : exp_f32(__fsub_rn(mx[g], nm));
            const float f1 = om == -INFINITY ? 0.0f : exp_f32(__fsub_rn(om, nm));
            sm[g] = __fmaf_rn(os, f1, __fmul_rn(sm[g], f0));
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float oa = __shfl_xor_sync(0xffffffffu, acc[g][e], o);
                acc[g][e] = __fmaf_rn(oa, f1, __fmul_rn(acc[g][e], f0));
            }
            mx[g] = nm;
        }
    }
    // merge the 4 warps through shared memory
    __shared__ float s_m[4][G], s_s[4][G];
    __shared__ float s_acc[4][G][D];
    if (grp == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int e = 0; e < 16; ++e) s_acc[warp][g][sl * 16 + e] = acc[g][e];
            if (sl == 0) {
                s_m[warp][g] = mx[g];
                s_s[warp][g] = sm[g];
            }
        }
    }
    __shared__ float s_f[4][G], s_L[G], s_M[G];
    __syncthreads();
    if (threadIdx.x < G) warp_merge_factors<G>(s_m, s_s, threadIdx.x, s_f, s_L, s_M);
    __syncthreads();
    for (int o = threadIdx.x; o < G * D; o += 128) {
        const int g = o / D, e = o % D;
        const float M = s_M[g], L = s_L[g];
        float A = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) A = __fmaf_rn(s_acc[w][g][e], s_f[w][g], A);
        const int h = hk * G + g;
        if (a.n_splits == 1) {
            const float val = L == 0.0f ? 0.0f : __fdiv_rn(A, L);
            if (a.oq) {
                const int64_t idx = ((int64_t)s * a.H + h) * D + e;
                store_q8_0_warp(val, a.oq + idx, a.od + idx / 32, lane);
            } else {
                reinterpret_cast<float *>(a.dst + h * a.d_nb1 + s * a.d_nb3)[e] = val;
            }
        } else {
            const int64_t row = (int64_t)s * a.H + h;
            float *pp = a.partials + (row * a.n_splits + split) * (D + 2);
            pp[e] = A;
            if (e == 0) {
                pp[D] = M;
                pp[D + 1] = L;
            }
        }
    }
    if (a.n_splits == 1) return;
    if (!cta_last_arrival(a.counters + blockIdx.x, (unsigned)a.n_splits)) return;
    // the G heads' partials are contiguous ([head][split][D + 2]): stage them in shared
    // memory with every load in flight, then merge in split order
    __shared__ float s_part[G * FA_HEADS_MAX_SPLITS * (D + 2)];
    const float *pbase = a.partials + ((int64_t)s * a.H + hk * G) * a.n_splits * (D + 2);
    stage_l2(s_part, pbase, G * a.n_splits * (D + 2));
    __syncthreads();
    __shared__ float s_fs[G][FA_HEADS_MAX_SPLITS], s_Ls[G];
    if (threadIdx.x < G)
        split_merge_factors(s_part + threadIdx.x * a.n_splits * (D + 2), a.n_splits, D, s_fs[threadIdx.x],
                            &s_Ls[threadIdx.x]);
    __syncthreads();
    for (int o = threadIdx.x; o < G * D; o += 128) {
        const int g = o / D, e = o % D;
        const float *pp = s_part + g * a.n_splits * (D + 2);
        const float L = s_Ls[g];
        float A = 0.0f;
        for (int sp = 0; sp < a.n_splits; ++sp) A = __fmaf_rn(pp[sp * (D + 2) + e], s_fs[g][sp], A);
        const float val = L == 0.0f ? 0.0f : __fdiv_rn(A, L);
        if (a.oq) {
            const int64_t idx = ((int64_t)s * a.H + hk * G + g) * D + e;
            store_q8_0_warp(val, a.oq + idx, a.od + idx / 32, lane);
        } else {
            reinterpret_cast<float *>(a.dst + (hk * G + g) * a.d_nb1 + s * a.d_nb3)[e] = val;
        }
    }
}

template <int D, bool F16>
static cudaError_t launch_fa_d(oasr_backend *be, const FaArgs &a, int QT, dim3 grid) {
    switch (QT) {
    case 1: return launch_k(be, fattn_split_kernel<D, 1, F16>, grid, dim3(128), 0, a);
    case 2: return launch_k(be, fattn_split_kernel<D, 2, F16>, grid, dim3(128), 0, a);
    case 4: return launch_k(be, fattn_split_kernel<D, 4, F16>, grid, dim3(128), 0, a);
    default: return launch_k(be, fattn_split_kernel<D, 8, F16>, grid, dim3(128), 0, a);
    }
}

int launch_flash_attn(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                      const oasr_tensor *mask, float scale, oasr_tensor *dst) {
    return launch_flash_attn_ex(be, q, k, v, mask, scale, dst, nullptr, nullptr);
}

// Split-KV scratch: `partials` of `partial_bytes` and `tickets` of `n_tickets` zeroed
// counters.  NULL partials = take them from the backend's (growable) scratch.
struct FaScratch {
    float *partials;
    size_t partial_bytes;
    unsigned int *tickets;
    int64_t n_tickets;
};

static int launch_flash_attn_split(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                                   const oasr_tensor *mask, float scale, oasr_tensor *dst, const float *q_bias,
                                   const int *nkv_dev, const FaScratch *fixed, const ActPlanes *out_q8 = nullptr,
                                   int out_family = FAMILY_Q8_0, int kv_static = 0);

// q_bias: optional [H*D] f32 added to q; nkv_dev: optional device KV length (k->ne[1] is the maximum)
int launch_flash_attn_ex(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                         const oasr_tensor *mask, float scale, oasr_tensor *dst, const float *q_bias,
                         const int *nkv_dev) {
    return launch_flash_attn_split(be, q, k, v, mask, scale, dst, q_bias, nkv_dev, nullptr);
}

int launch_flash_attn_decode_q8(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                                float scale, oasr_tensor *dst, const float *q_bias, const int *nkv_dev,
                                const ActPlanes &out_q8, int family, int kv_static) {
    return launch_flash_attn_split(be, q, k, v, nullptr, scale, dst, q_bias, nkv_dev, nullptr, &out_q8, family,
                                   kv_static);
}

bool flash_attn_decode_q8_supported(int H, int HKV, int D, int family) {
    const int G = HKV > 0 ? H / HKV : 0;
    if (D == 128) return family == FAMILY_Q8_0 && H % HKV == 0 && (G == 1 || G == 2 || G == 4);
    return D == 64 && H == HKV && H % 4 == 0;  // the 4-head kernel (one 256-value chunk per CTA)
}

// ---- allocation-free variant ------------------------------------------------------------
// File-scope device scratch for oasr_b200_flash_attn_ext_static: one copy per device,
// zero-initialised when the module loads.  The tickets must be zero when a launch
// starts; the last CTA of each split group resets its ticket, so they stay zero from
// one call to the next.  The partials need no initial value (every split writes its
// own slot before the merge reads it).
static __device__ __align__(256) float g_fa_static_partials[FA_STATIC_PARTIAL_BYTES / sizeof(float)];
static __device__ __align__(256) unsigned int g_fa_static_tickets[FA_STATIC_TICKETS];

int launch_flash_attn_static(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                             const oasr_tensor *mask, float scale, oasr_tensor *dst) {
    // symbol addresses, looked up once per device (the lookup may load the module,
    // so the first call on a device must not be inside a stream capture)
    static std::mutex mu;
    static void *partials[FA_STATIC_MAX_DEVICES] = {};
    static void *tickets[FA_STATIC_MAX_DEVICES] = {};
    if (be->device < 0 || be->device >= FA_STATIC_MAX_DEVICES)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext_static: device ordinal out of range");
    FaScratch fs;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!partials[be->device]) {
            cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
            if (cudaStreamIsCapturing(be->stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
                return oasr_internal_fail(be, OASR_STATUS_FAILED,
                                          "flash_attn_ext_static: first call on a device must precede stream capture");
            void *p = nullptr, *t = nullptr;
            OASR_CUDA_TRY(be, cudaGetSymbolAddress(&p, g_fa_static_partials));
            OASR_CUDA_TRY(be, cudaGetSymbolAddress(&t, g_fa_static_tickets));
            tickets[be->device] = t;
            partials[be->device] = p;
        }
        fs.partials = (float *)partials[be->device];
        fs.tickets = (unsigned int *)tickets[be->device];
    }
    fs.partial_bytes = FA_STATIC_PARTIAL_BYTES;
    fs.n_tickets = FA_STATIC_TICKETS;
    return launch_flash_attn_split(be, q, k, v, mask, scale, dst, nullptr, nullptr, &fs);
}

static int launch_flash_attn_split(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                                   const oasr_tensor *mask, float scale, oasr_tensor *dst, const float *q_bias,
                                   const int *nkv_dev, const FaScratch *fixed, const ActPlanes *out_q8,
                                   int out_family, int kv_static) {
    FaArgs a = {};
    a.q_bias = q_bias;
    a.nkv_dev = nkv_dev;
    const int D = (int)q->ne[0];
    a.q = (const char *)q->data;
    a.k = (const char *)k->data;
    a.v = (const char *)v->data;
    a.mask = mask ? (const char *)mask->data : nullptr;
    a.dst = (char *)dst->data;
    a.q_nb1 = q->nb[1]; a.q_nb2 = q->nb[2]; a.q_nb3 = q->nb[3];
    a.k_nb1 = k->nb[1]; a.k_nb2 = k->nb[2]; a.k_nb3 = k->nb[3];
    a.v_nb1 = v->nb[1]; a.v_nb2 = v->nb[2]; a.v_nb3 = v->nb[3];
    if (mask) {
        a.m_nb0 = mask->nb[0]; a.m_nb1 = mask->nb[1]; a.m_nb2 = mask->nb[2]; a.m_nb3 = mask->nb[3];
        a.m_ne2 = mask->ne[2]; a.m_ne3 = mask->ne[3];
    } else {
        a.m_nb0 = a.m_nb1 = a.m_nb2 = a.m_nb3 = 0;
        a.m_ne2 = a.m_ne3 = 1;
    }
    a.d_nb1 = dst->nb[1]; a.d_nb2 = dst->nb[2]; a.d_nb3 = dst->nb[3];
    a.NQ = (int)q->ne[1];
    a.H = (int)q->ne[2];
    a.S = (int)q->ne[3];
    a.HKV = (int)k->ne[2];
    a.NKV = (int)k->ne[1];
    a.G = a.H / a.HKV;
    a.QG = a.G * a.NQ;
    const int QT = a.QG >= 8 ? 8 : (a.QG >= 4 ? 4 : (a.QG >= 2 ? 2 : 1));
    a.n_qtiles = (a.QG + QT - 1) / QT;
    a.scale = scale;
    // one query per (sequence, head), f16 heads contiguous in a KV row: the 4-head kernel
    const bool heads = D == 64 && k->type == OASR_TYPE_F16 && v->type == OASR_TYPE_F16 && a.NQ == 1 && a.G == 1 &&
                       !mask && a.H % 4 == 0 && k->nb[2] == 2 * D && v->nb[2] == 2 * D &&
                       k->nb[1] % 16 == 0 && k->nb[3] % 16 == 0 && v->nb[1] % 16 == 0 && v->nb[3] % 16 == 0 &&
                       ((uintptr_t)k->data & 15) == 0 && ((uintptr_t)v->data & 15) == 0 &&
                       a.S * (int64_t)(a.H / 4) <= (1 << 16);
    // one query per (sequence, head) over head-major f16 caches with 256-byte rows: the GQA kernel
    const bool gqa = !heads && D == 128 && k->type == OASR_TYPE_F16 && v->type == OASR_TYPE_F16 && a.NQ == 1 &&
                     !mask && !q_bias && (a.G == 1 || a.G == 2 || a.G == 4) && k->nb[1] == 256 && v->nb[1] == 256 &&
                     k->nb[2] % 16 == 0 && k->nb[3] % 16 == 0 && v->nb[2] % 16 == 0 && v->nb[3] % 16 == 0 &&
                     q->nb[2] % 16 == 0 && q->nb[3] % 16 == 0 && ((uintptr_t)q->data & 15) == 0 &&
                     ((uintptr_t)k->data & 15) == 0 && ((uintptr_t)v->data & 15) == 0 &&
                     (int64_t)a.S * a.HKV <= 0x7fffffffLL;
    if (heads || gqa) a.kv_static = kv_static;

    if (out_q8) {
        if (!((gqa && out_family == FAMILY_Q8_0) || (heads && D == 64)))
            return oasr_internal_fail(be, OASR_STATUS_FAILED,
                                      "flash_attn: activation-plane output needs the GQA (q8_0) or 4-head decode kernel");
        a.oq = out_q8->qs;
        a.od = out_q8->d;
        a.obs = out_q8->bs16;
        a.oq_family = out_family;
    }
    const int64_t groups = heads ? (int64_t)a.S * (a.H / 4) : gqa ? (int64_t)a.S * a.HKV : (int64_t)a.HKV * a.S * a.n_qtiles;
    // The split plan depends on the kernel and the cache length only -- never on the
    // batch width, the other groups or the device -- so a sequence's output has the same
    // bits whatever batch it runs in and on whichever GPU (the reference's batched ==
    // serial property, and what lets a serving scheduler regroup sequences freely).
    // The counts are the one-wave plans of a 148-SM B200 at 8 sequences (Whisper-large
    // heads: 40 groups x 7 at 2 CTAs/SM; Qwen GQA: 64 groups x 4), at least 32 (64)
    // positions per split.  Tickets exist for 2^16 groups.
    int n_splits = 1;
    if (groups <= (1 << 16)) {
        // 4-head kernel: a cache of at most 512 positions (the decoder's self-attention,
        // n_text_ctx 448) is one split per CTA -- the outputs are written directly, with no
        // partials, tickets or merge, whose fixed cost exceeds the extra batches per warp
        if (heads) n_splits = a.NKV < FA_HEADS_SPLIT_MIN ? 1 : std::min(FA_SPLITS_HEADS, a.NKV / 32);
        else if (gqa) n_splits = std::min(FA_SPLITS_GQA, a.NKV / 32);
        else n_splits = std::min(FA_HEADS_MAX_SPLITS, a.NKV / 64);
        n_splits = std::max(1, n_splits);
    }
    a.n_splits = n_splits;
    a.kv_per_split = (a.NKV + n_splits - 1) / n_splits;
    a.partials = nullptr;
    a.counters = fixed ? fixed->tickets : be->counters;
    if (groups > 0x7fffffffLL) return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn: grid too large");
    if (n_splits > 1) {
        const size_t bytes = (size_t)a.S * a.H * a.NQ * n_splits * (D + 2) * sizeof(float);
        if (fixed) {
            if (bytes > fixed->partial_bytes || groups > fixed->n_tickets)
                return oasr_internal_fail(
                    be, OASR_STATUS_FAILED,
                    "flash_attn_ext_static: split-KV partials need " + std::to_string(bytes) + " bytes and " +
                        std::to_string(groups) + " tickets; the static scratch holds " +
                        std::to_string(fixed->partial_bytes) + " bytes and " + std::to_string(fixed->n_tickets) +
                        " tickets (use oasr_b200_flash_attn_ext)");
            a.partials = fixed->partials;
        } else {
            int st = 0;
            a.partials = (float *)oasr_internal_scratch(be, bytes, &st);
            if (st) return st;
        }
    }
    dim3 grid((unsigned)groups, n_splits);
    const bool f16 = k->type == OASR_TYPE_F16;
    cudaError_t e;
    if (heads) e = launch_k(be, fattn_heads_kernel<FA_HEADS_U>, grid, dim3(128), 0, a);
    else if (gqa) e = a.G == 1 ? launch_k(be, fattn_gqa_kernel<1, FA_GQA_U>, grid, dim3(128), 0, a)
                    : a.G == 2 ? launch_k(be, fattn_gqa_kernel<2, FA_GQA_U>, grid, dim3(128), 0, a)
                               : launch_k(be, fattn_gqa_kernel<4, FA_GQA_U>, grid, dim3(128), 0, a);
    else if (D == 64) e = f16 ? launch_fa_d<64, true>(be, a, QT, grid) : launch_fa_d<64, false>(be, a, QT, grid);
    else e = f16 ? launch_fa_d<128, true>(be, a, QT, grid) : launch_fa_d<128, false>(be, a, QT, grid);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "flash_attn launch", __LINE__);
    return oasr_internal_launch_check(be, "flash_attn");
}

}  // namespace oasr
