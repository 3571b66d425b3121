// mmv.cu -- K1: dequant-fused decode GEMV / skinny GEMM (M <= 8 activation rows).
//
// Replaces ggml-cuda's mul_mat_vec_q for the decode mul_mat nodes built by
// GgmlCpuGraphBuilder::mul_mat (cpu_graph.rs:3616-3686): weight rows stream
// from HBM exactly once with 128-bit non-allocating loads, the int8/int4
// quants are dotted against the pre-quantized activations with dp4a, and the
// per-block f32 term is formed exactly as ggml's CPU vec_dot forms it:
//   Q8_0 / Q4_0 (per 32):  (float)isum * (d_w * d_a)
//   Q4_K       (per 256):  (d_w*d_a)*(float)isum - (dmin_w*d_a)*(float)msum
// so GPU and CPU differ only in the order of the f32 sum over blocks.
//
// Work mapping: a row has `nitems` work items (Q8_0/Q4_0: one 32-block, Q4_K:
// one 64-element half of a 4-item super-block).  LPR = 2^lpr_log2 lanes share
// a row (LPR divides nitems, so every lane runs the same trip count and
// full-warp shuffles are safe); a warp covers 32/LPR rows per pass and RP
// passes, holding the RP weight items in registers while it loops over the M
// activation rows (activations are small and L1-resident).
#include "kernels.cuh"

namespace oasr {

static __device__ __forceinline__ int nib_lo(int v) { return v & 0x0F0F0F0F; }
static __device__ __forceinline__ int nib_hi(int v) { return (v >> 4) & 0x0F0F0F0F; }

// Canonical summation order (as mma_frag.cuh: every output is the sum of its per-block
// terms in block order).  A pass of the item loop gives each of the warp's lanes one item
// (block) of its row; the lanes stage their terms ([p][m][lane], rows of 33 floats so
// that neither the stores nor the folding reads collide in a bank) in the warp's shared
// slice, and lane L then adds, for the outputs it owns (o = L, L + 32, ...: sub-row, pass
// row p, activation m), the pass's items of that row in item order.
template <int RPM, int IPL>
static __device__ __forceinline__ void fold_pass(float (&out)[RPM], const float *stage, int lane, int lpr_log2,
                                                 int first_item, int nitems) {
    const int lpr = 1 << lpr_log2, rpp = 32 >> lpr_log2;
    const int outs = rpp * RPM;
#pragma unroll
    for (int k = 0; k < RPM; ++k) {
        const int o = lane + 32 * k;
        if (o >= outs) break;
        const int sub = o / RPM, pm = o - sub * RPM;
        for (int jj = 0; jj < lpr / IPL; ++jj) {
            if (first_item + jj * IPL >= nitems) break;
            out[k] = __fadd_rn(out[k], stage[pm * 33 + sub * (lpr / IPL) + jj]);
        }
    }
}

// ---- Q8_0 / Q4_0 -----------------------------------------------------------------------
template <int M, int RP, bool Q4>
__global__ void __launch_bounds__(128, 3)
    mmv_q8_kernel(const uint8_t *__restrict__ wqs, const uint16_t *__restrict__ wd, int64_t qs_ld, int64_t d_ld,
                  int64_t N, int nitems, int lpr_log2, const int8_t *__restrict__ aqs, const float *__restrict__ ad,
                  int K, float *__restrict__ y, int64_t y_ld) {
    constexpr int QB = Q4 ? 16 : 32;
    __shared__ float stage_all[4][33 * RP * M];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lpr = 1 << lpr_log2, rpp = 32 >> lpr_log2;
    const int sub = lane >> lpr_log2, j = lane & (lpr - 1);
    const int64_t wrow0 = ((int64_t)blockIdx.x * 4 + warp) * (int64_t)(rpp * RP);  // the warp's first row
    const int64_t row0 = wrow0 + sub;
    const int nb = K / 32;
    float *stage = stage_all[warp];
    float out[RP * M];  // outputs this lane folds (o = lane + 32 k)
#pragma unroll
    for (int i = 0; i < RP * M; ++i) out[i] = 0.0f;

    // every lane runs the same trip count (the warp folds each pass together);
    // items past the end of the row are never folded
    const int nit_pad = (nitems + lpr - 1) & ~(lpr - 1);
    int4 w0[RP], w1[RP];
    float dw[RP];
    auto load_w = [&](int it) {
        const bool itv = it < nitems;
#pragma unroll
        for (int p = 0; p < RP; ++p) {
            const int64_t row = row0 + (int64_t)p * rpp;
            if (itv && row < N) {
                const uint8_t *wp = wqs + row * qs_ld + (int64_t)it * QB;
                w0[p] = ldg_stream(wp);
                w1[p] = Q4 ? make_int4(0, 0, 0, 0) : ldg_stream(wp + 16);
                dw[p] = h2f(wd[row * d_ld + it]);
            } else {
                w0[p] = w1[p] = make_int4(0, 0, 0, 0);
                dw[p] = 0.0f;
            }
        }
    };
    // the weights do not depend on the previous kernel: start streaming them before
    // waiting for the activations (programmatic dependent launch)
    griddep_launch_dependents();
    load_w(j);
    griddep_wait();
    for (int it = j; it < nit_pad; it += lpr) {
        const bool itv = it < nitems;
        if (it != j) load_w(it);
        float term[RP * M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const int itc = itv ? it : 0;
            const int8_t *ap = aqs + (int64_t)m * K + (int64_t)itc * 32;
            const int4 a0 = __ldg(reinterpret_cast<const int4 *>(ap));
            const int4 a1 = __ldg(reinterpret_cast<const int4 *>(ap + 16));
            const float da = __ldg(ad + (int64_t)m * nb + itc);
#pragma unroll
            for (int p = 0; p < RP; ++p) {
                int s = 0;
                if (Q4) {
                    const int4 w = w0[p];
                    s = __dp4a((int)__vsub4(nib_lo(w.x), 0x08080808), a0.x, s);
                    s = __dp4a((int)__vsub4(nib_lo(w.y), 0x08080808), a0.y, s);
                    s = __dp4a((int)__vsub4(nib_lo(w.z), 0x08080808), a0.z, s);
                    s = __dp4a((int)__vsub4(nib_lo(w.w), 0x08080808), a0.w, s);
                    s = __dp4a((int)__vsub4(nib_hi(w.x), 0x08080808), a1.x, s);
                    s = __dp4a((int)__vsub4(nib_hi(w.y), 0x08080808), a1.y, s);
                    s = __dp4a((int)__vsub4(nib_hi(w.z), 0x08080808), a1.z, s);
                    s = __dp4a((int)__vsub4(nib_hi(w.w), 0x08080808), a1.w, s);
                } else {
                    s = __dp4a(w0[p].x, a0.x, s);
                    s = __dp4a(w0[p].y, a0.y, s);
                    s = __dp4a(w0[p].z, a0.z, s);
                    s = __dp4a(w0[p].w, a0.w, s);
                    s = __dp4a(w1[p].x, a1.x, s);
                    s = __dp4a(w1[p].y, a1.y, s);
                    s = __dp4a(w1[p].z, a1.z, s);
                    s = __dp4a(w1[p].w, a1.w, s);
                }
                term[p * M + m] = __fmul_rn((float)s, __fmul_rn(dw[p], da));
            }
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < RP * M; ++i) stage[i * 33 + lane] = term[i];
        __syncwarp();
        fold_pass<RP * M, 1>(out, stage, lane, lpr_log2, it - j, nitems);
    }
    const int outs = rpp * RP * M;
#pragma unroll
    for (int k = 0; k < RP * M; ++k) {
        const int o = lane + 32 * k;
        if (o >= outs) break;
        const int s2 = o / (RP * M), pm = o - s2 * (RP * M), p = pm / M, m = pm - p * M;
        const int64_t row = wrow0 + s2 + (int64_t)p * rpp;
        if (row < N) y[(int64_t)m * y_ld + row] = out[k];
    }
}

// ---- Q4_K ---------------------------------------------------------------------------------
static __device__ __forceinline__ int byte_of(const int4 &h, int i) {
    const int w = i < 4 ? h.y : (i < 8 ? h.z : h.w);  // scales[0..11] live in h.y..h.w
    return (w >> (8 * (i & 3))) & 0xFF;
}

// get_scale_min_k4 on the 12 packed scale bytes (layout: gguf/quants.py Q4_K.get_scale_min)
static __device__ __forceinline__ void scale_min(const int4 &h, int j, int &sc, int &m) {
    if (j < 4) {
        sc = byte_of(h, j) & 63;
        m = byte_of(h, j + 4) & 63;
    } else {
        sc = (byte_of(h, j + 4) & 0xF) | ((byte_of(h, j - 4) >> 6) << 4);
        m = (byte_of(h, j + 4) >> 4) | ((byte_of(h, j) >> 6) << 4);
    }
}

template <int M, int RP>
__global__ void __launch_bounds__(128, 3)
    mmv_q4k_kernel(const uint8_t *__restrict__ w, int64_t w_ld, int64_t N, int nitems, int lpr_log2,
                   const int8_t *__restrict__ aqs, const float *__restrict__ ad, const int16_t *__restrict__ abs16,
                   int K, float *__restrict__ y, int64_t y_ld) {
    __shared__ float stage_all[4][33 * RP * M];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lpr = 1 << lpr_log2, rpp = 32 >> lpr_log2;
    const int sub = lane >> lpr_log2, j = lane & (lpr - 1);
    const int64_t wrow0 = ((int64_t)blockIdx.x * 4 + warp) * (int64_t)(rpp * RP);
    const int64_t row0 = wrow0 + sub;
    const int nsb = K / 256;
    float *stage = stage_all[warp];
    float out[RP * M];  // outputs this lane folds (o = lane + 32 k)
#pragma unroll
    for (int i = 0; i < RP * M; ++i) out[i] = 0.0f;
    float term[RP * M];

    const int nit_pad = (nitems + lpr - 1) & ~(lpr - 1);
    // pull the first item's weight lines towards L2 before waiting for the
    // activations (programmatic dependent launch); holding them in registers
    // across the wait would spill at RP = 4
    griddep_launch_dependents();
    if (j < nitems) {
#pragma unroll
        for (int p = 0; p < RP; ++p) {
            const int64_t row = row0 + (int64_t)p * rpp;
            if (row < N) {
                const uint8_t *wp = w + row * w_ld + (int64_t)(j >> 2) * 144 + 32 * (j & 3);
                asm volatile("prefetch.global.L2 [%0];" ::"l"(wp + 16));
            }
        }
    }
    griddep_wait();
    for (int it = j; it < nit_pad; it += lpr) {
        const bool itv = it < nitems;
        const int sb = itv ? it >> 2 : 0, c = it & 3;
        int4 hdr[RP], q0[RP], q1[RP];
#pragma unroll
        for (int p = 0; p < RP; ++p) {
            const int64_t row = row0 + (int64_t)p * rpp;
            if (itv && row < N) {
                const uint8_t *wp = w + row * w_ld + (int64_t)sb * 144;
                hdr[p] = ldg_stream(wp);
                q0[p] = ldg_stream(wp + 16 + 32 * c);
                q1[p] = ldg_stream(wp + 32 + 32 * c);
            } else {
                hdr[p] = q0[p] = q1[p] = make_int4(0, 0, 0, 0);
            }
        }
        int sc0[RP], sc1[RP], mn0[RP], mn1[RP];
#pragma unroll
        for (int p = 0; p < RP; ++p) {
            scale_min(hdr[p], 2 * c, sc0[p], mn0[p]);
            scale_min(hdr[p], 2 * c + 1, sc1[p], mn1[p]);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const int8_t *ap = aqs + (int64_t)m * K + (int64_t)sb * 256 + 64 * c;
            const int4 l0 = __ldg(reinterpret_cast<const int4 *>(ap));
            const int4 l1 = __ldg(reinterpret_cast<const int4 *>(ap + 16));
            const int4 h0 = __ldg(reinterpret_cast<const int4 *>(ap + 32));
            const int4 h1 = __ldg(reinterpret_cast<const int4 *>(ap + 48));
            const float da = __ldg(ad + (int64_t)m * nsb + sb);
            const int2 bsv = __ldg(reinterpret_cast<const int2 *>(abs16 + (int64_t)m * (K / 16) + sb * 16 + 4 * c));
            const int bsA = (int)(int16_t)(bsv.x & 0xFFFF) + (int)(int16_t)(bsv.x >> 16);
            const int bsB = (int)(int16_t)(bsv.y & 0xFFFF) + (int)(int16_t)(bsv.y >> 16);
#pragma unroll
            for (int p = 0; p < RP; ++p) {
                int dlo = 0, dhi = 0;
                dlo = __dp4a(nib_lo(q0[p].x), l0.x, dlo);
                dlo = __dp4a(nib_lo(q0[p].y), l0.y, dlo);
                dlo = __dp4a(nib_lo(q0[p].z), l0.z, dlo);
                dlo = __dp4a(nib_lo(q0[p].w), l0.w, dlo);
                dlo = __dp4a(nib_lo(q1[p].x), l1.x, dlo);
                dlo = __dp4a(nib_lo(q1[p].y), l1.y, dlo);
                dlo = __dp4a(nib_lo(q1[p].z), l1.z, dlo);
                dlo = __dp4a(nib_lo(q1[p].w), l1.w, dlo);
                dhi = __dp4a(nib_hi(q0[p].x), h0.x, dhi);
                dhi = __dp4a(nib_hi(q0[p].y), h0.y, dhi);
                dhi = __dp4a(nib_hi(q0[p].z), h0.z, dhi);
                dhi = __dp4a(nib_hi(q0[p].w), h0.w, dhi);
                dhi = __dp4a(nib_hi(q1[p].x), h1.x, dhi);
                dhi = __dp4a(nib_hi(q1[p].y), h1.y, dhi);
                dhi = __dp4a(nib_hi(q1[p].z), h1.z, dhi);
                dhi = __dp4a(nib_hi(q1[p].w), h1.w, dhi);
                int isum = sc0[p] * dlo + sc1[p] * dhi;
                int msum = mn0[p] * bsA + mn1[p] * bsB;
                // the 4 items of a super-block sit on 4 aligned neighbouring lanes
                isum += __shfl_xor_sync(0xffffffffu, isum, 1);
                msum += __shfl_xor_sync(0xffffffffu, msum, 1);
                isum += __shfl_xor_sync(0xffffffffu, isum, 2);
                msum += __shfl_xor_sync(0xffffffffu, msum, 2);
                const float d = __fmul_rn(h2f((uint16_t)(hdr[p].x & 0xFFFF)), da);
                const float dm = __fmul_rn(h2f((uint16_t)((unsigned)hdr[p].x >> 16)), da);
                term[p * M + m] = __fsub_rn(__fmul_rn(d, (float)isum), __fmul_rn(dm, (float)msum));
            }
        }
        // lane j % 4 == 0 holds its super-block's terms: stage them, fold this pass's
        // super-blocks of each row in order
        __syncwarp();
        if ((j & 3) == 0) {
#pragma unroll
            for (int i = 0; i < RP * M; ++i) stage[i * 33 + (lane >> 2)] = term[i];
        }
        __syncwarp();
        fold_pass<RP * M, 4>(out, stage, lane, lpr_log2, it - j, nitems);
    }
    const int outs = rpp * RP * M;
#pragma unroll
    for (int k = 0; k < RP * M; ++k) {
        const int o = lane + 32 * k;
        if (o >= outs) break;
        const int s2 = o / (RP * M), pm = o - s2 * (RP * M), p = pm / M, m = pm - p * M;
        const int64_t row = wrow0 + s2 + (int64_t)p * rpp;
        if (row < N) y[(int64_t)m * y_ld + row] = out[k];
    }
}

// ---- F16 / F32 weights (activations read directly; optional fp16 rounding) ------------
template <int M, bool WF16, bool VEC>
__global__ void __launch_bounds__(128)
    mmv_float_kernel(const uint8_t *__restrict__ w, int64_t w_ld, int64_t N, int K, const char *__restrict__ x,
                     int64_t x_ld, bool x_f16, bool round16, float *__restrict__ y, int64_t y_ld) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = (int64_t)blockIdx.x * 4 + warp;
    if (row >= N) return;  // warp-uniform
    constexpr int E = VEC ? 8 : 1;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;
    const uint8_t *wr = w + row * w_ld;
    for (int k0 = lane * E; k0 < K; k0 += 32 * E) {
        float wv[E];
#pragma unroll
        for (int e = 0; e < E; ++e)
            wv[e] = WF16 ? h2f(reinterpret_cast<const uint16_t *>(wr)[k0 + e]) : reinterpret_cast<const float *>(wr)[k0 + e];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const char *xr = x + (int64_t)m * x_ld;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                float xv = x_f16 ? h2f(reinterpret_cast<const uint16_t *>(xr)[k0 + e]) : reinterpret_cast<const float *>(xr)[k0 + e];
                if (round16) xv = __half2float(__float2half_rn(xv));
                acc[m] = fmaf(wv[e], xv, acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = warp_sum(acc[m]);
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < M; ++m) y[(int64_t)m * y_ld + row] = acc[m];
    }
}

// ---- launchers ------------------------------------------------------------------------
// Lanes per row: cover a row in as few passes as possible while keeping most
// lanes busy (a power of two; 32 once the row has >= 24 items).
static int pick_lpr_log2(int nitems) {
    if (nitems >= 24) return 5;
    int l = 0;
    while ((1 << l) < nitems) ++l;
    return l;
}

// Rows per warp pass: the largest RP in {4, 2, 1} that still gives >= 2 CTAs per SM.
static int pick_rp(int64_t N, int lg, int sm_count) {
    const int64_t rpp = 32 >> lg;
    for (int rp = 4; rp > 1; rp >>= 1)
        if ((N + 4 * rpp * rp - 1) / (4 * rpp * rp) >= 2LL * sm_count) return rp;
    return 1;
}

template <int M, int RP>
static void launch_q8_rp(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int K, float *y, int64_t y_ld,
                         cudaStream_t st, bool q4, int lg) {
    const int64_t N = w->ne[1];
    const int rows_per_cta = 4 * (32 >> lg) * RP;
    const unsigned grid = (unsigned)((N + rows_per_cta - 1) / rows_per_cta);
    const uint8_t *wqs = w->qs + slice * N * w->qs_row_bytes;
    const uint16_t *wd = w->d + slice * N * w->d_row_elems;
    (void)st;
    if (q4)
        launch_k(be, mmv_q8_kernel<M, RP, true>, dim3(grid), dim3(128), 0, (const uint8_t *)wqs, (const uint16_t *)wd,
                 (int64_t)w->qs_row_bytes, (int64_t)w->d_row_elems, N, K / 32, lg, (const int8_t *)a.qs,
                 (const float *)a.d, K, y, y_ld);
    else
        launch_k(be, mmv_q8_kernel<M, RP, false>, dim3(grid), dim3(128), 0, (const uint8_t *)wqs, (const uint16_t *)wd,
                 (int64_t)w->qs_row_bytes, (int64_t)w->d_row_elems, N, K / 32, lg, (const int8_t *)a.qs,
                 (const float *)a.d, K, y, y_ld);
}

template <int M>
static void launch_q8(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int K, float *y, int64_t y_ld,
                      cudaStream_t st, bool q4, int sm_count) {
    const int lg = pick_lpr_log2(K / 32);
    switch (pick_rp(w->ne[1], lg, sm_count)) {
    case 4: launch_q8_rp<M, 4>(be, w, slice, a, K, y, y_ld, st, q4, lg); break;
    case 2: launch_q8_rp<M, 2>(be, w, slice, a, K, y, y_ld, st, q4, lg); break;
    default: launch_q8_rp<M, 1>(be, w, slice, a, K, y, y_ld, st, q4, lg); break;
    }
}

template <int M, int RP>
static void launch_q4k_rp(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int K, float *y, int64_t y_ld,
                          cudaStream_t st, int lg) {
    const int64_t N = w->ne[1];
    const int rows_per_cta = 4 * (32 >> lg) * RP;
    const unsigned grid = (unsigned)((N + rows_per_cta - 1) / rows_per_cta);
    (void)st;
    launch_k(be, mmv_q4k_kernel<M, RP>, dim3(grid), dim3(128), 0, (const uint8_t *)(w->qs + slice * N * w->qs_row_bytes),
             (int64_t)w->qs_row_bytes, N, K / 64, lg, (const int8_t *)a.qs, (const float *)a.d, (const int16_t *)a.bs16,
             K, y, y_ld);
}

template <int M>
static void launch_q4k(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int K, float *y, int64_t y_ld,
                       cudaStream_t st, int sm_count) {
    const int lg = std::max(2, pick_lpr_log2(K / 64));  // the 4 items of a super-block share aligned lanes
    switch (pick_rp(w->ne[1], lg, sm_count)) {
    case 4: launch_q4k_rp<M, 4>(be, w, slice, a, K, y, y_ld, st, lg); break;
    case 2: launch_q4k_rp<M, 2>(be, w, slice, a, K, y, y_ld, st, lg); break;
    default: launch_q4k_rp<M, 1>(be, w, slice, a, K, y, y_ld, st, lg); break;
    }
}

int launch_mmv_quant(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int M, int K,
                     float *y, int64_t y_ld) {
    if (w->tiles) return launch_mmv_tc(be, w, slice, a, M, K, y, y_ld);
    cudaStream_t st = be->stream;
    if (w->type == OASR_TYPE_Q4_K) {
        switch (M) {
        case 1: launch_q4k<1>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        case 2: launch_q4k<2>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        case 3: launch_q4k<3>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        case 4: launch_q4k<4>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        case 5: launch_q4k<5>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        case 6: launch_q4k<6>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        case 7: launch_q4k<7>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        default: launch_q4k<8>(be, w, slice, a, K, y, y_ld, st, be->sm_count); break;
        }
    } else {
        const bool q4 = w->type == OASR_TYPE_Q4_0;
        switch (M) {
        case 1: launch_q8<1>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        case 2: launch_q8<2>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        case 3: launch_q8<3>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        case 4: launch_q8<4>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        case 5: launch_q8<5>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        case 6: launch_q8<6>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        case 7: launch_q8<7>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        default: launch_q8<8>(be, w, slice, a, K, y, y_ld, st, q4, be->sm_count); break;
        }
    }
    return oasr_internal_launch_check(be, "mmv_quant");
}

template <int M>
static void launch_float_m(const oasr_weight *w, int64_t slice, const char *x, int64_t x_ld, bool x_f16, bool r16,
                           int K, float *y, int64_t y_ld, cudaStream_t st) {
    const int64_t N = w->ne[1];
    const unsigned grid = (unsigned)((N + 3) / 4);
    const uint8_t *wb = w->qs + slice * N * w->qs_row_bytes;
    const bool vec = K % 8 == 0;
    if (w->type == OASR_TYPE_F16) {
        if (vec) mmv_float_kernel<M, true, true><<<grid, 128, 0, st>>>(wb, w->qs_row_bytes, N, K, x, x_ld, x_f16, r16, y, y_ld);
        else mmv_float_kernel<M, true, false><<<grid, 128, 0, st>>>(wb, w->qs_row_bytes, N, K, x, x_ld, x_f16, r16, y, y_ld);
    } else {
        if (vec) mmv_float_kernel<M, false, true><<<grid, 128, 0, st>>>(wb, w->qs_row_bytes, N, K, x, x_ld, x_f16, r16, y, y_ld);
        else mmv_float_kernel<M, false, false><<<grid, 128, 0, st>>>(wb, w->qs_row_bytes, N, K, x, x_ld, x_f16, r16, y, y_ld);
    }
}

int launch_mmv_float(oasr_backend *be, const oasr_weight *w, int64_t slice, const char *x, int64_t x_ld_bytes,
                     bool x_f16, bool round_x_f16, int M, int K, float *y, int64_t y_ld) {
    cudaStream_t st = be->stream;
    switch (M) {
    case 1: launch_float_m<1>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    case 2: launch_float_m<2>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    case 3: launch_float_m<3>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    case 4: launch_float_m<4>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    case 5: launch_float_m<5>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    case 6: launch_float_m<6>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    case 7: launch_float_m<7>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    default: launch_float_m<8>(w, slice, x, x_ld_bytes, x_f16, round_x_f16, K, y, y_ld, st); break;
    }
    return oasr_internal_launch_check(be, "mmv_float");
}

}  // namespace oasr
