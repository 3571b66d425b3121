// ops.cu -- C-ABI entry points of the hot-path ops: argument validation with
// the reference's own rules, activation quantization into scratch, and
// dispatch to the GEMV (M <= 8) / GEMM (M > 8) / flash-attention kernels.
// SET_ROWS and the first-max argmax kernels live here too.
#include <math.h>

#include "kernels.cuh"
#include "model.cuh"

using namespace oasr;

namespace {

int type_size(int t) {
    switch (t) {
    case OASR_TYPE_F32: case OASR_TYPE_I32: return 4;
    case OASR_TYPE_F16: return 2;
    case OASR_TYPE_I64: return 8;
    default: return 0;
    }
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// ---- SET_ROWS --------------------------------------------------------------------------
template <bool F16DST, bool I64>
__global__ void set_rows_kernel(char *dst, int64_t d_nb1, int64_t d_nb2, int64_t d_nb3, int64_t d_rows,
                                const char *src, int64_t s_nb1, int64_t s_nb2, int64_t s_nb3, const void *rows,
                                int64_t n, int64_t ne0, int64_t ne2, int64_t ne3, int *err) {
    const int64_t total = n * ne2 * ne3;
    for (int64_t r = blockIdx.x; r < total; r += gridDim.x) {
        const int64_t i = r % n, i2 = (r / n) % ne2, i3 = r / (n * ne2);
        const int64_t dr = I64 ? reinterpret_cast<const int64_t *>(rows)[i] : reinterpret_cast<const int32_t *>(rows)[i];
        if (dr < 0 || dr >= d_rows) {
            if (threadIdx.x == 0) atomicOr(err, ERR_BAD_INDEX);
            continue;
        }
        const float *s = reinterpret_cast<const float *>(src + i * s_nb1 + i2 * s_nb2 + i3 * s_nb3);
        char *d = dst + dr * d_nb1 + i2 * d_nb2 + i3 * d_nb3;
        for (int64_t e = threadIdx.x; e < ne0; e += blockDim.x) {
            if (F16DST) reinterpret_cast<__half *>(d)[e] = __float2half_rn(s[e]);
            else reinterpret_cast<float *>(d)[e] = s[e];
        }
    }
}

// ---- first-max argmax ---------------------------------------------------------------------
__global__ void argmax_first_kernel(const char *x, int64_t nb1, int64_t n, int32_t *out) {
    griddep_launch_dependents();
    griddep_wait();
    const float *row = reinterpret_cast<const float *>(x + blockIdx.x * nb1);
    float best = -INFINITY;
    int64_t bi = -1;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (isfinite(v) && (bi < 0 || v > best)) { best = v; bi = i; }
    }
    // reduce: larger value wins, ties -> lower index; -1 means "no finite value"
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
    }
    __shared__ float sv[32];
    __shared__ int64_t si[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
        }
        if (lane == 0) out[blockIdx.x] = (int32_t)(bi < 0 ? 0 : bi);
    }
}

// larger value wins; ties (and "no finite value", bi < 0) resolve to the lower index
static __device__ __forceinline__ void argmax_merge(float &best, int64_t &bi, float ov, int64_t oi) {
    if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
}

static __device__ __forceinline__ void argmax_block(float &best, int64_t &bi) {
    __shared__ float sv[32];
    __shared__ int64_t si[32];
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : -1;
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
}

// Long rows (logits heads): CTA (chunk c, row) takes ARGMAX_CHUNK consecutive entries and
// records its first max; the last CTA of the row to finish merges the chunks' records.
constexpr int ARGMAX_CHUNK = 4096;

__global__ void __launch_bounds__(256) argmax_chunks_kernel(const float *x, int64_t ld, int64_t n, int nchunks,
                                                            float *pv, long long *pi, unsigned int *tickets,
                                                            int32_t *out) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = blockIdx.y, c = blockIdx.x;
    const float *xr = x + (int64_t)row * ld;
    const int64_t lo = (int64_t)c * ARGMAX_CHUNK, hi = min(n, lo + ARGMAX_CHUNK);
    float best = -INFINITY;
    int64_t bi = -1;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = xr[i];
        if (isfinite(v) && (bi < 0 || v > best)) { best = v; bi = i; }
    }
    argmax_block(best, bi);
    if (threadIdx.x == 0) {
        pv[(int64_t)row * nchunks + c] = best;
        pi[(int64_t)row * nchunks + c] = bi;
    }
    if (!cta_last_arrival(tickets + row, (unsigned)nchunks)) return;
    best = -INFINITY;
    bi = -1;
    for (int k = threadIdx.x; k < nchunks; k += blockDim.x)
        argmax_merge(best, bi, __ldcg(pv + (int64_t)row * nchunks + k), __ldcg(pi + (int64_t)row * nchunks + k));
    __syncthreads();  // argmax_block reuses its shared records
    argmax_block(best, bi);
    if (threadIdx.x == 0) out[row] = (int32_t)(bi < 0 ? 0 : bi);
}

}  // namespace

namespace oasr {
int launch_argmax_rows(oasr_backend *be, const float *x, int64_t ld, int64_t n, int rows, int32_t *out) {
    cudaError_t e;
    const int64_t nchunks = (n + ARGMAX_CHUNK - 1) / ARGMAX_CHUNK;
    if (nchunks > 1 && nchunks <= 65535 && rows <= 65535) {
        // chunk records from the scratch, one row ticket each (left at zero by the merging CTA)
        int st = 0;
        char *scr = (char *)oasr_internal_scratch(be, (size_t)rows * nchunks * (sizeof(float) + sizeof(long long)), &st);
        if (st) return st;
        long long *pi = reinterpret_cast<long long *>(scr);
        float *pv = reinterpret_cast<float *>(scr + (size_t)rows * nchunks * sizeof(long long));
        e = launch_k(be, argmax_chunks_kernel, dim3((unsigned)nchunks, (unsigned)rows), dim3(256), 0, x, ld, n,
                     (int)nchunks, pv, pi, be->counters, out);
    } else {
        e = launch_k(be, argmax_first_kernel, dim3((unsigned)rows), dim3(1024), 0, (const char *)x, ld * 4, n, out);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "argmax launch", __LINE__);
    return oasr_internal_launch_check(be, "argmax_first");
}

int mul_mat_planes(oasr_backend *be, const oasr_weight *w, const ActPlanes &a, int64_t rows, float *y, int64_t y_ld) {
    if (rows <= 8) return launch_mmv_quant(be, w, 0, a, (int)rows, (int)w->ne[0], y, y_ld);
    return launch_mmq(be, w, 0, a, rows, (int)w->ne[0], y, y_ld);
}

int mul_mat_planes_bias(oasr_backend *be, const oasr_weight *w, const ActPlanes &a, int64_t rows, float *y,
                        int64_t y_ld, const float *bias) {
    if (rows > 8 && mmq_fuses_bias(w, a)) return launch_mmq(be, w, 0, a, rows, (int)w->ne[0], y, y_ld, bias);
    const int st = mul_mat_planes(be, w, a, rows, y, y_ld);
    if (st || !bias) return st;
    if (y_ld != w->ne[1]) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat_planes_bias: rows must be dense");
    return launch_add_rows(be, y, bias, nullptr, rows, (int)w->ne[1]);
}
}  // namespace oasr

extern "C" {

int oasr_b200_mul_mat(oasr_backend *be, const oasr_weight *w, const oasr_tensor *x, oasr_tensor *dst, int32_t prec) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!w || !x || !dst || !x->data || !dst->data) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat: null argument");
    const int64_t K = w->ne[0], N = w->ne[1];
    // cpu_graph.rs:7188-7206 (ensure_can_mul_mat) and :3673-3678 (rhs types)
    if (x->ne[0] != K) return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_mul_mat lhs.ne0 must equal rhs.ne0");
    if (x->ne[2] % w->ne[2] || x->ne[3] % w->ne[3])
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_mul_mat batch dims are not broadcast-compatible");
    if (x->type != OASR_TYPE_F32 && x->type != OASR_TYPE_F16)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_mul_mat rhs must be F32 or F16");
    if (x->nb[0] != type_size(x->type)) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat: rhs rows must be contiguous");
    if (dst->type != OASR_TYPE_F32 || dst->ne[0] != N || dst->ne[1] != x->ne[1] || dst->ne[2] != x->ne[2] ||
        dst->ne[3] != x->ne[3] || dst->nb[0] != 4 || dst->nb[1] % 4 || dst->nb[2] % 4 || dst->nb[3] % 4)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat: dst must be f32 [N, M, ne2, ne3] with f32-aligned strides");
    if (prec != OASR_PREC_DEFAULT && prec != OASR_PREC_F32) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat: bad prec");
    const int64_t M = x->ne[1], ne2 = x->ne[2], ne3 = x->ne[3];
    if (M == 0 || ne2 == 0 || ne3 == 0) return OASR_STATUS_SUCCESS;
    const int64_t r2 = ne2 / w->ne[2], r3 = ne3 / w->ne[3];
    const bool quant = w->type == OASR_TYPE_Q8_0 || w->type == OASR_TYPE_Q4_0 || w->type == OASR_TYPE_Q4_K;
    if (quant) {
        const int family = w->type == OASR_TYPE_Q4_K ? FAMILY_Q8_K : FAMILY_Q8_0;
        const int64_t R = M * ne2 * ne3;
        void *scr = oasr_internal_scratch(be, act_planes_bytes(family, R, K), &st);
        if (st) return st;
        ActPlanes all = act_planes_at(scr, family, R, K);
        st = launch_quantize_act(be, x, family, all);
        if (st) return st;
        for (int64_t i3 = 0; i3 < ne3; ++i3)
            for (int64_t i2 = 0; i2 < ne2; ++i2) {
                const int64_t r0 = M * (i2 + ne2 * i3);
                const int64_t slice = (i2 / r2) + (i3 / r3) * w->ne[2];
                float *y = reinterpret_cast<float *>((char *)dst->data + i2 * dst->nb[2] + i3 * dst->nb[3]);
                const int64_t y_ld = dst->nb[1] / 4;
                const ActPlanes a = act_planes_offset(all, family, r0, K);
                if (M <= 8) st = launch_mmv_quant(be, w, slice, a, (int)M, (int)K, y, y_ld);
                else st = launch_mmq(be, w, slice, a, M, (int)K, y, y_ld);
                if (st) return st;
            }
        return OASR_STATUS_SUCCESS;
    }
    // F16 / F32 weights: ggml CPU converts f32 activations to f16 for F16
    // weights; GGML_PREC_F32 keeps the f32 range (cpu_graph.rs:157-165).
    const bool round16 = w->type == OASR_TYPE_F16 && x->type == OASR_TYPE_F32 && prec != OASR_PREC_F32;
    if (w->type == OASR_TYPE_F16 && prec != OASR_PREC_F32 && M > 8 && K % 64 == 0) {
        // fp16 operands (the vec_dot type of F16), f32 accumulation, on the tensor cores
        __half *x16 = (__half *)oasr_internal_scratch(be, align256((size_t)M * K * 2), &st);
        if (st) return st;
        for (int64_t i3 = 0; i3 < ne3; ++i3)
            for (int64_t i2 = 0; i2 < ne2; ++i2) {
                const int64_t slice = (i2 / r2) + (i3 / r3) * w->ne[2];
                const char *xp = (const char *)x->data + i2 * x->nb[2] + i3 * x->nb[3];
                if (x->type == OASR_TYPE_F32) {
                    st = launch_cast_f16(be, (const float *)xp, x->nb[1] / 4, nullptr, M, (int)K, x16, K);
                    if (st) return st;
                } else {
                    OASR_CUDA_TRY(be, cudaMemcpy2DAsync(x16, K * 2, xp, x->nb[1], K * 2, M, cudaMemcpyDeviceToDevice, be->stream));
                }
                float *y = reinterpret_cast<float *>((char *)dst->data + i2 * dst->nb[2] + i3 * dst->nb[3]);
                st = launch_gemm_f16(be, x16, K, (const __half *)(w->qs + slice * N * w->qs_row_bytes), K, (int)M, (int)N,
                                     (int)K, y, dst->nb[1] / 4, nullptr, false);
                if (st) return st;
            }
        return OASR_STATUS_SUCCESS;
    }
    for (int64_t i3 = 0; i3 < ne3; ++i3)
        for (int64_t i2 = 0; i2 < ne2; ++i2) {
            const int64_t slice = (i2 / r2) + (i3 / r3) * w->ne[2];
            for (int64_t m0 = 0; m0 < M; m0 += 8) {
                const int mc = (int)std::min<int64_t>(8, M - m0);
                const char *xp = (const char *)x->data + m0 * x->nb[1] + i2 * x->nb[2] + i3 * x->nb[3];
                float *y = reinterpret_cast<float *>((char *)dst->data + m0 * dst->nb[1] + i2 * dst->nb[2] + i3 * dst->nb[3]);
                st = launch_mmv_float(be, w, slice, xp, x->nb[1], x->type == OASR_TYPE_F16, round16, mc, (int)K, y,
                                      dst->nb[1] / 4);
                if (st) return st;
            }
        }
    return OASR_STATUS_SUCCESS;
}

int64_t oasr_b200_act_bytes(int32_t weight_type, int64_t K, int64_t rows) {
    if (rows < 0 || K <= 0) return OASR_STATUS_FAILED;
    if (weight_type == OASR_TYPE_Q8_0 || weight_type == OASR_TYPE_Q4_0)
        return K % 32 ? OASR_STATUS_FAILED : (int64_t)act_planes_bytes(FAMILY_Q8_0, rows, K);
    if (weight_type == OASR_TYPE_Q4_K) return K % 256 ? OASR_STATUS_FAILED : (int64_t)act_planes_bytes(FAMILY_Q8_K, rows, K);
    return OASR_STATUS_FAILED;
}

int oasr_b200_quantize_act(oasr_backend *be, int32_t weight_type, const oasr_tensor *x, void *qact, size_t qact_bytes) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!x || !qact) return oasr_internal_fail(be, OASR_STATUS_FAILED, "quantize_act: null argument");
    if ((x->type != OASR_TYPE_F32 && x->type != OASR_TYPE_F16) || x->nb[0] != type_size(x->type))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "quantize_act: x must be f32/f16 with contiguous rows");
    const int64_t R = x->ne[1] * x->ne[2] * x->ne[3];
    const int64_t need = oasr_b200_act_bytes(weight_type, x->ne[0], R);
    if (need < 0) return oasr_internal_fail(be, OASR_STATUS_FAILED, "quantize_act: unsupported weight type or K");
    if ((size_t)need > qact_bytes || ((uintptr_t)qact & 255))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "quantize_act: buffer too small or not 256-byte aligned");
    const int family = weight_type == OASR_TYPE_Q4_K ? FAMILY_Q8_K : FAMILY_Q8_0;
    return launch_quantize_act(be, x, family, act_planes_at(qact, family, R, x->ne[0]));
}

int oasr_b200_mul_mat_qact(oasr_backend *be, const oasr_weight *w, const void *qact, int64_t rows, oasr_tensor *dst) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!w || !qact || !dst) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat_qact: null argument");
    if (w->type != OASR_TYPE_Q8_0 && w->type != OASR_TYPE_Q4_0 && w->type != OASR_TYPE_Q4_K)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat_qact: weight must be Q8_0, Q4_0 or Q4_K");
    if (w->ne[2] != 1 || w->ne[3] != 1) return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat_qact: 2-D weights only");
    const int64_t K = w->ne[0], N = w->ne[1];
    if (dst->type != OASR_TYPE_F32 || dst->ne[0] != N || dst->ne[1] != rows || dst->ne[2] != 1 || dst->ne[3] != 1 ||
        dst->nb[0] != 4 || dst->nb[1] % 4)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "mul_mat_qact: dst must be f32 [N, rows]");
    if (rows == 0) return OASR_STATUS_SUCCESS;
    const int family = w->type == OASR_TYPE_Q4_K ? FAMILY_Q8_K : FAMILY_Q8_0;
    ActPlanes a = act_planes_at(const_cast<void *>(qact), family, rows, K);
    float *y = (float *)dst->data;
    if (rows <= 8) return launch_mmv_quant(be, w, 0, a, (int)rows, (int)K, y, dst->nb[1] / 4);
    return launch_mmq(be, w, 0, a, rows, (int)K, y, dst->nb[1] / 4);
}

// Argument checks shared by both attention entry points: a status; *empty is set
// when there is nothing to compute (no queries).
static int fa_validate(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                       const oasr_tensor *mask, float max_bias, float logit_softcap, int32_t prec,
                       oasr_tensor *dst, bool *empty) {
    *empty = false;
    if (!q || !k || !v || !dst) return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: null argument");
    if (max_bias != 0.0f || logit_softcap != 0.0f)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: max_bias/logit_softcap must be 0");
    if (prec != OASR_PREC_DEFAULT && prec != OASR_PREC_F32) return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: bad prec");
    // cpu_graph.rs:4156-4179 (types, contiguous rows) and :7476-7519 (shapes, mask)
    if (q->type != OASR_TYPE_F32) return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: q must be F32");
    if (k->type != v->type || (k->type != OASR_TYPE_F16 && k->type != OASR_TYPE_F32))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: k/v must both be F16 or F32");
    const int64_t D = q->ne[0];
    if (D != 64 && D != 128) return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: head_dim must be 64 or 128");
    if (k->ne[0] != D || v->ne[0] != D) return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: k/v head_dim mismatch");
    if (k->ne[2] <= 0 || q->ne[2] % k->ne[2] || q->ne[3] % k->ne[3])
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_mul_mat batch dims are not broadcast-compatible");
    if (q->ne[3] != k->ne[3] || q->ne[3] != v->ne[3])
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_flash_attn_ext q/k/v ne3 dimensions must match");
    if (k->ne[1] != v->ne[1]) return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_flash_attn_ext k/v ne1 dimensions must match");
    if (k->ne[2] != v->ne[2]) return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_flash_attn_ext k/v ne2 dimensions must match");
    const int es = type_size(k->type);
    if (q->nb[0] != 4 || k->nb[0] != es || v->nb[0] != es)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: rows must be contiguous");
    if (!aligned16(q->data) || !aligned16(k->data) || !aligned16(v->data) || q->nb[1] % 16 || q->nb[2] % 16 ||
        q->nb[3] % 16 || k->nb[1] % 16 || k->nb[2] % 16 || k->nb[3] % 16 || v->nb[1] % 16 || v->nb[2] % 16 ||
        v->nb[3] % 16)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: q/k/v rows must be 16-byte aligned");
    if (mask) {
        if (mask->type != OASR_TYPE_F16 || mask->ne[0] < k->ne[1] || mask->ne[1] < q->ne[1])
            return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: mask must be F16 covering [n_kv, n_q]");
        if (mask->ne[2] <= 0 || mask->ne[3] <= 0 || q->ne[2] % mask->ne[2] || q->ne[3] % mask->ne[3])
            return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_flash_attn_ext mask batch dims are not broadcast-compatible");
    }
    if (dst->type != OASR_TYPE_F32 || dst->ne[0] != D || dst->ne[1] != q->ne[2] || dst->ne[2] != q->ne[1] ||
        dst->ne[3] != q->ne[3] || dst->nb[0] != 4)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "flash_attn_ext: dst must be f32 [D, H, n_q, S]");
    *empty = q->ne[1] == 0 || q->ne[2] == 0 || q->ne[3] == 0;
    return OASR_STATUS_SUCCESS;
}

// ggml leaves S = 0 with no keys and writes zeros
static int fa_zero_fill(oasr_backend *be, const oasr_tensor *dst, int64_t D) {
    for (int64_t s = 0; s < dst->ne[3]; ++s)
        for (int64_t i = 0; i < dst->ne[2]; ++i)
            for (int64_t h = 0; h < dst->ne[1]; ++h)
                OASR_CUDA_TRY(be, cudaMemsetAsync((char *)dst->data + h * dst->nb[1] + i * dst->nb[2] + s * dst->nb[3], 0,
                                                  D * 4, be->stream));
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_flash_attn_ext(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                             const oasr_tensor *mask, float scale, float max_bias, float logit_softcap, int32_t prec,
                             oasr_tensor *dst) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    bool empty;
    st = fa_validate(be, q, k, v, mask, max_bias, logit_softcap, prec, dst, &empty);
    if (st || empty) return st;
    if (k->ne[1] == 0) return fa_zero_fill(be, dst, q->ne[0]);
    if (flash_attn_tc_eligible(q, k, mask, dst)) return launch_flash_attn_tc(be, q, k, v, scale, dst, false);
    return launch_flash_attn(be, q, k, v, mask, scale, dst);
}

int oasr_b200_flash_attn_causal(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                                float scale, int32_t prec, oasr_tensor *dst) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    bool empty;
    st = fa_validate(be, q, k, v, nullptr, 0.0f, 0.0f, prec, dst, &empty);
    if (st || empty) return st;
    const int64_t D = q->ne[0];
    if ((D != 64 && D != 128) || q->ne[1] < 64 || k->ne[1] < q->ne[1] || dst->nb[1] % 16 || dst->nb[2] % 16 ||
        dst->nb[3] % 16 || ((uintptr_t)dst->data & 15))
        return oasr_internal_fail(be, OASR_STATUS_FAILED,
                                  "flash_attn_causal: needs head_dim 64|128, n_q >= 64, n_kv >= n_q and 16-byte "
                                  "aligned dst rows (use flash_attn_ext with the mask)");
    return launch_flash_attn_tc(be, q, k, v, scale, dst, true);
}

int oasr_b200_flash_attn_ext_static(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k,
                                    const oasr_tensor *v, const oasr_tensor *mask, float scale, float max_bias,
                                    float logit_softcap, int32_t prec, oasr_tensor *dst) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    bool empty;
    st = fa_validate(be, q, k, v, mask, max_bias, logit_softcap, prec, dst, &empty);
    if (st || empty) return st;
    if (k->ne[1] == 0) return fa_zero_fill(be, dst, q->ne[0]);
    return launch_flash_attn_static(be, q, k, v, mask, scale, dst);
}

int oasr_b200_set_rows(oasr_backend *be, oasr_tensor *dst, const oasr_tensor *src, const oasr_tensor *rows) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!dst || !src || !rows) return oasr_internal_fail(be, OASR_STATUS_FAILED, "set_rows: null argument");
    if (src->type != OASR_TYPE_F32 || (dst->type != OASR_TYPE_F16 && dst->type != OASR_TYPE_F32))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "set_rows: src must be F32, dst F16 or F32");
    if (rows->type != OASR_TYPE_I32 && rows->type != OASR_TYPE_I64)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "set_rows: row indices must be I32 or I64");
    // cpu_graph.rs:4882 checks: indices 1-D along ne0 (ne3 > 1 rejected)
    if (rows->ne[1] != 1 || rows->ne[2] != 1 || rows->ne[3] != 1)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_set_rows indices.ne3 must equal 1");
    if (rows->ne[0] != src->ne[1] || src->ne[0] != dst->ne[0] || src->ne[2] != dst->ne[2] || src->ne[3] != dst->ne[3])
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "set_rows: shape mismatch");
    if (src->nb[0] != 4 || dst->nb[0] != type_size(dst->type) || rows->nb[0] != type_size(rows->type))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "set_rows: rows must be contiguous");
    const int64_t total = src->ne[1] * src->ne[2] * src->ne[3];
    if (total == 0) return OASR_STATUS_SUCCESS;
    const unsigned grid = (unsigned)std::min<int64_t>(total, 65535);
    const bool f16 = dst->type == OASR_TYPE_F16, i64 = rows->type == OASR_TYPE_I64;
#define OASR_SR(F, I)                                                                                             \
    set_rows_kernel<F, I><<<grid, 128, 0, be->stream>>>((char *)dst->data, dst->nb[1], dst->nb[2], dst->nb[3],     \
                                                        dst->ne[1], (const char *)src->data, src->nb[1], src->nb[2], \
                                                        src->nb[3], rows->data, src->ne[1], src->ne[0], src->ne[2],  \
                                                        src->ne[3], be->err_word)
    if (f16 && i64) OASR_SR(true, true);
    else if (f16) OASR_SR(true, false);
    else if (i64) OASR_SR(false, true);
    else OASR_SR(false, false);
#undef OASR_SR
    return oasr_internal_launch_check(be, "set_rows");
}

int oasr_b200_argmax_first(oasr_backend *be, const oasr_tensor *logits, oasr_tensor *out) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!logits || !out) return oasr_internal_fail(be, OASR_STATUS_FAILED, "argmax_first: null argument");
    // cpu_graph.rs:3752-3770: rank-2 contiguous f32 row matrix
    if (logits->type != OASR_TYPE_F32 || logits->ne[2] != 1 || logits->ne[3] != 1 || logits->nb[0] != 4)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "ggml_argmax_first input must be a rank-2 row matrix");
    if (out->type != OASR_TYPE_I32 || out->ne[0] != logits->ne[1])
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "argmax_first: out must be I32 [rows]");
    if (logits->ne[1] == 0) return OASR_STATUS_SUCCESS;
    if (logits->nb[1] % 4 == 0 && logits->ne[1] <= INT32_MAX)
        return launch_argmax_rows(be, (const float *)logits->data, logits->nb[1] / 4, logits->ne[0], (int)logits->ne[1],
                                  (int32_t *)out->data);
    argmax_first_kernel<<<(unsigned)logits->ne[1], 1024, 0, be->stream>>>((const char *)logits->data, logits->nb[1],
                                                                          logits->ne[0], (int32_t *)out->data);
    return oasr_internal_launch_check(be, "argmax_first");
}

}  // extern "C"
