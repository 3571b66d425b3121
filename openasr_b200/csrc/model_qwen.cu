// model_qwen.cu -- the Qwen3-ASR LLM decoder on the B200 kernels.
//
// Restates the graphs the reference builds for the decoder-only LLM stack:
//   layer      nn/decoder.rs:1850-2140 (llm_layer): RMSNorm * attn_norm ->
//              q|k|v -> per-head RMSNorm * q_norm / k_norm -> RoPE NEOX
//              (ggml_rope_ext, cpu_graph.rs:1135-1155) -> set_rows f16 K/V ->
//              flash_attn_ext (scale 1/sqrt(head_dim), native GQA) ->
//              attn_output -> residual -> RMSNorm * ffn_norm -> silu(gate) * up
//              -> down -> residual (nn/ffn.rs:64-91)
//   head       llm_transformer.rs:2096-2115 (build_fused_logits_top1):
//              RMSNorm * output_norm -> lm_head -> first-max argmax
//   prefill    llm_transformer.rs:3859-3895 (run_prefill): the prompt as one
//              causal pass under the f16 mask of build_causal_mask_f16_bits
//              (nn/decoder.rs:766-790)
//   decode     llm_transformer.rs:3203 (run_step) / :4983 (batched top-1): one
//              token per sequence attends over its live prefix
// Per layer the q|k|v weights are concatenated along N at load (raw blocks), and
// so are gate|up, so one GEMV / GEMM serves each group.  The q/k norms, RoPE and
// the f16 cache write run as one kernel per token row (qkv_post below) with the
// rotation angles from a host-built table, so they match the CPU restatement bit
// for bit.  A decode step is one CUDA graph whose inputs (tokens, position, KV
// length) live in device memory.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <string>
#include <vector>

#include "model.cuh"

using namespace oasr;

namespace {

constexpr int QWEN_HEAD_DIM = 128;  // head width the per-head kernels are written for
constexpr int QWEN_TC_MIN_ROWS = 64;  // prompt length from which attention runs on the tensor cores

struct QLayer {
    oasr_weight *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    __half *k_cache = nullptr, *v_cache = nullptr;  // [max_batch][n_kv_heads][max_pos][head_dim]
};

}  // namespace

struct oasr_qwen {
    oasr_backend *be;
    // scratch the captured decode step needs (reserved at load, and again before a
    // capture if the memory API's trim released it: scratch cannot grow during capture)
    size_t step_scratch;
    oasr_qwen_config cfg;
    cudaStream_t stream;
    int d, H, HKV, D, ffn, qw, kvw, P, B, Tmax;
    oasr_weight *tok_emb, *out_w;
    float *out_norm;
    float2 *rope;  // [max_pos][head_dim / 2] (cos, sin)
    std::vector<QLayer> layers;
    // prefill activations, max_batch * max_prefill rows
    float *x, *qkv, *q, *attn, *t, *gu;
    void *qa;
    __half *mask;  // causal f16 [n_tok][n_tok] of the last prefill
    int mask_tok;
    // decode activations, max_batch rows
    float *dx, *dqkv, *dq, *dattn, *dt, *dgu, *logits;
    void *dqa;
    int *tokens, *pos, *nkv, *history;
    int family;
    bool attn_q8;  // decode attention writes its output as the o_proj's q8_0 planes
    bool pdl;
    cudaGraphExec_t graph;
    int graph_batch;
    uint64_t graph_epoch;  // backend scratch epoch at capture
    std::vector<void *> allocs;
    std::vector<oasr_weight *> weights;
};

namespace {

// Work goes to the backend's current stream when the caller set a non-legacy one,
// else to the model's own stream (CUDA graph capture needs a non-legacy stream).
struct QStreamScope {
    oasr_backend *be;
    oasr_qwen *m;
    cudaStream_t saved_be, saved_m;
    QStreamScope(oasr_qwen *mm) : be(mm->be), m(mm), saved_be(mm->be->stream), saved_m(mm->stream) {
        if (be->stream) m->stream = be->stream;
        be->stream = m->stream;
    }
    ~QStreamScope() {
        be->stream = saved_be;
        m->stream = saved_m;
    }
};

#define Q_TRY(expr)                 \
    do {                            \
        int _st = (expr);           \
        if (_st) return _st;        \
    } while (0)

template <typename T>
int qalloc(oasr_qwen *m, T **p, size_t bytes) {
    *p = nullptr;
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc((void **)p, bytes);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(m->be, e, "cudaMalloc(qwen)", __LINE__);
    m->allocs.push_back(*p);
    return OASR_STATUS_SUCCESS;
}

int qfail(oasr_qwen *m, const std::string &msg) { return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "qwen: " + msg); }

int upload_vec(oasr_qwen *m, const oasr_named_tensor *t, int64_t n, float **out, const std::string &name) {
    if (!t || t->type != OASR_TYPE_F32 || t->bytes != (uint64_t)n * 4) return qfail(m, "missing or bad f32 tensor " + name);
    Q_TRY(qalloc(m, out, (size_t)n * 4));
    const cudaError_t e = cudaMemcpy(*out, t->data, (size_t)n * 4, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? OASR_STATUS_SUCCESS : oasr_internal_cuda_fail(m->be, e, "upload f32", __LINE__);
}

// 2-D weights [K, N_i] of one type concatenated along N (raw rows), uploaded as one
int upload_linear(oasr_qwen *m, const std::vector<const oasr_named_tensor *> &parts, int64_t K, oasr_weight **out,
                  const std::string &what) {
    int type = -1;
    int64_t N = 0;
    for (auto *p : parts) {
        if (!p || p->ne[0] != K || p->ne[2] != 1 || p->ne[3] != 1) return qfail(m, "missing or bad weight " + what);
        if (type < 0) type = p->type;
        if (p->type != type) return qfail(m, "mixed types in " + what);
        N += p->ne[1];
    }
    if (type != OASR_TYPE_Q8_0 && type != OASR_TYPE_Q4_0 && type != OASR_TYPE_Q4_K)
        return qfail(m, what + " must be Q8_0, Q4_0 or Q4_K");
    const int64_t rs = oasr_b200_row_size(type, K);
    if (rs <= 0) return qfail(m, "row size of " + what);
    std::vector<uint8_t> buf((size_t)(rs * N));
    size_t off = 0;
    for (auto *p : parts) {
        if (p->bytes != (uint64_t)(rs * p->ne[1])) return qfail(m, "byte count of " + what);
        memcpy(buf.data() + off, p->data, p->bytes);
        off += p->bytes;
    }
    const int64_t ne[4] = {K, N, 1, 1};
    Q_TRY(oasr_b200_weight_upload(m->be, buf.data(), buf.size(), type, ne, out));
    m->weights.push_back(*out);
    return OASR_STATUS_SUCCESS;
}

// ---- kernels --------------------------------------------------------------------------------
// One CTA per token row of the fused q|k|v projection [rows][(H + 2 HKV) * 128]:
// warp w takes heads w, w + warps, ... (query heads, then key heads, then value
// heads), 4 consecutive values per lane.  Query / key heads: RMSNorm over the
// head (double sum of float squares, as ggml_rms_norm), * q_norm / k_norm, then
// RoPE NEOX on the pairs (i, i + 64) with (cos, sin) of the row's position from
// `rope`; queries go to q_out [rows][H * 128] f32, keys and values to the f16
// caches [seq][kv head][max_pos][128].  Row r is token r % T of sequence r / T at
// position (pos_dev[sequence] or pos0) + r % T.
__global__ void __launch_bounds__(1024) qwen_qkv_post_kernel(const float *qkv, int64_t qkv_ld, int H, int HKV, int T,
                                                             const int *pos_dev, int pos0, const float *q_norm,
                                                             const float *k_norm, float eps, const float2 *rope,
                                                             float *q_out, __half *kc, __half *vc, int P, int *err) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t r = blockIdx.x;
    const int s = (int)(r / T), t = (int)(r % T);
    const int p = (pos_dev ? pos_dev[s] : pos0) + t;
    if (p < 0 || p >= P) {
        if (threadIdx.x == 0) atomicOr(err, ERR_BAD_INDEX);
        return;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float *row = qkv + r * qkv_ld;
    const float2 *cs = rope + (int64_t)p * (QWEN_HEAD_DIM / 2) + 4 * (lane & 15);
    for (int hh = warp; hh < H + 2 * HKV; hh += nw) {
        const float4 xv = *reinterpret_cast<const float4 *>(row + (int64_t)hh * QWEN_HEAD_DIM + 4 * lane);
        float v[4] = {xv.x, xv.y, xv.z, xv.w};
        if (hh >= H + HKV) {
            __half *dst = vc + (((int64_t)s * HKV + (hh - H - HKV)) * P + p) * QWEN_HEAD_DIM + 4 * lane;
            const __half2 h01 = __halves2half2(__float2half_rn(v[0]), __float2half_rn(v[1]));
            const __half2 h23 = __halves2half2(__float2half_rn(v[2]), __float2half_rn(v[3]));
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t *>(&h01);
            pk.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(dst) = pk;
            continue;
        }
        const bool isq = hh < H;
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += (double)__fmul_rn(v[j], v[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float mean = (float)(ss / (double)QWEN_HEAD_DIM);
        const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
        const float4 wv = *reinterpret_cast<const float4 *>((isq ? q_norm : k_norm) + 4 * lane);
        const float w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), w[j]);
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float other = __shfl_xor_sync(0xffffffffu, v[j], 16);
            const float2 c = cs[j];
            // first half: x0 cos - x1 sin; second half: x0 sin + x1 cos (x0 = first-half value)
            o[j] = lane < 16 ? __fsub_rn(__fmul_rn(v[j], c.x), __fmul_rn(other, c.y))
                             : __fadd_rn(__fmul_rn(other, c.y), __fmul_rn(v[j], c.x));
        }
        if (isq) {
            *reinterpret_cast<float4 *>(q_out + r * ((int64_t)H * QWEN_HEAD_DIM) + (int64_t)hh * QWEN_HEAD_DIM +
                                        4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
            __half *dst = kc + (((int64_t)s * HKV + (hh - H)) * P + p) * QWEN_HEAD_DIM + 4 * lane;
            const __half2 h01 = __halves2half2(__float2half_rn(o[0]), __float2half_rn(o[1]));
            const __half2 h23 = __halves2half2(__float2half_rn(o[2]), __float2half_rn(o[3]));
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t *>(&h01);
            pk.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(dst) = pk;
        }
    }
}

// causal f16 mask [n][n]: query t sees keys 0..t (build_causal_mask_f16_bits)
__global__ void causal_mask_kernel(__half *mask, int n) {
    const int64_t total = (int64_t)n * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        mask[i] = (i % n) > (i / n) ? __ushort_as_half((unsigned short)0xFC00) : __ushort_as_half((unsigned short)0);
}

int launch_qkv_post(oasr_qwen *m, const float *qkv, int64_t rows, int T, const int *pos_dev, int pos0, const QLayer &L,
                    float *q_out) {
    oasr_backend *be = m->be;
    const int warps = std::min(32, m->H + 2 * m->HKV);
    const cudaError_t e = launch_k(be, qwen_qkv_post_kernel, dim3((unsigned)rows), dim3(32 * warps), 0, qkv,
                                   (int64_t)(m->qw + 2 * m->kvw), m->H, m->HKV, T, pos_dev, pos0,
                                   (const float *)L.q_norm, (const float *)L.k_norm, m->cfg.rms_eps,
                                   (const float2 *)m->rope, q_out, L.k_cache, L.v_cache, m->P, be->err_word);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "qkv_post launch", __LINE__);
    return oasr_internal_launch_check(be, "qwen_qkv_post");
}

// attention of `nq` query rows per sequence over the sequence's cache rows
int attend(oasr_qwen *m, const QLayer &L, const float *q, int nq, int n, int nkv_max, const __half *mask,
           const int *nkv_dev, float *out, const ActPlanes *out_q8 = nullptr) {
    const int D = m->D, H = m->H, HKV = m->HKV, P = m->P;
    const int64_t qrow = (int64_t)m->qw * 4;
    oasr_tensor tq = make_tensor(OASR_TYPE_F32, q, D, nq, H, n, qrow, (int64_t)D * 4, qrow * nq);
    oasr_tensor tk = make_tensor(OASR_TYPE_F16, L.k_cache, D, nkv_max, HKV, n, (int64_t)D * 2, (int64_t)P * D * 2,
                                 (int64_t)HKV * P * D * 2);
    oasr_tensor tv = make_tensor(OASR_TYPE_F16, L.v_cache, D, nkv_max, HKV, n, (int64_t)D * 2, (int64_t)P * D * 2,
                                 (int64_t)HKV * P * D * 2);
    oasr_tensor to = make_tensor(OASR_TYPE_F32, out, D, H, nq, n, (int64_t)D * 4, qrow, qrow * nq);
    oasr_tensor tm;
    if (mask) {
        tm = make_tensor(OASR_TYPE_F16, mask, nkv_max, nq, 1, 1, (int64_t)nkv_max * 2, (int64_t)nkv_max * nq * 2,
                         (int64_t)nkv_max * nq * 2);
    }
    const float scale = 1.0f / sqrtf((float)D);
    // decode: the rows below *nkv_dev - 1 were written by earlier steps, so the attention loads
    // them before waiting on qkv_post (which writes the newest row)
    if (out_q8)
        return launch_flash_attn_decode_q8(m->be, &tq, &tk, &tv, scale, &to, nullptr, nkv_dev, *out_q8, FAMILY_Q8_0,
                                           KV_STATIC_OLD);
    // prompt passes of at least one 64-row tile: causal flash attention on the tcgen05 tensor cores
    if (mask && nq >= QWEN_TC_MIN_ROWS && nq == nkv_max) return launch_flash_attn_tc(m->be, &tq, &tk, &tv, scale, &to, true);
    return launch_flash_attn_ex(m->be, &tq, &tk, &tv, mask ? &tm : nullptr, scale, &to, nullptr, nkv_dev);
}

// ---- prefill: n sequences of T prompt rows, embeddings already in x -----------------------
int run_prefill(oasr_qwen *m, int n, int T) {
    oasr_backend *be = m->be;
    const int d = m->d, fam = m->family;
    const int64_t M = (int64_t)n * T;
    const ActPlanes qd = act_planes_at(m->qa, fam, M, d);
    const ActPlanes qq = act_planes_at(m->qa, fam, M, m->qw);
    const ActPlanes qf = act_planes_at(m->qa, fam, M, m->ffn);
    if (T > 1 && m->mask_tok != T) {
        causal_mask_kernel<<<std::max(1, std::min(be->sm_count * 8, (T * T + 255) / 256)), 256, 0, be->stream>>>(m->mask, T);
        Q_TRY(oasr_internal_launch_check(be, "causal_mask"));
        m->mask_tok = T;
    }
    Q_TRY(launch_resid_norm_quant(be, m->x, nullptr, nullptr, M, d, m->cfg.rms_eps, true, m->layers[0].attn_norm,
                                  nullptr, nullptr, &qd, fam));
    for (size_t l = 0; l < m->layers.size(); ++l) {
        const QLayer &L = m->layers[l];
        Q_TRY(mul_mat_planes(be, L.qkv, qd, M, m->qkv, m->qw + 2 * m->kvw));
        Q_TRY(launch_qkv_post(m, m->qkv, M, T, nullptr, 0, L, m->q));
        Q_TRY(attend(m, L, m->q, T, n, T, T > 1 ? m->mask : nullptr, nullptr, m->attn));
        oasr_tensor at = make_tensor(OASR_TYPE_F32, m->attn, m->qw, M, 1, 1, (int64_t)m->qw * 4, (int64_t)m->qw * 4 * M,
                                     (int64_t)m->qw * 4 * M);
        Q_TRY(launch_quantize_act(be, &at, fam, qq));
        Q_TRY(mul_mat_planes(be, L.o, qq, M, m->t, d));
        Q_TRY(launch_resid_norm_quant(be, m->x, m->t, nullptr, M, d, m->cfg.rms_eps, true, L.ffn_norm, nullptr, nullptr,
                                      &qd, fam));
        Q_TRY(mul_mat_planes(be, L.gu, qd, M, m->gu, 2 * m->ffn));
        Q_TRY(launch_swiglu_quant(be, m->gu, M, m->ffn, 2 * m->ffn, nullptr, &qf, fam));
        Q_TRY(mul_mat_planes(be, L.down, qf, M, m->t, d));
        if (l + 1 < m->layers.size())
            Q_TRY(launch_resid_norm_quant(be, m->x, m->t, nullptr, M, d, m->cfg.rms_eps, true,
                                          m->layers[l + 1].attn_norm, nullptr, nullptr, &qd, fam));
    }
    // the last prompt row of each sequence (hidden + pending down output) feeds the head
    OASR_CUDA_TRY(be, cudaMemcpy2DAsync(m->dx, (size_t)d * 4, m->x + (int64_t)(T - 1) * d, (size_t)T * d * 4,
                                        (size_t)d * 4, n, cudaMemcpyDeviceToDevice, be->stream));
    OASR_CUDA_TRY(be, cudaMemcpy2DAsync(m->dt, (size_t)d * 4, m->t + (int64_t)(T - 1) * d, (size_t)T * d * 4,
                                        (size_t)d * 4, n, cudaMemcpyDeviceToDevice, be->stream));
    const ActPlanes ql = act_planes_at(m->dqa, weight_family(m->out_w), n, d);
    Q_TRY(launch_resid_norm_quant(be, m->dx, m->dt, nullptr, n, d, m->cfg.rms_eps, true, m->out_norm, nullptr, nullptr,
                                  &ql, weight_family(m->out_w)));
    Q_TRY(mul_mat_planes(be, m->out_w, ql, n, m->logits, m->cfg.n_vocab));
    return launch_argmax_rows(be, m->logits, m->cfg.n_vocab, m->cfg.n_vocab, n, m->tokens);
}

// ---- one decode step: token of each of n sequences at device position *pos ----------------
// 9 launches per layer: RMSNorm+quantize -> q|k|v GEMV -> norms + RoPE + cache
// write -> attention (writes its output rows as q8_0 planes) -> o_proj GEMV ->
// residual + RMSNorm + quantize -> gate|up GEMV -> SiLU * up + quantize -> down GEMV
// (its residual is added by the next layer's first kernel).
int run_decode_step(oasr_qwen *m, int n) {
    oasr_backend *be = m->be;
    const int d = m->d, fam = m->family;
    const ActPlanes qd = act_planes_at(m->dqa, fam, n, d);
    const ActPlanes qq = act_planes_at(m->dqa, fam, n, m->qw);
    const ActPlanes qf = act_planes_at(m->dqa, fam, n, m->ffn);
    const int lfam = weight_family(m->out_w);
    const ActPlanes ql = act_planes_at(m->dqa, lfam, n, d);
    Q_TRY(launch_embed_q8_0(be, m->tok_emb, m->tokens, n, nullptr, m->pos, m->P, m->dx));
    Q_TRY(launch_resid_norm_quant(be, m->dx, nullptr, nullptr, n, d, m->cfg.rms_eps, true, m->layers[0].attn_norm,
                                  nullptr, nullptr, &qd, fam));
    for (size_t l = 0; l < m->layers.size(); ++l) {
        const QLayer &L = m->layers[l];
        const bool last = l + 1 == m->layers.size();
        Q_TRY(mul_mat_planes(be, L.qkv, qd, n, m->dqkv, m->qw + 2 * m->kvw));
        Q_TRY(launch_qkv_post(m, m->dqkv, n, 1, m->pos, 0, L, m->dq));
        if (m->attn_q8) {
            // the attention writes its output rows as the o_proj's q8_0 input planes
            Q_TRY(attend(m, L, m->dq, 1, n, m->P, nullptr, m->nkv, m->dattn, &qq));
        } else {
            Q_TRY(attend(m, L, m->dq, 1, n, m->P, nullptr, m->nkv, m->dattn));
            oasr_tensor at = make_tensor(OASR_TYPE_F32, m->dattn, m->qw, n, 1, 1, (int64_t)m->qw * 4,
                                         (int64_t)m->qw * 4 * n, (int64_t)m->qw * 4 * n);
            Q_TRY(launch_quantize_act(be, &at, fam, qq));
        }
        Q_TRY(mul_mat_planes(be, L.o, qq, n, m->dt, d));
        Q_TRY(launch_resid_norm_quant(be, m->dx, m->dt, nullptr, n, d, m->cfg.rms_eps, true, L.ffn_norm, nullptr,
                                      nullptr, &qd, fam));
        Q_TRY(mul_mat_planes(be, L.gu, qd, n, m->dgu, 2 * m->ffn));
        Q_TRY(launch_swiglu_quant(be, m->dgu, n, m->ffn, 2 * m->ffn, nullptr, &qf, fam));
        Q_TRY(mul_mat_planes(be, L.down, qf, n, m->dt, d));
        Q_TRY(launch_resid_norm_quant(be, m->dx, m->dt, nullptr, n, d, m->cfg.rms_eps, true,
                                      last ? m->out_norm : m->layers[l + 1].attn_norm, nullptr, nullptr,
                                      last ? &ql : &qd, last ? lfam : fam));
    }
    Q_TRY(mul_mat_planes(be, m->out_w, ql, n, m->logits, m->cfg.n_vocab));
    return launch_argmax_rows(be, m->logits, m->cfg.n_vocab, m->cfg.n_vocab, n, m->tokens);
}

int decode_step_graph(oasr_qwen *m, int n) {
    oasr_backend *be = m->be;
    if (be->scratch_bytes < m->step_scratch) {
        int st = 0;
        oasr_internal_scratch(be, m->step_scratch, &st);
        if (st) return st;
    }
    // re-capture when the batch changes or the backend's scratch (which the graph's
    // attention partials and argmax records live in) was reallocated since the capture
    if (m->graph && (m->graph_batch != n || m->graph_epoch != be->scratch_epoch)) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    if (!m->graph) {
        cudaGraph_t g;
        OASR_CUDA_TRY(be, cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        be->pdl = m->pdl;
        int st = run_decode_step(m, n);
        if (st == OASR_STATUS_SUCCESS) st = launch_decode_advance(be, m->tokens, m->pos, m->nkv, m->history, n, m->P);
        be->pdl = false;
        const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (st) return st;
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "cudaStreamEndCapture", __LINE__);
        const cudaError_t ie = cudaGraphInstantiate(&m->graph, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return oasr_internal_cuda_fail(be, ie, "cudaGraphInstantiate", __LINE__);
        m->graph_batch = n;
        m->graph_epoch = be->scratch_epoch;
    }
    OASR_CUDA_TRY(be, cudaGraphLaunch(m->graph, m->stream));
    return OASR_STATUS_SUCCESS;
}

// every slot at position pos (its KV length pos + 1)
int set_position(oasr_qwen *m, int pos) {
    std::vector<int> v(2 * (size_t)m->B);
    for (int b = 0; b < m->B; ++b) {
        v[b] = pos;
        v[m->B + b] = pos + 1;
    }
    OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->pos, v.data(), (size_t)m->B * 4, cudaMemcpyHostToDevice, m->stream));
    OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->nkv, v.data() + m->B, (size_t)m->B * 4, cudaMemcpyHostToDevice, m->stream));
    return OASR_STATUS_SUCCESS;
}

// prompt embeddings -> x, prefill, then the selected tokens become the inputs of position T
int prefill_from(oasr_qwen *m, const float *emb, bool on_device, int n, int T) {
    OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->x, emb, (size_t)n * T * m->d * 4,
                                         on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, m->stream));
    Q_TRY(run_prefill(m, n, T));
    Q_TRY(set_position(m, T - 1));
    return launch_decode_advance(m->be, m->tokens, m->pos, m->nkv, m->history, n, m->P);
}

bool prefill_args_ok(oasr_qwen *m, const float *emb, int n_seq, int n_tok) {
    return m && emb && n_seq >= 1 && n_seq <= m->B && n_tok >= 1 && n_tok <= m->Tmax && n_tok < m->P;
}

}  // namespace

extern "C" {

int oasr_b200_qwen_free(oasr_qwen *m) {
    if (!m) return OASR_STATUS_SUCCESS;
    cudaSetDevice(m->be->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    for (auto *w : m->weights) oasr_b200_weight_free(m->be, w);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_qwen_load(oasr_backend *be, const oasr_qwen_config *cfg, const oasr_named_tensor *tensors,
                        int32_t n_tensors, oasr_qwen **out) {
    if (!out) return OASR_STATUS_FAILED;
    *out = nullptr;
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!cfg || !tensors || cfg->head_dim != QWEN_HEAD_DIM || cfg->n_heads < 1 || cfg->n_kv_heads < 1 ||
        cfg->n_heads % cfg->n_kv_heads || cfg->d_model % 256 || (cfg->n_heads * cfg->head_dim) % 256 ||
        cfg->ffn % 256 || cfg->n_layers < 1 || cfg->n_vocab < 1 || cfg->max_batch < 1 || cfg->max_batch > 8 ||
        cfg->max_pos < 2 || cfg->max_prefill < 1 || cfg->max_prefill >= cfg->max_pos || !(cfg->rms_eps > 0.0f) ||
        !(cfg->rope_theta > 0.0f))
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "qwen_load: unsupported config");
    std::map<std::string, const oasr_named_tensor *> tm;
    for (int i = 0; i < n_tensors; ++i) tm[tensors[i].name] = &tensors[i];
    auto T_ = [&](const std::string &nm) -> const oasr_named_tensor * {
        auto it = tm.find(nm);
        return it == tm.end() ? nullptr : it->second;
    };
    oasr_qwen *m = new oasr_qwen();
    m->be = be;
    m->cfg = *cfg;
    m->d = cfg->d_model;
    m->H = cfg->n_heads;
    m->HKV = cfg->n_kv_heads;
    m->D = cfg->head_dim;
    m->ffn = cfg->ffn;
    m->qw = m->H * m->D;
    m->kvw = m->HKV * m->D;
    m->P = cfg->max_pos;
    m->B = cfg->max_batch;
    m->Tmax = cfg->max_prefill;
    m->graph = nullptr;
    m->graph_batch = 0;
    m->mask_tok = 0;
    m->stream = nullptr;
    auto fail = [&](int s) {
        oasr_b200_qwen_free(m);
        return s;
    };
#define L_TRY(expr)                 \
    do {                            \
        int _s = (expr);            \
        if (_s) return fail(_s);    \
    } while (0)
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(OASR_STATUS_ALLOC_FAILED);
    const int d = m->d, B = m->B, P = m->P, D = m->D, HKV = m->HKV;
    {
        const oasr_named_tensor *te = T_("token_embd.weight");
        if (!te || te->type != OASR_TYPE_Q8_0 || te->ne[0] != d || te->ne[1] != cfg->n_vocab)
            return fail(qfail(m, "token_embd.weight must be Q8_0 [d_model, n_vocab]"));
        L_TRY(upload_linear(m, {te}, d, &m->tok_emb, "token_embd.weight"));
        const oasr_named_tensor *to = T_("output.weight");
        if (to) {
            if (to->ne[1] != cfg->n_vocab) return fail(qfail(m, "output.weight must be [d_model, n_vocab]"));
            L_TRY(upload_linear(m, {to}, d, &m->out_w, "output.weight"));
        } else {
            m->out_w = m->tok_emb;  // tied embeddings
        }
    }
    L_TRY(upload_vec(m, T_("output_norm.weight"), d, &m->out_norm, "output_norm.weight"));
    for (int l = 0; l < cfg->n_layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        QLayer L;
        const oasr_named_tensor *wq = T_(p + "attn_q.weight"), *wk = T_(p + "attn_k.weight"), *wv = T_(p + "attn_v.weight");
        if (!wq || !wk || !wv || wq->ne[1] != m->qw || wk->ne[1] != m->kvw || wv->ne[1] != m->kvw)
            return fail(qfail(m, "attention projections of " + p + " do not match the head counts"));
        L_TRY(upload_linear(m, {wq, wk, wv}, d, &L.qkv, p + "attn_qkv"));
        const oasr_named_tensor *wo = T_(p + "attn_output.weight");
        if (!wo || wo->ne[1] != d) return fail(qfail(m, p + "attn_output.weight must be [n_heads * head_dim, d_model]"));
        L_TRY(upload_linear(m, {wo}, m->qw, &L.o, p + "attn_output"));
        const oasr_named_tensor *wg = T_(p + "ffn_gate.weight"), *wu = T_(p + "ffn_up.weight");
        if (!wg || !wu || wg->ne[1] != m->ffn || wu->ne[1] != m->ffn) return fail(qfail(m, p + "ffn_gate/up must be [d_model, ffn]"));
        L_TRY(upload_linear(m, {wg, wu}, d, &L.gu, p + "ffn_gate_up"));
        const oasr_named_tensor *wdn = T_(p + "ffn_down.weight");
        if (!wdn || wdn->ne[1] != d) return fail(qfail(m, p + "ffn_down.weight must be [ffn, d_model]"));
        L_TRY(upload_linear(m, {wdn}, m->ffn, &L.down, p + "ffn_down"));
        L_TRY(upload_vec(m, T_(p + "attn_norm.weight"), d, &L.attn_norm, p + "attn_norm.weight"));
        L_TRY(upload_vec(m, T_(p + "ffn_norm.weight"), d, &L.ffn_norm, p + "ffn_norm.weight"));
        L_TRY(upload_vec(m, T_(p + "attn_q_norm.weight"), D, &L.q_norm, p + "attn_q_norm.weight"));
        L_TRY(upload_vec(m, T_(p + "attn_k_norm.weight"), D, &L.k_norm, p + "attn_k_norm.weight"));
        const size_t cache = (size_t)B * HKV * P * D * 2;
        L_TRY(qalloc(m, &L.k_cache, cache));
        L_TRY(qalloc(m, &L.v_cache, cache));
        // zeroed like the reference's KV arena (allocate_zeroed_llm_resident_kv_arena)
        if (cudaMemset(L.k_cache, 0, cache) != cudaSuccess || cudaMemset(L.v_cache, 0, cache) != cudaSuccess)
            return fail(qfail(m, "KV cache zeroing failed"));
        m->layers.push_back(L);
    }
    m->family = weight_family(m->layers[0].qkv);
    for (const QLayer &L : m->layers)
        if (weight_family(L.qkv) != m->family || weight_family(L.o) != m->family || weight_family(L.gu) != m->family ||
            weight_family(L.down) != m->family)
            return fail(qfail(m, "layer weights must share one activation family"));
    {
        const char *pdl_env = getenv("OASR_B200_PDL");
        m->pdl = !(pdl_env && strcmp(pdl_env, "0") == 0);
        // q8_0 activations (Q8_0 / Q4_0 weights) and 1, 2 or 4 query heads per kv head: the GQA
        // decode kernel quantizes the attention rows itself (measured faster than quantizing
        // them in the o_proj GEMV's prologue, 7.1 us per layer, or in a separate launch)
        m->attn_q8 = flash_attn_decode_q8_supported(m->H, m->HKV, m->D, m->family);
    }
    // rotation table: theta_i = p * theta_scale^i accumulated by repeated multiplication
    // (ggml_rope_cache_init), cos / sin from the host's libm like the CPU op
    {
        std::vector<float2> tab((size_t)P * (D / 2));
        const float theta_scale = powf(cfg->rope_theta, -2.0f / (float)D);
        for (int p = 0; p < P; ++p) {
            float theta = (float)p;
            for (int i = 0; i < D / 2; ++i) {
                tab[(size_t)p * (D / 2) + i] = make_float2(cosf(theta), sinf(theta));
                theta *= theta_scale;
            }
        }
        L_TRY(qalloc(m, &m->rope, tab.size() * sizeof(float2)));
        if (cudaMemcpy(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(qfail(m, "rope table upload failed"));
    }
    const int64_t M = (int64_t)B * m->Tmax;
    const int kmax = std::max(std::max(d, m->qw), m->ffn);
    const int qkvw = m->qw + 2 * m->kvw;
    L_TRY(qalloc(m, &m->x, (size_t)M * d * 4));
    L_TRY(qalloc(m, &m->qkv, (size_t)M * qkvw * 4));
    L_TRY(qalloc(m, &m->q, (size_t)M * m->qw * 4));
    L_TRY(qalloc(m, &m->attn, (size_t)M * m->qw * 4));
    L_TRY(qalloc(m, &m->t, (size_t)M * d * 4));
    L_TRY(qalloc(m, &m->gu, (size_t)M * 2 * m->ffn * 4));
    L_TRY(qalloc(m, (uint8_t **)&m->qa, act_planes_bytes(FAMILY_Q8_K, M, kmax)));  // the larger layout covers both families
    L_TRY(qalloc(m, &m->mask, (size_t)m->Tmax * m->Tmax * 2));
    L_TRY(qalloc(m, &m->dx, (size_t)B * d * 4));
    L_TRY(qalloc(m, &m->dqkv, (size_t)B * qkvw * 4));
    L_TRY(qalloc(m, &m->dq, (size_t)B * m->qw * 4));
    L_TRY(qalloc(m, &m->dattn, (size_t)B * m->qw * 4));
    L_TRY(qalloc(m, &m->dt, (size_t)B * d * 4));
    L_TRY(qalloc(m, &m->dgu, (size_t)B * 2 * m->ffn * 4));
    L_TRY(qalloc(m, &m->logits, (size_t)B * cfg->n_vocab * 4));
    L_TRY(qalloc(m, (uint8_t **)&m->dqa, act_planes_bytes(FAMILY_Q8_K, B, kmax)));
    L_TRY(qalloc(m, &m->tokens, (size_t)B * 4));
    L_TRY(qalloc(m, &m->pos, (size_t)B * 4));  // per slot
    L_TRY(qalloc(m, &m->nkv, (size_t)B * 4));
    L_TRY(qalloc(m, &m->history, (size_t)B * P * 4));
    // flash-decode partials for the largest split configuration of a decode step,
    // reserved now so that no step (and no graph capture) has to grow the scratch
    m->step_scratch = (size_t)std::max<int64_t>(64ll << 20, (int64_t)B * m->H * 16 * (D + 2) * 4);
    L_TRY(oasr_b200_reserve_scratch(be, m->step_scratch));
#undef L_TRY
    *out = m;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_qwen_prefill(oasr_qwen *m, const float *emb, int32_t emb_on_device, int32_t n_seq, int32_t n_tok,
                           float *logits, int32_t *next) {
    if (!prefill_args_ok(m, emb, n_seq, n_tok)) return m ? qfail(m, "prefill: bad arguments") : OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    QStreamScope sc(m);
    Q_TRY(prefill_from(m, emb, emb_on_device != 0, n_seq, n_tok));
    if (logits)
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(logits, m->logits, (size_t)n_seq * m->cfg.n_vocab * 4,
                                             cudaMemcpyDeviceToHost, m->stream));
    if (next) OASR_CUDA_TRY(m->be, cudaMemcpyAsync(next, m->tokens, n_seq * 4, cudaMemcpyDeviceToHost, m->stream));
    OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
    return oasr_b200_synchronize(m->be);
}

int oasr_b200_qwen_decode_step(oasr_qwen *m, const int32_t *tokens, int32_t n_seq, int32_t pos, float *logits,
                               int32_t *next) {
    if (!m || n_seq < 1 || n_seq > m->B || pos < 0 || pos >= m->P) return m ? qfail(m, "decode_step: bad arguments") : OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    QStreamScope sc(m);
    if (tokens) OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->tokens, tokens, n_seq * 4, cudaMemcpyHostToDevice, m->stream));
    Q_TRY(set_position(m, pos));
    Q_TRY(run_decode_step(m, n_seq));
    if (logits)
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(logits, m->logits, (size_t)n_seq * m->cfg.n_vocab * 4,
                                             cudaMemcpyDeviceToHost, m->stream));
    if (next) OASR_CUDA_TRY(m->be, cudaMemcpyAsync(next, m->tokens, n_seq * 4, cudaMemcpyDeviceToHost, m->stream));
    OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
    return oasr_b200_synchronize(m->be);
}

int oasr_b200_qwen_generate(oasr_qwen *m, const float *emb, int32_t emb_on_device, int32_t n_seq, int32_t n_tok,
                            int32_t n_new, int32_t eos, int32_t stop_at_eos, int32_t *tokens_out,
                            int32_t tokens_on_device) {
    if (!prefill_args_ok(m, emb, n_seq, n_tok) || n_new < 1 || (int64_t)n_tok + n_new > m->P || !tokens_out)
        return m ? qfail(m, "generate: bad arguments") : OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    QStreamScope sc(m);
    Q_TRY(prefill_from(m, emb, emb_on_device != 0, n_seq, n_tok));
    std::vector<int32_t> last(n_seq);
    for (int i = 0; i < n_new - 1; ++i) {
        if (m->be->abort_cb && m->be->abort_cb(m->be->abort_data)) return OASR_STATUS_ABORTED;  // step checkpoint
        if (stop_at_eos) {
            OASR_CUDA_TRY(m->be, cudaMemcpyAsync(last.data(), m->tokens, n_seq * 4, cudaMemcpyDeviceToHost, m->stream));
            OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
            bool all = true;
            for (int b = 0; b < n_seq; ++b) all = all && last[b] == eos;
            if (all) break;
        }
        Q_TRY(decode_step_graph(m, n_seq));
    }
    // tokens_out[s][i] = history[s][n_tok + i]
    OASR_CUDA_TRY(m->be, cudaMemcpy2DAsync(tokens_out, (size_t)n_new * 4, m->history + n_tok, (size_t)m->P * 4,
                                           (size_t)n_new * 4, n_seq,
                                           tokens_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                           m->stream));
    if (!tokens_on_device) {
        OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
        return oasr_b200_synchronize(m->be);
    }
    return oasr_internal_launch_check(m->be, "qwen_generate");
}

int oasr_b200_qwen_read_kv(oasr_qwen *m, int32_t layer, int32_t seq, int32_t n_pos, uint16_t *k_out, uint16_t *v_out) {
    if (!m || layer < 0 || layer >= (int)m->layers.size() || seq < 0 || seq >= m->B || n_pos < 0 || n_pos > m->P)
        return m ? qfail(m, "read_kv: bad arguments") : OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    QStreamScope sc(m);
    const QLayer &L = m->layers[layer];
    const size_t row = (size_t)m->D * 2;
    for (int which = 0; which < 2; ++which) {
        uint16_t *dst = which ? v_out : k_out;
        const __half *src = which ? L.v_cache : L.k_cache;
        if (!dst || n_pos == 0) continue;
        // [kv head][n_pos][D] from [seq][kv head][max_pos][D]
        OASR_CUDA_TRY(m->be, cudaMemcpy2DAsync(dst, row * n_pos, src + (size_t)seq * m->HKV * m->P * m->D,
                                               row * m->P, row * n_pos, m->HKV, cudaMemcpyDeviceToHost, m->stream));
    }
    OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
    return oasr_b200_synchronize(m->be);
}

}  // extern "C"
