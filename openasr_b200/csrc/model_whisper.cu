// model_whisper.cu -- Whisper encoder-decoder on the B200 kernels.
//
// Restates the graphs the reference builds per utterance:
//   frontend   whisper/mel.rs (pad/trim to 30 s, reflect-centred STFT n_fft 400
//              hop 160 with a periodic Hann window, Slaney mel filterbank,
//              log10 floor 1e-10, max-8 dynamic range, (x+4)/4)
//   prelude    whisper/ggml_executor.rs:640-730 (conv1d k3 s1 p1 + GELU,
//              conv1d k3 s2 p1 + GELU, + positional embedding); ggml_conv_1d =
//              im2col to fp16 + fp16 dot with f32 accumulation
//   encoder    ggml_executor.rs:1509-1810 (pre-LN blocks: LN -> q(+b), k, v(+b)
//              -> flash_attn_ext(scale 1/sqrt(64)) -> out(+b) -> residual ->
//              LN -> fc1(+b) -> GELU -> fc2(+b) -> residual), final LN
//   decoder    ggml_decoder_graph.rs:2840-3010 (token + position embedding,
//              self-attention over the f16 self-KV cache, cross-attention over
//              the f16 cross-KV cache, MLP, final LN, logits) + first-max argmax
// with the hot ops on the kernels of this library.  Per-layer q|k|v weights are
// concatenated along N at load (raw blocks, exact) so one GEMV serves all three.
// A decoder step is captured once into a CUDA graph; token ids, the position
// and the KV length live in device memory, so the graph replays for every step
// and the greedy argmax feeds the next step without a host round trip.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <string>
#include <vector>

#include "model.cuh"

using namespace oasr;

namespace {

constexpr int N_FFT = 400, HOP = 160, N_SAMPLES_30S = 480000, N_MEL_FRAMES = 3000;
constexpr float LN_EPS = 1e-5f;

struct EncLayer {
    oasr_weight *qkv = nullptr, *o = nullptr, *fc1 = nullptr, *fc2 = nullptr;
    float *ln1_g, *ln1_b, *ln2_g, *ln2_b, *b_qkv, *b_o, *b_fc1, *b_fc2;
};

struct DecLayer {
    oasr_weight *qkv = nullptr, *o = nullptr, *cq = nullptr, *ckv = nullptr, *co = nullptr, *fc1 = nullptr, *fc2 = nullptr;
    float *ln1_g, *ln1_b, *lnc_g, *lnc_b, *ln2_g, *ln2_b;
    float *b_qkv, *b_o, *b_cq, *b_ckv, *b_co, *b_fc1, *b_fc2;
    __half *self_k, *self_v, *cross_kv;
};

}  // namespace

struct oasr_whisper {
    oasr_backend *be;
    // scratch the captured decode step needs (reserved at load, and again before a
    // capture if the memory API's trim released it: scratch cannot grow during capture)
    size_t step_scratch;
    oasr_whisper_config cfg;
    cudaStream_t stream;
    int d, H, ffn, K1p, K2p, T_enc, B;
    __half *conv1_w, *conv2_w;
    float *conv1_b, *conv2_b, *enc_pos;
    std::vector<EncLayer> enc;
    float *lnp_g, *lnp_b;
    oasr_weight *tok_emb;
    float *dec_pos;
    std::vector<DecLayer> dec;
    float *lnd_g, *lnd_b;
    // frontend
    float *window, *filters, *audio, *power, *mel;
    float2 *twiddle;
    int *max_key;
    // encoder activations, B * T_enc rows
    __half *im2col;
    float *c1, *x, *qkv, *attn, *t, *f;
    void *qa_d, *qa_f;
    // decoder activations, B rows
    float *dx, *dqkv, *dq, *dattn, *dt, *df, *logits;
    bool fused_dec;  // decoder GEMVs run as dgemv (prologue/epilogue fused), see run_decode_step
    bool attn_planes;  // the fused step's attentions emit the out-projections' activation planes
    bool pdl;        // programmatic dependent launch inside the step graph (OASR_B200_PDL=0 turns it off)
    void *dqa_d, *dqa_f, *dqa_lm;
    int *tokens, *pos, *nkv, *history;
    // serving: per-slot done flags and token budgets, the prompt on the device, admission lists
    int *done, *budget, *prompt_dev, *serve_io;
    int enc_family, dec_family;
    cudaGraphExec_t graph;
    int graph_batch;
    uint64_t graph_epoch;  // backend scratch epoch at capture
    // serve step graphs per power-of-two width (1, 2, 4, 8) and the serving parameters they hold
    cudaGraphExec_t serve_graph[4];
    uint64_t serve_epoch[4];
    int serve_key[3];  // n_prompt, eot, stop_at_eot of the captured serve graphs
    std::vector<void *> allocs;
    std::vector<oasr_weight *> weights;
};

namespace {

// Work goes to the backend's current stream when the caller set a non-legacy one
// (so callers can order and time it), else to the model's own stream; CUDA
// graph capture needs a non-legacy stream.
struct StreamScope {
    oasr_backend *be;
    oasr_whisper *m;
    cudaStream_t saved_be, saved_m;
    StreamScope(oasr_whisper *mm) : be(mm->be), m(mm), saved_be(mm->be->stream), saved_m(mm->stream) {
        if (be->stream) m->stream = be->stream;
        be->stream = m->stream;
    }
    ~StreamScope() {
        be->stream = saved_be;
        m->stream = saved_m;
    }
};

template <typename T>
int dalloc(oasr_whisper *m, T **p, size_t bytes) {
    *p = nullptr;
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc((void **)p, bytes);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(m->be, e, "cudaMalloc(whisper)", __LINE__);
    m->allocs.push_back(*p);
    return OASR_STATUS_SUCCESS;
}

const oasr_named_tensor *find(const std::map<std::string, const oasr_named_tensor *> &tm, const std::string &n) {
    auto it = tm.find(n);
    return it == tm.end() ? nullptr : it->second;
}

#define W_TRY(expr)                 \
    do {                            \
        int _st = (expr);           \
        if (_st) return _st;        \
    } while (0)

int upload_f32(oasr_whisper *m, const oasr_named_tensor *t, int64_t n, float **out, const char *name) {
    if (!t || t->type != OASR_TYPE_F32 || t->bytes != (uint64_t)n * 4)
        return oasr_internal_fail(m->be, OASR_STATUS_FAILED, std::string("whisper: missing or bad f32 tensor ") + name);
    W_TRY(dalloc(m, out, (size_t)n * 4));
    cudaError_t e = cudaMemcpy(*out, t->data, (size_t)n * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(m->be, e, "upload f32", __LINE__);
    return OASR_STATUS_SUCCESS;
}

// concatenate 2-D weights [K, N_i] of one type along N (raw rows) and upload
int upload_cat(oasr_whisper *m, const std::vector<const oasr_named_tensor *> &parts, int64_t K, oasr_weight **out,
               const std::string &what) {
    int type = -1;
    int64_t N = 0;
    for (auto *p : parts) {
        if (!p || p->ne[0] != K || p->ne[2] != 1 || p->ne[3] != 1)
            return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper: missing or bad weight " + what);
        if (type < 0) type = p->type;
        if (p->type != type) return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper: mixed types in " + what);
        N += p->ne[1];
    }
    const int64_t rs = oasr_b200_row_size(type, K);
    std::vector<uint8_t> buf((size_t)(rs * N));
    size_t off = 0;
    for (auto *p : parts) {
        if (p->bytes != (uint64_t)(rs * p->ne[1])) return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper: byte count " + what);
        memcpy(buf.data() + off, p->data, p->bytes);
        off += p->bytes;
    }
    const int64_t ne[4] = {K, N, 1, 1};
    W_TRY(oasr_b200_weight_upload(m->be, buf.data(), buf.size(), type, ne, out));
    m->weights.push_back(*out);
    return OASR_STATUS_SUCCESS;
}

// [b_0 | b_1 | ...] with missing biases as zeros
int upload_bias_cat(oasr_whisper *m, const std::vector<const oasr_named_tensor *> &parts, int64_t each, float **out) {
    std::vector<float> b(parts.size() * each, 0.0f);
    for (size_t i = 0; i < parts.size(); ++i) {
        if (!parts[i]) continue;
        if (parts[i]->type != OASR_TYPE_F32 || parts[i]->bytes != (uint64_t)each * 4)
            return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper: bad bias tensor");
        memcpy(b.data() + i * each, parts[i]->data, each * 4);
    }
    W_TRY(dalloc(m, out, b.size() * 4));
    cudaError_t e = cudaMemcpy(*out, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? OASR_STATUS_SUCCESS : oasr_internal_cuda_fail(m->be, e, "upload bias", __LINE__);
}

// conv weight ggml [KW=3, IC, OC] f16 -> f16 [OC][K_pad] (row oc: ic*3 + k), zero padded
int upload_conv(oasr_whisper *m, const oasr_named_tensor *t, int IC, int OC, int K_pad, __half **out) {
    if (!t || t->type != OASR_TYPE_F16 || t->ne[0] != 3 || t->ne[1] != IC || t->ne[2] != OC)
        return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper: bad conv weight");
    std::vector<uint16_t> w((size_t)OC * K_pad, 0);
    const uint16_t *src = (const uint16_t *)t->data;
    for (int oc = 0; oc < OC; ++oc)
        memcpy(&w[(size_t)oc * K_pad], src + (size_t)oc * IC * 3, (size_t)IC * 3 * 2);
    W_TRY(dalloc(m, out, w.size() * 2));
    cudaError_t e = cudaMemcpy(*out, w.data(), w.size() * 2, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? OASR_STATUS_SUCCESS : oasr_internal_cuda_fail(m->be, e, "upload conv", __LINE__);
}

int alloc_planes(oasr_whisper *m, void **p, int family, int64_t R, int64_t K) {
    return dalloc(m, (uint8_t **)p, act_planes_bytes(family, R, K));
}

// ---- encoder ----------------------------------------------------------------------------------
// utterance i of the batch writes its cross-attention K|V into slot slot_of[i] (identity when null)
int run_encoder(oasr_whisper *m, int n, const int *slot_of = nullptr) {
    oasr_backend *be = m->be;
    const int d = m->d, H = m->H, T = m->T_enc, nm = m->cfg.n_mels;
    const int64_t M = (int64_t)n * T;
    const int ef = m->enc_family;
    // conv stem: im2col (fp16) + fp16 tensor-core GEMM + bias + GELU, twice
    W_TRY(launch_im2col_f16(be, m->mel, (int64_t)nm * N_MEL_FRAMES, N_MEL_FRAMES, 1, n, nm, N_MEL_FRAMES, N_MEL_FRAMES,
                            3, 1, 1, m->im2col, m->K1p));
    W_TRY(launch_gemm_f16(be, m->im2col, m->K1p, m->conv1_w, m->K1p, n * N_MEL_FRAMES, d, m->K1p, m->c1, d,
                          m->conv1_b, true));
    W_TRY(launch_im2col_f16(be, m->c1, (int64_t)N_MEL_FRAMES * d, 1, d, n, d, N_MEL_FRAMES, T, 3, 2, 1, m->im2col,
                            m->K2p));
    W_TRY(launch_gemm_f16(be, m->im2col, m->K2p, m->conv2_w, m->K2p, (int)M, d, m->K2p, m->x, d, m->conv2_b, true));
    for (int b = 0; b < n; ++b) W_TRY(launch_add_rows(be, m->x + (int64_t)b * T * d, nullptr, m->enc_pos, T, d));

    const ActPlanes qd = act_planes_at(m->qa_d, ef, M, d);
    const ActPlanes qf = act_planes_at(m->qa_f, ef, M, m->ffn);
    const float scale = 1.0f / sqrtf(64.0f);
    for (size_t l = 0; l < m->enc.size(); ++l) {
        const EncLayer &L = m->enc[l];
        const float *pend = l == 0 ? nullptr : m->t;
        const float *pend_b = l == 0 ? nullptr : m->enc[l - 1].b_fc2;
        W_TRY(launch_resid_norm_quant(be, m->x, pend, pend_b, M, d, LN_EPS, false, L.ln1_g, L.ln1_b, nullptr, &qd, ef));
        W_TRY(mul_mat_planes_bias(be, L.qkv, qd, M, m->qkv, 3 * d, L.b_qkv));
        const int64_t ld = 3 * d * 4;
        oasr_tensor q = make_tensor(OASR_TYPE_F32, m->qkv, 64, T, H, n, ld, 256, ld * T);
        oasr_tensor k = make_tensor(OASR_TYPE_F32, m->qkv + d, 64, T, H, n, ld, 256, ld * T);
        oasr_tensor v = make_tensor(OASR_TYPE_F32, m->qkv + 2 * d, 64, T, H, n, ld, 256, ld * T);
        oasr_tensor o = make_tensor(OASR_TYPE_F32, m->attn, 64, H, T, n, 256, (int64_t)d * 4, (int64_t)d * 4 * T);
        W_TRY(oasr_b200_flash_attn_ext(be, &q, &k, &v, nullptr, scale, 0.0f, 0.0f, OASR_PREC_DEFAULT, &o));
        oasr_tensor at = make_tensor(OASR_TYPE_F32, m->attn, d, M, 1, 1, (int64_t)d * 4, (int64_t)d * 4 * M, (int64_t)d * 4 * M);
        W_TRY(launch_quantize_act(be, &at, ef, qd));
        W_TRY(mul_mat_planes(be, L.o, qd, M, m->t, d));
        W_TRY(launch_resid_norm_quant(be, m->x, m->t, L.b_o, M, d, LN_EPS, false, L.ln2_g, L.ln2_b, nullptr, &qd, ef));
        W_TRY(mul_mat_planes(be, L.fc1, qd, M, m->f, m->ffn));
        W_TRY(launch_bias_gelu_quant(be, m->f, L.b_fc1, M, m->ffn, nullptr, &qf, ef));
        W_TRY(mul_mat_planes(be, L.fc2, qf, M, m->t, d));
    }
    // final LN -> encoder output (f32, kept in x) + quantized copy for the cross-KV projections
    const int df = m->dec_family;
    const ActPlanes qx = act_planes_at(m->qa_d, df, M, d);
    W_TRY(launch_resid_norm_quant(be, m->x, m->t, m->enc.back().b_fc2, M, d, LN_EPS, false, m->lnp_g, m->lnp_b, m->x,
                                  &qx, df));
    // cross-attention K|V per decoder layer, stored fp16 [slot][T][2d]
    for (size_t l = 0; l < m->dec.size(); ++l) {
        const DecLayer &L = m->dec[l];
        W_TRY(mul_mat_planes(be, L.ckv, qx, M, m->qkv, 2 * d));
        if (!slot_of) {
            W_TRY(launch_cast_f16(be, m->qkv, 2 * d, L.b_ckv, M, 2 * d, L.cross_kv, 2 * d));
        } else {
            for (int i = 0; i < n; ++i)
                W_TRY(launch_cast_f16(be, m->qkv + (int64_t)i * T * 2 * d, 2 * d, L.b_ckv, T, 2 * d,
                                      L.cross_kv + (int64_t)slot_of[i] * T * 2 * d, 2 * d));
        }
    }
    return OASR_STATUS_SUCCESS;
}

// ---- one decoder step for n sequences at device position *pos -------------------------------
// The decoder step with fused GEMVs (dgemv.cu): 12 launches per layer.
//   LN1 planes -> qkv (q, self-K/V row out) -> self-attention (writes its output as the
//   out-projection's activation planes; with heads not a multiple of 4 the out-projection
//   quantizes them in its prologue instead) -> out-proj -> residual + LN -> cross-q ->
//   cross-attention (+b_cq, same output planes) -> cross-out -> residual + LN -> fc1 ->
//   GELU + quantize -> fc2 -> residual + next LN1 (after the last layer: the final LN
//   into the head's q8_0 planes).
// Both attentions issue their first K/V loads before waiting on their predecessor: the
// cross K/V were written before the step graph started, and of the self K/V only the
// newest row (*nkv - 1) comes from the qkv GEMV in front; *nkv itself only changes in the
// position advance that closes the step (or in a host copy between steps).
static int run_decode_step_fused(oasr_whisper *m, int n) {
    oasr_backend *be = m->be;
    const int d = m->d, H = m->H, T = m->T_enc, P = m->cfg.n_text_ctx;
    const int df = m->dec_family;
    const ActPlanes qd = act_planes_at(m->dqa_d, df, n, d);
    const ActPlanes qf = act_planes_at(m->dqa_f, df, n, m->ffn);
    const ActPlanes ql = act_planes_at(m->dqa_lm, FAMILY_Q8_0, n, d);
    const float scale = 1.0f / sqrtf(64.0f);
    W_TRY(launch_embed_q8_0(be, m->tok_emb, m->tokens, n, m->dec_pos, m->pos, P, m->dx));
    W_TRY(launch_resid_norm_quant(be, m->dx, nullptr, nullptr, n, d, LN_EPS, false, m->dec[0].ln1_g, m->dec[0].ln1_b,
                                  nullptr, &qd, df));
    for (size_t l = 0; l < m->dec.size(); ++l) {
        const DecLayer &L = m->dec[l];
        const bool last = l + 1 == m->dec.size();
        W_TRY(launch_dgemv_qkv(be, L.qkv, qd, n, L.b_qkv, d, m->dq, L.self_k, L.self_v, (int64_t)P * d, m->pos, P));
        {
            oasr_tensor q = make_tensor(OASR_TYPE_F32, m->dq, 64, 1, H, n, (int64_t)d * 4, 256, (int64_t)d * 4);
            oasr_tensor k = make_tensor(OASR_TYPE_F16, L.self_k, 64, P, H, n, (int64_t)d * 2, 128, (int64_t)P * d * 2);
            oasr_tensor v = make_tensor(OASR_TYPE_F16, L.self_v, 64, P, H, n, (int64_t)d * 2, 128, (int64_t)P * d * 2);
            oasr_tensor o = make_tensor(OASR_TYPE_F32, m->dattn, 64, H, 1, n, 256, (int64_t)d * 4, (int64_t)d * 4);
            if (m->attn_planes)
                W_TRY(launch_flash_attn_decode_q8(be, &q, &k, &v, scale, &o, nullptr, m->nkv, qd, df, KV_STATIC_OLD));
            else W_TRY(launch_flash_attn_ex(be, &q, &k, &v, nullptr, scale, &o, nullptr, m->nkv));
        }
        if (m->attn_planes) W_TRY(mul_mat_planes(be, L.o, qd, n, m->dt, d));
        else W_TRY(launch_dgemv_quant(be, L.o, m->dattn, n, m->dt, d));
        W_TRY(launch_resid_norm_quant(be, m->dx, m->dt, L.b_o, n, d, LN_EPS, false, L.lnc_g, L.lnc_b, nullptr, &qd, df));
        W_TRY(mul_mat_planes(be, L.cq, qd, n, m->dq, d));
        {
            oasr_tensor q = make_tensor(OASR_TYPE_F32, m->dq, 64, 1, H, n, (int64_t)d * 4, 256, (int64_t)d * 4);
            oasr_tensor k = make_tensor(OASR_TYPE_F16, L.cross_kv, 64, T, H, n, (int64_t)d * 4, 128, (int64_t)T * d * 4);
            oasr_tensor v = make_tensor(OASR_TYPE_F16, L.cross_kv + d, 64, T, H, n, (int64_t)d * 4, 128, (int64_t)T * d * 4);
            oasr_tensor o = make_tensor(OASR_TYPE_F32, m->dattn, 64, H, 1, n, 256, (int64_t)d * 4, (int64_t)d * 4);
            if (m->attn_planes)
                W_TRY(launch_flash_attn_decode_q8(be, &q, &k, &v, scale, &o, L.b_cq, nullptr, qd, df, KV_STATIC_ALL));
            else W_TRY(launch_flash_attn_ex(be, &q, &k, &v, nullptr, scale, &o, L.b_cq, nullptr));
        }
        if (m->attn_planes) W_TRY(mul_mat_planes(be, L.co, qd, n, m->dt, d));
        else W_TRY(launch_dgemv_quant(be, L.co, m->dattn, n, m->dt, d));
        W_TRY(launch_resid_norm_quant(be, m->dx, m->dt, L.b_co, n, d, LN_EPS, false, L.ln2_g, L.ln2_b, nullptr, &qd, df));
        W_TRY(mul_mat_planes(be, L.fc1, qd, n, m->df, m->ffn));
        W_TRY(launch_bias_gelu_quant(be, m->df, L.b_fc1, n, m->ffn, nullptr, &qf, df));
        W_TRY(mul_mat_planes(be, L.fc2, qf, n, m->dt, d));
        const float *g_next = last ? m->lnd_g : m->dec[l + 1].ln1_g;
        const float *b_next = last ? m->lnd_b : m->dec[l + 1].ln1_b;
        W_TRY(launch_resid_norm_quant(be, m->dx, m->dt, L.b_fc2, n, d, LN_EPS, false, g_next, b_next, nullptr,
                                      last ? &ql : &qd, last ? FAMILY_Q8_0 : df));
    }
    W_TRY(mul_mat_planes(be, m->tok_emb, ql, n, m->logits, m->cfg.n_vocab));
    W_TRY(launch_argmax_rows(be, m->logits, m->cfg.n_vocab, m->cfg.n_vocab, n, m->tokens));
    return OASR_STATUS_SUCCESS;
}

int run_decode_step(oasr_whisper *m, int n) {
    if (m->fused_dec) return run_decode_step_fused(m, n);
    oasr_backend *be = m->be;
    const int d = m->d, H = m->H, T = m->T_enc, P = m->cfg.n_text_ctx;
    const int df = m->dec_family;
    const ActPlanes qd = act_planes_at(m->dqa_d, df, n, d);
    const ActPlanes qf = act_planes_at(m->dqa_f, df, n, m->ffn);
    const ActPlanes ql = act_planes_at(m->dqa_lm, FAMILY_Q8_0, n, d);
    const float scale = 1.0f / sqrtf(64.0f);
    W_TRY(launch_embed_q8_0(be, m->tok_emb, m->tokens, n, m->dec_pos, m->pos, P, m->dx));
    for (size_t l = 0; l < m->dec.size(); ++l) {
        const DecLayer &L = m->dec[l];
        const float *pend = l == 0 ? nullptr : m->dt;
        const float *pend_b = l == 0 ? nullptr : m->dec[l - 1].b_fc2;
        W_TRY(launch_resid_norm_quant(be, m->dx, pend, pend_b, n, d, LN_EPS, false, L.ln1_g, L.ln1_b, nullptr, &qd, df));
        W_TRY(mul_mat_planes(be, L.qkv, qd, n, m->dqkv, 3 * d));
        W_TRY(launch_qkv_split_kv_write(be, m->dqkv, L.b_qkv, n, d, m->dq, L.self_k, L.self_v, (int64_t)P * d, m->pos, P));
        {
            oasr_tensor q = make_tensor(OASR_TYPE_F32, m->dq, 64, 1, H, n, (int64_t)d * 4, 256, (int64_t)d * 4);
            oasr_tensor k = make_tensor(OASR_TYPE_F16, L.self_k, 64, P, H, n, (int64_t)d * 2, 128, (int64_t)P * d * 2);
            oasr_tensor v = make_tensor(OASR_TYPE_F16, L.self_v, 64, P, H, n, (int64_t)d * 2, 128, (int64_t)P * d * 2);
            oasr_tensor o = make_tensor(OASR_TYPE_F32, m->dattn, 64, H, 1, n, 256, (int64_t)d * 4, (int64_t)d * 4);
            W_TRY(launch_flash_attn_ex(be, &q, &k, &v, nullptr, scale, &o, nullptr, m->nkv));
        }
        oasr_tensor at = make_tensor(OASR_TYPE_F32, m->dattn, d, n, 1, 1, (int64_t)d * 4, (int64_t)d * 4 * n, (int64_t)d * 4 * n);
        W_TRY(launch_quantize_act(be, &at, df, qd));
        W_TRY(mul_mat_planes(be, L.o, qd, n, m->dt, d));
        W_TRY(launch_resid_norm_quant(be, m->dx, m->dt, L.b_o, n, d, LN_EPS, false, L.lnc_g, L.lnc_b, nullptr, &qd, df));
        W_TRY(mul_mat_planes(be, L.cq, qd, n, m->dq, d));
        {
            oasr_tensor q = make_tensor(OASR_TYPE_F32, m->dq, 64, 1, H, n, (int64_t)d * 4, 256, (int64_t)d * 4);
            oasr_tensor k = make_tensor(OASR_TYPE_F16, L.cross_kv, 64, T, H, n, (int64_t)d * 4, 128, (int64_t)T * d * 4);
            oasr_tensor v = make_tensor(OASR_TYPE_F16, L.cross_kv + d, 64, T, H, n, (int64_t)d * 4, 128, (int64_t)T * d * 4);
            oasr_tensor o = make_tensor(OASR_TYPE_F32, m->dattn, 64, H, 1, n, 256, (int64_t)d * 4, (int64_t)d * 4);
            W_TRY(launch_flash_attn_ex(be, &q, &k, &v, nullptr, scale, &o, L.b_cq, nullptr));
        }
        W_TRY(launch_quantize_act(be, &at, df, qd));
        W_TRY(mul_mat_planes(be, L.co, qd, n, m->dt, d));
        W_TRY(launch_resid_norm_quant(be, m->dx, m->dt, L.b_co, n, d, LN_EPS, false, L.ln2_g, L.ln2_b, nullptr, &qd, df));
        W_TRY(mul_mat_planes(be, L.fc1, qd, n, m->df, m->ffn));
        W_TRY(launch_bias_gelu_quant(be, m->df, L.b_fc1, n, m->ffn, nullptr, &qf, df));
        W_TRY(mul_mat_planes(be, L.fc2, qf, n, m->dt, d));
    }
    W_TRY(launch_resid_norm_quant(be, m->dx, m->dt, m->dec.back().b_fc2, n, d, LN_EPS, false, m->lnd_g, m->lnd_b,
                                  nullptr, &ql, FAMILY_Q8_0));
    W_TRY(mul_mat_planes(be, m->tok_emb, ql, n, m->logits, m->cfg.n_vocab));
    W_TRY(launch_argmax_rows(be, m->logits, m->cfg.n_vocab, m->cfg.n_vocab, n, m->tokens));
    return OASR_STATUS_SUCCESS;
}

__global__ void fill_tokens_kernel(int *tokens, int n, int value) {
    griddep_wait();
    if (threadIdx.x < n) tokens[threadIdx.x] = value;
}

int decode_step_graph(oasr_whisper *m, int n) {
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
        // inside the step graph every kernel waits on its predecessor with griddepcontrol,
        // so successive launches overlap their prologues (programmatic dependent launch)
        be->pdl = m->pdl;
        int st = run_decode_step(m, n);
        if (st == OASR_STATUS_SUCCESS)
            st = launch_decode_advance(be, m->tokens, m->pos, m->nkv, m->history, n, (int)m->cfg.n_text_ctx);
        be->pdl = false;
        cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (st) return st;
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "cudaStreamEndCapture", __LINE__);
        e = cudaGraphInstantiate(&m->graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "cudaGraphInstantiate", __LINE__);
        m->graph_batch = n;
        m->graph_epoch = be->scratch_epoch;
    }
    OASR_CUDA_TRY(be, cudaGraphLaunch(m->graph, m->stream));
    return OASR_STATUS_SUCCESS;
}

// every slot at position pos (its KV length pos + 1)
int set_position(oasr_whisper *m, int pos) {
    std::vector<int> v(2 * (size_t)m->B);
    for (int b = 0; b < m->B; ++b) {
        v[b] = pos;
        v[m->B + b] = pos + 1;
    }
    OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->pos, v.data(), (size_t)m->B * 4, cudaMemcpyHostToDevice, m->stream));
    OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->nkv, v.data() + m->B, (size_t)m->B * 4, cudaMemcpyHostToDevice, m->stream));
    return OASR_STATUS_SUCCESS;
}

// ---- serving: continuous batching over a queue of utterances --------------------------------
// (seq2seq_serve_batch.rs:224-640 run_batch / decode_continuous_batch)

// admission: slot slots[i] starts utterance i of the group -- position 0, the first prompt
// token as its input, its generated-token budget
__global__ void serve_admit_kernel(const int *io, int n, const int *prompt, int *tokens, int *pos, int *nkv,
                                   int *done, int *budget) {
    const int i = threadIdx.x;
    if (i >= n) return;
    const int b = io[i];
    tokens[b] = prompt[0];
    pos[b] = 0;
    nkv[b] = 1;
    done[b] = 0;
    budget[b] = io[n + i];
}

// every slot parked (done) at position 0: slots outside the active set compute harmlessly
__global__ void serve_park_kernel(int n, const int *prompt, int *tokens, int *pos, int *nkv, int *done, int *budget) {
    const int b = threadIdx.x;
    if (b >= n) return;
    tokens[b] = prompt[0];
    pos[b] = 0;
    nkv[b] = 1;
    done[b] = 1;
    budget[b] = 1;
}

int width_index(int w) { return w <= 1 ? 0 : w <= 2 ? 1 : w <= 4 ? 2 : 3; }

// one serve step of `w` slots: the decode step, then the per-slot advance with teacher-forced
// prompts and done detection; one CUDA graph per power-of-two width
int serve_step_graph(oasr_whisper *m, int w, const ServeCtl &sc) {
    oasr_backend *be = m->be;
    if (be->scratch_bytes < m->step_scratch) {
        int st = 0;
        oasr_internal_scratch(be, m->step_scratch, &st);
        if (st) return st;
    }
    const int gi = width_index(w);
    cudaGraphExec_t &g = m->serve_graph[gi];
    if (g && m->serve_epoch[gi] != be->scratch_epoch) {
        cudaGraphExecDestroy(g);
        g = nullptr;
    }
    if (!g) {
        cudaGraph_t graph;
        OASR_CUDA_TRY(be, cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        be->pdl = m->pdl;
        int st = run_decode_step(m, w);
        if (st == OASR_STATUS_SUCCESS)
            st = launch_decode_advance(be, m->tokens, m->pos, m->nkv, m->history, w, (int)m->cfg.n_text_ctx, sc);
        be->pdl = false;
        const cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
        if (st) return st;
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "cudaStreamEndCapture", __LINE__);
        const cudaError_t ie = cudaGraphInstantiate(&g, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return oasr_internal_cuda_fail(be, ie, "cudaGraphInstantiate", __LINE__);
        m->serve_epoch[gi] = be->scratch_epoch;
    }
    OASR_CUDA_TRY(be, cudaGraphLaunch(g, m->stream));
    return OASR_STATUS_SUCCESS;
}

// move slot `src`'s whole state to slot `dst` (compaction before a narrower width): its
// cross-attention K|V, self-attention K/V rows, position, input, flags and history
int serve_move_slot(oasr_whisper *m, int src, int dst) {
    oasr_backend *be = m->be;
    const int64_t d = m->d, T = m->T_enc, P = m->cfg.n_text_ctx;
    for (const DecLayer &L : m->dec) {
        OASR_CUDA_TRY(be, cudaMemcpyAsync(L.cross_kv + dst * T * 2 * d, L.cross_kv + src * T * 2 * d,
                                          (size_t)(T * 2 * d * 2), cudaMemcpyDeviceToDevice, m->stream));
        OASR_CUDA_TRY(be, cudaMemcpyAsync(L.self_k + dst * P * d, L.self_k + src * P * d, (size_t)(P * d * 2),
                                          cudaMemcpyDeviceToDevice, m->stream));
        OASR_CUDA_TRY(be, cudaMemcpyAsync(L.self_v + dst * P * d, L.self_v + src * P * d, (size_t)(P * d * 2),
                                          cudaMemcpyDeviceToDevice, m->stream));
    }
    for (int *a : {m->tokens, m->pos, m->nkv, m->done, m->budget})
        OASR_CUDA_TRY(be, cudaMemcpyAsync(a + dst, a + src, 4, cudaMemcpyDeviceToDevice, m->stream));
    OASR_CUDA_TRY(be, cudaMemcpyAsync(m->history + dst * P, m->history + src * P, (size_t)P * 4,
                                      cudaMemcpyDeviceToDevice, m->stream));
    return OASR_STATUS_SUCCESS;
}

}  // namespace

namespace oasr {

void whisper_hann_window(float *w, int n) {
    const float scale = 3.14159265358979323846f * 2.0f / (float)n;
    for (int i = 0; i < n; ++i) w[i] = 0.5f - 0.5f * cosf(scale * (float)i);
}

static float hz_to_mel_slaney(float hz) {
    const float f_sp = 200.0f / 3.0f, min_log_hz = 1000.0f;
    const float min_log_mel = (min_log_hz - 0.0f) / f_sp;
    const float logstep = logf(6.4f) / 27.0f;
    return hz >= min_log_hz ? min_log_mel + logf(hz / min_log_hz) / logstep : (hz - 0.0f) / f_sp;
}

static float mel_to_hz_slaney(float mel) {
    const float f_sp = 200.0f / 3.0f, min_log_hz = 1000.0f;
    const float min_log_mel = (min_log_hz - 0.0f) / f_sp;
    const float logstep = logf(6.4f) / 27.0f;
    return mel >= min_log_mel ? min_log_hz * expf(logstep * (mel - min_log_mel)) : 0.0f + f_sp * mel;
}

void whisper_mel_filters(float *filt, int n_mels, int n_fft, float sr) {
    const int bins = n_fft / 2 + 1;
    const float mel_min = hz_to_mel_slaney(0.0f), mel_max = hz_to_mel_slaney(8000.0f);
    std::vector<float> hz(n_mels + 2);
    for (int i = 0; i < n_mels + 2; ++i) {
        const float ratio = (float)i / (float)(n_mels + 1);
        hz[i] = mel_to_hz_slaney(mel_min + ratio * (mel_max - mel_min));
    }
    for (int m = 0; m < n_mels; ++m) {
        const float left = hz[m], center = hz[m + 1], right = hz[m + 2];
        const float enorm = 2.0f / (right - left);
        for (int b = 0; b < bins; ++b) {
            const float f = (float)b * sr / (float)n_fft;
            const float lower = (f - left) / (center - left), upper = (right - f) / (right - center);
            float w = lower < upper ? lower : upper;
            w = w > 0.0f ? w : 0.0f;
            filt[m * bins + b] = w * enorm;
        }
    }
}

}  // namespace oasr

extern "C" {

int oasr_b200_whisper_free(oasr_whisper *m) {
    if (!m) return OASR_STATUS_SUCCESS;
    cudaSetDevice(m->be->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    for (cudaGraphExec_t g : m->serve_graph)
        if (g) cudaGraphExecDestroy(g);
    for (auto *w : m->weights) oasr_b200_weight_free(m->be, w);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_whisper_load(oasr_backend *be, const oasr_whisper_config *cfg, const oasr_named_tensor *tensors,
                           int32_t n_tensors, oasr_whisper **out) {
    if (!out) return OASR_STATUS_FAILED;
    *out = nullptr;
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!cfg || !tensors || cfg->d_model % 64 || cfg->n_heads * 64 != cfg->d_model || cfg->max_batch < 1 ||
        cfg->max_batch > 8 || cfg->n_audio_ctx * 2 != N_MEL_FRAMES || cfg->n_enc_layers < 1 || cfg->n_dec_layers < 1)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "whisper_load: unsupported config");
    std::map<std::string, const oasr_named_tensor *> tm;
    for (int i = 0; i < n_tensors; ++i) tm[tensors[i].name] = &tensors[i];
    oasr_whisper *m = new oasr_whisper();
    m->be = be;
    m->cfg = *cfg;
    m->d = cfg->d_model;
    m->H = cfg->n_heads;
    m->ffn = 4 * cfg->d_model;
    m->T_enc = cfg->n_audio_ctx;
    m->B = cfg->max_batch;
    {
        // serving width capped by the device memory left for per-slot state once the
        // weights are resident (serve_batch_vram_capped_max_batch, serve_batch_env.rs:295-315)
        // device bytes of the resident weights: raw blocks + decode tiles, and for Q4_K the
        // tensor-core GEMM's fp16 operand (2 B per element = 3.6x the 4.5-bit blocks)
        uint64_t used = 0;
        for (int i = 0; i < n_tensors; ++i)
            used += tensors[i].bytes * (tensors[i].type == OASR_TYPE_Q4_K ? 6 : 3);
        size_t free_b = 0, total_b = 0;
        if (cfg->max_batch > 2 && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
            const uint64_t avail = free_b > used ? free_b - used : 0;
            m->B = oasr_b200_serve_batch_vram_cap(cfg->max_batch, oasr::whisper_slot_bytes(cfg), avail,
                                                  oasr::serve_vram_reserve_bytes());
        }
    }
    m->K1p = (3 * cfg->n_mels + 63) / 64 * 64;
    m->K2p = (3 * cfg->d_model + 63) / 64 * 64;
    m->graph = nullptr;
    m->graph_batch = 0;
    m->stream = nullptr;
    for (int i = 0; i < 4; ++i) {
        m->serve_graph[i] = nullptr;
        m->serve_epoch[i] = 0;
    }
    m->serve_key[0] = m->serve_key[1] = m->serve_key[2] = -1;
    auto fail = [&](int s) {
        oasr_b200_whisper_free(m);
        return s;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(OASR_STATUS_ALLOC_FAILED);
    const int d = m->d, B = m->B, T = m->T_enc, P = cfg->n_text_ctx, nm = cfg->n_mels;
    auto T_ = [&](const std::string &n) { return find(tm, n); };
#define L_TRY(expr)                 \
    do {                            \
        int _s = (expr);            \
        if (_s) return fail(_s);    \
    } while (0)
    // prelude
    L_TRY(upload_conv(m, T_("encoder.conv1.weight"), nm, d, m->K1p, &m->conv1_w));
    L_TRY(upload_conv(m, T_("encoder.conv2.weight"), d, d, m->K2p, &m->conv2_w));
    L_TRY(upload_f32(m, T_("encoder.conv1.bias"), d, &m->conv1_b, "encoder.conv1.bias"));
    L_TRY(upload_f32(m, T_("encoder.conv2.bias"), d, &m->conv2_b, "encoder.conv2.bias"));
    L_TRY(upload_f32(m, T_("encoder.positional_embedding"), (int64_t)T * d, &m->enc_pos, "encoder.positional_embedding"));
    for (int l = 0; l < cfg->n_enc_layers; ++l) {
        const std::string p = "encoder.blocks." + std::to_string(l) + ".";
        EncLayer L;
        L_TRY(upload_cat(m, {T_(p + "attn.query.weight"), T_(p + "attn.key.weight"), T_(p + "attn.value.weight")}, d, &L.qkv, p + "attn.qkv"));
        L_TRY(upload_cat(m, {T_(p + "attn.out.weight")}, d, &L.o, p + "attn.out"));
        L_TRY(upload_cat(m, {T_(p + "mlp.0.weight")}, d, &L.fc1, p + "mlp.0"));
        L_TRY(upload_cat(m, {T_(p + "mlp.2.weight")}, m->ffn, &L.fc2, p + "mlp.2"));
        L_TRY(upload_bias_cat(m, {T_(p + "attn.query.bias"), nullptr, T_(p + "attn.value.bias")}, d, &L.b_qkv));
        L_TRY(upload_f32(m, T_(p + "attn.out.bias"), d, &L.b_o, "attn.out.bias"));
        L_TRY(upload_f32(m, T_(p + "mlp.0.bias"), m->ffn, &L.b_fc1, "mlp.0.bias"));
        L_TRY(upload_f32(m, T_(p + "mlp.2.bias"), d, &L.b_fc2, "mlp.2.bias"));
        L_TRY(upload_f32(m, T_(p + "attn_ln.weight"), d, &L.ln1_g, "attn_ln.weight"));
        L_TRY(upload_f32(m, T_(p + "attn_ln.bias"), d, &L.ln1_b, "attn_ln.bias"));
        L_TRY(upload_f32(m, T_(p + "mlp_ln.weight"), d, &L.ln2_g, "mlp_ln.weight"));
        L_TRY(upload_f32(m, T_(p + "mlp_ln.bias"), d, &L.ln2_b, "mlp_ln.bias"));
        m->enc.push_back(L);
    }
    L_TRY(upload_f32(m, T_("encoder.ln_post.weight"), d, &m->lnp_g, "encoder.ln_post.weight"));
    L_TRY(upload_f32(m, T_("encoder.ln_post.bias"), d, &m->lnp_b, "encoder.ln_post.bias"));
    // decoder
    {
        const oasr_named_tensor *te = T_("decoder.token_embedding.weight");
        if (!te || te->type != OASR_TYPE_Q8_0 || te->ne[0] != d || te->ne[1] != cfg->n_vocab)
            return fail(oasr_internal_fail(be, OASR_STATUS_FAILED, "whisper: token embedding must be Q8_0 [d, vocab]"));
        L_TRY(upload_cat(m, {te}, d, &m->tok_emb, "decoder.token_embedding"));
    }
    L_TRY(upload_f32(m, T_("decoder.positional_embedding"), (int64_t)P * d, &m->dec_pos, "decoder.positional_embedding"));
    for (int l = 0; l < cfg->n_dec_layers; ++l) {
        const std::string p = "decoder.blocks." + std::to_string(l) + ".";
        DecLayer L;
        L_TRY(upload_cat(m, {T_(p + "attn.query.weight"), T_(p + "attn.key.weight"), T_(p + "attn.value.weight")}, d, &L.qkv, p + "attn.qkv"));
        L_TRY(upload_cat(m, {T_(p + "attn.out.weight")}, d, &L.o, p + "attn.out"));
        L_TRY(upload_cat(m, {T_(p + "cross_attn.query.weight")}, d, &L.cq, p + "cross_attn.query"));
        L_TRY(upload_cat(m, {T_(p + "cross_attn.key.weight"), T_(p + "cross_attn.value.weight")}, d, &L.ckv, p + "cross_attn.kv"));
        L_TRY(upload_cat(m, {T_(p + "cross_attn.out.weight")}, d, &L.co, p + "cross_attn.out"));
        L_TRY(upload_cat(m, {T_(p + "mlp.0.weight")}, d, &L.fc1, p + "mlp.0"));
        L_TRY(upload_cat(m, {T_(p + "mlp.2.weight")}, m->ffn, &L.fc2, p + "mlp.2"));
        L_TRY(upload_bias_cat(m, {T_(p + "attn.query.bias"), nullptr, T_(p + "attn.value.bias")}, d, &L.b_qkv));
        L_TRY(upload_f32(m, T_(p + "attn.out.bias"), d, &L.b_o, "attn.out.bias"));
        L_TRY(upload_f32(m, T_(p + "cross_attn.query.bias"), d, &L.b_cq, "cross_attn.query.bias"));
        L_TRY(upload_bias_cat(m, {nullptr, T_(p + "cross_attn.value.bias")}, d, &L.b_ckv));
        L_TRY(upload_f32(m, T_(p + "cross_attn.out.bias"), d, &L.b_co, "cross_attn.out.bias"));
        L_TRY(upload_f32(m, T_(p + "mlp.0.bias"), m->ffn, &L.b_fc1, "mlp.0.bias"));
        L_TRY(upload_f32(m, T_(p + "mlp.2.bias"), d, &L.b_fc2, "mlp.2.bias"));
        L_TRY(upload_f32(m, T_(p + "attn_ln.weight"), d, &L.ln1_g, "attn_ln.weight"));
        L_TRY(upload_f32(m, T_(p + "attn_ln.bias"), d, &L.ln1_b, "attn_ln.bias"));
        L_TRY(upload_f32(m, T_(p + "cross_attn_ln.weight"), d, &L.lnc_g, "cross_attn_ln.weight"));
        L_TRY(upload_f32(m, T_(p + "cross_attn_ln.bias"), d, &L.lnc_b, "cross_attn_ln.bias"));
        L_TRY(upload_f32(m, T_(p + "mlp_ln.weight"), d, &L.ln2_g, "mlp_ln.weight"));
        L_TRY(upload_f32(m, T_(p + "mlp_ln.bias"), d, &L.ln2_b, "mlp_ln.bias"));
        L_TRY(dalloc(m, &L.self_k, (size_t)B * P * d * 2));
        L_TRY(dalloc(m, &L.self_v, (size_t)B * P * d * 2));
        L_TRY(dalloc(m, &L.cross_kv, (size_t)B * T * 2 * d * 2));
        // slots that never held an utterance read zeros, not stale memory
        if (cudaMemset(L.cross_kv, 0, (size_t)B * T * 2 * d * 2) != cudaSuccess)
            return fail(oasr_internal_fail(be, OASR_STATUS_FAILED, "whisper: cross-K/V clear failed"));
        m->dec.push_back(L);
    }
    L_TRY(upload_f32(m, T_("decoder.ln.weight"), d, &m->lnd_g, "decoder.ln.weight"));
    L_TRY(upload_f32(m, T_("decoder.ln.bias"), d, &m->lnd_b, "decoder.ln.bias"));
    m->enc_family = weight_family(m->enc[0].fc1);
    m->dec_family = weight_family(m->dec[0].fc1);
    if (weight_family(m->dec[0].ckv) != m->dec_family)
        return fail(oasr_internal_fail(be, OASR_STATUS_FAILED, "whisper: decoder weights must share one type family"));
    {
        // fused decoder GEMVs need every decoder linear in decode tiles;
        // OASR_B200_DECODE_FUSION=off keeps the unfused kernel sequence
        const char *pdl_env = getenv("OASR_B200_PDL");
        m->pdl = !(pdl_env && strcmp(pdl_env, "0") == 0);
        const char *env = getenv("OASR_B200_DECODE_FUSION");
        m->fused_dec = !(env && strcmp(env, "off") == 0) && B <= 8;
        for (const DecLayer &L : m->dec)
            m->fused_dec = m->fused_dec && dgemv_supported(L.qkv, false) && dgemv_supported(L.o, true) &&
                           dgemv_supported(L.cq, false) && dgemv_supported(L.co, true) &&
                           dgemv_supported(L.fc1, false) && dgemv_supported(L.fc2, false);
        if (m->fused_dec) L_TRY(dgemv_configure(be));
        // the 4-head decode attention (heads a multiple of 4) quantizes its 256-value output
        // chunks itself, so the out-projections run as plain GEMVs (measured faster than
        // quantizing the attention rows in every GEMV CTA's prologue)
        m->attn_planes = m->fused_dec && flash_attn_decode_q8_supported(m->H, m->H, 64, m->dec_family);
    }
    // frontend tables (host-computed like the reference's plan, whisper/mel.rs:64-96)
    {
        std::vector<float> win(N_FFT), filt((size_t)nm * (N_FFT / 2 + 1));
        std::vector<float2> tw(N_FFT);
        whisper_hann_window(win.data(), N_FFT);
        whisper_mel_filters(filt.data(), nm, N_FFT, 16000.0f);
        for (int j = 0; j < N_FFT; ++j) {
            const double a = 2.0 * 3.14159265358979323846 * (double)j / (double)N_FFT;
            tw[j] = make_float2((float)cos(a), (float)-sin(a));
        }
        L_TRY(dalloc(m, &m->window, N_FFT * 4));
        L_TRY(dalloc(m, &m->filters, filt.size() * 4));
        L_TRY(dalloc(m, &m->twiddle, N_FFT * sizeof(float2)));
        cudaMemcpy(m->window, win.data(), N_FFT * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(m->filters, filt.data(), filt.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(m->twiddle, tw.data(), N_FFT * sizeof(float2), cudaMemcpyHostToDevice);
    }
    const int64_t M = (int64_t)B * T;
    L_TRY(dalloc(m, &m->audio, (size_t)B * N_SAMPLES_30S * 4));
    L_TRY(dalloc(m, &m->power, (size_t)B * N_MEL_FRAMES * (N_FFT / 2 + 1) * 4));
    L_TRY(dalloc(m, &m->mel, (size_t)B * nm * N_MEL_FRAMES * 4));
    L_TRY(dalloc(m, &m->max_key, (size_t)B * 4));
    L_TRY(dalloc(m, &m->im2col, (size_t)B * N_MEL_FRAMES * std::max(m->K1p, m->K2p) * 2));
    L_TRY(dalloc(m, &m->c1, (size_t)B * N_MEL_FRAMES * d * 4));
    L_TRY(dalloc(m, &m->x, (size_t)M * d * 4));
    L_TRY(dalloc(m, &m->qkv, (size_t)M * 3 * d * 4));
    L_TRY(dalloc(m, &m->attn, (size_t)M * d * 4));
    L_TRY(dalloc(m, &m->t, (size_t)M * d * 4));
    L_TRY(dalloc(m, &m->f, (size_t)M * m->ffn * 4));
    L_TRY(alloc_planes(m, &m->qa_d, FAMILY_Q8_K, M, d));  // the larger family layout covers both
    L_TRY(alloc_planes(m, &m->qa_f, FAMILY_Q8_K, M, m->ffn));
    L_TRY(dalloc(m, &m->dx, (size_t)B * d * 4));
    L_TRY(dalloc(m, &m->dqkv, (size_t)B * 3 * d * 4));
    L_TRY(dalloc(m, &m->dq, (size_t)B * d * 4));
    L_TRY(dalloc(m, &m->dattn, (size_t)B * d * 4));
    L_TRY(dalloc(m, &m->dt, (size_t)B * d * 4));
    L_TRY(dalloc(m, &m->df, (size_t)B * m->ffn * 4));
    L_TRY(dalloc(m, &m->logits, (size_t)B * cfg->n_vocab * 4));
    L_TRY(alloc_planes(m, &m->dqa_d, FAMILY_Q8_K, B, d));
    L_TRY(alloc_planes(m, &m->dqa_f, FAMILY_Q8_K, B, m->ffn));
    L_TRY(alloc_planes(m, &m->dqa_lm, FAMILY_Q8_0, B, d));
    L_TRY(dalloc(m, &m->tokens, (size_t)B * 4));
    L_TRY(dalloc(m, &m->pos, (size_t)B * 4));  // per slot
    L_TRY(dalloc(m, &m->nkv, (size_t)B * 4));
    L_TRY(dalloc(m, &m->history, (size_t)B * P * 4));
    L_TRY(dalloc(m, &m->done, (size_t)B * 4));
    L_TRY(dalloc(m, &m->budget, (size_t)B * 4));
    L_TRY(dalloc(m, &m->prompt_dev, (size_t)P * 4));
    L_TRY(dalloc(m, &m->serve_io, (size_t)4 * B * 4));
    // flash-decode partials for the largest split configuration seen by a decoder step
    m->step_scratch = (size_t)std::max<int64_t>(64ll << 20, (int64_t)B * m->H * 1024 * 66 * 4);
    L_TRY(oasr_b200_reserve_scratch(be, m->step_scratch));
#undef L_TRY
    *out = m;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_whisper_mel(oasr_whisper *m, const float *pcm, const int64_t *n_samples, int32_t n_utts, float *mel_out) {
    if (!m || !pcm || !n_samples || n_utts < 1 || n_utts > m->B) return OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    StreamScope sc(m);
    const int nm = m->cfg.n_mels;
    // pad / trim every clip to 30 s (whisper/mel.rs pad_or_trim_audio)
    int64_t off = 0;
    OASR_CUDA_TRY(m->be, cudaMemsetAsync(m->audio, 0, (size_t)n_utts * N_SAMPLES_30S * 4, m->stream));
    for (int b = 0; b < n_utts; ++b) {
        if (n_samples[b] < 1) return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper_mel: empty clip");
        const int64_t take = std::min<int64_t>(n_samples[b], N_SAMPLES_30S);
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->audio + (int64_t)b * N_SAMPLES_30S, pcm + off, take * 4,
                                             cudaMemcpyHostToDevice, m->stream));
        off += n_samples[b];
    }
    W_TRY(launch_mel(m->be, m->audio, n_utts, N_SAMPLES_30S, N_MEL_FRAMES, nm, m->window, m->twiddle, m->filters,
                     m->power, m->mel, m->max_key));
    if (mel_out) {
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(mel_out, m->mel, (size_t)n_utts * nm * N_MEL_FRAMES * 4,
                                             cudaMemcpyDeviceToHost, m->stream));
        OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
    }
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_whisper_encode(oasr_whisper *m, const float *mel_host, int32_t n_utts, float *enc_out) {
    if (!m || n_utts < 1 || n_utts > m->B) return OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    StreamScope sc(m);
    if (mel_host)
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->mel, mel_host, (size_t)n_utts * m->cfg.n_mels * N_MEL_FRAMES * 4,
                                             cudaMemcpyHostToDevice, m->stream));
    W_TRY(run_encoder(m, n_utts));
    if (enc_out)
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(enc_out, m->x, (size_t)n_utts * m->T_enc * m->d * 4, cudaMemcpyDeviceToHost,
                                             m->stream));
    OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
    return oasr_b200_synchronize(m->be);
}

int oasr_b200_whisper_decode_step(oasr_whisper *m, const int32_t *tokens, int32_t n_utts, int32_t pos, float *logits,
                                  int32_t *next) {
    if (!m || !tokens || n_utts < 1 || n_utts > m->B || pos < 0 || pos >= m->cfg.n_text_ctx) return OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    StreamScope sc(m);
    OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->tokens, tokens, n_utts * 4, cudaMemcpyHostToDevice, m->stream));
    W_TRY(set_position(m, pos));
    W_TRY(run_decode_step(m, n_utts));
    if (logits)
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(logits, m->logits, (size_t)n_utts * m->cfg.n_vocab * 4,
                                             cudaMemcpyDeviceToHost, m->stream));
    if (next) OASR_CUDA_TRY(m->be, cudaMemcpyAsync(next, m->tokens, n_utts * 4, cudaMemcpyDeviceToHost, m->stream));
    OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
    return oasr_b200_synchronize(m->be);
}

int oasr_b200_whisper_mel_device(oasr_whisper *m, const float *pcm_dev, const int64_t *n_samples, int32_t n_utts) {
    if (!m || !pcm_dev || !n_samples || n_utts < 1 || n_utts > m->B) return OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    StreamScope sc(m);
    int64_t off = 0;
    OASR_CUDA_TRY(m->be, cudaMemsetAsync(m->audio, 0, (size_t)n_utts * N_SAMPLES_30S * 4, m->stream));
    for (int b = 0; b < n_utts; ++b) {
        if (n_samples[b] < 1) return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper_mel: empty clip");
        const int64_t take = std::min<int64_t>(n_samples[b], N_SAMPLES_30S);
        OASR_CUDA_TRY(m->be, cudaMemcpyAsync(m->audio + (int64_t)b * N_SAMPLES_30S, pcm_dev + off, take * 4,
                                             cudaMemcpyDeviceToDevice, m->stream));
        off += n_samples[b];
    }
    return launch_mel(m->be, m->audio, n_utts, N_SAMPLES_30S, N_MEL_FRAMES, m->cfg.n_mels, m->window, m->twiddle,
                      m->filters, m->power, m->mel, m->max_key);
}

int oasr_b200_whisper_generate(oasr_whisper *m, int32_t n_utts, const int32_t *prompt, int32_t n_prompt, int32_t n_new,
                               int32_t eot, int32_t stop_at_eot, int32_t *tokens_out, int32_t tokens_on_device) {
    if (!m || !prompt || n_utts < 1 || n_utts > m->B || n_prompt < 1 || n_new < 1 ||
        n_prompt + n_new > m->cfg.n_text_ctx || !tokens_out)
        return OASR_STATUS_FAILED;
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    StreamScope sc(m);
    W_TRY(run_encoder(m, n_utts));
    const int P = m->cfg.n_text_ctx;
    W_TRY(set_position(m, 0));
    std::vector<int32_t> last(n_utts);
    for (int i = 0; i < n_prompt + n_new - 1; ++i) {
        if (m->be->abort_cb && m->be->abort_cb(m->be->abort_data)) return OASR_STATUS_ABORTED;  // step checkpoint
        if (i < n_prompt) {
            // prompt token i for every sequence: one device-side fill, no host buffer to keep alive
            fill_tokens_kernel<<<1, 32, 0, m->stream>>>(m->tokens, n_utts, prompt[i]);
        }
        W_TRY(decode_step_graph(m, n_utts));
        if (stop_at_eot && i >= n_prompt - 1) {
            OASR_CUDA_TRY(m->be, cudaMemcpyAsync(last.data(), m->tokens, n_utts * 4, cudaMemcpyDeviceToHost, m->stream));
            OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
            bool all = true;
            for (int b = 0; b < n_utts; ++b) all = all && last[b] == eot;
            if (all) break;
        }
    }
    // tokens_out[b][i] = history[b][n_prompt + i]
    OASR_CUDA_TRY(m->be, cudaMemcpy2DAsync(tokens_out, (size_t)n_new * 4, m->history + n_prompt, (size_t)P * 4,
                                           (size_t)n_new * 4, n_utts,
                                           tokens_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                           m->stream));
    if (!tokens_on_device) {
        OASR_CUDA_TRY(m->be, cudaStreamSynchronize(m->stream));
        return oasr_b200_synchronize(m->be);
    }
    return oasr_internal_launch_check(m->be, "whisper_generate");
}


int oasr_b200_whisper_max_batch(oasr_whisper *m) { return m ? m->B : 0; }

int oasr_b200_whisper_serve(oasr_whisper *m, const float *pcm, const int64_t *n_samples, int32_t n_utts,
                            const int32_t *prompt, int32_t n_prompt, const int32_t *budgets, int32_t max_new,
                            int32_t eot, int32_t stop_at_eot, int32_t max_width, int32_t check_every,
                            int32_t *tokens_out, int32_t *lengths_out, oasr_serve_stats *stats) {
    const int P = m ? (int)m->cfg.n_text_ctx : 0;
    if (!m || !pcm || !n_samples || n_utts < 1 || !prompt || n_prompt < 1 || max_new < 1 ||
        n_prompt + max_new > P || !tokens_out || !lengths_out || max_width < 0 || check_every < 1)
        return m ? oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper_serve: bad arguments") : OASR_STATUS_FAILED;
    for (int r = 0; r < n_utts; ++r)
        if (n_samples[r] < 1 || (budgets && (budgets[r] < 1 || budgets[r] > max_new)))
            return oasr_internal_fail(m->be, OASR_STATUS_FAILED, "whisper_serve: empty clip or budget out of range");
    int st = oasr_internal_precheck(m->be);
    if (st) return st;
    StreamScope sc(m);
    oasr_backend *be = m->be;
    const int W = max_width > 0 ? std::min(max_width, m->B) : m->B;
    std::vector<int64_t> off(n_utts + 1, 0);
    for (int r = 0; r < n_utts; ++r) off[r + 1] = off[r] + n_samples[r];
    OASR_CUDA_TRY(be, cudaMemcpyAsync(m->prompt_dev, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, m->stream));
    // the captured step graphs hold the serving parameters: re-capture when they change
    if (m->serve_key[0] != n_prompt || m->serve_key[1] != eot || m->serve_key[2] != (stop_at_eot != 0)) {
        for (cudaGraphExec_t &g : m->serve_graph)
            if (g) {
                cudaGraphExecDestroy(g);
                g = nullptr;
            }
        m->serve_key[0] = n_prompt;
        m->serve_key[1] = eot;
        m->serve_key[2] = stop_at_eot != 0;
    }
    const ServeCtl ctl{m->prompt_dev, n_prompt, m->done, m->budget, eot, stop_at_eot != 0};
    serve_park_kernel<<<1, 32, 0, m->stream>>>(m->B, m->prompt_dev, m->tokens, m->pos, m->nkv, m->done, m->budget);
    W_TRY(oasr_internal_launch_check(be, "serve_park"));

    std::vector<int> slot_req(m->B, -1);  // request held by each slot, -1 = free
    std::vector<int> slot_age(m->B, 0);   // steps a slot has run since its admission
    int next = 0, active = 0, width = 0;
    oasr_serve_stats stt = {};
    // admit queued requests into the free slots below `width`: log-mel and encoder of the
    // group (cross-attention K|V straight into the slots), then the slots' start state
    auto admit = [&]() -> int {
        std::vector<int> slots, reqs;
        for (int b = 0; b < width && next < n_utts; ++b)
            if (slot_req[b] < 0) {
                slots.push_back(b);
                reqs.push_back(next++);
            }
        if (slots.empty()) return OASR_STATUS_SUCCESS;
        const int k = (int)slots.size();
        OASR_CUDA_TRY(be, cudaMemsetAsync(m->audio, 0, (size_t)k * N_SAMPLES_30S * 4, m->stream));
        for (int i = 0; i < k; ++i) {
            const int64_t take = std::min<int64_t>(n_samples[reqs[i]], N_SAMPLES_30S);
            OASR_CUDA_TRY(be, cudaMemcpyAsync(m->audio + (int64_t)i * N_SAMPLES_30S, pcm + off[reqs[i]], take * 4,
                                              cudaMemcpyHostToDevice, m->stream));
        }
        W_TRY(launch_mel(be, m->audio, k, N_SAMPLES_30S, N_MEL_FRAMES, m->cfg.n_mels, m->window, m->twiddle,
                         m->filters, m->power, m->mel, m->max_key));
        W_TRY(run_encoder(m, k, slots.data()));
        std::vector<int> io(2 * k);
        for (int i = 0; i < k; ++i) {
            io[i] = slots[i];
            io[k + i] = budgets ? budgets[reqs[i]] : max_new;
            slot_req[slots[i]] = reqs[i];
            slot_age[slots[i]] = 0;
        }
        OASR_CUDA_TRY(be, cudaMemcpyAsync(m->serve_io, io.data(), io.size() * 4, cudaMemcpyHostToDevice, m->stream));
        serve_admit_kernel<<<1, 32, 0, m->stream>>>(m->serve_io, k, m->prompt_dev, m->tokens, m->pos, m->nkv,
                                                    m->done, m->budget);
        W_TRY(oasr_internal_launch_check(be, "serve_admit"));
        active += k;
        ++stt.admissions;
        return OASR_STATUS_SUCCESS;
    };
    width = oasr_b200_serve_batch_width(std::min(n_utts, W), W);
    stt.max_width = width;
    W_TRY(admit());
    std::vector<int> done(m->B), pos(m->B);
    while (active > 0) {
        if (be->abort_cb && be->abort_cb(be->abort_data)) return OASR_STATUS_ABORTED;  // step checkpoint
        // steps to the next harvest: check_every, cut at the earliest step a slot reaches
        // its budget (a slot with budget b finishes after n_prompt - 1 + b steps; one
        // that meets eot earlier idles at most check_every - 1 steps)
        int chunk = check_every;
        for (int b = 0; b < width; ++b) {
            const int r = slot_req[b];
            if (r < 0) continue;
            const int left = n_prompt - 1 + (budgets ? budgets[r] : max_new) - slot_age[b];
            chunk = std::min(chunk, std::max(1, left));
        }
        for (int i = 0; i < chunk; ++i) W_TRY(serve_step_graph(m, width, ctl));
        for (int b = 0; b < width; ++b) slot_age[b] += chunk;
        stt.steps += chunk;
        OASR_CUDA_TRY(be, cudaMemcpyAsync(done.data(), m->done, (size_t)width * 4, cudaMemcpyDeviceToHost, m->stream));
        OASR_CUDA_TRY(be, cudaMemcpyAsync(pos.data(), m->pos, (size_t)width * 4, cudaMemcpyDeviceToHost, m->stream));
        OASR_CUDA_TRY(be, cudaStreamSynchronize(m->stream));
        // harvest: a finished slot's generated tokens are history[n_prompt .. pos + 1]
        for (int b = 0; b < width; ++b) {
            const int r = slot_req[b];
            if (r < 0 || !done[b]) continue;
            const int count = pos[b] + 2 - n_prompt;
            lengths_out[r] = count;
            OASR_CUDA_TRY(be, cudaMemcpyAsync(tokens_out + (int64_t)r * max_new, m->history + (int64_t)b * P + n_prompt,
                                              (size_t)count * 4, cudaMemcpyDeviceToHost, m->stream));
            slot_req[b] = -1;
            --active;
        }
        // refill the free slots; widen when more requests wait than the width holds
        // (try_rebucket_active_slots), else narrow to the bucket of the active count
        // (try_shrink_active_slots), compacting the active slots to the front
        const int pending = n_utts - next;
        const int want = oasr_b200_serve_batch_width(std::min(active + pending, W), W);
        if (want > width) {
            width = want;
            ++stt.width_changes;
        }
        if (pending > 0) W_TRY(admit());
        if (next >= n_utts && active > 0) {
            const int narrow = oasr_b200_serve_batch_width(active, W);
            if (narrow < width) {
                int dst = 0;
                for (int src = 0; src < width; ++src) {
                    if (slot_req[src] < 0) continue;
                    while (slot_req[dst] >= 0 && dst < src) ++dst;
                    if (dst < src) {
                        W_TRY(serve_move_slot(m, src, dst));
                        slot_req[dst] = slot_req[src];
                        slot_age[dst] = slot_age[src];
                        slot_req[src] = -1;
                    }
                }
                width = narrow;
                ++stt.width_changes;
            }
        }
        stt.max_width = std::max(stt.max_width, width);
    }
    OASR_CUDA_TRY(be, cudaStreamSynchronize(m->stream));
    if (stats) *stats = stt;
    return oasr_b200_synchronize(be);
}

int oasr_b200_whisper_transcribe(oasr_whisper *m, const float *pcm, const int64_t *n_samples, int32_t n_utts,
                                 const int32_t *prompt, int32_t n_prompt, int32_t n_new, int32_t eot, int32_t stop_at_eot,
                                 int32_t *tokens_out) {
    W_TRY(oasr_b200_whisper_mel(m, pcm, n_samples, n_utts, nullptr));
    return oasr_b200_whisper_generate(m, n_utts, prompt, n_prompt, n_new, eot, stop_at_eot, tokens_out, 0);
}

}  // extern "C"
