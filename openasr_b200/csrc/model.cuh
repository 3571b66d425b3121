// model.cuh -- launchers shared by the model drivers (model_whisper.cu, model_qwen.cu).
#pragma once

#include "kernels.cuh"

namespace oasr {

int launch_resid_norm_quant(oasr_backend *be, float *x, const float *add, const float *add_bias, int64_t rows, int n,
                            float eps, bool rms, const float *gamma, const float *beta, float *out_f32,
                            const ActPlanes *q, int family);
int launch_bias_gelu_quant(oasr_backend *be, const float *x, const float *bias, int64_t rows, int n, float *out_f32,
                           const ActPlanes *q, int family);
int launch_swiglu_quant(oasr_backend *be, const float *gu, int64_t rows, int n, int64_t gu_ld, float *out_f32,
                        const ActPlanes *q, int family);
// Decode-step state is per sequence (slot): pos_dev[b] is the cache row sequence b writes in
// this step, nkv[b] = pos_dev[b] + 1 its attention length, so sequences at different positions
// share one step (the serving scheduler refills a slot while the others continue).
int launch_qkv_split_kv_write(oasr_backend *be, const float *qkv, const float *bias3, int B, int d, float *q_out,
                              __half *kc, __half *vc, int64_t cache_seq_stride, const int *pos_dev, int max_pos);
int launch_embed_q8_0(oasr_backend *be, const oasr_weight *emb, const int *tokens, int B, const float *pos_emb,
                      const int *pos_dev, int max_pos, float *x);
int launch_add_rows(oasr_backend *be, float *x, const float *bias, const float *add, int64_t rows, int n);
// Serving control of the decode-step epilogue: the prompt every slot starts with (device,
// n_prompt tokens), per-slot done flags and generated-token budgets, the end token.
// prompt == nullptr is the lockstep mode (every slot advances; the host feeds the prompt).
struct ServeCtl {
    const int *prompt;
    int n_prompt;
    int *done;
    const int *budget;
    int eot;
    int stop_at_eot;
};
// decode-step epilogue per slot b < n: history[b][pos[b] + 1] = tokens[b], pos[b] += 1,
// nkv[b] = pos[b] + 1; with a ServeCtl, teacher-forced prompt inputs and done detection
// (elementwise.cu decode_advance_kernel)
int launch_decode_advance(oasr_backend *be, int *tokens, int *pos, int *nkv, int *history, int n, int P,
                          const ServeCtl &sc = ServeCtl{});
int launch_cast_f16(oasr_backend *be, const float *src, int64_t src_ld, const float *bias, int64_t rows, int cols,
                    __half *dst, int64_t dst_ld);
int launch_im2col_f16(oasr_backend *be, const float *src, int64_t s_b, int64_t s_ic, int64_t s_t, int B, int IC,
                      int T_in, int T_out, int KW, int stride, int pad, __half *dst, int K_pad);
int launch_mel(oasr_backend *be, const float *audio, int B, int n_samples, int n_frames, int n_mels,
               const float *window, const float2 *twiddle, const float *filters, float *power, float *mel,
               int *max_key);
int launch_gemm_f16(oasr_backend *be, const __half *A, int64_t lda, const __half *B, int64_t ldb, int M, int N, int K,
                    float *y, int64_t y_ld, const float *bias, bool gelu);
int launch_argmax_rows(oasr_backend *be, const float *x, int64_t ld, int64_t n, int rows, int32_t *out);

// Fused decoder GEMVs (dgemv.cu): the weight's decode tiles against up to 8 activation
// rows; quantize-in-prologue (attention output) and QKV / KV-write epilogue forms.
int dgemv_configure(oasr_backend *be);
bool dgemv_supported(const oasr_weight *w, bool quant_prologue);
int launch_dgemv(oasr_backend *be, const oasr_weight *w, const ActPlanes &in, int M, float *y, int64_t y_ld);
int launch_dgemv_quant(oasr_backend *be, const oasr_weight *w, const float *h, int M, float *y, int64_t y_ld);
int launch_dgemv_qkv(oasr_backend *be, const oasr_weight *w, const ActPlanes &in, int M, const float *bias3, int d,
                     float *q_out, __half *kc, __half *vc, int64_t cache_seq_stride, const int *pos_dev, int max_pos);

// y[rows][N] = w . activation planes (rows <= 8: GEMV, else tensor-core / chunked GEMM)
int mul_mat_planes(oasr_backend *be, const oasr_weight *w, const ActPlanes &a, int64_t rows, float *y, int64_t y_ld);
// the same plus a per-column bias: in the tensor-core GEMM's store where it can, else an add launch
int mul_mat_planes_bias(oasr_backend *be, const oasr_weight *w, const ActPlanes &a, int64_t rows, float *y,
                        int64_t y_ld, const float *bias);

inline int weight_family(const oasr_weight *w) { return w->type == OASR_TYPE_Q4_K ? FAMILY_Q8_K : FAMILY_Q8_0; }

// tensor descriptor helper: contiguous-row views with explicit byte strides
inline oasr_tensor make_tensor(int type, const void *data, int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3,
                               int64_t nb1, int64_t nb2, int64_t nb3) {
    oasr_tensor t;
    t.type = type;
    t.flags = 0;
    t.data = const_cast<void *>(data);
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = ne2; t.ne[3] = ne3;
    t.nb[0] = type == OASR_TYPE_F16 ? 2 : 4;
    t.nb[1] = nb1; t.nb[2] = nb2; t.nb[3] = nb3;
    return t;
}

// serving width rules (serve_policy.cpp): the device bytes of one Whisper serving slot and the
// VRAM reserve the width cap keeps free
uint64_t whisper_slot_bytes(const oasr_whisper_config *c);
uint64_t serve_vram_reserve_bytes();

// Host-side helpers shared with the CPU oracle's frontend definition (whisper/mel.rs):
// periodic Hann window (scale first), Slaney mel filterbank (ratio-first edges).
void whisper_hann_window(float *w, int n);
void whisper_mel_filters(float *f, int n_mels, int n_fft, float sample_rate);

}  // namespace oasr
