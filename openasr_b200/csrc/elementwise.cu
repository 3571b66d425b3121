// elementwise.cu -- the row/elementwise ops around the hot ops in the Whisper
// and Qwen graphs, fused so that a decoder step launches few kernels:
//   residual add + LayerNorm / RMSNorm (+gamma, beta) + activation quantization
//   bias + GELU (+ quantization), fused QKV split + f16 KV-cache write,
//   token embedding (Q8_0 get_rows) + positional add, im2col (f16), casts,
//   SiLU * up (+ quantization), the decode-step advance and the Whisper log-mel
//   frontend.
// Rounding follows ggml's CPU ops (nn/decoder.rs, whisper/ggml_executor.rs call
// ggml_norm, ggml_rms_norm, ggml_mul, ggml_add, ggml_gelu, ggml_silu): norms sum
// in double, every add/mul rounds separately (no FMA contraction), GELU reads
// the same fp16 table ggml builds, SiLU's e^x is the decode path's exp_f32
// (fmath.cuh), and quantization matches quant_act.cu.
#include <math.h>

#include "fmath.cuh"
#include "kernels.cuh"
#include "model.cuh"

namespace oasr {

// ---- block reductions -----------------------------------------------------------------------
template <typename T>
static __device__ __forceinline__ T block_sum(T v, T *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    T r = 0;
    for (int i = 0; i < nw; ++i) r += sh[i];  // same order in every thread
    return r;
}

static __device__ __forceinline__ float gelu_tab(float r, const uint16_t *tab) {
    if (r <= -10.0f) return 0.0f;
    if (r >= 10.0f) return r;
    return h2f(tab[__half_as_ushort(__float2half_rn(r))]);
}

// Quantize one row held in shared memory (n floats) into the activation planes.
// q8_0: 8 threads per 32-block; q8_K: one warp per 256-super-block (first-max).
static __device__ void quantize_row_smem(const float *y, int n, int64_t r, int family, const ActPlanes &a) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (family == FAMILY_Q8_0) {
        for (int g = tid; g < n / 4; g += nt) {
            const int k0 = 4 * g;
            float v[4] = {y[k0], y[k0 + 1], y[k0 + 2], y[k0 + 3]};
            const unsigned gmask = 0xFFu << (threadIdx.x & 24);
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
            amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 4));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
            uint32_t packed = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) packed |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[i], id)) << (8 * i);
            *reinterpret_cast<uint32_t *>(a.qs + r * n + k0) = packed;
            if ((k0 & 31) == 0) a.d[r * (n / 32) + k0 / 32] = __half2float(__float2half_rn(d));
        }
    } else {
        const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
        for (int sb = warp; sb < n / 256; sb += nw) {
            const int k0 = sb * 256 + lane * 8;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = y[k0 + i];
            float amax = -1.0f, maxv = 0.0f;
            int idx = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (fabsf(v[i]) > amax) { amax = fabsf(v[i]); maxv = v[i]; idx = k0 + i; }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
                const float ov = __shfl_xor_sync(0xffffffffu, maxv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (oa > amax || (oa == amax && oi < idx)) { amax = oa; maxv = ov; idx = oi; }
            }
            int q[8];
            float d = 0.0f;
            if (amax == 0.0f) {
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = 0;
            } else {
                const float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
                d = __frcp_rn(iscale);
            }
            int sum = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) sum += q[i];
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            uint2 pk;
            pk.x = (uint32_t)(uint8_t)q[0] | (uint32_t)(uint8_t)q[1] << 8 | (uint32_t)(uint8_t)q[2] << 16 | (uint32_t)(uint8_t)q[3] << 24;
            pk.y = (uint32_t)(uint8_t)q[4] | (uint32_t)(uint8_t)q[5] << 8 | (uint32_t)(uint8_t)q[6] << 16 | (uint32_t)(uint8_t)q[7] << 24;
            *reinterpret_cast<uint2 *>(a.qs + r * n + k0) = pk;
            if ((lane & 1) == 0) a.bs16[r * (n / 16) + k0 / 16] = (int16_t)sum;
            if (lane == 0) a.d[r * (n / 256) + sb] = d;
            if (a.qs16) {
                __half2 h[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = __halves2half2(__int2half_rn(q[2 * i]), __int2half_rn(q[2 * i + 1]));
                *reinterpret_cast<int4 *>(a.qs16 + r * n + k0) = *reinterpret_cast<int4 *>(h);
                if ((lane & 1) == 0) a.bs16h[r * (n / 16) + k0 / 16] = __int2half_rn(sum);
            }
        }
    }
}

// x[r] (+)= add[r] + bias ; y = norm(x[r]) (* gamma + beta) -> out_f32 and/or quantized planes
__global__ void resid_norm_quant_kernel(float *x, const float *add, const float *add_bias, int n, float eps, int rms,
                                        const float *gamma, const float *beta, float *out_f32, ActPlanes q,
                                        int family) {
    extern __shared__ float srow[];
    __shared__ double sh_d[32];
    griddep_launch_dependents();
    griddep_wait();
    const int64_t r = blockIdx.x;
    float *xr = x + r * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        if (add) {
            const float t = add_bias ? __fadd_rn(add[r * n + i], add_bias[i]) : add[r * n + i];
            v = __fadd_rn(v, t);
            xr[i] = v;
        }
        srow[i] = v;
    }
    __syncthreads();
    float scale;
    if (rms) {
        double s = 0.0;
        for (int i = threadIdx.x; i < n; i += blockDim.x) s += (double)__fmul_rn(srow[i], srow[i]);
        s = block_sum(s, sh_d);
        const float mean = (float)(s / (double)n);
        scale = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
        for (int i = threadIdx.x; i < n; i += blockDim.x) srow[i] = __fmul_rn(srow[i], scale);
    } else {
        double s = 0.0;
        for (int i = threadIdx.x; i < n; i += blockDim.x) s += (double)srow[i];
        s = block_sum(s, sh_d);
        const float mean = (float)(s / (double)n);
        double s2 = 0.0;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float v = __fsub_rn(srow[i], mean);
            srow[i] = v;
            s2 += (double)__fmul_rn(v, v);
        }
        s2 = block_sum(s2, sh_d);
        const float var = (float)(s2 / (double)n);
        scale = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
        for (int i = threadIdx.x; i < n; i += blockDim.x) srow[i] = __fmul_rn(srow[i], scale);
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = srow[i];
        if (gamma) v = __fmul_rn(v, gamma[i]);
        if (beta) v = __fadd_rn(v, beta[i]);
        srow[i] = v;
        if (out_f32) out_f32[r * n + i] = v;
    }
    __syncthreads();
    if (q.qs) quantize_row_smem(srow, n, r, family, q);
}

// y = gelu(x + bias) -> out_f32 and/or quantized planes (fc1 -> fc2 boundary)
__global__ void bias_gelu_quant_kernel(const float *x, const float *bias, int n, const uint16_t *tab, float *out_f32,
                                       ActPlanes q, int family) {
    extern __shared__ float srow[];
    griddep_launch_dependents();
    griddep_wait();
    const int64_t r = blockIdx.x;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[r * n + i];
        if (bias) v = __fadd_rn(v, bias[i]);
        v = gelu_tab(v, tab);
        srow[i] = v;
        if (out_f32) out_f32[r * n + i] = v;
    }
    __syncthreads();
    if (q.qs) quantize_row_smem(srow, n, r, family, q);
}

// y = silu(g) * u (Qwen SwiGLU: ggml_silu then ggml_mul) -> quantized planes
__global__ void swiglu_quant_kernel(const float *gu, int n, int64_t gu_ld, float *out_f32, ActPlanes q, int family) {
    extern __shared__ float srow[];
    griddep_launch_dependents();
    griddep_wait();
    const int64_t r = blockIdx.x;
    const float *g = gu + r * gu_ld, *u = g + n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float s = __fdiv_rn(g[i], __fadd_rn(1.0f, exp_f32(-g[i])));
        const float v = __fmul_rn(s, u[i]);
        srow[i] = v;
        if (out_f32) out_f32[r * n + i] = v;
    }
    __syncthreads();
    if (q.qs) quantize_row_smem(srow, n, r, family, q);
}

// Whisper fused-QKV output [b][3d] + bias -> q [b][d] (f32); k, v -> f16 caches at row *pos
__global__ void qkv_split_kv_write_kernel(const float *qkv, const float *bias3, int d, float *q_out, __half *kc,
                                          __half *vc, int64_t cache_seq_stride, const int *pos_dev, int *err,
                                          int max_pos) {
    griddep_launch_dependents();
    griddep_wait();
    const int b = blockIdx.x;
    const int pos = pos_dev[b];
    if (pos < 0 || pos >= max_pos) {
        if (threadIdx.x == 0) atomicOr(err, ERR_BAD_INDEX);
        return;
    }
    const float *row = qkv + (int64_t)b * 3 * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        q_out[(int64_t)b * d + i] = bias3 ? __fadd_rn(row[i], bias3[i]) : row[i];
        const float kv = bias3 ? __fadd_rn(row[d + i], bias3[d + i]) : row[d + i];
        const float vv = bias3 ? __fadd_rn(row[2 * d + i], bias3[2 * d + i]) : row[2 * d + i];
        kc[b * cache_seq_stride + (int64_t)pos * d + i] = __float2half_rn(kv);
        vc[b * cache_seq_stride + (int64_t)pos * d + i] = __float2half_rn(vv);
    }
}

// x[b] = dequant(tok_emb Q8_0 row tokens[b]) + pos_emb[pos[b]]  (ggml_get_rows + ggml_add)
__global__ void embed_q8_0_kernel(const uint8_t *qs, const uint16_t *dsc, int d, int vocab, const int *tokens,
                                  const float *pos_emb, const int *pos_dev, int max_pos, float *x, int *err) {
    griddep_launch_dependents();
    griddep_wait();
    const int b = blockIdx.x;
    const int tok = tokens[b], pos = pos_dev ? pos_dev[b] : 0;
    if (tok < 0 || tok >= vocab || pos < 0 || pos >= max_pos) {
        if (threadIdx.x == 0) atomicOr(err, ERR_BAD_INDEX);
        return;
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float e = __fmul_rn((float)(int8_t)qs[(int64_t)tok * d + i], h2f(dsc[(int64_t)tok * (d / 32) + i / 32]));
        x[(int64_t)b * d + i] = pos_emb ? __fadd_rn(e, pos_emb[(int64_t)pos * d + i]) : e;
    }
}

// x[r][i] += bias[i] (+ add[r][i])
__global__ void add_rows_kernel(float *x, const float *bias, const float *add, int64_t rows, int n) {
    griddep_launch_dependents();
    griddep_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * n; i += (int64_t)gridDim.x * blockDim.x) {
        float v = x[i];
        if (bias) v = __fadd_rn(v, bias[i % n]);
        if (add) v = __fadd_rn(v, add[i]);
        x[i] = v;
    }
}

// dst[r][c] = fp16(src[r][c] (+ bias[c])), r < rows, c < cols; zero for c in [cols, dst_ld)
__global__ void cast_f16_kernel(const float *src, int64_t src_ld, const float *bias, int64_t rows, int cols,
                                __half *dst, int64_t dst_ld) {
    griddep_launch_dependents();
    griddep_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * dst_ld; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / dst_ld;
        const int c = (int)(i % dst_ld);
        float v = 0.0f;
        if (c < cols) {
            v = src[r * src_ld + c];
            if (bias) v = __fadd_rn(v, bias[c]);
        }
        dst[i] = __float2half_rn(v);
    }
}

// conv1d im2col (ggml_im2col, fp16 result): dst[b*T_out + t][ic*KW + k] = src_b(ic, t*s + k - p)
__global__ void im2col_f16_kernel(const float *src, int64_t s_b, int64_t s_ic, int64_t s_t, int B, int IC, int T_in,
                                  int T_out, int KW, int stride, int pad, __half *dst, int K_pad) {
    const int64_t total = (int64_t)B * T_out * K_pad;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % K_pad);
        const int64_t rt = i / K_pad;
        const int t = (int)(rt % T_out), b = (int)(rt / T_out);
        float v = 0.0f;
        if (c < IC * KW) {
            const int ic = c / KW, k = c % KW;
            const int ti = t * stride + k - pad;
            if (ti >= 0 && ti < T_in) v = src[b * s_b + ic * s_ic + (int64_t)ti * s_t];
        }
        dst[i] = __float2half_rn(v);
    }
}

// ---- Whisper log-mel frontend (whisper/mel.rs) ------------------------------------------------
// power[b][f][k] = |sum_n x_pad[f*hop + n] w[n] e^{-2 pi i k n / N}|^2, reflect-padded by N/2
__global__ void stft_power_kernel(const float *audio, int B, int n_samples, int n_frames, const float *window,
                                  const float2 *twiddle, int n_fft, int hop, float *power) {
    extern __shared__ float frame[];
    const int f = blockIdx.x, b = blockIdx.y;
    const float *x = audio + (int64_t)b * n_samples;
    const int pad = n_fft / 2;
    for (int n = threadIdx.x; n < n_fft; n += blockDim.x) {
        int idx = f * hop + n - pad;
        if (idx < 0) idx = -idx;                                    // reflect, no edge repeat
        if (idx >= n_samples) idx = 2 * (n_samples - 1) - idx;
        frame[n] = __fmul_rn(x[idx], window[n]);
    }
    __syncthreads();
    const int bins = n_fft / 2 + 1;
    for (int k = threadIdx.x; k < bins; k += blockDim.x) {
        float re = 0.0f, im = 0.0f;
        int j = 0;
        for (int n = 0; n < n_fft; ++n) {
            const float2 t = twiddle[j];
            re = fmaf(frame[n], t.x, re);
            im = fmaf(frame[n], t.y, im);
            j += k;
            if (j >= n_fft) j -= n_fft;
        }
        power[((int64_t)b * n_frames + f) * bins + k] = __fadd_rn(__fmul_rn(re, re), __fmul_rn(im, im));
    }
}

static __device__ __forceinline__ int float_order_key(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
static __device__ __forceinline__ float float_from_key(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7FFFFFFF); }

// mel[b][m][f] = log10(max(sum_k filt[m][k] power[b][f][k], 1e-10)); per-utterance max key
__global__ void mel_log_kernel(const float *power, const float *filters, int n_mels, int bins, int n_frames,
                               float *mel, int *max_key) {
    const int f = blockIdx.x, b = blockIdx.y;
    const float *p = power + ((int64_t)b * n_frames + f) * bins;
    int local = float_order_key(-INFINITY);
    for (int m = threadIdx.x; m < n_mels; m += blockDim.x) {
        float s = 0.0f;
        for (int k = 0; k < bins; ++k) s = fmaf(p[k], filters[m * bins + k], s);
        const float v = log10f(fmaxf(s, 1e-10f));
        mel[((int64_t)b * n_mels + m) * n_frames + f] = v;
        local = max(local, float_order_key(v));
    }
    atomicMax(max_key + b, local);
}

__global__ void mel_norm_kernel(float *mel, int64_t per_utt, const int *max_key) {
    const int b = blockIdx.y;
    const float floor = __fsub_rn(float_from_key(max_key[b]), 8.0f);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per_utt; i += (int64_t)gridDim.x * blockDim.x) {
        float *v = mel + b * per_utt + i;
        *v = __fdiv_rn(__fadd_rn(fmaxf(*v, floor), 4.0f), 4.0f);
    }
}

// After a decode step the selected tokens become the inputs of position pos + 1
// (history[b][pos + 1]) and the device position and KV length advance by one.
// The end of a decode step, per sequence b < n (position pos[b], KV length nkv[b] = pos[b] + 1):
// record the step's selected token tokens[b] as history[b][pos + 1] and advance the position.
// With a serving control block (sc.prompt != null) every slot also feeds its own next input:
// the prompt token while pos + 1 is inside the prompt (teacher forcing, so slots at different
// positions share one step), else the selected token; a slot whose token is `eot` (when
// stop_at_eot), whose generated count reached its budget or whose context is full is marked
// done and parks (its position, input and history stay until the host refills the slot).
__global__ void decode_advance_kernel(int *tokens, int *pos, int *nkv, int *history, int n, int P, ServeCtl sc) {
    griddep_wait();
    const int b = threadIdx.x;
    if (b >= n) return;
    const int p = pos[b];
    if (!sc.prompt) {
        if (p + 1 < P) history[b * P + p + 1] = tokens[b];
        pos[b] = p + 1;
        nkv[b] = p + 2;
        return;
    }
    if (sc.done[b]) return;
    const int q = p + 1;
    int tok = tokens[b];
    bool fin = false;
    if (q < sc.n_prompt) {
        tok = sc.prompt[q];
    } else {
        history[b * P + q] = tok;
        const int generated = q - sc.n_prompt + 1;
        fin = (sc.stop_at_eot && tok == sc.eot) || generated >= sc.budget[b] || q + 1 >= P;
    }
    tokens[b] = tok;
    if (fin) {
        sc.done[b] = 1;
    } else {
        pos[b] = q;
        nkv[b] = q + 1;
    }
}

// ---- launchers --------------------------------------------------------------------------------------
static int blocks_for(int64_t work, int threads, oasr_backend *be) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, (int64_t)be->sm_count * 32));
}

// ---- chunk-parallel row kernels ---------------------------------------------------------------
// One warp per chunk of 32*E elements (E = 8 for the q8_K family: one 256 super-block;
// E = 4 for q8_0: four 32-blocks of 8 lanes), every operand loaded before any
// arithmetic, so a row costs one memory round trip instead of one per element
// group.  Arithmetic as resid_norm_quant / bias_gelu_quant above.

template <int E>
static __device__ __forceinline__ void ldE(const float *p, float (&v)[E]) {
    if (E == 8) {
        const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[E > 4 ? 4 : 0] = b.x; v[E > 5 ? 5 : 0] = b.y; v[E > 6 ? 6 : 0] = b.z; v[E > 7 ? 7 : 0] = b.w;
    } else {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    }
}

template <int E>
static __device__ __forceinline__ void stE(float *p, const float (&v)[E]) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    if (E == 8) *reinterpret_cast<float4 *>(p + 4) = make_float4(v[E > 4 ? 4 : 0], v[E > 5 ? 5 : 0], v[E > 6 ? 6 : 0], v[E > 7 ? 7 : 0]);
}

// quantize one warp chunk (lane holds E consecutive values at k0 = chunk*32*E + E*lane) of row r
template <int E>
static __device__ __forceinline__ void quant_chunk(const float (&v)[E], int64_t r, int n, int k0, int lane,
                                                   const ActPlanes &a) {
    if (E == 8) {
        // q8_K: one super-block per warp, first-max
        float amax = -1.0f, maxv = 0.0f;
        int idx = 0;
#pragma unroll
        for (int i = 0; i < E; ++i)
            if (fabsf(v[i]) > amax) { amax = fabsf(v[i]); maxv = v[i]; idx = k0 + i; }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
            const float ov = __shfl_xor_sync(0xffffffffu, maxv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (oa > amax || (oa == amax && oi < idx)) { amax = oa; maxv = ov; idx = oi; }
        }
        int q[E];
        float d = 0.0f;
        if (amax == 0.0f) {
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = 0;
        } else {
            const float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
            d = __frcp_rn(iscale);
        }
        int sum = 0;
#pragma unroll
        for (int i = 0; i < E; ++i) sum += q[i];
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        uint2 pk;
        pk.x = (uint32_t)(uint8_t)q[0] | (uint32_t)(uint8_t)q[1] << 8 | (uint32_t)(uint8_t)q[2] << 16 |
               (uint32_t)(uint8_t)q[3] << 24;
        pk.y = (uint32_t)(uint8_t)q[E > 4 ? 4 : 0] | (uint32_t)(uint8_t)q[E > 5 ? 5 : 0] << 8 |
               (uint32_t)(uint8_t)q[E > 6 ? 6 : 0] << 16 | (uint32_t)(uint8_t)q[E > 7 ? 7 : 0] << 24;
        *reinterpret_cast<uint2 *>(a.qs + r * n + k0) = pk;
        if ((lane & 1) == 0) a.bs16[r * (n / 16) + k0 / 16] = (int16_t)sum;
        if (lane == 0) a.d[r * (n / 256) + k0 / 256] = d;
        if (a.qs16) {
            __half2 h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                h[i] = __halves2half2(__int2half_rn(q[(2 * i) % E]), __int2half_rn(q[(2 * i + 1) % E]));
            *reinterpret_cast<int4 *>(a.qs16 + r * n + k0) = *reinterpret_cast<int4 *>(h);
            if ((lane & 1) == 0) a.bs16h[r * (n / 16) + k0 / 16] = __int2half_rn(sum);
        }
    } else {
        // q8_0: 8 lanes per 32-block
        const unsigned gmask = 0xFFu << (lane & 24);
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 4));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
        uint32_t packed = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) packed |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[i], id)) << (8 * i);
        *reinterpret_cast<uint32_t *>(a.qs + r * n + k0) = packed;
        if ((k0 & 31) == 0) a.d[r * (n / 32) + k0 / 32] = __half2float(__float2half_rn(d));
    }
}

// CTA = one row, warp = one chunk: x (+)= add + bias; y = norm(x)(*gamma + beta) -> out_f32 / planes
template <int E>
__global__ void ln_quant_chunks_kernel(float *x, const float *add, const float *add_bias, int n, float eps, int rms,
                                       const float *gamma, const float *beta, float *out_f32, ActPlanes q) {
    __shared__ double sh[32];
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t r = blockIdx.x;
    const int k0 = warp * 32 * E + E * lane;
    float g[E], b[E], ad[E], ab[E];
    // parameters do not depend on the previous kernel
    if (gamma) ldE<E>(gamma + k0, g);
    if (beta) ldE<E>(beta + k0, b);
    if (add_bias) ldE<E>(add_bias + k0, ab);
    griddep_wait();
    float v[E];
    ldE<E>(x + r * n + k0, v);
    if (add) {
        ldE<E>(add + r * n + k0, ad);
#pragma unroll
        for (int i = 0; i < E; ++i) v[i] = __fadd_rn(v[i], add_bias ? __fadd_rn(ad[i], ab[i]) : ad[i]);
        stE<E>(x + r * n + k0, v);
    }
    auto block_sum_d = [&](double s) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sh[warp] = s;
        __syncthreads();
        double t = 0.0;
        for (int i = 0; i < nw; ++i) t += sh[i];
        __syncthreads();
        return t;
    };
    float scale;
    if (rms) {
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < E; ++i) s += (double)__fmul_rn(v[i], v[i]);
        s = block_sum_d(s);
        scale = __frcp_rn(__fsqrt_rn(__fadd_rn((float)(s / (double)n), eps)));
    } else {
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < E; ++i) s += (double)v[i];
        const float mean = (float)(block_sum_d(s) / (double)n);
        double s2 = 0.0;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            v[i] = __fsub_rn(v[i], mean);
            s2 += (double)__fmul_rn(v[i], v[i]);
        }
        scale = __frcp_rn(__fsqrt_rn(__fadd_rn((float)(block_sum_d(s2) / (double)n), eps)));
    }
#pragma unroll
    for (int i = 0; i < E; ++i) {
        float u = __fmul_rn(v[i], scale);
        if (gamma) u = __fmul_rn(u, g[i]);
        if (beta) u = __fadd_rn(u, b[i]);
        v[i] = u;
    }
    if (out_f32) stE<E>(out_f32 + r * n + k0, v);
    if (q.qs) quant_chunk<E>(v, r, n, k0, lane, q);
}

// warp = one (row, chunk): y = gelu(x + bias) -> out_f32 / planes
template <int E>
__global__ void gelu_quant_chunks_kernel(const float *x, const float *bias, int n, int64_t n_chunks,
                                         const uint16_t *tab, float *out_f32, ActPlanes q) {
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (w >= n_chunks) return;  // warp-uniform
    const int per_row = n / (32 * E);
    const int64_t r = w / per_row;
    const int k0 = (int)(w - r * per_row) * 32 * E + E * lane;
    float bb[E], v[E];
    if (bias) ldE<E>(bias + k0, bb);
    griddep_wait();
    ldE<E>(x + r * n + k0, v);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = gelu_tab(bias ? __fadd_rn(v[i], bb[i]) : v[i], tab);
    if (out_f32) stE<E>(out_f32 + r * n + k0, v);
    if (q.qs) quant_chunk<E>(v, r, n, k0, lane, q);
}

// warp = one (row, chunk): y = silu(gate) * up -> out_f32 / planes (gate|up -> down boundary);
// arithmetic as swiglu_quant_kernel
template <int E>
__global__ void swiglu_quant_chunks_kernel(const float *gu, int n, int64_t gu_ld, int64_t n_chunks, float *out_f32,
                                           ActPlanes q) {
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (w >= n_chunks) return;  // warp-uniform
    const int per_row = n / (32 * E);
    const int64_t r = w / per_row;
    const int k0 = (int)(w - r * per_row) * 32 * E + E * lane;
    griddep_wait();
    float g[E], u[E], v[E];
    ldE<E>(gu + r * gu_ld + k0, g);
    ldE<E>(gu + r * gu_ld + n + k0, u);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, exp_f32(-g[i]))), u[i]);
    if (out_f32) stE<E>(out_f32 + r * n + k0, v);
    if (q.qs) quant_chunk<E>(v, r, n, k0, lane, q);
}

int launch_resid_norm_quant(oasr_backend *be, float *x, const float *add, const float *add_bias, int64_t rows, int n,
                            float eps, bool rms, const float *gamma, const float *beta, float *out_f32,
                            const ActPlanes *q, int family) {
    ActPlanes qq{};
    if (q) qq = *q;
    cudaError_t e;
    // chunk-parallel form when a row is whole warp chunks (<= 32 warps) of the planes' family
    const int E = (!q || family == FAMILY_Q8_K) ? 8 : 4;
    if (n % (32 * E) == 0 && n / (32 * E) <= 32 && (!q || family != FAMILY_Q8_K || n % 256 == 0)) {
        const dim3 block(32 * (n / (32 * E)));
        if (E == 8)
            e = launch_k(be, ln_quant_chunks_kernel<8>, dim3((unsigned)rows), block, 0, x, add, add_bias, n, eps,
                         rms ? 1 : 0, gamma, beta, out_f32, qq);
        else
            e = launch_k(be, ln_quant_chunks_kernel<4>, dim3((unsigned)rows), block, 0, x, add, add_bias, n, eps,
                         rms ? 1 : 0, gamma, beta, out_f32, qq);
    } else {
        e = launch_k(be, resid_norm_quant_kernel, dim3((unsigned)rows), dim3(256), n * sizeof(float), x, add, add_bias,
                     n, eps, rms ? 1 : 0, gamma, beta, out_f32, qq, family);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "resid_norm_quant launch", __LINE__);
    return oasr_internal_launch_check(be, "resid_norm_quant");
}

int launch_bias_gelu_quant(oasr_backend *be, const float *x, const float *bias, int64_t rows, int n, float *out_f32,
                           const ActPlanes *q, int family) {
    ActPlanes qq{};
    if (q) qq = *q;
    cudaError_t e;
    const int E = (!q || family == FAMILY_Q8_K) ? 8 : 4;
    if (n % (32 * E) == 0) {
        const int64_t chunks = rows * (n / (32 * E));
        // two warps (chunks) per CTA: small CTAs share SMs with the GEMVs around them under
        // programmatic dependent launch (decode step 1708 against 1719 us with 8 warps)
        constexpr int wpb = 2;
        const unsigned grid = (unsigned)((chunks + wpb - 1) / wpb);
        if (E == 8)
            e = launch_k(be, gelu_quant_chunks_kernel<8>, dim3(grid), dim3(32 * wpb), 0, x, bias, n, chunks,
                         (const uint16_t *)be->gelu_table, out_f32, qq);
        else
            e = launch_k(be, gelu_quant_chunks_kernel<4>, dim3(grid), dim3(32 * wpb), 0, x, bias, n, chunks,
                         (const uint16_t *)be->gelu_table, out_f32, qq);
    } else {
        e = launch_k(be, bias_gelu_quant_kernel, dim3((unsigned)rows), dim3(256), n * sizeof(float), x, bias, n,
                     (const uint16_t *)be->gelu_table, out_f32, qq, family);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "bias_gelu_quant launch", __LINE__);
    return oasr_internal_launch_check(be, "bias_gelu_quant");
}

int launch_swiglu_quant(oasr_backend *be, const float *gu, int64_t rows, int n, int64_t gu_ld, float *out_f32,
                        const ActPlanes *q, int family) {
    ActPlanes qq{};
    if (q) qq = *q;
    cudaError_t e;
    const int E = (!q || family == FAMILY_Q8_K) ? 8 : 4;
    if (n % (32 * E) == 0 && gu_ld % 4 == 0) {
        const int64_t chunks = rows * (n / (32 * E));
        const unsigned grid = (unsigned)((chunks + 7) / 8);
        if (E == 8)
            e = launch_k(be, swiglu_quant_chunks_kernel<8>, dim3(grid), dim3(256), 0, gu, n, gu_ld, chunks, out_f32, qq);
        else
            e = launch_k(be, swiglu_quant_chunks_kernel<4>, dim3(grid), dim3(256), 0, gu, n, gu_ld, chunks, out_f32, qq);
    } else {
        e = launch_k(be, swiglu_quant_kernel, dim3((unsigned)rows), dim3(256), n * sizeof(float), gu, n, gu_ld, out_f32,
                     qq, family);
    }
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "swiglu_quant launch", __LINE__);
    return oasr_internal_launch_check(be, "swiglu_quant");
}

int launch_qkv_split_kv_write(oasr_backend *be, const float *qkv, const float *bias3, int B, int d, float *q_out,
                              __half *kc, __half *vc, int64_t cache_seq_stride, const int *pos_dev, int max_pos) {
    const cudaError_t e = launch_k(be, qkv_split_kv_write_kernel, dim3(B), dim3(256), 0, qkv, bias3, d, q_out, kc, vc,
                                   cache_seq_stride, pos_dev, be->err_word, max_pos);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "qkv_split launch", __LINE__);
    return oasr_internal_launch_check(be, "qkv_split_kv_write");
}

int launch_embed_q8_0(oasr_backend *be, const oasr_weight *emb, const int *tokens, int B, const float *pos_emb,
                      const int *pos_dev, int max_pos, float *x) {
    const cudaError_t e = launch_k(be, embed_q8_0_kernel, dim3(B), dim3(256), 0, (const uint8_t *)emb->qs,
                                   (const uint16_t *)emb->d, (int)emb->ne[0], (int)emb->ne[1], tokens, pos_emb, pos_dev,
                                   max_pos, x, be->err_word);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "embed launch", __LINE__);
    return oasr_internal_launch_check(be, "embed_q8_0");
}

int launch_decode_advance(oasr_backend *be, int *tokens, int *pos, int *nkv, int *history, int n, int P,
                          const ServeCtl &sc) {
    const cudaError_t e = launch_k(be, decode_advance_kernel, dim3(1), dim3(32), 0, tokens, pos, nkv, history, n, P, sc);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "decode_advance launch", __LINE__);
    return oasr_internal_launch_check(be, "decode_advance");
}

int launch_add_rows(oasr_backend *be, float *x, const float *bias, const float *add, int64_t rows, int n) {
    add_rows_kernel<<<blocks_for(rows * n, 256, be), 256, 0, be->stream>>>(x, bias, add, rows, n);
    return oasr_internal_launch_check(be, "add_rows");
}

// The same cast 8 columns per thread: two 16-byte loads of src (and of the bias), one
// 16-byte store of 8 halves (dense rows, 16-byte aligned, cols a multiple of 8).
__global__ void cast_f16_x8_kernel(const float *src, int64_t src_ld, const float *bias, int64_t rows, int cols,
                                   __half *dst, int64_t dst_ld) {
    griddep_launch_dependents();
    griddep_wait();
    const int per_row = cols / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * per_row; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / per_row;
        const int c = 8 * (int)(i - r * per_row);
        const float4 a = *reinterpret_cast<const float4 *>(src + r * src_ld + c);
        const float4 b = *reinterpret_cast<const float4 *>(src + r * src_ld + c + 4);
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        if (bias) {
            const float4 p = *reinterpret_cast<const float4 *>(bias + c);
            const float4 q = *reinterpret_cast<const float4 *>(bias + c + 4);
            const float w[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], w[j]);
        }
        __half2 h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __halves2half2(__float2half_rn(v[2 * j]), __float2half_rn(v[2 * j + 1]));
        *reinterpret_cast<int4 *>(dst + r * dst_ld + c) = *reinterpret_cast<const int4 *>(h);
    }
}

int launch_cast_f16(oasr_backend *be, const float *src, int64_t src_ld, const float *bias, int64_t rows, int cols,
                    __half *dst, int64_t dst_ld) {
    const bool x8 = cols % 8 == 0 && dst_ld == cols && src_ld % 4 == 0 && dst_ld % 8 == 0 &&
                    ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0 && ((uintptr_t)bias & 15) == 0;
    if (x8)
        cast_f16_x8_kernel<<<blocks_for(rows * (cols / 8), 256, be), 256, 0, be->stream>>>(src, src_ld, bias, rows, cols,
                                                                                         dst, dst_ld);
    else
        cast_f16_kernel<<<blocks_for(rows * dst_ld, 256, be), 256, 0, be->stream>>>(src, src_ld, bias, rows, cols, dst,
                                                                                   dst_ld);
    return oasr_internal_launch_check(be, "cast_f16");
}

int launch_im2col_f16(oasr_backend *be, const float *src, int64_t s_b, int64_t s_ic, int64_t s_t, int B, int IC,
                      int T_in, int T_out, int KW, int stride, int pad, __half *dst, int K_pad) {
    im2col_f16_kernel<<<blocks_for((int64_t)B * T_out * K_pad, 256, be), 256, 0, be->stream>>>(
        src, s_b, s_ic, s_t, B, IC, T_in, T_out, KW, stride, pad, dst, K_pad);
    return oasr_internal_launch_check(be, "im2col_f16");
}

int launch_mel(oasr_backend *be, const float *audio, int B, int n_samples, int n_frames, int n_mels,
               const float *window, const float2 *twiddle, const float *filters, float *power, float *mel,
               int *max_key) {
    const int n_fft = 400, hop = 160, bins = n_fft / 2 + 1;
    cudaMemsetAsync(max_key, 0x80, B * sizeof(int), be->stream);  // very negative keys
    stft_power_kernel<<<dim3(n_frames, B), 256, n_fft * sizeof(float), be->stream>>>(audio, B, n_samples, n_frames,
                                                                                      window, twiddle, n_fft, hop, power);
    mel_log_kernel<<<dim3(n_frames, B), 128, 0, be->stream>>>(power, filters, n_mels, bins, n_frames, mel, max_key);
    const int64_t per = (int64_t)n_mels * n_frames;
    mel_norm_kernel<<<dim3(blocks_for(per, 256, be), B), 256, 0, be->stream>>>(mel, per, max_key);
    return oasr_internal_launch_check(be, "mel");
}

}  // namespace oasr
