/*
 * oracle.h -- CPU restatement of the ggml semantics that OpenASR's inference
 * hot path relies on.  TEST INFRASTRUCTURE ONLY: the product
 * (openasr_b200/, include/oasr_b200.h) never links, loads or calls this code.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it,
 * and only as the checker / the timed CPU baseline.
 *
 * Why a restatement: the reference executes every tensor op in a vendored ggml
 * fork (crates/openasr-core/third_party/openasr-ggml, an un-vendored git
 * submodule, .gitmodules:1-3) that is empty in the reference checkout, and the
 * reference's Rust workspace has no toolchain here.  The arithmetic below
 * restates ggml's public block formats and op semantics; every function names
 * the reference call site it follows.
 *
 * Pinning:
 *   - block formats / dequant / Q8_0 + Q4_0 quantizers: bit-exact against
 *     the gguf Python package 0.19.0 (gguf/quants.py) -- tests/golden/.
 *   - mul_mat layout and flash_attn_ext layout/mask/GQA: pinned against the
 *     reference's own known-answer tests (cpu_graph.rs:12827, :12860, :12892,
 *     :13471, :13900, :13950) re-run through this oracle in tests/.
 *   - activation quantization before the integer block dot (q8_0 / q8_K),
 *     GELU's fp16 table, flash-attention's f16 V accumulator and the f32
 *     summation order: ggml-CPU internals whose source is absent from the
 *     reference checkout -> "parity unpinned" for those details; they are
 *     restated from upstream ggml's public behaviour.
 */
#ifndef OASR_ORACLE_H
#define OASR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (reference: crates/openasr-core/src/ggml_runtime/ffi.rs:338-346) */
enum {
    OO_TYPE_F32 = 0,
    OO_TYPE_F16 = 1,
    OO_TYPE_Q4_0 = 2,
    OO_TYPE_Q8_0 = 8,
    OO_TYPE_Q4_K = 12,
    OO_TYPE_Q8_K = 15,
    OO_TYPE_I32 = 26,
};

/* ggml_status (ffi.rs:102-117) */
enum {
    OO_STATUS_ALLOC_FAILED = -2,
    OO_STATUS_FAILED = -1,
    OO_STATUS_SUCCESS = 0,
};

/* Mirrors the ggml_tensor prefix the reference reads (ffi.rs:24-30):
 * type, ne[4] (elements per dim, ne0 fastest), nb[4] (byte strides), data. */
typedef struct {
    int32_t type;
    int32_t _pad;
    void *data;
    int64_t ne[4];
    int64_t nb[4];
} oo_tensor;

/* ---- scalar helpers ---------------------------------------------------- */
uint16_t oo_f32_to_f16(float f);   /* round-to-nearest-even, like F16C _cvtss_sh */
float oo_f16_to_f32(uint16_t h);
int oo_nearest_int(float f);       /* ggml's magic-number nearest_int (ties-to-even) */

/* ---- deterministic synthetic data -------------------------------------- */
/* x[i] = mean + std * N(0,1), element i drawn from SplitMix64 state
 * seed + (offset+i+1)*0x9E3779B97F4A7C15 via Box-Muller on pairs. */
void oo_synth_normal(uint64_t seed, uint64_t offset, float *x, int64_t n, float mean, float std);
uint64_t oo_splitmix64(uint64_t state);

/* ---- block formats ------------------------------------------------------ */
int64_t oo_block_elems(int type);
int64_t oo_block_bytes(int type);
int64_t oo_row_size(int type, int64_t ne0);
/* quantize k floats (k multiple of block size) of type Q8_0 / Q4_0 / Q4_K / Q8_K */
int oo_quantize_row(int type, const float *x, void *y, int64_t k);
/* multi-row quantize, rows of ne0 elements, OpenMP over rows */
int oo_quantize_rows(int type, const float *x, void *y, int64_t nrows, int64_t ne0);
int oo_dequantize_row(int type, const void *x, float *y, int64_t k);

/* ---- ops ------------------------------------------------------------------ */
/* dst = mul_mat(w, x): dst[n, m, i2, i3] = dot(w[:, n, i2/r2, i3/r3], x[:, m, i2, i3])
 * (cpu_graph.rs:3651-3686, :7188-7206).  Activations are converted to the
 * weight type's vec_dot type (Q8_0/Q4_0 -> q8_0, Q4_K -> q8_K, F16 -> f16). */
int oo_mul_mat(const oo_tensor *w, const oo_tensor *x, oo_tensor *dst);

/* flash_attn_ext (cpu_graph.rs:4144-4220, :7476-7519).  q f32 [D, n_q, H, S];
 * k, v f16|f32 [D, n_kv, H_kv, S]; optional mask f16 [n_kv, >=n_q, *, *];
 * dst f32 [D, H, n_q, S].  mode 0 = ggml CPU (f16 V accumulator when v is
 * f16), mode 1 = f32 V accumulator. */
enum { OO_FA_GGML = 0, OO_FA_F32 = 1, OO_FA_TC128 = 2 };
/* OO_FA_TC128: the arithmetic of a tensor-core flash attention -- q, k, v rounded
 * to fp16, scores in 128-key blocks with a running max in the base-2 domain,
 * probabilities rounded to fp16 for the P.V product, f32 rescaling; a mask may
 * only hide keys (entries 0 or -inf).  Used to check the GPU tensor-core
 * attention (encoder; the Qwen causal prompt pass) -- ggml's CUDA backend makes
 * the same fp16 conversion of f32 K/V; the ggml CPU semantics are modes 0 and 1. */
int oo_flash_attn_ext(const oo_tensor *q, const oo_tensor *k, const oo_tensor *v,
                      const oo_tensor *mask, float scale, int mode, oo_tensor *dst);

/* set_rows (cpu_graph.rs:4882): dst[:, rows[i], i2, i3] = convert(src[:, i, i2, i3]) */
int oo_set_rows(oo_tensor *dst, const oo_tensor *src, const int64_t *rows, int64_t n_rows);

/* first-max argmax over each row of a [n, rows] f32 matrix (cpu_graph.rs:3750-3765) */
void oo_argmax_first(const float *x, int64_t n, int64_t rows, int32_t *out);

/* elementwise / row ops used by the model graphs (ggml semantics) */
void oo_norm(const float *x, float *y, int64_t n, int64_t rows, float eps);      /* ggml_norm */
void oo_rms_norm(const float *x, float *y, int64_t n, int64_t rows, float eps);  /* ggml_rms_norm */
void oo_gelu(const float *x, float *y, int64_t n);                                 /* ggml_gelu (fp16 table) */
void oo_silu(const float *x, float *y, int64_t n);                                 /* ggml_silu, e^x as oo_expf */
/* ggml_rope_ext NEOX mode on [D, H, T] rows: positions[t]; n_dims = D */
void oo_rope_neox(float *x, int64_t D, int64_t H, int64_t T, const int32_t *pos, float freq_base);

/* ---- the decode path's canonical arithmetic -------------------------------------------
 * ggml's CPU ops leave the f32 summation order to the ISA (AVX2 and AVX-512 builds of
 * ggml differ in the last bits); this restatement fixes one order per op -- the order the
 * B200 kernels use -- so that greedy transcripts can be compared bit for bit.  The
 * quantized mul_mat above already sums its per-block terms in block order (ggml's
 * vec_dot loop order), which every device mul_mat path follows.  The functions below
 * restate the other reductions of a decode step. */

/* e^x: Cody-Waite reduction (ln2 split as fdlibm's float split), degree-7 Taylor
 * polynomial in Horner form with fmaf, scaling by 2^n (two steps below 2^-126).  Used by
 * the SiLU and by the decode attentions' softmax. */
float oo_expf(float x);

/* LayerNorm (rms = 0) / RMSNorm (rms = 1) of rows of n, without gain or bias, with the
 * device's reduction tree: layout E > 0 = one warp per 32E-element chunk (lane l of warp
 * w sums elements 32Ew + El .. +E-1 in double, the warp adds lanes by an xor butterfly,
 * the warps' sums are added in warp order); E = 0 = the 256-thread row kernel (thread i
 * sums elements i, i + 256, ...).  Means and variances are sums / n rounded to float. */
void oo_norm_dev(const float *x, float *y, int64_t n, int64_t rows, float eps, int rms, int E);

/* Decode attention as the device kernels compute it (flash_attn_ext with one query
 * tile).  kind: OO_FAK_SPLIT (generic split-KV kernel: D 64 / 128, masks, f16 or f32
 * K/V), OO_FAK_HEADS (4-head kernel: D 64, f16, one query, no mask, H % 4 == 0),
 * OO_FAK_GQA (GQA kernel: D 128, f16, one query, no mask, G in {1, 2, 4}).  The KV
 * range [0, k->ne[1]) is the live prefix; nkv_max is the cache length the split plan
 * is taken from (>= k->ne[1]).  Shapes and dst as oo_flash_attn_ext. */
enum { OO_FAK_SPLIT = 0, OO_FAK_HEADS = 1, OO_FAK_GQA = 2 };
int oo_fa_device(const oo_tensor *q, const oo_tensor *k, const oo_tensor *v, const oo_tensor *mask, float scale,
                 int kind, int64_t nkv_max, oo_tensor *dst);
/* the split count the device plans for `kind` over a cache of nkv_max positions with
 * `groups` CTA groups (fattn.cu) */
int oo_fa_device_splits(int kind, int64_t nkv_max, int64_t groups);

#ifdef __cplusplus
}
#endif
#endif
