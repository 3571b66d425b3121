// kernels.cuh -- launcher declarations shared by the backend's .cu files.
#pragma once

#include <algorithm>

#include "common.cuh"

namespace oasr {

enum { FAMILY_Q8_0 = 0, FAMILY_Q8_K = 1 };

// Planar quantized activations in scratch (see quant_act.cu).  The q8_K
// family also carries fp16 copies of the quants and 16-wide sums (exact
// small integers) when the row count reaches the tensor-core GEMM (R > 8).
struct ActPlanes {
    int8_t *qs;      // [R][K]
    float *d;        // [R][K/32] (q8_0) or [R][K/256] (q8_K)
    int16_t *bs16;   // [R][K/16] (q8_K only)
    __half *qs16;    // [R][K]    (q8_K, R > 8)
    __half *bs16h;   // [R][K/16] (q8_K, R > 8)
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

inline bool act_has_f16(int family, int64_t R) { return family == FAMILY_Q8_K && R > 8; }

inline size_t act_planes_bytes(int family, int64_t R, int64_t K) {
    size_t b = align256((size_t)(R * K));
    if (family == FAMILY_Q8_0) return b + align256((size_t)(R * (K / 32)) * 4);
    b += align256((size_t)(R * (K / 256)) * 4) + align256((size_t)(R * (K / 16)) * 2);
    if (act_has_f16(family, R)) b += align256((size_t)(R * K) * 2) + align256((size_t)(R * (K / 16)) * 2);
    return b;
}

inline ActPlanes act_planes_at(void *base, int family, int64_t R, int64_t K) {
    uint8_t *p = (uint8_t *)base;
    ActPlanes a;
    a.qs = (int8_t *)p;
    p += align256((size_t)(R * K));
    a.d = (float *)p;
    a.bs16 = nullptr;
    a.qs16 = nullptr;
    a.bs16h = nullptr;
    if (family == FAMILY_Q8_K) {
        p += align256((size_t)(R * (K / 256)) * 4);
        a.bs16 = (int16_t *)p;
        p += align256((size_t)(R * (K / 16)) * 2);
        if (act_has_f16(family, R)) {
            a.qs16 = (__half *)p;
            p += align256((size_t)(R * K) * 2);
            a.bs16h = (__half *)p;
        }
    }
    return a;
}

// row offset r0 into planes laid out for K-element rows
inline ActPlanes act_planes_offset(const ActPlanes &a, int family, int64_t r0, int64_t K) {
    ActPlanes s = a;
    s.qs = a.qs + r0 * K;
    s.d = a.d + r0 * (K / (family == FAMILY_Q8_0 ? 32 : 256));
    if (a.bs16) s.bs16 = a.bs16 + r0 * (K / 16);
    if (a.qs16) s.qs16 = a.qs16 + r0 * K;
    if (a.bs16h) s.bs16h = a.bs16h + r0 * (K / 16);
    return s;
}

int launch_quantize_act(oasr_backend *be, const oasr_tensor *x, int family, const ActPlanes &p);

// decode GEMV (M <= 8 activation rows sharing one weight slice)
int launch_mmv_quant(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int M, int K,
                     float *y, int64_t y_ld);
// decode GEMV on the integer tensor-core path over the weight's decode tiles (mmv_tc.cu)
bool mmv_tiles_supported(int type, int64_t K);
size_t mmv_tiles_bytes(int type, int64_t N, int64_t K, int64_t slices);
cudaError_t build_mmv_tiles(oasr_weight *w, cudaStream_t st);
int launch_mmv_tc(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int M, int K, float *y,
                  int64_t y_ld);
int launch_mmv_float(oasr_backend *be, const oasr_weight *w, int64_t slice, const char *x, int64_t x_ld_bytes,
                     bool x_f16, bool round_x_f16, int M, int K, float *y, int64_t y_ld);

// prefill / encoder GEMM (M > 8); Q8_0 on tcgen05 needs the block-major scale copy
bool mmq_q80_tc_supported(int type, int64_t N, int64_t K);
cudaError_t build_q80_scales_t(oasr_weight *w, cudaStream_t st);
cudaError_t build_q40_expanded(oasr_weight *w, cudaStream_t st);  // w->qs8 from a Q4_0 weight's nibble plane
bool mmq_q4k_tc_supported(int type, int64_t K);
size_t q4k_operand_bytes(int64_t N, int64_t K, int64_t slices, size_t *meta_bytes);  // h16 bytes; *meta_bytes k_meta
cudaError_t build_q4k_operand(oasr_weight *w, cudaStream_t st);  // w->h16, w->k_meta from the raw Q4_K rows
// M > 8 GEMM; bias (optional, [N]) is added to each output in the store, only on the Q4_K
// tensor-core path (mmq_fuses_bias)
bool mmq_fuses_bias(const oasr_weight *w, const ActPlanes &a);
int launch_mmq(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
               float *y, int64_t y_ld, const float *bias = nullptr);

// attention
bool flash_attn_tc_eligible(const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *mask,
                            const oasr_tensor *dst);
// tcgen05 flash attention for long query blocks (fattn_tc.cu): head_dim 64 or 128,
// no mask or (causal) key j visible to query i when j <= i + n_kv - n_q
int launch_flash_attn_tc(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                         float scale, oasr_tensor *dst, bool causal);
int launch_flash_attn(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                      const oasr_tensor *mask, float scale, oasr_tensor *dst);
int launch_flash_attn_ex(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                         const oasr_tensor *mask, float scale, oasr_tensor *dst, const float *q_bias,
                         const int *nkv_dev);
// Decode attention (one query per head) whose output rows [S][H * D] leave as the next
// mul_mat's activation planes (act_planes_at layout of `family` for S rows of H * D)
// instead of f32: the GQA kernel (head-major f16 caches, D 128, q8_0) or the 4-head kernel
// (heads contiguous per KV row, D 64, q8_0 or q8_K).  Fails for shapes that take neither;
// flash_attn_decode_q8_supported tells in advance.  `dst` describes the output shape only.
// kv_static (4-head kernel only): which K/V rows no launch this one can overlap under
// programmatic dependent launch writes, so that its first loads go before the wait on
// the predecessor: none, all, or all but the newest live row (*nkv_dev - 1, which the
// predecessor writes; *nkv_dev itself is then final before the launch).
enum : int { KV_STATIC_NONE = 0, KV_STATIC_ALL = 1, KV_STATIC_OLD = 2 };
int launch_flash_attn_decode_q8(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                                float scale, oasr_tensor *dst, const float *q_bias, const int *nkv_dev,
                                const ActPlanes &out_q8, int family, int kv_static = 0);
bool flash_attn_decode_q8_supported(int H, int HKV, int D, int family);
// allocation-free split-KV attention over file-scope device scratch (fattn.cu)
constexpr size_t FA_STATIC_PARTIAL_BYTES = (size_t)4 << 20;  // 4 MiB of split partials
constexpr int64_t FA_STATIC_TICKETS = 1024;                   // split groups (one ticket each)
constexpr int FA_STATIC_MAX_DEVICES = 64;
int launch_flash_attn_static(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                             const oasr_tensor *mask, float scale, oasr_tensor *dst);

}  // namespace oasr
