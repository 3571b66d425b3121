// kernels.cuh -- launcher declarations shared by the backend's .cu files.
#pragma once

#include <algorithm>

#include "common.cuh"

namespace oasr {

enum { FAMILY_Q8_0 = 0, FAMILY_Q8_K = 1 };

// Planar quantized activations in scratch (see quant_act.cu).
struct ActPlanes {
    int8_t *qs;    // [R][K]
    float *d;      // [R][K/32] (q8_0) or [R][K/256] (q8_K)
    int16_t *bs16; // [R][K/16] (q8_K only)
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

inline size_t act_planes_bytes(int family, int64_t R, int64_t K) {
    size_t b = align256((size_t)(R * K));
    if (family == FAMILY_Q8_0) return b + align256((size_t)(R * (K / 32)) * 4);
    return b + align256((size_t)(R * (K / 256)) * 4) + align256((size_t)(R * (K / 16)) * 2);
}

inline ActPlanes act_planes_at(void *base, int family, int64_t R, int64_t K) {
    uint8_t *p = (uint8_t *)base;
    ActPlanes a;
    a.qs = (int8_t *)p;
    p += align256((size_t)(R * K));
    a.d = (float *)p;
    if (family == FAMILY_Q8_0) {
        a.bs16 = nullptr;
    } else {
        p += align256((size_t)(R * (K / 256)) * 4);
        a.bs16 = (int16_t *)p;
    }
    return a;
}

int launch_quantize_act(oasr_backend *be, const oasr_tensor *x, int family, const ActPlanes &p);

// decode GEMV (M <= 8 activation rows sharing one weight slice)
int launch_mmv_quant(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int M, int K,
                     float *y, int64_t y_ld);
int launch_mmv_float(oasr_backend *be, const oasr_weight *w, int64_t slice, const char *x, int64_t x_ld_bytes,
                     bool x_f16, bool round_x_f16, int M, int K, float *y, int64_t y_ld);

// prefill / encoder GEMM (M > 8)
int launch_mmq(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
               float *y, int64_t y_ld);

// attention
int launch_flash_attn(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                      const oasr_tensor *mask, float scale, oasr_tensor *dst);

}  // namespace oasr
