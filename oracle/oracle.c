/*
 * oracle.c -- CPU restatement of ggml's block formats and the semantics of the
 * ops on OpenASR's inference hot path.  TEST INFRASTRUCTURE ONLY (see
 * oracle.h): used by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg as the checker and the timed CPU baseline; never by the
 * product.
 *
 * Built with -ffp-contract=off so that every float operation below rounds
 * exactly where it is written; explicit fmaf() marks where ggml's SIMD kernels
 * fuse.  Summation order is this file's canonical order (ggml's own order
 * differs per ISA, so only the per-block terms are ggml-defined).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define QK8_0 32
#define QK4_0 32
#define QK_K 256

typedef struct { uint16_t d; int8_t qs[QK8_0]; } blk_q8_0;               /* 34 B */
typedef struct { uint16_t d; uint8_t qs[QK4_0 / 2]; } blk_q4_0;          /* 18 B */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[QK_K / 2]; } blk_q4_K; /* 144 B */
typedef struct { float d; int8_t qs[QK_K]; int16_t bsums[QK_K / 16]; } blk_q8_K;        /* 292 B */

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0 block size (gguf/constants.py Q8_0: 32, 34)");
_Static_assert(sizeof(blk_q4_0) == 18, "q4_0 block size (gguf/constants.py Q4_0: 32, 18)");
_Static_assert(sizeof(blk_q4_K) == 144, "q4_K block size (gguf/constants.py Q4_K: 256, 144)");
_Static_assert(sizeof(blk_q8_K) == 292, "q8_K block size (gguf/constants.py Q8_K: 256, 292)");

/* ------------------------------------------------------------------------ */
/* fp16                                                                      */
/* ------------------------------------------------------------------------ */
uint16_t oo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m24 = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t h = m24 >> shift;
        uint32_t rem = m24 & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static float f16_table[65536];
static pthread_once_t f16_once = PTHREAD_ONCE_INIT;
static float f16_to_f32_bits(uint16_t h);
static void f16_table_init(void) {
    for (uint32_t i = 0; i < 65536; ++i) f16_table[i] = f16_to_f32_bits((uint16_t)i);
}

/* table lookup (like ggml's ggml_table_f32_f16), filled from the bit-level conversion below */
float oo_f16_to_f32(uint16_t h) {
    pthread_once(&f16_once, f16_table_init);
    return f16_table[h];
}

static inline float f16(uint16_t h) { return f16_table[h]; }

static float f16_to_f32_bits(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else {
            int e = -1;
            do { e++; mant <<= 1; } while (!(mant & 0x400u));
            mant &= 0x3ffu;
            x = sign | ((uint32_t)(112 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1f) {
        x = sign | 0x7f800000u | (mant << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ggml's nearest_int: add 1.5*2^23 and read the mantissa (round half to even) */
int oo_nearest_int(float fval) {
    float val = fval + 12582912.f;
    int32_t i;
    memcpy(&i, &val, 4);
    return (i & 0x007fffff) - 0x00400000;
}

/* ------------------------------------------------------------------------ */
/* synthetic data: SplitMix64 -> Box-Muller                                  */
/* ------------------------------------------------------------------------ */
uint64_t oo_splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

#define OO_GAMMA 0x9E3779B97F4A7C15ULL
#define OO_TWO_PI 6.283185307179586476925286766559

void oo_synth_normal(uint64_t seed, uint64_t offset, float *x, int64_t n, float mean, float std) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint64_t j = offset + (uint64_t)i;
        uint64_t p = j >> 1;
        uint64_t a = oo_splitmix64(seed + (2 * p + 1) * OO_GAMMA);
        uint64_t b = oo_splitmix64(seed + (2 * p + 2) * OO_GAMMA);
        double u1 = (double)((a >> 11) + 1) * 0x1p-53;
        double u2 = (double)(b >> 11) * 0x1p-53;
        double r = sqrt(-2.0 * log(u1));
        double z = (j & 1) ? r * sin(OO_TWO_PI * u2) : r * cos(OO_TWO_PI * u2);
        x[i] = (float)((double)mean + (double)std * z);
    }
}

/* ------------------------------------------------------------------------ */
/* block formats                                                             */
/* ------------------------------------------------------------------------ */
int64_t oo_block_elems(int type) {
    switch (type) {
    case OO_TYPE_F32: case OO_TYPE_F16: case OO_TYPE_I32: return 1;
    case OO_TYPE_Q8_0: case OO_TYPE_Q4_0: return 32;
    case OO_TYPE_Q4_K: case OO_TYPE_Q8_K: return 256;
    default: return 0;
    }
}

int64_t oo_block_bytes(int type) {
    switch (type) {
    case OO_TYPE_F32: case OO_TYPE_I32: return 4;
    case OO_TYPE_F16: return 2;
    case OO_TYPE_Q8_0: return (int64_t)sizeof(blk_q8_0);
    case OO_TYPE_Q4_0: return (int64_t)sizeof(blk_q4_0);
    case OO_TYPE_Q4_K: return (int64_t)sizeof(blk_q4_K);
    case OO_TYPE_Q8_K: return (int64_t)sizeof(blk_q8_K);
    default: return 0;
    }
}

int64_t oo_row_size(int type, int64_t ne0) {
    int64_t be = oo_block_elems(type);
    if (be == 0 || ne0 % be) return -1;
    return ne0 / be * oo_block_bytes(type);
}

/* quantize_row_q8_0_ref (restated): d = amax/127, q = roundf(x * (1/d)). */
static void quantize_q8_0(const float *x, blk_q8_0 *y, int64_t k) {
    for (int64_t i = 0; i < k / QK8_0; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; ++j) {
            float v = fabsf(x[i * QK8_0 + j]);
            amax = amax > v ? amax : v;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = oo_f32_to_f16(d);
        for (int j = 0; j < QK8_0; ++j) y[i].qs[j] = (int8_t)roundf(x[i * QK8_0 + j] * id);
    }
}

/* quantize_row_q4_0_ref (restated): d = max/-8 (signed value of the first
 * largest |x|), q = min(15, trunc(x/d + 8.5)). */
static void quantize_q4_0(const float *x, blk_q4_0 *y, int64_t k) {
    for (int64_t i = 0; i < k / QK4_0; ++i) {
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK4_0; ++j) {
            const float v = x[i * QK4_0 + j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = oo_f32_to_f16(d);
        for (int j = 0; j < QK4_0 / 2; ++j) {
            const float x0 = x[i * QK4_0 + j] * id;
            const float x1 = x[i * QK4_0 + QK4_0 / 2 + j] * id;
            int q0 = (int8_t)(x0 + 8.5f);
            int q1 = (int8_t)(x1 + 8.5f);
            q0 = q0 < 15 ? q0 : 15;
            q1 = q1 < 15 ? q1 : 15;
            y[i].qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* quantize_row_q8_K_ref (restated): the activation format for Q4_K's dot.
 * iscale = -127/max (max = signed value of the first largest |x|),
 * q = min(127, nearest_int(iscale*x)), d = 1/iscale, bsums over 16. */
static void quantize_q8_K(const float *x, blk_q8_K *y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; ++i) {
        const float *xb = x + i * QK_K;
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < QK_K; ++j) {
            float ax = fabsf(xb[j]);
            if (ax > amax) { amax = ax; max = xb[j]; }
        }
        if (amax == 0.0f) {
            y[i].d = 0.0f;
            memset(y[i].qs, 0, sizeof(y[i].qs));
            memset(y[i].bsums, 0, sizeof(y[i].bsums));
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < QK_K; ++j) {
            int v = oo_nearest_int(iscale * xb[j]);
            y[i].qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int j = 0; j < QK_K / 16; ++j) {
            int s = 0;
            for (int l = 0; l < 16; ++l) s += y[i].qs[j * 16 + l];
            y[i].bsums[j] = (int16_t)s;
        }
        y[i].d = 1.0f / iscale;
    }
}

/* get_scale_min_k4: 6-bit scale and min of sub-block j from the 12 packed bytes
 * (layout cross-checked against gguf/quants.py Q4_K.get_scale_min). */
static inline void scale_min_k4(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* A simple deterministic Q4_K encoder for synthetic weights (NOT ggml's
 * make_qkx2_quants search): per 32-element sub-block, scale = (max-min)/15 and
 * min = -min(0, x); 6-bit sub-scales relative to fp16 d / dmin.  Any valid
 * Q4_K encoding is acceptable because the GPU and the oracle consume the same
 * bytes; decoding follows ggml exactly. */
static void quantize_q4_K(const float *x, blk_q4_K *y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; ++i) {
        const float *xb = x + i * QK_K;
        float scale[8], mins[8];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; ++j) {
            float mn = xb[32 * j], mx = xb[32 * j];
            for (int l = 1; l < 32; ++l) {
                float v = xb[32 * j + l];
                mn = v < mn ? v : mn;
                mx = v > mx ? v : mx;
            }
            if (mn > 0.0f) mn = 0.0f;
            scale[j] = (mx - mn) / 15.0f;
            mins[j] = -mn;
            max_scale = scale[j] > max_scale ? scale[j] : max_scale;
            max_min = mins[j] > max_min ? mins[j] : max_min;
        }
        uint16_t dh = oo_f32_to_f16(max_scale / 63.0f);
        uint16_t dminh = oo_f32_to_f16(max_min / 63.0f);
        const float d = oo_f16_to_f32(dh), dmin = oo_f16_to_f32(dminh);
        int sc[8], mq[8];
        for (int j = 0; j < 8; ++j) {
            int s = d > 0.0f ? oo_nearest_int(scale[j] / d) : 0;
            int m = dmin > 0.0f ? oo_nearest_int(mins[j] / dmin) : 0;
            sc[j] = s < 0 ? 0 : (s > 63 ? 63 : s);
            mq[j] = m < 0 ? 0 : (m > 63 ? 63 : m);
        }
        y[i].d = dh;
        y[i].dmin = dminh;
        for (int j = 0; j < 4; ++j) {
            y[i].scales[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            y[i].scales[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
            y[i].scales[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
        }
        uint8_t q[QK_K];
        for (int j = 0; j < 8; ++j) {
            const float dl = d * (float)sc[j];
            const float ml = dmin * (float)mq[j];
            for (int l = 0; l < 32; ++l) {
                int v = dl > 0.0f ? oo_nearest_int((xb[32 * j + l] + ml) / dl) : 0;
                q[32 * j + l] = (uint8_t)(v < 0 ? 0 : (v > 15 ? 15 : v));
            }
        }
        for (int c = 0; c < 4; ++c)
            for (int l = 0; l < 32; ++l)
                y[i].qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
}

int oo_quantize_row(int type, const float *x, void *y, int64_t k) {
    int64_t be = oo_block_elems(type);
    if (be == 0 || k % be) return OO_STATUS_FAILED;
    switch (type) {
    case OO_TYPE_Q8_0: quantize_q8_0(x, (blk_q8_0 *)y, k); return 0;
    case OO_TYPE_Q4_0: quantize_q4_0(x, (blk_q4_0 *)y, k); return 0;
    case OO_TYPE_Q4_K: quantize_q4_K(x, (blk_q4_K *)y, k); return 0;
    case OO_TYPE_Q8_K: quantize_q8_K(x, (blk_q8_K *)y, k); return 0;
    case OO_TYPE_F16:
        for (int64_t i = 0; i < k; ++i) ((uint16_t *)y)[i] = oo_f32_to_f16(x[i]);
        return 0;
    case OO_TYPE_F32: memcpy(y, x, (size_t)k * 4); return 0;
    default: return OO_STATUS_FAILED;
    }
}

int oo_quantize_rows(int type, const float *x, void *y, int64_t nrows, int64_t ne0) {
    int64_t rs = oo_row_size(type, ne0);
    if (rs < 0) return OO_STATUS_FAILED;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t r = 0; r < nrows; ++r)
        bad |= oo_quantize_row(type, x + r * ne0, (char *)y + r * rs, ne0) != 0;
    return bad ? OO_STATUS_FAILED : 0;
}

int oo_dequantize_row(int type, const void *vx, float *y, int64_t k) {
    int64_t be = oo_block_elems(type);
    if (be == 0 || k % be) return OO_STATUS_FAILED;
    switch (type) {
    case OO_TYPE_Q8_0: {
        const blk_q8_0 *x = (const blk_q8_0 *)vx;
        for (int64_t i = 0; i < k / QK8_0; ++i) {
            const float d = oo_f16_to_f32(x[i].d);
            for (int j = 0; j < QK8_0; ++j) y[i * QK8_0 + j] = (float)x[i].qs[j] * d;
        }
        return 0;
    }
    case OO_TYPE_Q4_0: {
        const blk_q4_0 *x = (const blk_q4_0 *)vx;
        for (int64_t i = 0; i < k / QK4_0; ++i) {
            const float d = oo_f16_to_f32(x[i].d);
            for (int j = 0; j < QK4_0 / 2; ++j) {
                y[i * QK4_0 + j] = (float)((x[i].qs[j] & 0xF) - 8) * d;
                y[i * QK4_0 + j + QK4_0 / 2] = (float)((x[i].qs[j] >> 4) - 8) * d;
            }
        }
        return 0;
    }
    case OO_TYPE_Q4_K: {
        const blk_q4_K *x = (const blk_q4_K *)vx;
        for (int64_t i = 0; i < k / QK_K; ++i) {
            const float d = oo_f16_to_f32(x[i].d);
            const float min = oo_f16_to_f32(x[i].dmin);
            const uint8_t *q = x[i].qs;
            float *yb = y + i * QK_K;
            for (int c = 0; c < 4; ++c) {
                int sc, m;
                scale_min_k4(2 * c, x[i].scales, &sc, &m);
                const float d1 = d * (float)sc, m1 = min * (float)m;
                scale_min_k4(2 * c + 1, x[i].scales, &sc, &m);
                const float d2 = d * (float)sc, m2 = min * (float)m;
                for (int l = 0; l < 32; ++l) yb[64 * c + l] = d1 * (float)(q[32 * c + l] & 0xF) - m1;
                for (int l = 0; l < 32; ++l) yb[64 * c + 32 + l] = d2 * (float)(q[32 * c + l] >> 4) - m2;
            }
        }
        return 0;
    }
    case OO_TYPE_Q8_K: {
        const blk_q8_K *x = (const blk_q8_K *)vx;
        for (int64_t i = 0; i < k / QK_K; ++i)
            for (int j = 0; j < QK_K; ++j) y[i * QK_K + j] = x[i].d * (float)x[i].qs[j];
        return 0;
    }
    case OO_TYPE_F16:
        for (int64_t i = 0; i < k; ++i) y[i] = oo_f16_to_f32(((const uint16_t *)vx)[i]);
        return 0;
    case OO_TYPE_F32: memcpy(y, vx, (size_t)k * 4); return 0;
    default: return OO_STATUS_FAILED;
    }
}

/* ------------------------------------------------------------------------ */
/* block dot products (ggml vec_dot semantics; per-block term then f32 sum)  */
/* ------------------------------------------------------------------------ */
static float dot_q8_0_q8_0(const blk_q8_0 *x, const blk_q8_0 *y, int64_t nb) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        int sumi = 0;
        for (int j = 0; j < QK8_0; ++j) sumi += (int)x[b].qs[j] * (int)y[b].qs[j];
        const float dd = f16(x[b].d) * f16(y[b].d);
        sumf += (float)sumi * dd;
    }
    return sumf;
}

static float dot_q4_0_q8_0(const blk_q4_0 *x, const blk_q8_0 *y, int64_t nb) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        int sumi = 0;
        for (int j = 0; j < QK4_0 / 2; ++j) {
            sumi += ((x[b].qs[j] & 0xF) - 8) * (int)y[b].qs[j];
            sumi += ((x[b].qs[j] >> 4) - 8) * (int)y[b].qs[j + QK4_0 / 2];
        }
        const float dd = f16(x[b].d) * f16(y[b].d);
        sumf += (float)sumi * dd;
    }
    return sumf;
}

/* per super-block: isum = sum_j sc_j * <q4_j, q8_j>, msum = sum_j m_j * bsum32_j,
 * term = (d_x*d_y)*isum - (dmin_x*d_y)*msum */
static float dot_q4_K_q8_K(const blk_q4_K *x, const blk_q8_K *y, int64_t nb) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        int isum = 0, msum = 0;
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            scale_min_k4(j, x[b].scales, &sc, &m);
            const int c = j >> 1, hi = j & 1;
            int dot = 0;
            for (int l = 0; l < 32; ++l) {
                int q = hi ? (x[b].qs[32 * c + l] >> 4) : (x[b].qs[32 * c + l] & 0xF);
                dot += q * (int)y[b].qs[32 * j + l];
            }
            isum += sc * dot;
            msum += m * ((int)y[b].bsums[2 * j] + (int)y[b].bsums[2 * j + 1]);
        }
        const float d = f16(x[b].d) * y[b].d;
        const float dmin = f16(x[b].dmin) * y[b].d;
        const float t1 = d * (float)isum;
        const float t2 = dmin * (float)msum;
        sumf += t1 - t2;
    }
    return sumf;
}

static float dot_f16_f16(const uint16_t *x, const uint16_t *y, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)(f16(x[i]) * f16(y[i]));
    return (float)s;
}

static float dot_f32_f32(const float *x, const float *y, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)(x[i] * y[i]);
    return (float)s;
}

static int vec_dot_type(int wtype) {
    switch (wtype) {
    case OO_TYPE_Q8_0: case OO_TYPE_Q4_0: return OO_TYPE_Q8_0;
    case OO_TYPE_Q4_K: return OO_TYPE_Q8_K;
    case OO_TYPE_F16: return OO_TYPE_F16;
    case OO_TYPE_F32: return OO_TYPE_F32;
    default: return -1;
    }
}

int oo_mul_mat(const oo_tensor *w, const oo_tensor *x, oo_tensor *dst) {
    pthread_once(&f16_once, f16_table_init);
    const int64_t K = w->ne[0], N = w->ne[1];
    if (x->ne[0] != K) return OO_STATUS_FAILED;
    if (x->ne[2] % w->ne[2] || x->ne[3] % w->ne[3]) return OO_STATUS_FAILED;
    if (x->type != OO_TYPE_F32 && x->type != OO_TYPE_F16) return OO_STATUS_FAILED;
    if (dst->type != OO_TYPE_F32 || dst->ne[0] != N || dst->ne[1] != x->ne[1] ||
        dst->ne[2] != x->ne[2] || dst->ne[3] != x->ne[3])
        return OO_STATUS_FAILED;
    const int vt = vec_dot_type(w->type);
    if (vt < 0) return OO_STATUS_FAILED;
    const int64_t rs = oo_row_size(vt, K);
    if (rs < 0 || oo_row_size(w->type, K) < 0) return OO_STATUS_FAILED;
    const int64_t M = x->ne[1], ne2 = x->ne[2], ne3 = x->ne[3];
    const int64_t r2 = ne2 / w->ne[2], r3 = ne3 / w->ne[3];
    const int64_t nrows = M * ne2 * ne3;
    char *xq = (char *)malloc((size_t)(nrows * rs));
    if (!xq) return OO_STATUS_ALLOC_FAILED;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t r = 0; r < nrows; ++r) {
        const int64_t m = r % M, i2 = (r / M) % ne2, i3 = r / (M * ne2);
        const char *src = (const char *)x->data + m * x->nb[1] + i2 * x->nb[2] + i3 * x->nb[3];
        float *tmp = (float *)malloc((size_t)K * 4);
        if (!tmp) { bad = 1; continue; }
        for (int64_t k = 0; k < K; ++k) {
            const char *p = src + k * x->nb[0];
            tmp[k] = x->type == OO_TYPE_F32 ? *(const float *)p : oo_f16_to_f32(*(const uint16_t *)p);
        }
        if (vt == OO_TYPE_F16 && x->type == OO_TYPE_F16) {
            for (int64_t k = 0; k < K; ++k)
                ((uint16_t *)(xq + r * rs))[k] = *(const uint16_t *)(src + k * x->nb[0]);
        } else {
            bad |= oo_quantize_row(vt, tmp, xq + r * rs, K) != 0;
        }
        free(tmp);
    }
    if (bad) { free(xq); return OO_STATUS_FAILED; }
    const int64_t total = nrows * N;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < total; ++t) {
        const int64_t n = t % N, r = t / N;
        const int64_t m = r % M, i2 = (r / M) % ne2, i3 = r / (M * ne2);
        const char *wr = (const char *)w->data + n * w->nb[1] + (i2 / r2) * w->nb[2] + (i3 / r3) * w->nb[3];
        const char *xr = xq + r * rs;
        float v;
        switch (w->type) {
        case OO_TYPE_Q8_0: v = dot_q8_0_q8_0((const blk_q8_0 *)wr, (const blk_q8_0 *)xr, K / QK8_0); break;
        case OO_TYPE_Q4_0: v = dot_q4_0_q8_0((const blk_q4_0 *)wr, (const blk_q8_0 *)xr, K / QK4_0); break;
        case OO_TYPE_Q4_K: v = dot_q4_K_q8_K((const blk_q4_K *)wr, (const blk_q8_K *)xr, K / QK_K); break;
        case OO_TYPE_F16: v = dot_f16_f16((const uint16_t *)wr, (const uint16_t *)xr, K); break;
        default: v = dot_f32_f32((const float *)wr, (const float *)xr, K); break;
        }
        *(float *)((char *)dst->data + n * dst->nb[0] + m * dst->nb[1] + i2 * dst->nb[2] + i3 * dst->nb[3]) = v;
    }
    free(xq);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* flash_attn_ext                                                            */
/* ------------------------------------------------------------------------ */
static inline float load_elem(const char *p, int type) {
    return type == OO_TYPE_F32 ? *(const float *)p : oo_f16_to_f32(*(const uint16_t *)p);
}

static float r16(float x) { return oo_f16_to_f32(oo_f32_to_f16(x)); }

/* tensor-core arithmetic (see oracle.h, OO_FA_TC128); mask entries 0 (visible) or -inf (hidden).
 * K and V of each (sequence, kv head) are rounded to fp16 once into contiguous rows; the
 * per-query arithmetic below is unchanged by that (same values, same summation order). */
static int fa_tc128(const oo_tensor *q, const oo_tensor *k, const oo_tensor *v, const oo_tensor *mask, float scale,
                    oo_tensor *dst) {
    const int64_t D = q->ne[0], NQ = q->ne[1], H = q->ne[2], S = q->ne[3];
    const int64_t NKV = k->ne[1], HKV = k->ne[2];
    const int64_t G = H / HKV;
    const float sl2 = scale * 1.4426950408889634f;
    int bad = 0;
    for (int64_t s = 0; s < S; ++s)
        for (int64_t hk = 0; hk < HKV; ++hk) {
            float *kr16 = (float *)malloc((size_t)(2 * NKV * D) * sizeof(float));
            if (!kr16) return OO_STATUS_ALLOC_FAILED;
            float *vr16 = kr16 + NKV * D;
#pragma omp parallel for schedule(static)
            for (int64_t j = 0; j < NKV; ++j)
                for (int64_t d = 0; d < D; ++d) {
                    kr16[j * D + d] = r16(load_elem((const char *)k->data + d * k->nb[0] + j * k->nb[1] + hk * k->nb[2] + s * k->nb[3], k->type));
                    vr16[j * D + d] = r16(load_elem((const char *)v->data + d * v->nb[0] + j * v->nb[1] + hk * v->nb[2] + s * v->nb[3], v->type));
                }
#pragma omp parallel for schedule(dynamic, 4) reduction(| : bad)
            for (int64_t ir = 0; ir < NQ * G; ++ir) {
                const int64_t h = hk * G + ir / NQ, iq = ir % NQ;
                float *qv = (float *)malloc((size_t)D * 4 * 3 + 128 * 4);
                if (!qv) { bad = 1; continue; }
                float *o = qv + D, *ot = qv + 2 * D, *x = qv + 3 * D;
                const char *pq = (const char *)q->data + iq * q->nb[1] + h * q->nb[2] + s * q->nb[3];
                for (int64_t d = 0; d < D; ++d) { qv[d] = r16(*(const float *)(pq + d * q->nb[0])); o[d] = 0.0f; }
                const char *mp = mask ? (const char *)mask->data + iq * mask->nb[1] + (h % mask->ne[2]) * mask->nb[2] +
                                            (s % mask->ne[3]) * mask->nb[3]
                                      : NULL;
                float m = -INFINITY, l = 0.0f;
                for (int64_t j0 = 0; j0 < NKV; j0 += 128) {
                    const int64_t nv = NKV - j0 < 128 ? NKV - j0 : 128;
                    float tmax = -INFINITY;
                    for (int64_t i = 0; i < nv; ++i) {
                        /* mask: 0 = visible, -inf = hidden (the kernel takes no other values) */
                        if (mp && oo_f16_to_f32(*(const uint16_t *)(mp + (j0 + i) * mask->nb[0])) == -INFINITY) {
                            x[i] = -INFINITY;
                            continue;
                        }
                        const float *kr = kr16 + (j0 + i) * D;
                        double acc = 0.0;
                        for (int64_t d = 0; d < D; ++d) acc += (double)(qv[d] * kr[d]);
                        x[i] = (float)acc * sl2;
                        tmax = tmax > x[i] ? tmax : x[i];
                    }
                    const float mnew = m > tmax ? m : tmax;
                    const float alpha = mnew == -INFINITY ? 1.0f : exp2f(m - mnew);
                    float tsum = 0.0f;
                    for (int64_t i = 0; i < 128; i += 2) {
                        const float p0 = i < nv && x[i] != -INFINITY ? exp2f(x[i] - mnew) : 0.0f;
                        const float p1 = i + 1 < nv && x[i + 1] != -INFINITY ? exp2f(x[i + 1] - mnew) : 0.0f;
                        tsum += p0 + p1;
                        if (i < nv) x[i] = r16(p0);
                        if (i + 1 < nv) x[i + 1] = r16(p1);
                    }
                    for (int64_t d = 0; d < D; ++d) {
                        double acc = 0.0;
                        for (int64_t i = 0; i < nv; ++i) acc += (double)(x[i] * vr16[(j0 + i) * D + d]);
                        ot[d] = (float)acc;
                    }
                    for (int64_t d = 0; d < D; ++d) o[d] = fmaf(o[d], alpha, ot[d]);
                    l = l * alpha + tsum;
                    m = mnew;
                }
                const float inv = l == 0.0f ? 0.0f : 1.0f / l;
                float *out = (float *)((char *)dst->data + h * dst->nb[1] + iq * dst->nb[2] + s * dst->nb[3]);
                for (int64_t d = 0; d < D; ++d) out[d] = o[d] * inv;
                free(qv);
            }
            free(kr16);
        }
    return bad ? OO_STATUS_ALLOC_FAILED : 0;
}

int oo_flash_attn_ext(const oo_tensor *q, const oo_tensor *k, const oo_tensor *v,
                      const oo_tensor *mask, float scale, int mode, oo_tensor *dst) {
    const int64_t DK = q->ne[0], NQ = q->ne[1], H = q->ne[2], S = q->ne[3];
    const int64_t NKV = k->ne[1], HKV = k->ne[2], DV = v->ne[0];
    if (q->type != OO_TYPE_F32 || k->ne[0] != DK) return OO_STATUS_FAILED;
    if (k->type != v->type || (k->type != OO_TYPE_F16 && k->type != OO_TYPE_F32)) return OO_STATUS_FAILED;
    if (v->ne[1] != NKV || v->ne[2] != HKV || k->ne[3] != S || v->ne[3] != S) return OO_STATUS_FAILED;
    if (HKV == 0 || H % HKV) return OO_STATUS_FAILED;
    if (mask && (mask->type != OO_TYPE_F16 || mask->ne[0] < NKV || mask->ne[1] < NQ ||
                 H % mask->ne[2] || S % mask->ne[3]))
        return OO_STATUS_FAILED;
    if (dst->type != OO_TYPE_F32 || dst->ne[0] != DV || dst->ne[1] != H || dst->ne[2] != NQ || dst->ne[3] != S)
        return OO_STATUS_FAILED;
    const int64_t rk2 = H / HKV;
    if (mode == OO_FA_TC128) {
        if (mask) /* visible / hidden masks only */
            for (int64_t i3 = 0; i3 < mask->ne[3]; ++i3)
                for (int64_t i2 = 0; i2 < mask->ne[2]; ++i2)
                    for (int64_t i1 = 0; i1 < NQ; ++i1)
                        for (int64_t i0 = 0; i0 < NKV; ++i0) {
                            const float mv = oo_f16_to_f32(*(const uint16_t *)((const char *)mask->data + i0 * mask->nb[0] +
                                                                               i1 * mask->nb[1] + i2 * mask->nb[2] +
                                                                               i3 * mask->nb[3]));
                            if (mv != 0.0f && mv != -INFINITY) return OO_STATUS_FAILED;
                        }
        return fa_tc128(q, k, v, mask, scale, dst);
    }
    const int f16acc = (mode == OO_FA_GGML) && v->type == OO_TYPE_F16;
    int bad = 0;
#pragma omp parallel for schedule(dynamic, 4) reduction(| : bad)
    for (int64_t ir = 0; ir < NQ * H * S; ++ir) {
        const int64_t iq3 = ir / (H * NQ);
        const int64_t iq2 = (ir - iq3 * H * NQ) / NQ;
        const int64_t iq1 = ir - iq3 * H * NQ - iq2 * NQ;
        const int64_t ik2 = iq2 / rk2;
        float *qc = (float *)malloc((size_t)(DK + 2 * DV) * 4);
        uint16_t *vkq16 = (uint16_t *)malloc((size_t)DV * 2);
        if (!qc || !vkq16) { free(qc); free(vkq16); bad = 1; continue; }
        float *vkq32 = qc + DK, *vrow = qc + DK + DV;
        const char *pq = (const char *)q->data + iq1 * q->nb[1] + iq2 * q->nb[2] + iq3 * q->nb[3];
        for (int64_t d = 0; d < DK; ++d) {
            float qv = *(const float *)(pq + d * q->nb[0]);
            qc[d] = k->type == OO_TYPE_F16 ? oo_f16_to_f32(oo_f32_to_f16(qv)) : qv;
        }
        memset(vkq32, 0, (size_t)DV * 4);
        memset(vkq16, 0, (size_t)DV * 2);
        const char *mp = mask ? (const char *)mask->data + iq1 * mask->nb[1] +
                                    (iq2 % mask->ne[2]) * mask->nb[2] + (iq3 % mask->ne[3]) * mask->nb[3]
                              : NULL;
        float S_ = 0.0f, M_ = -INFINITY;
        for (int64_t ic = 0; ic < NKV; ++ic) {
            const float mv = mp ? oo_f16_to_f32(*(const uint16_t *)(mp + ic * mask->nb[0])) : 0.0f;
            if (mv == -INFINITY) continue;
            const char *kr = (const char *)k->data + ic * k->nb[1] + ik2 * k->nb[2] + iq3 * k->nb[3];
            double acc = 0.0;
            for (int64_t d = 0; d < DK; ++d) acc += (double)(qc[d] * load_elem(kr + d * k->nb[0], k->type));
            float s = (float)acc;
            s = s * scale;
            s += mv;
            const float Mold = M_;
            float ms = 1.0f, vs = 1.0f;
            const char *vr = (const char *)v->data + ic * v->nb[1] + ik2 * v->nb[2] + iq3 * v->nb[3];
            if (s > M_) {
                M_ = s;
                ms = expf(Mold - M_);
                if (f16acc)
                    for (int64_t d = 0; d < DV; ++d) vkq16[d] = oo_f32_to_f16(oo_f16_to_f32(vkq16[d]) * ms);
                else
                    for (int64_t d = 0; d < DV; ++d) vkq32[d] *= ms;
            } else {
                vs = expf(s - M_);
            }
            if (f16acc) {
                for (int64_t d = 0; d < DV; ++d)
                    vkq16[d] = oo_f32_to_f16(fmaf(load_elem(vr + d * v->nb[0], v->type), vs, oo_f16_to_f32(vkq16[d])));
            } else {
                for (int64_t d = 0; d < DV; ++d) vrow[d] = load_elem(vr + d * v->nb[0], v->type);
                for (int64_t d = 0; d < DV; ++d) vkq32[d] = fmaf(vrow[d], vs, vkq32[d]);
            }
            S_ = S_ * ms + vs;
        }
        if (f16acc)
            for (int64_t d = 0; d < DV; ++d) vkq32[d] = oo_f16_to_f32(vkq16[d]);
        const float S_inv = S_ == 0.0f ? 0.0f : 1.0f / S_;
        float *out = (float *)((char *)dst->data + iq2 * dst->nb[1] + iq1 * dst->nb[2] + iq3 * dst->nb[3]);
        for (int64_t d = 0; d < DV; ++d) out[d] = vkq32[d] * S_inv;
        free(qc);
        free(vkq16);
    }
    return bad ? OO_STATUS_ALLOC_FAILED : 0;
}

/* ------------------------------------------------------------------------ */
/* set_rows / argmax / row ops                                               */
/* ------------------------------------------------------------------------ */
int oo_set_rows(oo_tensor *dst, const oo_tensor *src, const int64_t *rows, int64_t n_rows) {
    if (src->type != OO_TYPE_F32 || (dst->type != OO_TYPE_F32 && dst->type != OO_TYPE_F16)) return OO_STATUS_FAILED;
    if (src->ne[0] != dst->ne[0] || src->ne[1] != n_rows || src->ne[2] != dst->ne[2] || src->ne[3] != dst->ne[3])
        return OO_STATUS_FAILED;
    for (int64_t i = 0; i < n_rows; ++i)
        if (rows[i] < 0 || rows[i] >= dst->ne[1]) return OO_STATUS_FAILED;
    for (int64_t i3 = 0; i3 < src->ne[3]; ++i3)
        for (int64_t i2 = 0; i2 < src->ne[2]; ++i2)
            for (int64_t i = 0; i < n_rows; ++i) {
                const char *s = (const char *)src->data + i * src->nb[1] + i2 * src->nb[2] + i3 * src->nb[3];
                char *d = (char *)dst->data + rows[i] * dst->nb[1] + i2 * dst->nb[2] + i3 * dst->nb[3];
                for (int64_t e = 0; e < src->ne[0]; ++e) {
                    float f = *(const float *)(s + e * src->nb[0]);
                    if (dst->type == OO_TYPE_F32) *(float *)(d + e * dst->nb[0]) = f;
                    else *(uint16_t *)(d + e * dst->nb[0]) = oo_f32_to_f16(f);
                }
            }
    return 0;
}

void oo_argmax_first(const float *x, int64_t n, int64_t rows, int32_t *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        int64_t best = -1;
        float bv = 0.0f;
        for (int64_t i = 0; i < n; ++i) {
            const float v = xr[i];
            if (!isfinite(v)) continue;
            if (best < 0 || v > bv) { best = i; bv = v; }
        }
        out[r] = (int32_t)(best < 0 ? 0 : best);
    }
}

void oo_norm(const float *x, float *y, int64_t n, int64_t rows, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; ++i) sum += (double)xr[i];
        const float mean = (float)(sum / (double)n);
        double sum2 = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            const float v = xr[i] - mean;
            yr[i] = v;
            sum2 += (double)(v * v);
        }
        const float variance = (float)(sum2 / (double)n);
        const float scale = 1.0f / sqrtf(variance + eps);
        for (int64_t i = 0; i < n; ++i) yr[i] *= scale;
    }
}

void oo_rms_norm(const float *x, float *y, int64_t n, int64_t rows, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; ++i) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / (double)n);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < n; ++i) yr[i] = xr[i] * scale;
    }
}

/* ggml_gelu on CPU: tanh-approximation GELU evaluated through an fp16 lookup
 * table indexed by the fp16 bits of x, identity above 10 and zero below -10. */
static uint16_t gelu_table[65536];
static pthread_once_t gelu_once = PTHREAD_ONCE_INIT;

static float gelu_f32(float x) {
    const float GELU_COEF_A = 0.044715f;
    const float SQRT_2_OVER_PI = 0.79788456080286535587989211986876f;
    return 0.5f * x * (1.0f + tanhf(SQRT_2_OVER_PI * x * (1.0f + GELU_COEF_A * x * x)));
}

static void gelu_table_init(void) {
    for (uint32_t i = 0; i < 65536; ++i) gelu_table[i] = oo_f32_to_f16(gelu_f32(oo_f16_to_f32((uint16_t)i)));
}

void oo_gelu(const float *x, float *y, int64_t n) {
    pthread_once(&gelu_once, gelu_table_init);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i];
        if (v <= -10.0f) y[i] = 0.0f;
        else if (v >= 10.0f) y[i] = v;
        else y[i] = oo_f16_to_f32(gelu_table[oo_f32_to_f16(v)]);
    }
}

void oo_silu(const float *x, float *y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) y[i] = x[i] / (1.0f + oo_expf(-x[i]));
}

void oo_rope_neox(float *x, int64_t D, int64_t H, int64_t T, const int32_t *pos, float freq_base) {
    const float theta_scale = powf(freq_base, -2.0f / (float)D);
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        float theta = (float)pos[t];
        for (int64_t i = 0; i < D / 2; ++i) {
            const float c = cosf(theta), s = sinf(theta);
            for (int64_t h = 0; h < H; ++h) {
                float *row = x + (t * H + h) * D;
                const float x0 = row[i], x1 = row[i + D / 2];
                row[i] = x0 * c - x1 * s;
                row[i + D / 2] = x0 * s + x1 * c;
            }
            theta *= theta_scale;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* the decode path's canonical arithmetic (see oracle.h)                     */
/* ------------------------------------------------------------------------ */
static float pow2i(int k) { /* 2^k, -126 <= k <= 127 */
    uint32_t b = (uint32_t)(k + 127) << 23;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

float oo_expf(float x) {
    if (!(x == x)) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    const float t = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-t, 0.693145751953125f, x);
    r = fmaf(-t, 1.428606765330187045e-06f, r);
    float p = 1.9841270113e-04f;
    p = fmaf(p, r, 1.3888889225e-03f);
    p = fmaf(p, r, 8.3333337680e-03f);
    p = fmaf(p, r, 4.1666667908e-02f);
    p = fmaf(p, r, 1.6666667163e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int n = (int)t;
    if (n > 127) return (p * pow2i(127)) * 2.0f;
    if (n < -126) return (p * pow2i(n + 64)) * pow2i(-64);
    return p * pow2i(n);
}

/* xor butterfly over `n` (power of two) lanes: after level o every lane holds
 * v[l] + v[l ^ o]; returns lane 0's final value (all lanes agree: + commutes) */
static double butterfly_d(double *v, int n) {
    for (int o = n / 2; o > 0; o >>= 1)
        for (int l = 0; l < n; ++l)
            if (l < (l ^ o)) {
                const double s = v[l] + v[l ^ o];
                v[l] = s;
                v[l ^ o] = s;
            }
    return v[0];
}

static float butterfly_f(float *v, int n) {
    for (int o = n / 2; o > 0; o >>= 1)
        for (int l = 0; l < n; ++l)
            if (l < (l ^ o)) {
                const float s = v[l] + v[l ^ o];
                v[l] = s;
                v[l ^ o] = s;
            }
    return v[0];
}

/* the device's double reduction of per-element values x[i] (squared when sq) over a
 * row of n: E > 0 chunk kernel, E == 0 256-thread kernel (elementwise.cu) */
static double dev_row_sum(const float *x, int64_t n, int E, int sq) {
    double lanes[32];
    double t = 0.0;
    if (E > 0) {
        const int64_t nw = n / (32 * E);
        for (int64_t w = 0; w < nw; ++w) {
            for (int l = 0; l < 32; ++l) {
                double s = 0.0;
                for (int i = 0; i < E; ++i) {
                    const float v = x[w * 32 * E + (int64_t)E * l + i];
                    s += (double)(sq ? v * v : v);
                }
                lanes[l] = s;
            }
            t += butterfly_d(lanes, 32);
        }
    } else {
        for (int w = 0; w < 8; ++w) {
            for (int l = 0; l < 32; ++l) {
                double s = 0.0;
                for (int64_t i = 32 * w + l; i < n; i += 256) {
                    const float v = x[i];
                    s += (double)(sq ? v * v : v);
                }
                lanes[l] = s;
            }
            t += butterfly_d(lanes, 32);
        }
    }
    return t;
}

void oo_norm_dev(const float *x, float *y, int64_t n, int64_t rows, float eps, int rms, int E) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        if (rms) {
            const float mean = (float)(dev_row_sum(xr, n, E, 1) / (double)n);
            const float scale = 1.0f / sqrtf(mean + eps);
            for (int64_t i = 0; i < n; ++i) yr[i] = xr[i] * scale;
        } else {
            const float mean = (float)(dev_row_sum(xr, n, E, 0) / (double)n);
            for (int64_t i = 0; i < n; ++i) yr[i] = xr[i] - mean;
            const float var = (float)(dev_row_sum(yr, n, E, 1) / (double)n);
            const float scale = 1.0f / sqrtf(var + eps);
            for (int64_t i = 0; i < n; ++i) yr[i] = yr[i] * scale;
        }
    }
}

/* ---- decode attention, device order ------------------------------------------------- */
#define FA_SPLITS_HEADS 7
#define FA_HEADS_SPLIT_MIN 513 /* shorter caches run unsplit in the 4-head kernel */
#define FA_SPLITS_GQA 4
#define FA_SPLITS_MAX 16

int oo_fa_device_splits(int kind, int64_t nkv_max, int64_t groups) {
    if (groups > (1 << 16)) return 1;
    int64_t n = kind == OO_FAK_HEADS ? (nkv_max < FA_HEADS_SPLIT_MIN                ? 1
                                        : nkv_max / 32 < FA_SPLITS_HEADS ? nkv_max / 32
                                                                         : FA_SPLITS_HEADS)
              : kind == OO_FAK_GQA   ? (nkv_max / 32 < FA_SPLITS_GQA ? nkv_max / 32 : FA_SPLITS_GQA)
                                     : (nkv_max / 64 < FA_SPLITS_MAX ? nkv_max / 64 : FA_SPLITS_MAX);
    return n < 1 ? 1 : (int)n;
}

/* online-softmax state of one lane group: running max, sum, D accumulators */
typedef struct { float m, l; float a[128]; } fa_state;

static void fa_state_init(fa_state *s, int D) {
    s->m = -INFINITY;
    s->l = 0.0f;
    for (int e = 0; e < D; ++e) s->a[e] = 0.0f;
}

/* a absorbs its shuffle partner b: a = a * f(a) + b * f(b), b's product fused */
static void fa_combine(fa_state *a, const fa_state *b, int D) {
    const float nm = fmaxf(a->m, b->m);
    const float f0 = a->m == -INFINITY ? 0.0f : oo_expf(a->m - nm);
    const float f1 = b->m == -INFINITY ? 0.0f : oo_expf(b->m - nm);
    a->l = fmaf(b->l, f1, a->l * f0);
    for (int e = 0; e < D; ++e) a->a[e] = fmaf(b->a[e], f1, a->a[e] * f0);
    a->m = nm;
}

/* merge of parts in order (the 4 warps of a CTA, or the splits of a row):
 * M = max m, L = sum l f, A = sum a f (f = e^(m - M)), each product fused into its sum */
static void fa_merge(const fa_state *parts, int n, int D, fa_state *out) {
    float M = -INFINITY;
    for (int i = 0; i < n; ++i) M = fmaxf(M, parts[i].m);
    float L = 0.0f;
    for (int e = 0; e < D; ++e) out->a[e] = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float f = parts[i].m == -INFINITY ? 0.0f : oo_expf(parts[i].m - M);
        L = fmaf(parts[i].l, f, L);
        for (int e = 0; e < D; ++e) out->a[e] = fmaf(parts[i].a[e], f, out->a[e]);
    }
    out->m = M;
    out->l = L;
}

/* dot of q and a K row as a lane group computes it: lane sl of `lanes` takes dims
 * per*sl .. per*sl + per - 1 in an fmaf chain, then the xor butterfly of the group */
static float fa_dot(const float *q, const float *kr, int lanes, int per) {
    float d[16];
    for (int sl = 0; sl < lanes; ++sl) {
        float s = 0.0f;
        for (int e = 0; e < per; ++e) s = fmaf(q[per * sl + e], kr[per * sl + e], s);
        d[sl] = s;
    }
    return butterfly_f(d, lanes);
}

/* rows of one (sequence, kv head): K/V rows [nkv][D] as f32 (converted from f16 exactly) */
typedef struct {
    const float *k, *v;  /* [nkv][D] */
    const float *mask;   /* [nkv] or NULL (one query row) */
    int64_t nkv;
} fa_rows;

/* fattn_split_kernel: one query row, positions [kv0, kv1) */
static void fa_split_part(const float *q, const fa_rows *r, int D, float scale, int64_t kv0, int64_t kv1,
                          fa_state *out, fa_state *scratch /* [16] */) {
    const int LPP = D / 8, PPW = 32 / LPP, U = 4;
    fa_state *grp = scratch;
    fa_state warps[4];
    for (int w = 0; w < 4; ++w) {
        for (int g = 0; g < PPW; ++g) fa_state_init(&grp[g], D);
        for (int64_t pb = kv0 + (int64_t)w * PPW; pb < kv1; pb += 4 * PPW * U)
            for (int u = 0; u < U; ++u)
                for (int g = 0; g < PPW; ++g) {
                    const int64_t p = pb + (int64_t)u * 4 * PPW + g;
                    if (p >= kv1) continue;
                    float sc = fa_dot(q, r->k + p * D, LPP, 8) * scale;
                    if (r->mask) {
                        const float mv = r->mask[p];
                        if (mv == -INFINITY) continue;
                        sc = sc + mv;
                    }
                    fa_state *s = &grp[g];
                    const float mnew = fmaxf(s->m, sc);
                    const float corr = oo_expf(s->m - mnew);
                    const float wgt = oo_expf(sc - mnew);
                    s->l = fmaf(s->l, corr, wgt);
                    const float *vr = r->v + p * D;
                    for (int e = 0; e < D; ++e) s->a[e] = fmaf(wgt, vr[e], s->a[e] * corr);
                    s->m = mnew;
                }
        /* position groups: level o = LPP, 2 LPP, ... pairs group g with g ^ (o / LPP) */
        for (int lvl = 1; lvl < PPW; lvl <<= 1) {
            fa_state nxt[4];
            for (int g = 0; g < PPW; ++g) {
                nxt[g] = grp[g];
                fa_combine(&nxt[g], &grp[g ^ lvl], D);
            }
            for (int g = 0; g < PPW; ++g) grp[g] = nxt[g];
        }
        warps[w] = grp[0];
    }
    fa_merge(warps, 4, D, out);
}

/* fattn_heads_kernel<8>: one (sequence, head), D 64, positions [kv0, kv1) */
static void fa_heads_part(const float *q, const fa_rows *r, float scale, int64_t kv0, int64_t kv1, fa_state *out) {
    const int D = 64, U = 8;
    fa_state warps[4];
    for (int w = 0; w < 4; ++w) {
        fa_state *s = &warps[w];
        fa_state_init(s, D);
        for (int64_t pb = kv0 + w; pb < kv1; pb += 4 * U) {
            float sc[8], wv[8];
            float mb = -INFINITY;
            for (int u = 0; u < U; ++u) {
                const int64_t p = pb + 4 * u;
                sc[u] = p < kv1 ? fa_dot(q, r->k + p * D, 8, 8) * scale : -INFINITY;
                mb = fmaxf(mb, sc[u]);
            }
            const float mnew = fmaxf(s->m, mb);
            for (int u = 0; u < U; ++u) wv[u] = oo_expf(sc[u] - mnew);
            const float corr = oo_expf(s->m - mnew);
            s->l = s->l * corr;
            for (int e = 0; e < D; ++e) s->a[e] = s->a[e] * corr;
            for (int u = 0; u < U; ++u) {
                const int64_t p = pb + 4 * u;
                s->l = s->l + wv[u];
                for (int e = 0; e < D; ++e) s->a[e] = fmaf(wv[u], p < kv1 ? r->v[p * D + e] : 0.0f, s->a[e]);
            }
            s->m = mnew;
        }
    }
    fa_merge(warps, 4, D, out);
}

/* fattn_gqa_kernel<G, 2>: one (sequence, kv head) and its G query heads, D 128,
 * positions [kv0, kv1); q = G rows of 128, out = G states */
static void fa_gqa_part(const float *q, int G, const fa_rows *r, float scale, int64_t kv0, int64_t kv1,
                        fa_state *out, fa_state *scratch /* [4 warps][4 groups][G] */) {
    const int D = 128, U = 2;
    for (int w = 0; w < 4; ++w)
        for (int grp = 0; grp < 4; ++grp) {
            fa_state *st = scratch + (w * 4 + grp) * G;
            for (int g = 0; g < G; ++g) fa_state_init(&st[g], D);
            for (int64_t pb = kv0 + 4 * w; pb < kv1; pb += 16 * U) {
                float sc[4][2];
                for (int u = 0; u < U; ++u) {
                    const int64_t p = pb + grp + 16 * u;
                    for (int g = 0; g < G; ++g)
                        sc[g][u] = p < kv1 ? fa_dot(q + g * D, r->k + p * D, 8, 16) * scale : -INFINITY;
                }
                for (int g = 0; g < G; ++g) {
                    float mb = sc[g][0];
                    for (int u = 1; u < U; ++u) mb = fmaxf(mb, sc[g][u]);
                    const float mnew = fmaxf(st[g].m, mb);
                    if (mnew == -INFINITY) continue;
                    const float corr = oo_expf(st[g].m - mnew);
                    st[g].l = st[g].l * corr;
                    for (int e = 0; e < D; ++e) st[g].a[e] = st[g].a[e] * corr;
                    st[g].m = mnew;
                }
                for (int u = 0; u < U; ++u) {
                    const int64_t p = pb + grp + 16 * u;
                    for (int g = 0; g < G; ++g) {
                        if (sc[g][u] == -INFINITY) continue;
                        const float wgt = oo_expf(sc[g][u] - st[g].m);
                        st[g].l = st[g].l + wgt;
                        for (int e = 0; e < D; ++e) st[g].a[e] = fmaf(wgt, r->v[p * D + e], st[g].a[e]);
                    }
                }
            }
        }
    for (int g = 0; g < G; ++g) {
        fa_state warps[4];
        for (int w = 0; w < 4; ++w) {
            fa_state grp4[4];
            for (int grp = 0; grp < 4; ++grp) grp4[grp] = scratch[(w * 4 + grp) * G + g];
            for (int lvl = 1; lvl < 4; lvl <<= 1) {
                fa_state nxt[4];
                for (int x = 0; x < 4; ++x) {
                    nxt[x] = grp4[x];
                    fa_combine(&nxt[x], &grp4[x ^ lvl], D);
                }
                for (int x = 0; x < 4; ++x) grp4[x] = nxt[x];
            }
            warps[w] = grp4[0];
        }
        fa_merge(warps, 4, D, &out[g]);
    }
}

static float elem_f(const char *p, int type) {
    return type == OO_TYPE_F32 ? *(const float *)p : oo_f16_to_f32(*(const uint16_t *)p);
}

int oo_fa_device(const oo_tensor *q, const oo_tensor *k, const oo_tensor *v, const oo_tensor *mask, float scale,
                 int kind, int64_t nkv_max, oo_tensor *dst) {
    pthread_once(&f16_once, f16_table_init);
    const int64_t D = q->ne[0], NQ = q->ne[1], H = q->ne[2], S = q->ne[3];
    const int64_t NKV = k->ne[1], HKV = k->ne[2];
    if (q->type != OO_TYPE_F32 || k->ne[0] != D || v->ne[0] != D || k->type != v->type) return OO_STATUS_FAILED;
    if (k->type != OO_TYPE_F16 && k->type != OO_TYPE_F32) return OO_STATUS_FAILED;
    if (v->ne[1] != NKV || v->ne[2] != HKV || k->ne[3] != S || v->ne[3] != S || HKV == 0 || H % HKV) return OO_STATUS_FAILED;
    if (nkv_max < NKV) return OO_STATUS_FAILED;
    if (dst->type != OO_TYPE_F32 || dst->ne[0] != D || dst->ne[1] != H || dst->ne[2] != NQ || dst->ne[3] != S)
        return OO_STATUS_FAILED;
    const int64_t G = H / HKV;
    if (kind == OO_FAK_HEADS && !(D == 64 && k->type == OO_TYPE_F16 && NQ == 1 && G == 1 && !mask && H % 4 == 0))
        return OO_STATUS_FAILED;
    if (kind == OO_FAK_GQA && !(D == 128 && k->type == OO_TYPE_F16 && NQ == 1 && !mask && (G == 1 || G == 2 || G == 4)))
        return OO_STATUS_FAILED;
    if (kind == OO_FAK_SPLIT && !(D == 64 || D == 128)) return OO_STATUS_FAILED;
    const int f16 = k->type == OO_TYPE_F16;
    const int64_t QG = G * NQ, QT = QG >= 8 ? 8 : QG >= 4 ? 4 : QG >= 2 ? 2 : 1;
    const int64_t groups = kind == OO_FAK_HEADS ? S * (H / 4) : kind == OO_FAK_GQA ? S * HKV : HKV * S * ((QG + QT - 1) / QT);
    const int ns = oo_fa_device_splits(kind, nkv_max, groups);
    const int64_t per = (NKV + ns - 1) / ns;
    int bad = 0;
#pragma omp parallel for schedule(dynamic, 1) collapse(2) reduction(| : bad)
    for (int64_t s = 0; s < S; ++s)
        for (int64_t hk = 0; hk < HKV; ++hk) {
            fa_rows r;
            float *kv = (float *)malloc((size_t)(2 * NKV * D + NKV + 4 * D) * sizeof(float));
            fa_state *st = (fa_state *)malloc(sizeof(fa_state) * (size_t)(16 * 4 + 2 * FA_SPLITS_MAX * 4 + 4));
            if (!kv || !st) { free(kv); free(st); bad = 1; continue; }
            float *kf = kv, *vf = kv + NKV * D, *mrow = kv + 2 * NKV * D, *qv = mrow + NKV;
            for (int64_t p = 0; p < NKV; ++p)
                for (int64_t d = 0; d < D; ++d) {
                    kf[p * D + d] = elem_f((const char *)k->data + d * k->nb[0] + p * k->nb[1] + hk * k->nb[2] + s * k->nb[3], k->type);
                    vf[p * D + d] = elem_f((const char *)v->data + d * v->nb[0] + p * v->nb[1] + hk * v->nb[2] + s * v->nb[3], v->type);
                }
            r.k = kf;
            r.v = vf;
            r.nkv = NKV;
            fa_state *parts = st + 64;       /* [splits][G] */
            fa_state *res = parts + FA_SPLITS_MAX * 4;
            for (int64_t g = 0; g < G; ++g)
                for (int64_t iq = 0; iq < NQ; ++iq) {
                    const int64_t h = hk * G + g;
                    if (kind == OO_FAK_GQA && iq > 0) break;
                    /* the query as the kernel holds it: rounded to f16 over f16 K/V */
                    const int64_t gq = kind == OO_FAK_GQA ? G : 1;
                    for (int64_t gg = 0; gg < gq; ++gg) {
                        const int64_t hh = kind == OO_FAK_GQA ? hk * G + gg : h;
                        for (int64_t d = 0; d < D; ++d) {
                            const float x = *(const float *)((const char *)q->data + d * q->nb[0] + iq * q->nb[1] + hh * q->nb[2] + s * q->nb[3]);
                            qv[gg * D + d] = f16 ? oo_f16_to_f32(oo_f32_to_f16(x)) : x;
                        }
                    }
                    if (kind == OO_FAK_GQA && g > 0) break;  /* all G heads at once */
                    r.mask = NULL;
                    if (mask) {
                        for (int64_t p = 0; p < NKV; ++p)
                            mrow[p] = oo_f16_to_f32(*(const uint16_t *)((const char *)mask->data + p * mask->nb[0] + iq * mask->nb[1] +
                                                                       (h % mask->ne[2]) * mask->nb[2] + (s % mask->ne[3]) * mask->nb[3]));
                        r.mask = mrow;
                    }
                    for (int sp = 0; sp < ns; ++sp) {
                        const int64_t kv0 = sp * per, kv1 = kv0 + per < NKV ? kv0 + per : NKV;
                        if (kind == OO_FAK_HEADS) fa_heads_part(qv, &r, scale, kv0, kv1, &parts[sp]);
                        else if (kind == OO_FAK_GQA) {
                            fa_state tmp[4];
                            fa_gqa_part(qv, (int)G, &r, scale, kv0, kv1, tmp, st);
                            for (int64_t gg = 0; gg < G; ++gg) parts[gg * FA_SPLITS_MAX + sp] = tmp[gg];
                        } else fa_split_part(qv, &r, (int)D, scale, kv0, kv1, &parts[sp], st);
                    }
                    const int64_t nout = kind == OO_FAK_GQA ? G : 1;
                    for (int64_t gg = 0; gg < nout; ++gg) {
                        const fa_state *pp = kind == OO_FAK_GQA ? parts + gg * FA_SPLITS_MAX : parts;
                        const fa_state *fin = pp;
                        if (ns > 1) {
                            fa_merge(pp, ns, (int)D, res);
                            fin = res;
                        }
                        const int64_t hh = kind == OO_FAK_GQA ? hk * G + gg : h;
                        float *out = (float *)((char *)dst->data + hh * dst->nb[1] + iq * dst->nb[2] + s * dst->nb[3]);
                        for (int64_t d = 0; d < D; ++d) out[d] = fin->l == 0.0f ? 0.0f : fin->a[d] / fin->l;
                    }
                }
            free(kv);
            free(st);
        }
    return bad ? OO_STATUS_ALLOC_FAILED : 0;
}
