// host_quant.cpp -- host-side ggml block encoders and the deterministic
// synthetic-data generator of the backend library (no device work).
//
// oasr_b200_quantize_chunk is the backend's answer to ggml_quantize_chunk
// (crates/openasr-core/src/ggml_runtime/ffi.rs:623), which the reference calls
// when it writes quantized packs (gguf_write.rs:522-599).  Q8_0 and Q4_0 follow
// ggml's reference quantizers (quantize_row_q8_0_ref / quantize_row_q4_0_ref:
// d = amax/127 with roundf; d = max/-8 with trunc(x/d + 8.5)).  Q4_K uses a
// simple min/max encoder per 32-element sub-block (a valid Q4_K encoding, not
// ggml's iterative search): every consumer decodes the same bytes.
//
// Compiled with -ffp-contract=off so each float operation rounds where written.

#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "../../include/oasr_b200.h"

namespace {

uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    const uint32_t mant = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    const int32_t e = (int32_t)exp - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        const uint32_t m = mant | 0x800000u;
        const int sh = 14 - e;
        uint32_t h = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, mant = h & 0x3ffu, x;
    if (exp == 0) {
        if (!mant) {
            x = sign;
        } else {
            int e = 0;
            while (!(mant & 0x400u)) { mant <<= 1; ++e; }
            x = sign | ((uint32_t)(113 - e) << 23) | ((mant & 0x3ffu) << 13);
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

int nearest_int(float v) {
    float t = v + 12582912.f;
    int32_t i;
    memcpy(&i, &t, 4);
    return (i & 0x007fffff) - 0x00400000;
}

void q8_0_row(const float *x, uint8_t *y, int64_t k) {
    for (int64_t b = 0; b < k / 32; ++b, y += 34) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, fabsf(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        memcpy(y, &dh, 2);
        for (int j = 0; j < 32; ++j) y[2 + j] = (uint8_t)(int8_t)roundf(xb[j] * id);
    }
}

void q4_0_row(const float *x, uint8_t *y, int64_t k) {
    for (int64_t b = 0; b < k / 32; ++b, y += 18) {
        const float *xb = x + b * 32;
        float amax = 0.0f, maxv = 0.0f;
        for (int j = 0; j < 32; ++j)
            if (amax < fabsf(xb[j])) { amax = fabsf(xb[j]); maxv = xb[j]; }
        const float d = maxv / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        memcpy(y, &dh, 2);
        for (int j = 0; j < 16; ++j) {
            int a = (int8_t)(xb[j] * id + 8.5f), c = (int8_t)(xb[16 + j] * id + 8.5f);
            a = std::min(a, 15);
            c = std::min(c, 15);
            y[2 + j] = (uint8_t)(a | (c << 4));
        }
    }
}

void q4_K_row(const float *x, uint8_t *y, int64_t k) {
    for (int64_t b = 0; b < k / 256; ++b, y += 144) {
        const float *xb = x + b * 256;
        float scale[8], mins[8], smax = 0.0f, mmax = 0.0f;
        for (int j = 0; j < 8; ++j) {
            float lo = xb[32 * j], hi = xb[32 * j];
            for (int l = 1; l < 32; ++l) {
                lo = std::min(lo, xb[32 * j + l]);
                hi = std::max(hi, xb[32 * j + l]);
            }
            lo = std::min(lo, 0.0f);
            scale[j] = (hi - lo) / 15.0f;
            mins[j] = -lo;
            smax = std::max(smax, scale[j]);
            mmax = std::max(mmax, mins[j]);
        }
        const uint16_t dh = f32_to_f16(smax / 63.0f), mh = f32_to_f16(mmax / 63.0f);
        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        int sc[8], mq[8];
        for (int j = 0; j < 8; ++j) {
            sc[j] = std::clamp(d > 0.0f ? nearest_int(scale[j] / d) : 0, 0, 63);
            mq[j] = std::clamp(dmin > 0.0f ? nearest_int(mins[j] / dmin) : 0, 0, 63);
        }
        memcpy(y, &dh, 2);
        memcpy(y + 2, &mh, 2);
        uint8_t *s = y + 4;
        for (int j = 0; j < 4; ++j) {
            s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            s[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
            s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
        }
        uint8_t q[256];
        for (int j = 0; j < 8; ++j) {
            const float dl = d * (float)sc[j], ml = dmin * (float)mq[j];
            for (int l = 0; l < 32; ++l)
                q[32 * j + l] = (uint8_t)std::clamp(dl > 0.0f ? nearest_int((xb[32 * j + l] + ml) / dl) : 0, 0, 15);
        }
        uint8_t *qs = y + 16;
        for (int c = 0; c < 4; ++c)
            for (int l = 0; l < 32; ++l) qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
}

template <class F>
void parallel_rows(int64_t n, F &&f) {
    unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    int64_t nt = std::min<int64_t>(hw, std::max<int64_t>(1, n / 64));
    if (nt <= 1) {
        f(0, n);
        return;
    }
    std::vector<std::thread> th;
    for (int64_t t = 0; t < nt; ++t) {
        int64_t a = n * t / nt, b = n * (t + 1) / nt;
        th.emplace_back([=, &f] { f(a, b); });
    }
    for (auto &t : th) t.join();
}

}  // namespace

extern "C" int64_t oasr_b200_row_size(int32_t type, int64_t ne0) {
    switch (type) {
    case OASR_TYPE_F32: case OASR_TYPE_I32: return ne0 * 4;
    case OASR_TYPE_I64: return ne0 * 8;
    case OASR_TYPE_F16: return ne0 * 2;
    case OASR_TYPE_Q8_0: return ne0 % 32 ? -1 : ne0 / 32 * 34;
    case OASR_TYPE_Q4_0: return ne0 % 32 ? -1 : ne0 / 32 * 18;
    case OASR_TYPE_Q4_K: return ne0 % 256 ? -1 : ne0 / 256 * 144;
    default: return -1;
    }
}

extern "C" int64_t oasr_b200_quantize_chunk(int32_t type, const float *src, void *dst, int64_t start_row,
                                            int64_t nrows, int64_t n_per_row) {
    const int64_t rs = oasr_b200_row_size(type, n_per_row);
    if (rs < 0 || !src || !dst || nrows < 0 || start_row < 0) return OASR_STATUS_FAILED;
    if (type != OASR_TYPE_Q8_0 && type != OASR_TYPE_Q4_0 && type != OASR_TYPE_Q4_K && type != OASR_TYPE_F16 &&
        type != OASR_TYPE_F32)
        return OASR_STATUS_FAILED;
    const float *x = src + start_row * n_per_row;
    uint8_t *y = (uint8_t *)dst + start_row * rs;
    parallel_rows(nrows, [&](int64_t a, int64_t b) {
        for (int64_t r = a; r < b; ++r) {
            const float *xr = x + r * n_per_row;
            uint8_t *yr = y + r * rs;
            switch (type) {
            case OASR_TYPE_Q8_0: q8_0_row(xr, yr, n_per_row); break;
            case OASR_TYPE_Q4_0: q4_0_row(xr, yr, n_per_row); break;
            case OASR_TYPE_Q4_K: q4_K_row(xr, yr, n_per_row); break;
            case OASR_TYPE_F16:
                for (int64_t i = 0; i < n_per_row; ++i) ((uint16_t *)yr)[i] = f32_to_f16(xr[i]);
                break;
            default: memcpy(yr, xr, (size_t)n_per_row * 4); break;
            }
        }
    });
    return nrows * rs;
}

extern "C" int oasr_b200_synth_normal(uint64_t seed, uint64_t offset, float *x, int64_t n, float mean, float std) {
    if (!x || n < 0) return OASR_STATUS_FAILED;
    const uint64_t G = 0x9E3779B97F4A7C15ULL;
    auto mix = [](uint64_t z) {
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        return z ^ (z >> 31);
    };
    parallel_rows(n / 4096 + 1, [&](int64_t a, int64_t b) {
        for (int64_t c = a; c < b; ++c)
            for (int64_t i = c * 4096; i < std::min<int64_t>(n, (c + 1) * 4096); ++i) {
                const uint64_t j = offset + (uint64_t)i, p = j >> 1;
                const uint64_t ua = mix(seed + (2 * p + 1) * G), ub = mix(seed + (2 * p + 2) * G);
                const double u1 = (double)((ua >> 11) + 1) * 0x1p-53, u2 = (double)(ub >> 11) * 0x1p-53;
                const double r = sqrt(-2.0 * log(u1));
                const double two_pi = 6.283185307179586476925286766559;
                const double z = (j & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
                x[i] = (float)((double)mean + (double)std * z);
            }
    });
    return OASR_STATUS_SUCCESS;
}
