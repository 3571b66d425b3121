// quant_act.cu -- on-device activation quantization to ggml's vec_dot types.
//
// ggml's CPU mul_mat converts every activation row to the weight type's
// vec_dot type before the integer block dot: Q8_0/Q4_0 weights -> q8_0 (per 32:
// d = amax/127, q = roundf(x/d), d stored as fp16), Q4_K weights -> q8_K (per
// 256: iscale = -127/max, q = min(127, rint(iscale*x)), d = 1/iscale, 16-wide
// partial sums).  These kernels reproduce that rounding exactly (IEEE division
// and reciprocal, roundf / rint) and write planar scratch:
//   q8_0: qs[R][K] int8 | d[R][K/32] f32 (the fp16-rounded scale)
//   q8_K: qs[R][K] int8 | d[R][K/256] f32 | bs16[R][K/16] int16
// Reference call sites: mul_mat_impl (cpu_graph.rs:3651-3686) feeding
// ggml_mul_mat (ffi.rs:694).
#include "kernels.cuh"

namespace oasr {

// x rows: element (k, r) at x + row_offset(r) + k*esize, r = m + M*(i2 + ne2*i3)
struct ActRows {
    const char *base;
    int64_t nb1, nb2, nb3;
    int M, ne2;
    __device__ __forceinline__ const char *row(int64_t r) const {
        const int64_t m = r % M, t = r / M;
        return base + m * nb1 + (t % ne2) * nb2 + (t / ne2) * nb3;
    }
};

template <bool F16>
__device__ __forceinline__ float load_act(const char *row, int k) {
    if (F16) return __half2float(reinterpret_cast<const __half *>(row)[k]);
    return reinterpret_cast<const float *>(row)[k];
}

// 8 threads per 32-element block, 4 elements each.
template <bool F16>
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(ActRows xr, int K, int64_t R, int8_t *__restrict__ qs,
                                                            float *__restrict__ dsc) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t groups_per_row = K / 4;
    const int64_t total = R * groups_per_row;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = g / groups_per_row;
        const int k0 = (int)(g - r * groups_per_row) * 4;
        const char *row = xr.row(r);
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = load_act<F16>(row, k0 + i);
        // the 8 lanes of one block are always active together (K % 32 == 0)
        const unsigned gmask = 0xFFu << (threadIdx.x & 24);
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, 4));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
        uint32_t packed = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int q = (int)roundf(__fmul_rn(v[i], id));
            packed |= (uint32_t)(uint8_t)(int8_t)q << (8 * i);
        }
        *reinterpret_cast<uint32_t *>(qs + r * K + k0) = packed;
        if ((k0 & 31) == 0) dsc[r * (K / 32) + k0 / 32] = __half2float(__float2half_rn(d));
    }
}

// one warp per 256-element super-block, 8 elements per lane
template <bool F16>
__global__ void __launch_bounds__(256) quantize_q8_K_kernel(ActRows xr, int K, int64_t R, int8_t *__restrict__ qs,
                                                            float *__restrict__ dsc, int16_t *__restrict__ bs16,
                                                            __half *__restrict__ qs16, __half *__restrict__ bs16h) {
    griddep_launch_dependents();
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nsb = K / 256;
    const int64_t total = R * nsb;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t s = warp0; s < total; s += nwarps) {
        const int64_t r = s / nsb;
        const int sb = (int)(s - r * nsb);
        const char *row = xr.row(r);
        const int k0 = sb * 256 + lane * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = load_act<F16>(row, k0 + i);
        // first (lowest index) element of largest |x|
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
        int8_t q[8];
        float d;
        if (amax == 0.0f) {
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = 0;
            d = 0.0f;
        } else {
            const float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = (int8_t)min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
            d = __frcp_rn(iscale);
        }
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += q[i];
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        uint2 pk;
        pk.x = (uint32_t)(uint8_t)q[0] | (uint32_t)(uint8_t)q[1] << 8 | (uint32_t)(uint8_t)q[2] << 16 |
               (uint32_t)(uint8_t)q[3] << 24;
        pk.y = (uint32_t)(uint8_t)q[4] | (uint32_t)(uint8_t)q[5] << 8 | (uint32_t)(uint8_t)q[6] << 16 |
               (uint32_t)(uint8_t)q[7] << 24;
        *reinterpret_cast<uint2 *>(qs + r * K + k0) = pk;
        if ((lane & 1) == 0) bs16[r * (K / 16) + k0 / 16] = (int16_t)sum;
        if (lane == 0) dsc[r * nsb + sb] = d;
        if (qs16) {
            // exact fp16 copies (|q| <= 127, |16-sum| <= 2032) for the tensor-core GEMM
            __half2 h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __halves2half2(__int2half_rn(q[2 * i]), __int2half_rn(q[2 * i + 1]));
            *reinterpret_cast<int4 *>(qs16 + r * K + k0) = *reinterpret_cast<int4 *>(h);
            if ((lane & 1) == 0) bs16h[r * (K / 16) + k0 / 16] = __int2half_rn(sum);
        }
    }
}

int launch_quantize_act(oasr_backend *be, const oasr_tensor *x, int family, const ActPlanes &p) {
    ActRows xr{(const char *)x->data, x->nb[1], x->nb[2], x->nb[3], (int)x->ne[1], (int)x->ne[2]};
    const int K = (int)x->ne[0];
    const int64_t R = x->ne[1] * x->ne[2] * x->ne[3];
    const bool f16 = x->type == OASR_TYPE_F16;
    const int threads = 256;
    if (family == FAMILY_Q8_0) {
        const int64_t work = R * (K / 4);
        const int blocks = (int)std::min<int64_t>((work + threads - 1) / threads, (int64_t)be->sm_count * 16);
        const cudaError_t e = f16 ? launch_k(be, quantize_q8_0_kernel<true>, dim3(blocks), dim3(threads), 0, xr, K, R, p.qs, p.d)
                                  : launch_k(be, quantize_q8_0_kernel<false>, dim3(blocks), dim3(threads), 0, xr, K, R, p.qs, p.d);
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "quantize_q8_0 launch", __LINE__);
    } else {
        const int64_t work = R * (K / 256) * 32;
        const int blocks = (int)std::min<int64_t>((work + threads - 1) / threads, (int64_t)be->sm_count * 16);
        const cudaError_t e =
            f16 ? launch_k(be, quantize_q8_K_kernel<true>, dim3(blocks), dim3(threads), 0, xr, K, R, p.qs, p.d, p.bs16, p.qs16, p.bs16h)
                : launch_k(be, quantize_q8_K_kernel<false>, dim3(blocks), dim3(threads), 0, xr, K, R, p.qs, p.d, p.bs16, p.qs16, p.bs16h);
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "quantize_q8_K launch", __LINE__);
    }
    return oasr_internal_launch_check(be, "quantize_act");
}

}  // namespace oasr
