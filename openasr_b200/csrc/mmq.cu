// mmq.cu -- K2 entry: quantized GEMM for M > 8 activation rows (encoder,
// prefill).  This first revision tiles the M rows into groups of 8 and runs
// the K1 GEMV kernel per group (same exact per-block arithmetic, weights
// re-read per group from L2).
#include "kernels.cuh"

namespace oasr {

int launch_mmq(oasr_backend *be, const oasr_weight *w, int64_t slice, const ActPlanes &a, int64_t M, int K,
               float *y, int64_t y_ld) {
    const bool k_family = w->type == OASR_TYPE_Q4_K;
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        const int mc = (int)std::min<int64_t>(8, M - m0);
        ActPlanes s;
        s.qs = a.qs + m0 * K;
        s.d = a.d + m0 * (K / (k_family ? 256 : 32));
        s.bs16 = k_family ? a.bs16 + m0 * (K / 16) : nullptr;
        int st = launch_mmv_quant(be, w, slice, s, mc, K, y + m0 * y_ld, y_ld);
        if (st) return st;
    }
    return OASR_STATUS_SUCCESS;
}

}  // namespace oasr
