// selftest.cu -- exercises the failure path of the bounded pipeline waits.
//
// Every tcgen05 / TMA kernel of this library waits on mbarriers with a bound
// (tc_common.cuh mbar_wait): when a producer never arrives, the waiting role gives
// up, records ERR_TIMEOUT in the backend's device error word and unwinds, so the
// context stays usable and oasr_b200_synchronize reports EXECUTION_FAILED instead of
// the GPU hanging.  This entry point runs that path on purpose: one CTA initialises
// an mbarrier that expects one arrival, never arrives, and waits with a short bound.
// No fault, no trap and no unbounded loop is involved.
#include "tc_common.cuh"

namespace oasr {

__global__ void bounded_wait_selftest_kernel(int *err, long long limit) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, limit);  // nobody arrives
    __syncthreads();
}

}  // namespace oasr

extern "C" int oasr_b200_selftest_bounded_wait(oasr_backend *be, int64_t limit_cycles) {
    const int st = oasr_internal_precheck(be);
    if (st) return st;
    if (limit_cycles < 1 || limit_cycles > oasr::kMbarWaitLimit)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "selftest_bounded_wait: limit out of range");
    oasr::bounded_wait_selftest_kernel<<<1, 32, 0, be->stream>>>(be->err_word, (long long)limit_cycles);
    const int lst = oasr_internal_launch_check(be, "bounded_wait_selftest");
    if (lst) return lst;
    return oasr_b200_synchronize(be);
}
