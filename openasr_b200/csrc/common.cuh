// common.cuh -- shared definitions of the B200 backend (host + device).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <utility>

#include "../../include/oasr_b200.h"

namespace oasr {

constexpr int QK8_0 = 32;
constexpr int QK4_0 = 32;
constexpr int QK_K = 256;
constexpr int BYTES_Q8_0 = 34;
constexpr int BYTES_Q4_0 = 18;
constexpr int BYTES_Q4_K = 144;

// ggml block layouts (host side; gguf/constants.py GGML_QUANT_SIZES)
struct BlockQ8_0 { uint16_t d; int8_t qs[QK8_0]; };
struct BlockQ4_0 { uint16_t d; uint8_t qs[QK4_0 / 2]; };
struct BlockQ4_K { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[QK_K / 2]; };
static_assert(sizeof(BlockQ8_0) == BYTES_Q8_0, "q8_0");
static_assert(sizeof(BlockQ4_0) == BYTES_Q4_0, "q4_0");
static_assert(sizeof(BlockQ4_K) == BYTES_Q4_K, "q4_K");

// Device error word bits: a kernel that detects a bad input sets one and
// returns instead of touching memory out of bounds.
enum : int {
    ERR_NONE = 0,
    ERR_BAD_INDEX = 1,   // set_rows / get_rows index out of range
    ERR_BAD_SHAPE = 2,   // launch geometry inconsistent with the descriptors
    ERR_TIMEOUT = 4,     // a bounded wait (mbarrier, pipeline hand-off) gave up
};

}  // namespace oasr

// A resident weight: ggml [ne0=K, ne1=N, ne2, ne3] of `type`, repacked.
struct oasr_weight {
    int32_t type;
    int64_t ne[4];
    // Q8_0 / Q4_0: qs plane [slices][N][K or K/2] bytes + d plane [slices][N][K/32] fp16
    // Q4_K / F16 / F32: ggml bytes in `qs`, d unused
    uint8_t *qs;
    uint16_t *d;
    int64_t qs_row_bytes;    // bytes per row in the qs plane
    int64_t d_row_elems;     // fp16 scales per row in the d plane
    uint8_t *tiles;          // decode-tile copy for the tensor-core GEMV (Q4_K, Q8_0), or null
    float *dT;               // Q8_0 / Q4_0: block-major f32 scales [slices][K/32][N] for the tensor-core GEMM, or null
    int8_t *qs8;             // Q4_0: the quants expanded to int8 (q - 8) [slices][N][K] for that GEMM, or null
    __half *h16;             // Q4_K: sub-scale x quant as fp16 [slices][N][K] for the tensor-core GEMM, or null
    float *k_meta;           // Q4_K: per super-block d, dmin, mins of weight-row pairs for that GEMM, or null
    uint64_t device_bytes;
};

struct oasr_backend {
    int device;
    int sm_count;
    int cc_major, cc_minor;
    cudaStream_t own_stream;
    cudaStream_t stream;
    // activation scratch: quantized activations, flash-decode partials, counters
    uint8_t *scratch;
    size_t scratch_bytes;
    uint64_t scratch_epoch;   // bumped whenever the scratch is reallocated (captured graphs hold its address)
    unsigned int *counters;   // zero-initialised; kernels leave them at zero
    int *err_word;            // device error word (oasr::ERR_*)
    uint16_t *gelu_table;     // 65536-entry fp16 GELU table (ggml CPU semantics)
    std::atomic<int> poisoned;  // sticky ggml_status once a device error is seen
    oasr_abort_callback abort_cb;
    void *abort_data;
    uint64_t weight_bytes;
    int64_t n_weights;
    std::string last_error;
    bool pdl;  // launch with programmatic stream serialization (dependent kernels overlap)
    bool decode_tiles;  // build decode tiles at upload (OASR_B200_DECODE_GEMV=dp4a turns it off)
    // weight upload staging: two pinned host buffers, each reused once the copy that last
    // read it has completed (its event), allocated at the first upload
    void *stage[2];
    cudaEvent_t stage_done[2];
    // memory API v1 bookkeeping (memory_api.cu): a generation that every change of the
    // backend's allocations bumps, allocation counters, the owned-bytes high water, the
    // quarantine state, the last failure, and the last quote issued
    std::atomic<uint64_t> mem_generation;
    uint64_t mem_alloc_count, mem_alloc_failures, mem_high_water;
    uint64_t quarantine_generation;
    int quarantined;
    int last_status;
    int64_t last_native_error;
    uint64_t quote_token, quote_fingerprint, quote_generation;
};

// fixed device bytes every backend holds besides weights and scratch (split-KV tickets,
// error word, GELU table)
constexpr uint64_t kBackendFixedBytes = (uint64_t)(1 << 16) * 4 + 4 + 65536 * 2;
inline uint64_t oasr_internal_owned_device_bytes(const oasr_backend *be) {
    return be->weight_bytes + be->scratch_bytes + kBackendFixedBytes;
}
// record an allocation (ok) or a failed allocation, and bump the memory generation
void oasr_internal_mem_event(oasr_backend *be, bool ok);
// weight-upload staging: two pinned buffers of kUploadStageBytes (allocated on demand)
constexpr size_t kUploadStageBytes = 16ull << 20;
cudaError_t oasr_internal_stage_alloc(oasr_backend *be);
void oasr_internal_stage_release(oasr_backend *be);
// free the activation scratch after the stream drains (the next use reallocates it and
// bumps scratch_epoch, so captured step graphs are re-captured)
void oasr_internal_scratch_release(oasr_backend *be);

#define OASR_CUDA_TRY(be, expr)                                                          \
    do {                                                                                 \
        cudaError_t _e = (expr);                                                         \
        if (_e != cudaSuccess) return oasr_internal_cuda_fail((be), _e, #expr, __LINE__);\
    } while (0)

int oasr_internal_cuda_fail(oasr_backend *be, cudaError_t e, const char *what, int line);
int oasr_internal_fail(oasr_backend *be, int status, const std::string &msg);
int oasr_internal_precheck(oasr_backend *be);  // poison / abort check before enqueueing
int oasr_internal_launch_check(oasr_backend *be, const char *what);
void *oasr_internal_scratch(oasr_backend *be, size_t bytes, int *status);

// ---- programmatic dependent launch ----------------------------------------------------
// A kernel launched with PDL may start while its predecessor in the stream is
// still running: it must call griddep_wait() before reading anything the
// predecessor writes (and before writing anything the predecessor reads).
// Work that touches neither (e.g. streaming constant weights into registers)
// can precede the wait.  Both instructions are no-ops for a normal launch.
static __device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
static __device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Hint: start streaming [p, p + bytes) from HBM into L2 (p 16-byte aligned, bytes a
// multiple of 16).  Nothing waits on it; a kernel issues it for data that does not
// depend on its predecessor (weights) before griddep_wait(), so under programmatic
// dependent launch the stream overlaps the predecessor's tail.
static __device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_k(oasr_backend *be, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = be->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = be->pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- last-CTA ticket ------------------------------------------------------------------
// "The last CTA to finish does the rest": call with every thread of the CTA after its
// global stores.  bar.sync orders those stores before thread 0's release-acquire
// atomic (release is cumulative over the barrier), so the CTA that draws ticket
// total-1 sees every other CTA's stores; it resets the ticket, so each launch leaves
// it at zero.  Read other CTAs' data with L2 loads (ld.cg / __ldcg).
static __device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int *p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

static __device__ __forceinline__ bool cta_last_arrival(unsigned int *ticket, unsigned int total) {
    __shared__ unsigned int s_last_flag;
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool last = atom_add_acq_rel_gpu(ticket, 1u) == total - 1;
        if (last) atomicExch(ticket, 0u);  // every other CTA has drawn its ticket
        s_last_flag = last;
    }
    __syncthreads();
    return s_last_flag != 0;
}

// ---- device helpers --------------------------------------------------------------
// cp.async (global -> shared, completion by group): 16 bytes (both addresses 16-byte
// aligned) or 4 bytes
static __device__ __forceinline__ void cp_async16(void *smem_dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(src)
                 : "memory");
}
static __device__ __forceinline__ void cp_async4(void *smem_dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(src)
                 : "memory");
}
static __device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
static __device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
static __device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

static __device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

static __device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

static __device__ __forceinline__ int4 ldg_stream(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

static __device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
