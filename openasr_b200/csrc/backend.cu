// backend.cu -- device/backend lifecycle, status and poisoning, activation
// scratch, resident weight upload (raw quantized blocks, repacked without
// dequantizing) and supports_op.  Mirrors the ggml backend device interface
// the reference binds in crates/openasr-core/src/ggml_runtime/ffi.rs:566-598
// and its status contract (ffi.rs:102-117, cpu_graph.rs:7893-7935, :8380-8405).

#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cstdlib>
#include <thread>
#include <vector>

#include "kernels.cuh"

using namespace oasr;

namespace {
constexpr size_t kCounterSlots = 1 << 16;  // flash-decode split counters
static_assert(kBackendFixedBytes == kCounterSlots * 4 + 4 + 65536 * 2, "fixed backend bytes");
constexpr size_t kDefaultScratch = 64ull << 20;

uint16_t host_f32_to_f16(float f) { return __half_as_ushort(__float2half_rn(f)); }
float host_f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ggml CPU evaluates GELU through a 65536-entry fp16 table:
// table[h] = fp16(0.5 x (1 + tanh(sqrt(2/pi) x (1 + 0.044715 x^2)))), x = fp32(h).
void build_gelu_table(std::vector<uint16_t> &t) {
    t.resize(65536);
    const float A = 0.044715f, S = 0.79788456080286535587989211986876f;
    for (uint32_t i = 0; i < 65536; ++i) {
        const float x = host_f16_to_f32((uint16_t)i);
        const float inner = S * x * (1.0f + A * x * x);
        t[i] = host_f32_to_f16(0.5f * x * (1.0f + tanhf(inner)));
    }
}
// ---- weight upload: raw blocks through pinned staging, planes split on the device --------
constexpr size_t kStageBytes = kUploadStageBytes;

// host copy into a staging buffer, spread over up to 8 threads for large chunks (a single
// core's memcpy is slower than the host-to-device link)
void par_memcpy(void *dst, const void *src, size_t n) {
    const int nt = n >= (4u << 20) ? 8 : n >= (1u << 20) ? 2 : 1;
    if (nt == 1) {
        memcpy(dst, src, n);
        return;
    }
    const size_t per = (n / nt + 63) & ~(size_t)63;
    std::vector<std::thread> th;
    for (int t = 1; t < nt; ++t) {
        const size_t o = std::min(n, per * t), e = std::min(n, o + per);
        if (e > o) th.emplace_back([=] { memcpy((char *)dst + o, (const char *)src + o, e - o); });
    }
    memcpy(dst, src, std::min(n, per));
    for (auto &x : th) x.join();
}

}  // namespace

cudaError_t oasr_internal_stage_alloc(oasr_backend *be) {
    for (int i = 0; i < 2; ++i) {
        if (be->stage[i]) continue;
        cudaError_t e = cudaHostAlloc(&be->stage[i], kStageBytes, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&be->stage_done[i], cudaEventDisableTiming);
        oasr_internal_mem_event(be, e == cudaSuccess);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

void oasr_internal_stage_release(oasr_backend *be) {
    for (int i = 0; i < 2; ++i) {
        if (be->stage_done[i]) cudaEventSynchronize(be->stage_done[i]);
        if (be->stage[i]) cudaFreeHost(be->stage[i]);
        if (be->stage_done[i]) cudaEventDestroy(be->stage_done[i]);
        be->stage[i] = nullptr;
        be->stage_done[i] = nullptr;
    }
    be->mem_generation.fetch_add(1);
}

void oasr_internal_scratch_release(oasr_backend *be) {
    cudaStreamSynchronize(be->stream);
    if (be->scratch) cudaFree(be->scratch);
    be->scratch = nullptr;
    be->scratch_bytes = 0;
    ++be->scratch_epoch;
    be->mem_generation.fetch_add(1);
}

namespace {

// bytes at `src` (any host memory) -> device `dst`: chunk i is copied into staging buffer
// i % 2 while the asynchronous copy of chunk i - 1 runs
cudaError_t upload_staged(oasr_backend *be, void *dst, const void *src, size_t bytes) {
    cudaError_t e = oasr_internal_stage_alloc(be);
    for (size_t off = 0, i = 0; e == cudaSuccess && off < bytes; ++i) {
        const size_t n = std::min(kStageBytes, bytes - off);
        const int b = (int)(i & 1);
        e = cudaEventSynchronize(be->stage_done[b]);
        if (e != cudaSuccess) break;
        par_memcpy(be->stage[b], (const char *)src + off, n);
        e = cudaMemcpyAsync((char *)dst + off, be->stage[b], n, cudaMemcpyHostToDevice, be->stream);
        if (e == cudaSuccess) e = cudaEventRecord(be->stage_done[b], be->stream);
        off += n;
    }
    return e;
}

// raw Q8_0 / Q4_0 blocks [rows][nb][bb] -> quant plane [rows][nb * qb] + fp16 scale plane
// [rows][nb] (one thread per block; the scale is the block's first two bytes)
__global__ void split_blocks_kernel(const uint8_t *raw, int64_t nblocks, int64_t nb, int bb, int64_t qs_row, uint8_t *qs,
                                    uint16_t *d) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nblocks; i += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t *blk = raw + i * bb;
        const int64_t r = i / nb, b = i - r * nb;
        d[i] = (uint16_t)(blk[0] | (blk[1] << 8));
        const int qb = bb - 2;
        uint8_t *q = qs + r * qs_row + b * qb;
        for (int j = 0; j < qb; ++j) q[j] = blk[2 + j];
    }
}
}  // namespace

void oasr_internal_mem_event(oasr_backend *be, bool ok) {
    if (ok) ++be->mem_alloc_count;
    else ++be->mem_alloc_failures;
    be->mem_generation.fetch_add(1);
    be->mem_high_water = std::max(be->mem_high_water, oasr_internal_owned_device_bytes(be));
}

int oasr_internal_fail(oasr_backend *be, int status, const std::string &msg) {
    if (be) {
        be->last_error = msg;
        if (status != OASR_STATUS_SUCCESS) be->last_status = status;
    }
    return status;
}

int oasr_internal_cuda_fail(oasr_backend *be, cudaError_t e, const char *what, int line) {
    char buf[512];
    snprintf(buf, sizeof buf, "%s failed at backend.cu:%d: %s", what, line, cudaGetErrorString(e));
    int st = e == cudaErrorMemoryAllocation ? OASR_STATUS_ALLOC_FAILED : OASR_STATUS_EXECUTION_FAILED;
    if (be) be->last_native_error = (int64_t)e;
    if (e == cudaErrorIllegalAddress || e == cudaErrorLaunchFailure || e == cudaErrorIllegalInstruction ||
        e == cudaErrorMisalignedAddress || e == cudaErrorHardwareStackError || e == cudaErrorECCUncorrectable ||
        e == cudaErrorNoDevice || e == cudaErrorDevicesUnavailable)
        st = OASR_STATUS_DEVICE_LOST;
    if (be && st != OASR_STATUS_ALLOC_FAILED) {
        int expected = 0;
        be->poisoned.compare_exchange_strong(expected, st == OASR_STATUS_DEVICE_LOST ? OASR_STATUS_DEVICE_LOST
                                                                                     : OASR_STATUS_BACKEND_POISONED);
    }
    return oasr_internal_fail(be, st, buf);
}

int oasr_internal_precheck(oasr_backend *be) {
    if (!be) return OASR_STATUS_FAILED;
    int p = be->poisoned.load();
    if (p) return OASR_STATUS_BACKEND_POISONED;
    if (be->abort_cb && be->abort_cb(be->abort_data)) return OASR_STATUS_ABORTED;
    if (cudaSetDevice(be->device) != cudaSuccess) return OASR_STATUS_DEVICE_LOST;
    return OASR_STATUS_SUCCESS;
}

int oasr_internal_launch_check(oasr_backend *be, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, what, __LINE__);
    return OASR_STATUS_SUCCESS;
}

// Returns scratch of at least `bytes` (grows by reallocation outside any
// capture; the stream is synchronised first because in-flight kernels may
// still read the old buffer).
void *oasr_internal_scratch(oasr_backend *be, size_t bytes, int *status) {
    *status = OASR_STATUS_SUCCESS;
    if (bytes <= be->scratch_bytes) return be->scratch;
    size_t nb = std::max(bytes + (bytes >> 2), be->scratch_bytes * 2);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(be->stream, &cs);
    if (cs != cudaStreamCaptureStatusNone) {
        *status = oasr_internal_fail(be, OASR_STATUS_ALLOC_FAILED,
                                     "activation scratch too small during stream capture; call oasr_b200_reserve_scratch first");
        return nullptr;
    }
    cudaError_t e = cudaStreamSynchronize(be->stream);
    if (e != cudaSuccess) {
        *status = oasr_internal_cuda_fail(be, e, "cudaStreamSynchronize(scratch grow)", __LINE__);
        return nullptr;
    }
    if (be->scratch) cudaFree(be->scratch);
    be->scratch = nullptr;
    be->scratch_bytes = 0;
    e = cudaMalloc(&be->scratch, nb);
    if (e != cudaSuccess) {
        oasr_internal_mem_event(be, false);
        *status = oasr_internal_cuda_fail(be, e, "cudaMalloc(scratch)", __LINE__);
        return nullptr;
    }
    be->scratch_bytes = nb;
    ++be->scratch_epoch;
    oasr_internal_mem_event(be, true);
    return be->scratch;
}

extern "C" {

int oasr_b200_device_count(int32_t *count) {
    if (!count) return OASR_STATUS_FAILED;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) n = 0;
    *count = n;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_init(int32_t ordinal, oasr_backend **out) {
    if (!out) return OASR_STATUS_FAILED;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || ordinal < 0 || ordinal >= n) return OASR_STATUS_FAILED;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, ordinal) != cudaSuccess) return OASR_STATUS_DEVICE_LOST;
    if (prop.major != 10) return OASR_STATUS_FAILED;  // kernels are built for sm_100a only
    oasr_backend *be = new oasr_backend();
    be->device = ordinal;
    be->sm_count = prop.multiProcessorCount;
    be->cc_major = prop.major;
    be->cc_minor = prop.minor;
    be->poisoned = 0;
    be->abort_cb = nullptr;
    be->abort_data = nullptr;
    be->weight_bytes = 0;
    be->n_weights = 0;
    be->scratch = nullptr;
    be->scratch_bytes = 0;
    be->pdl = false;
    {
        // decode GEMV path: tensor-core tiles by default, the dp4a kernel on request
        const char *env = getenv("OASR_B200_DECODE_GEMV");
        be->decode_tiles = !(env && strcmp(env, "dp4a") == 0);
    }
    int st = OASR_STATUS_SUCCESS;
    std::vector<uint16_t> gelu;
    build_gelu_table(gelu);
    cudaSetDevice(ordinal);
    if (cudaStreamCreateWithFlags(&be->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&be->counters, kCounterSlots * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&be->err_word, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&be->gelu_table, 65536 * sizeof(uint16_t)) != cudaSuccess ||
        cudaMemset(be->counters, 0, kCounterSlots * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(be->err_word, 0, sizeof(int)) != cudaSuccess ||
        cudaMemcpy(be->gelu_table, gelu.data(), 65536 * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
        delete be;
        return OASR_STATUS_ALLOC_FAILED;
    }
    be->stream = be->own_stream;
    oasr_internal_scratch(be, kDefaultScratch, &st);
    if (st != OASR_STATUS_SUCCESS) {
        oasr_b200_free(be);
        return st;
    }
    *out = be;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_free(oasr_backend *be) {
    if (!be) return OASR_STATUS_SUCCESS;
    cudaSetDevice(be->device);
    cudaStreamSynchronize(be->stream);
    if (be->scratch) cudaFree(be->scratch);
    if (be->counters) cudaFree(be->counters);
    if (be->err_word) cudaFree(be->err_word);
    if (be->gelu_table) cudaFree(be->gelu_table);
    for (int i = 0; i < 2; ++i) {
        if (be->stage[i]) cudaFreeHost(be->stage[i]);
        if (be->stage_done[i]) cudaEventDestroy(be->stage_done[i]);
    }
    if (be->own_stream) cudaStreamDestroy(be->own_stream);
    delete be;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_props(oasr_backend *be, oasr_device_props *out) {
    if (!be || !out) return OASR_STATUS_FAILED;
    memset(out, 0, sizeof *out);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, be->device) != cudaSuccess) return OASR_STATUS_DEVICE_LOST;
    snprintf(out->name, sizeof out->name, "CUDA%d", be->device);
    snprintf(out->description, sizeof out->description, "%s (sm_%d%d, oasr_b200 abi %d)", prop.name, prop.major,
             prop.minor, OASR_B200_ABI_VERSION);
    out->ordinal = be->device;
    out->device_type = 1;
    out->sm_count = prop.multiProcessorCount;
    out->cc_major = prop.major;
    out->cc_minor = prop.minor;
    out->cancel_mechanism = OASR_CANCEL_NATIVE;
    out->cancel_observation = OASR_CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT;
    size_t fr = 0, tot = 0;
    cudaSetDevice(be->device);
    cudaMemGetInfo(&fr, &tot);
    out->memory_free = fr;
    out->memory_total = tot;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_set_stream(oasr_backend *be, void *stream) {
    if (!be) return OASR_STATUS_FAILED;
    be->stream = (cudaStream_t)stream;  // NULL is CUDA's legacy default stream
    return OASR_STATUS_SUCCESS;
}

void *oasr_b200_get_stream(oasr_backend *be) { return be ? (void *)be->stream : nullptr; }

int oasr_b200_synchronize(oasr_backend *be) {
    if (!be) return OASR_STATUS_FAILED;
    int p = be->poisoned.load();
    if (p) return OASR_STATUS_BACKEND_POISONED;
    cudaSetDevice(be->device);
    cudaError_t e = cudaStreamSynchronize(be->stream);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "cudaStreamSynchronize", __LINE__);
    int err = 0;
    e = cudaMemcpy(&err, be->err_word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "read error word", __LINE__);
    if (err) {
        cudaMemset(be->err_word, 0, sizeof(int));
        return oasr_internal_fail(be, OASR_STATUS_EXECUTION_FAILED,
                                  err & ERR_BAD_INDEX   ? "kernel rejected an out-of-range row index"
                                  : err & ERR_BAD_SHAPE ? "kernel rejected inconsistent launch geometry"
                                                        : "a kernel's bounded wait on its pipeline timed out");
    }
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_synchronize_ex(oasr_backend *be, oasr_cancel_capability *cap) {
    if (cap) {
        cap->mechanism = be ? OASR_CANCEL_NATIVE : OASR_CANCEL_DISABLED;
        cap->observation_granularity = be ? OASR_CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT : OASR_CANCEL_OBSERVATION_NONE;
    }
    return oasr_b200_synchronize(be);
}

int oasr_b200_set_abort_callback(oasr_backend *be, oasr_abort_callback cb, void *data) {
    if (!be) return OASR_STATUS_FAILED;
    be->abort_cb = cb;
    be->abort_data = data;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_mem_stats(oasr_backend *be, oasr_mem_stats *out) {
    if (!be || !out) return OASR_STATUS_FAILED;
    memset(out, 0, sizeof *out);
    out->weight_bytes = be->weight_bytes;
    out->scratch_bytes = be->scratch_bytes;
    out->n_weights = be->n_weights;
    size_t fr = 0, tot = 0;
    cudaSetDevice(be->device);
    cudaMemGetInfo(&fr, &tot);
    out->device_free = fr;
    out->device_total = tot;
    return OASR_STATUS_SUCCESS;
}

const char *oasr_b200_last_error(oasr_backend *be) { return be ? be->last_error.c_str() : "null backend"; }

int oasr_b200_reserve_scratch(oasr_backend *be, size_t bytes) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    oasr_internal_scratch(be, bytes, &st);
    return st;
}

// ---- resident weights ----------------------------------------------------------------
int oasr_b200_weight_upload(oasr_backend *be, const void *host, size_t bytes, int32_t type, const int64_t ne[4],
                            oasr_weight **out) {
    if (!out) return OASR_STATUS_FAILED;
    *out = nullptr;
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!host || !ne) return oasr_internal_fail(be, OASR_STATUS_FAILED, "weight_upload: null argument");
    if (type != OASR_TYPE_Q8_0 && type != OASR_TYPE_Q4_0 && type != OASR_TYPE_Q4_K && type != OASR_TYPE_F16 &&
        type != OASR_TYPE_F32)
        return oasr_internal_fail(be, OASR_STATUS_FAILED, "weight_upload: unsupported type");
    for (int i = 0; i < 4; ++i)
        if (ne[i] <= 0) return oasr_internal_fail(be, OASR_STATUS_FAILED, "weight_upload: bad shape");
    const int64_t rs = oasr_b200_row_size(type, ne[0]);
    if (rs < 0) return oasr_internal_fail(be, OASR_STATUS_FAILED, "weight_upload: ne0 not a multiple of the block");
    const int64_t rows = ne[1] * ne[2] * ne[3];
    if ((size_t)(rs * rows) != bytes) return oasr_internal_fail(be, OASR_STATUS_FAILED, "weight_upload: byte count");
    oasr_weight *w = new oasr_weight();
    w->type = type;
    for (int i = 0; i < 4; ++i) w->ne[i] = ne[i];
    w->qs = nullptr;
    w->d = nullptr;
    // the pack's raw blocks cross to the device once, through the pinned staging ring
    // (bulk host-to-device copies); Q8_0 / Q4_0 blocks are split into planes there
    cudaError_t e;
    if (type == OASR_TYPE_Q8_0 || type == OASR_TYPE_Q4_0) {
        const int bb = type == OASR_TYPE_Q8_0 ? BYTES_Q8_0 : BYTES_Q4_0;
        const int qb = bb - 2;  // quant bytes per block (32 or 16)
        const int64_t nb = ne[0] / 32;
        w->qs_row_bytes = nb * qb;
        w->d_row_elems = nb;
        const size_t qs_bytes = (size_t)(rows * w->qs_row_bytes), d_bytes = (size_t)(rows * nb) * 2;
        w->device_bytes = qs_bytes + d_bytes;
        void *raw = nullptr;
        e = cudaMalloc(&w->qs, qs_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&w->d, d_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&raw, bytes);
        if (e == cudaSuccess) e = upload_staged(be, raw, host, bytes);
        if (e == cudaSuccess) {
            const int64_t nblocks = rows * nb;
            const unsigned grid = (unsigned)std::min<int64_t>((nblocks + 255) / 256, (int64_t)be->sm_count * 16);
            split_blocks_kernel<<<grid, 256, 0, be->stream>>>((const uint8_t *)raw, nblocks, nb, bb, w->qs_row_bytes,
                                                              (uint8_t *)w->qs, (uint16_t *)w->d);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
        if (raw) cudaFree(raw);
    } else {
        w->qs_row_bytes = rs;
        w->d_row_elems = 0;
        w->device_bytes = bytes;
        e = cudaMalloc(&w->qs, bytes);
        if (e == cudaSuccess) e = upload_staged(be, w->qs, host, bytes);
        if (e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
    }
    w->tiles = nullptr;
    w->dT = nullptr;
    w->qs8 = nullptr;
    w->h16 = nullptr;
    w->k_meta = nullptr;
    if (e == cudaSuccess && mmq_q80_tc_supported(type, ne[1], ne[0])) {
        // the tensor-core GEMM's operands: block-major f32 scales, and for Q4_0 the quants
        // expanded to int8 (the GEMM then runs as Q8_0 on them, bit for bit the Q4_0 dot)
        const size_t db = (size_t)(ne[2] * ne[3] * (ne[0] / 32) * ne[1]) * sizeof(float);
        const size_t qb = type == OASR_TYPE_Q4_0 ? (size_t)(rows * ne[0]) : 0;
        e = cudaMalloc(&w->dT, db);
        if (e == cudaSuccess) e = build_q80_scales_t(w, be->stream);
        if (e == cudaSuccess && qb) e = cudaMalloc(&w->qs8, qb);
        if (e == cudaSuccess && qb) e = build_q40_expanded(w, be->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
        if (e == cudaSuccess) w->device_bytes += db + qb;
    }
    if (e == cudaSuccess && mmq_q4k_tc_supported(type, ne[0])) {
        // the tensor-core GEMM's operands: fp16 sub-scale x quant rows and per super-block
        // metadata, built once on the device from the raw blocks
        size_t mb = 0;
        const size_t hb = q4k_operand_bytes(ne[1], ne[0], ne[2] * ne[3], &mb);
        e = cudaMalloc(&w->h16, hb);
        if (e == cudaSuccess) e = cudaMalloc(&w->k_meta, mb);
        if (e == cudaSuccess) e = build_q4k_operand(w, be->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
        if (e == cudaSuccess) w->device_bytes += hb + mb;
    }
    if (e == cudaSuccess && be->decode_tiles && mmv_tiles_supported(type, ne[0])) {
        // decode-tile copy for the tensor-core GEMV, built on the device from the planes above
        const size_t tb = mmv_tiles_bytes(type, ne[1], ne[0], ne[2] * ne[3]);
        e = cudaMalloc(&w->tiles, tb);
        if (e == cudaSuccess) e = build_mmv_tiles(w, be->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
        if (e == cudaSuccess) w->device_bytes += tb;
    }
    if (e != cudaSuccess) {
        if (w->qs) cudaFree(w->qs);
        if (w->d) cudaFree(w->d);
        if (w->tiles) cudaFree(w->tiles);
        if (w->dT) cudaFree(w->dT);
        if (w->qs8) cudaFree(w->qs8);
        if (w->h16) cudaFree(w->h16);
        if (w->k_meta) cudaFree(w->k_meta);
        delete w;
        oasr_internal_mem_event(be, false);
        return oasr_internal_cuda_fail(be, e, "weight_upload", __LINE__);
    }
    be->weight_bytes += w->device_bytes;
    be->n_weights += 1;
    oasr_internal_mem_event(be, true);
    *out = w;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_weight_free(oasr_backend *be, oasr_weight *w) {
    if (!w) return OASR_STATUS_SUCCESS;
    if (be) {
        cudaSetDevice(be->device);
        cudaStreamSynchronize(be->stream);
        be->weight_bytes -= w->device_bytes;
        be->n_weights -= 1;
        be->mem_generation.fetch_add(1);
    }
    if (w->qs) cudaFree(w->qs);
    if (w->d) cudaFree(w->d);
    if (w->tiles) cudaFree(w->tiles);
    if (w->dT) cudaFree(w->dT);
    if (w->qs8) cudaFree(w->qs8);
    if (w->h16) cudaFree(w->h16);
    if (w->k_meta) cudaFree(w->k_meta);
    delete w;
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_weight_download(oasr_backend *be, const oasr_weight *w, void *host, size_t bytes) {
    int st = oasr_internal_precheck(be);
    if (st) return st;
    if (!w || !host) return OASR_STATUS_FAILED;
    const int64_t rs = oasr_b200_row_size(w->type, w->ne[0]);
    const int64_t rows = w->ne[1] * w->ne[2] * w->ne[3];
    if ((size_t)(rs * rows) != bytes) return oasr_internal_fail(be, OASR_STATUS_FAILED, "weight_download: byte count");
    OASR_CUDA_TRY(be, cudaStreamSynchronize(be->stream));
    uint8_t *dst = (uint8_t *)host;
    if (w->type == OASR_TYPE_Q8_0 || w->type == OASR_TYPE_Q4_0) {
        const int bb = w->type == OASR_TYPE_Q8_0 ? BYTES_Q8_0 : BYTES_Q4_0, qb = bb - 2;
        const int64_t nb = w->d_row_elems;
        std::vector<uint8_t> qs((size_t)(rows * w->qs_row_bytes));
        std::vector<uint16_t> d((size_t)(rows * nb));
        OASR_CUDA_TRY(be, cudaMemcpy(qs.data(), w->qs, qs.size(), cudaMemcpyDeviceToHost));
        OASR_CUDA_TRY(be, cudaMemcpy(d.data(), w->d, d.size() * 2, cudaMemcpyDeviceToHost));
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t b = 0; b < nb; ++b) {
                uint8_t *blk = dst + r * rs + b * bb;
                memcpy(blk, &d[(size_t)(r * nb + b)], 2);
                memcpy(blk + 2, &qs[(size_t)(r * w->qs_row_bytes + b * qb)], qb);
            }
    } else {
        OASR_CUDA_TRY(be, cudaMemcpy(dst, w->qs, bytes, cudaMemcpyDeviceToHost));
    }
    return OASR_STATUS_SUCCESS;
}

int oasr_b200_weight_info(const oasr_weight *w, int32_t *type, int64_t ne[4], uint64_t *device_bytes) {
    if (!w) return OASR_STATUS_FAILED;
    if (type) *type = w->type;
    if (ne)
        for (int i = 0; i < 4; ++i) ne[i] = w->ne[i];
    if (device_bytes) *device_bytes = w->device_bytes;
    return OASR_STATUS_SUCCESS;
}

// ---- capability probe (backend.rs:295-323 probes mul_mat(W[256,32], X f32 [256,8])) ----
int oasr_b200_supports_op(oasr_backend *be, int32_t op, const oasr_tensor *src0, const oasr_tensor *src1) {
    if (!be || !src0) return 0;
    switch (op) {
    case OASR_OP_MUL_MAT: {
        if (!src1) return 0;
        const int t = src0->type;
        if (t != OASR_TYPE_Q8_0 && t != OASR_TYPE_Q4_0 && t != OASR_TYPE_Q4_K && t != OASR_TYPE_F16 &&
            t != OASR_TYPE_F32)
            return 0;
        if (src1->type != OASR_TYPE_F32 && src1->type != OASR_TYPE_F16) return 0;
        if (src0->ne[0] != src1->ne[0] || oasr_b200_row_size(t, src0->ne[0]) < 0) return 0;
        if (src0->ne[2] <= 0 || src0->ne[3] <= 0 || src1->ne[2] % src0->ne[2] || src1->ne[3] % src0->ne[3]) return 0;
        return 1;
    }
    case OASR_OP_FLASH_ATTN_EXT: {
        // src0 = q, src1 = k
        if (!src1 || src0->type != OASR_TYPE_F32) return 0;
        if (src1->type != OASR_TYPE_F16 && src1->type != OASR_TYPE_F32) return 0;
        const int64_t D = src0->ne[0];
        if (D != 64 && D != 128) return 0;
        if (src1->ne[2] <= 0 || src0->ne[2] % src1->ne[2]) return 0;
        return 1;
    }
    case OASR_OP_SET_ROWS:
        return src0->type == OASR_TYPE_F16 || src0->type == OASR_TYPE_F32;
    case OASR_OP_ARGMAX_FIRST:
        return src0->type == OASR_TYPE_F32;
    default:
        return 0;
    }
}

}  // extern "C"
