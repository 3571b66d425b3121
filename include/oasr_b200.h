/*
 * oasr_b200.h -- C ABI of the B200 (sm_100a) backend for OpenASR's inference
 * hot path: quantized-weight GGML_OP_MUL_MAT and f16-KV GGML_OP_FLASH_ATTN_EXT,
 * plus the KV write (SET_ROWS) and the greedy first-max argmax that sit next
 * to them in every decoder step.
 *
 * The reference reaches its device backends through ggml's backend/plugin C
 * ABI declared in crates/openasr-core/src/ggml_runtime/ffi.rs:399-1057.  This
 * header exposes the same operations as plain functions over plain pointers
 * and sizes (no torch or ggml types), so the openasr-core side needs only a
 * thin `extern "C"` block.  Each entry point names the
 * reference interface it replaces.
 *
 * Conventions (identical to ggml's):
 *   - a tensor is {type, data, ne[4], nb[4]}: ne0 is the fastest dimension,
 *     nb are byte strides -- ggml's tensor geometry as GgmlTensorLayoutPrefix
 *     reads it (ffi.rs:24-30), see oasr_tensor for how it differs;
 *   - every function returns a ggml_status value (ffi.rs:102-117) and never
 *     aborts the process;
 *   - device tensors live in this device's memory; ops are enqueued on the
 *     backend's stream and complete asynchronously; oasr_b200_synchronize()
 *     returns the merged submit + completion status (ffi.rs:107-113);
 *   - a device-side failure (CUDA error, kernel error word) poisons the
 *     backend: later calls return OASR_STATUS_BACKEND_POISONED (cpu_graph.rs:7893-7935).
 *   - one backend instance serves one stream at a time (ffi.rs:334-336,
 *     "one graph compute per backend at a time"): its activation scratch is
 *     shared by the ops it enqueues.
 */
#ifndef OASR_B200_H
#define OASR_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OASR_B200_ABI_VERSION 1

/* enum ggml_status -- ffi.rs:102-117 */
enum oasr_status {
    OASR_STATUS_ALLOC_FAILED = -2,
    OASR_STATUS_FAILED = -1,
    OASR_STATUS_SUCCESS = 0,
    OASR_STATUS_ABORTED = 1,
    OASR_STATUS_EXECUTION_FAILED = 2,
    OASR_STATUS_DEVICE_LOST = 3,
    OASR_STATUS_BACKEND_POISONED = 4,
};

/* enum ggml_type ids -- ffi.rs:338-346 */
enum oasr_type {
    OASR_TYPE_F32 = 0,
    OASR_TYPE_F16 = 1,
    OASR_TYPE_Q4_0 = 2,
    OASR_TYPE_Q8_0 = 8,
    OASR_TYPE_Q4_K = 12,
    OASR_TYPE_I32 = 26,
    OASR_TYPE_I64 = 27,
};

/* ggml_prec -- ffi.rs:15-16 (GGML_PREC_DEFAULT / GGML_PREC_F32) */
enum oasr_prec {
    OASR_PREC_DEFAULT = 0,
    OASR_PREC_F32 = 10,
};

/* ops answered by oasr_b200_supports_op (ggml_backend_dev_supports_op, ffi.rs:566-598) */
enum oasr_op {
    OASR_OP_MUL_MAT = 1,
    OASR_OP_FLASH_ATTN_EXT = 2,
    OASR_OP_SET_ROWS = 3,
    OASR_OP_ARGMAX_FIRST = 4,
};

/* GGML_BACKEND_GRAPH_CANCEL_* mechanisms and observation granularities -- ffi.rs:118-124 */
enum oasr_cancel_mechanism {
    OASR_CANCEL_DISABLED = 0,
    OASR_CANCEL_NATIVE = 1,
    OASR_CANCEL_SEGMENTED = 2,
};
enum oasr_cancel_observation {
    OASR_CANCEL_OBSERVATION_NONE = 0,
    OASR_CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT = 1,
    OASR_CANCEL_OBSERVATION_GRAPH_COMPLETION = 2,
};

/* struct ggml_backend_graph_cancel_capability (GgmlBackendGraphCancelCapability,
 * ffi.rs:125-131): how a compute call honours the abort callback, reported with its
 * terminal status (ggml_backend_graph_compute_with_abort's out parameter, ffi.rs:453-459).
 * The host accepts the pairs validate_graph_cancel_capability lists (cpu_graph.rs:7974-8002). */
typedef struct oasr_cancel_capability {
    int32_t mechanism;               /* enum oasr_cancel_mechanism */
    int32_t observation_granularity; /* enum oasr_cancel_observation */
} oasr_cancel_capability;

/* A tensor: ggml's geometry (type, ne, nb with ne[0] fastest and nb byte strides),
 * laid out like GgmlTensorLayoutPrefix (ffi.rs:24-30: c_int type, a pointer, i64 ne[4],
 * usize nb[4]) -- but the pointer is the tensor's data (ggml_tensor.data), where that
 * prefix has the buffer handle.  It is not a view of struct ggml_tensor: a host fills
 * it from a ggml_tensor's type / data / ne / nb fields (INTEGRATION.md shows the
 * conversion). */
typedef struct oasr_tensor {
    int32_t type;  /* enum oasr_type */
    int32_t flags; /* reserved, 0 (the padding GgmlTensorLayoutPrefix leaves after type) */
    void *data;    /* device pointer (host pointer only where a function says so) */
    int64_t ne[4]; /* elements per dimension, ne[0] fastest */
    int64_t nb[4]; /* byte strides */
} oasr_tensor;

typedef struct oasr_device_props {
    char name[64];          /* ggml_backend_dev_name, e.g. "CUDA0" */
    char description[256];  /* ggml_backend_dev_description */
    int32_t ordinal;
    int32_t device_type;    /* GGML_BACKEND_DEVICE_TYPE_GPU = 1 (ffi.rs:93-97) */
    int32_t sm_count;
    int32_t cc_major, cc_minor;
    int32_t cancel_mechanism;   /* OASR_CANCEL_NATIVE */
    int32_t cancel_observation; /* OASR_CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT */
    uint64_t memory_total, memory_free; /* ggml_backend_dev_memory */
} oasr_device_props;

typedef struct oasr_mem_stats {
    uint64_t weight_bytes;   /* resident weights (usage WEIGHTS, ffi.rs:141) */
    uint64_t scratch_bytes;  /* activation scratch (usage COMPUTE, ffi.rs:142) */
    uint64_t device_total, device_free;
    int64_t n_weights;
} oasr_mem_stats;

/* ggml_abort_callback (ffi.rs:334-336, GgmlAbortCallback: extern "C" fn(*mut c_void) -> bool):
 * return true to abort.  Called on the thread that enqueues work; must be lock-free. */
typedef bool (*oasr_abort_callback)(void *data);

typedef struct oasr_backend oasr_backend; /* one device + one stream */
typedef struct oasr_weight oasr_weight;   /* a resident quantized weight */

/* ---- device / backend lifecycle (ffi.rs:566-598: ggml_backend_dev_*) ------ */
int oasr_b200_device_count(int32_t *count);
int oasr_b200_init(int32_t ordinal, oasr_backend **out);       /* ggml_backend_dev_init */
int oasr_b200_free(oasr_backend *be);                          /* ggml_backend_free */
int oasr_b200_props(oasr_backend *be, oasr_device_props *out); /* ggml_backend_dev_get_props */
/* 1 if supported, 0 if not (ggml_backend_dev_supports_op; probe in backend.rs:295-323) */
int oasr_b200_supports_op(oasr_backend *be, int32_t op, const oasr_tensor *src0, const oasr_tensor *src1);
/* Enqueue subsequent work on `stream` (a cudaStream_t of this device; NULL is
 * CUDA's legacy default stream).  A new backend starts on a non-blocking
 * stream of its own, which oasr_b200_get_stream returns. */
int oasr_b200_set_stream(oasr_backend *be, void *stream);
void *oasr_b200_get_stream(oasr_backend *be);
int oasr_b200_synchronize(oasr_backend *be);                   /* merged completion status */
/* The merged completion status together with the cancel capability of the work it
 * completes (ggml_backend_graph_compute_with_abort's status + *cancel_capability,
 * ffi.rs:453-459): the abort callback is polled before every enqueue and between the
 * steps of the model drivers' decode loops, so a live backend reports
 * {OASR_CANCEL_NATIVE, OASR_CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT}; a NULL backend
 * returns OASR_STATUS_FAILED with {OASR_CANCEL_DISABLED, OASR_CANCEL_OBSERVATION_NONE}.
 * `cancel_capability` may be NULL. */
int oasr_b200_synchronize_ex(oasr_backend *be, oasr_cancel_capability *cancel_capability);
/* Entry point lookup by name, as ggml_backend_reg_get_proc_address (ffi.rs:599;
 * backend.rs:1290) answers a loader: "ggml_backend_memory_get_api_v1" ->
 * oasr_b200_memory_get_api_v1, and every oasr_b200_* function of this header by its
 * own name; NULL for any other name.  Host-only (no device needed). */
void *oasr_b200_get_proc_address(const char *name);
int oasr_b200_set_abort_callback(oasr_backend *be, oasr_abort_callback cb, void *data);
int oasr_b200_mem_stats(oasr_backend *be, oasr_mem_stats *out);
const char *oasr_b200_last_error(oasr_backend *be);
/* Pre-size the activation scratch (bytes) so no later op allocates. */
int oasr_b200_reserve_scratch(oasr_backend *be, size_t bytes);

/* ---- resident weights (ggml_backend_dev_buffer_from_host_ptr, ffi.rs:588;
 *      cpu_graph.rs:9497 maybe_allocate_weight_buffer_from_host_ptr) ------------
 * `host` holds ggml row-major blocks for a [ne0=K, ne1=N, ne2, ne3] tensor of
 * `type`; the raw blocks are copied to HBM and repacked without dequantizing
 * (Q8_0/Q4_0: quants and fp16 scales split into two 16-byte-aligned planes;
 * Q4_K and F16/F32 keep ggml's layout).  The host buffer may be freed after
 * the call returns. */
int oasr_b200_weight_upload(oasr_backend *be, const void *host, size_t bytes, int32_t type,
                            const int64_t ne[4], oasr_weight **out);
int oasr_b200_weight_free(oasr_backend *be, oasr_weight *w);
/* Copy the resident weight back as ggml bytes (inverse of the repack). */
int oasr_b200_weight_download(oasr_backend *be, const oasr_weight *w, void *host, size_t bytes);
int oasr_b200_weight_info(const oasr_weight *w, int32_t *type, int64_t ne[4], uint64_t *device_bytes);

/* ---- hot-path ops ------------------------------------------------------------ */
/* GGML_OP_MUL_MAT (ggml_mul_mat ffi.rs:694; builder cpu_graph.rs:3616-3686):
 * dst[n, m, i2, i3] = sum_k w[k, n, i2/r2, i3/r3] * x[k, m, i2, i3].
 * x: f32 or f16 device tensor [K, M, ne2, ne3] with contiguous rows; dst: f32
 * [N, M, ne2, ne3].  Activations are quantized to the weight type's ggml
 * vec_dot type (Q8_0/Q4_0 -> q8_0 per 32, Q4_K -> q8_K per 256) and dotted
 * with integer block arithmetic and f32 accumulation; prec = OASR_PREC_F32
 * (ggml_mul_mat_set_prec, ffi.rs:699) keeps f32 activations for F16 weights. */
int oasr_b200_mul_mat(oasr_backend *be, const oasr_weight *w, const oasr_tensor *x, oasr_tensor *dst,
                      int32_t prec);

/* The two halves of oasr_b200_mul_mat, for callers that feed one activation
 * to several weights (fused QKV / gate+up read the same normed rows).  ggml's
 * mul_mat first converts src1 into the weight's vec_dot type (its wdata
 * buffer) and then runs the block dots; these expose that split.
 * oasr_b200_act_bytes: device bytes of `rows` converted rows of K elements
 * for weights of `weight_type` (negative status if unsupported).
 * oasr_b200_quantize_act: convert x (f32|f16 [K, rows], contiguous rows) into
 * the caller's device buffer `qact`.
 * oasr_b200_mul_mat_qact: dst f32 [N, rows] = w . qact (qact from
 * oasr_b200_quantize_act with the same weight type and K). */
int64_t oasr_b200_act_bytes(int32_t weight_type, int64_t K, int64_t rows);
int oasr_b200_quantize_act(oasr_backend *be, int32_t weight_type, const oasr_tensor *x, void *qact, size_t qact_bytes);
int oasr_b200_mul_mat_qact(oasr_backend *be, const oasr_weight *w, const void *qact, int64_t rows, oasr_tensor *dst);

/* GGML_OP_FLASH_ATTN_EXT (ggml_flash_attn_ext ffi.rs:755-764; builder
 * cpu_graph.rs:4144-4220, checks :7476-7519).
 * q f32 [D, n_q, H, S]; k, v f16 or f32 [D, n_kv, H_kv, S] (rows contiguous,
 * other strides free: KV-cache views); mask NULL or f16 [>=n_kv, >=n_q, H|1, S|1];
 * dst f32 [D, H, n_q, S] (ggml's permuted output).  H % H_kv == 0 (GQA).
 * max_bias and logit_softcap must be 0 (every hot call site passes 0). */
int oasr_b200_flash_attn_ext(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k,
                             const oasr_tensor *v, const oasr_tensor *mask, float scale, float max_bias,
                             float logit_softcap, int32_t prec, oasr_tensor *dst);

/* GGML_OP_FLASH_ATTN_EXT under the causal mask, with no mask tensor read.  No
 * reference counterpart: the reference passes the mask of
 * build_causal_mask_f16_bits (nn/decoder.rs:766-790; the Qwen prompt pass,
 * llm_transformer.rs:3859-3895), under which key j is visible to query i when
 * j <= i + n_kv - n_q; a host that knows its mask is that one can call this
 * instead and skip the n_q x n_kv mask.  Runs on the tcgen05 tensor cores with
 * fp16 operands and fp16 probabilities (the arithmetic ggml's CUDA backend
 * uses): head_dim 64 or 128, n_q >= 64, n_kv >= n_q; other shapes fail with
 * OASR_STATUS_FAILED (use oasr_b200_flash_attn_ext with the mask).  Arguments
 * otherwise as oasr_b200_flash_attn_ext (no mask argument). */
int oasr_b200_flash_attn_causal(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k, const oasr_tensor *v,
                                float scale, int32_t prec, oasr_tensor *dst);

/* Allocation-free GGML_OP_FLASH_ATTN_EXT.  No reference counterpart.
 * For callers that must not allocate device memory once they are running: a
 * host whose memory planner reserves the GPU's budget up front and treats any
 * later allocation as a failure, or a real-time decode loop where a
 * cudaMalloc (which may synchronise the device) would stall the audio
 * pipeline.  oasr_b200_flash_attn_ext may grow the backend's scratch; this
 * call never allocates or frees device or host memory.
 * Same arguments, checks and results as oasr_b200_flash_attn_ext for every
 * shape that call runs through its split-KV kernels (decode and short
 * prefill); it always uses those kernels, never the tensor-core encoder path
 * (whose staging copies need backend scratch).  The split-KV partials and
 * tickets live in a file-scope device array: 4 MiB of partials and 1024
 * tickets, held on every GPU that loads the library until the process exits.
 * A shape that needs more fails with OASR_STATUS_FAILED and a message naming
 * both sizes, and nothing is launched.
 *  - The tickets must be zero when a launch starts: they are zero when the
 *    module loads and every launch leaves them at zero.  The partials need no
 *    initial value (each split writes its slot before the merge reads it).
 *  - Calls that overlap on one device (two streams, two backends, or two
 *    host threads without ordering) share that array and race: serialise them.
 *  - The first call on a device looks the array's address up
 *    (cudaGetSymbolAddress, which may load the module); make that first call
 *    before any stream capture.  A first call made during capture is refused. */
int oasr_b200_flash_attn_ext_static(oasr_backend *be, const oasr_tensor *q, const oasr_tensor *k,
                                    const oasr_tensor *v, const oasr_tensor *mask, float scale, float max_bias,
                                    float logit_softcap, int32_t prec, oasr_tensor *dst);

/* GGML_OP_SET_ROWS (ggml_set_rows ffi.rs:884; cpu_graph.rs:4882): write f32 rows
 * of src [D, n, ne2, ne3] into dst (f16|f32) rows rows[i] (I32 or I64 [n]). */
int oasr_b200_set_rows(oasr_backend *be, oasr_tensor *dst, const oasr_tensor *src, const oasr_tensor *rows);

/* First-max argmax (ggml_argmax_first ffi.rs:706; cpu_graph.rs:3750-3765): for
 * each row of f32 logits [n, rows] the lowest index whose finite value is
 * maximal; out I32 [rows]. */
int oasr_b200_argmax_first(oasr_backend *be, const oasr_tensor *logits, oasr_tensor *out);

/* ---- memory API v1 (the optional table the plugin loader resolves through
 * ggml_backend_reg_get_proc_address("ggml_backend_memory_get_api_v1"); layouts and
 * constants of ffi.rs:144-333, fixed widths checked by backend_memory.rs:697-704:
 * domain id 24 B, request 88 B, claim 96 B, quote 48 B, stats 152 B, table 64 B).
 * Every `dev` / `backend` handle here is an oasr_backend (one device + one stream).
 * Count protocol (backend_memory.rs:193-356): a call with a null array returns the
 * item count in *count; a call with an array of *count items fills at most that many
 * and sets *count to the number written, failing (OASR_STATUS_FAILED, *count = the
 * number needed) when the array is too small.  Domains: 1 device-local HBM (heap 0,
 * the backend's weights, activation scratch and tables), 2 host-pinned (heap 1, the
 * weight-upload staging buffers).  Request kinds: BUFFER (an engine-owned device
 * buffer, claimed, committed by the engine), HOST_IMPORT (a host weight payload
 * copied to HBM by oasr_b200_weight_upload: device claim plus staging), GRAPH_PRIVATE
 * (the backend's activation scratch; reserve_private grows it), TRANSFER (the
 * pinned staging buffers; reserve_private allocates them).  A quote carries the
 * stats generation and a token; reserve_private refuses a quote whose token,
 * request fingerprint or generation no longer matches (any allocation, free, trim
 * or quarantine bumps the generation).  reserve_private with a null claim array is
 * the sizing query and changes nothing.  trim (flags ignored) synchronises the
 * stream and releases the activation scratch and the staging buffers (graphs
 * captured before must be re-captured: the model drivers do so themselves).
 * quarantine poisons the backend (later calls: OASR_STATUS_BACKEND_POISONED) and
 * records the reason; stats then report health QUARANTINED.  Like every other call on
 * a backend, these come from one thread at a time per backend (the last quote issued
 * and the generation are per-backend state). */
#define OASR_MEMORY_ABI_V1 1u
enum {
    OASR_MEMORY_DOMAIN_DEVICE_LOCAL = 1, OASR_MEMORY_DOMAIN_HOST_PAGEABLE = 2, OASR_MEMORY_DOMAIN_HOST_PINNED = 3,
    OASR_MEMORY_DOMAIN_UNIFIED = 4, OASR_MEMORY_DOMAIN_FILE_BACKED = 5
};
enum {
    OASR_MEMORY_REQUEST_BUFFER = 1, OASR_MEMORY_REQUEST_HOST_IMPORT = 2, OASR_MEMORY_REQUEST_GRAPH_PRIVATE = 3,
    OASR_MEMORY_REQUEST_TRANSFER = 4
};
enum {
    OASR_MEMORY_QUOTE_PROVISIONAL = 1u << 0, OASR_MEMORY_QUOTE_HAS_RESIDUAL_UNCERTAINTY = 1u << 1,
    OASR_MEMORY_QUOTE_OPAQUE_DRIVER_COSTS_REQUIRE_DOMAIN_HEADROOM = 1u << 2
};
enum { OASR_MEMORY_STATS_BUDGET_UNAVAILABLE = 1u << 0 };
enum {
    OASR_MEMORY_CLAIM_EXACT = 1u << 0, OASR_MEMORY_CLAIM_CONSERVATIVE_UPPER = 1u << 1,
    OASR_MEMORY_CLAIM_DRIVER_ESTIMATE = 1u << 2, OASR_MEMORY_CLAIM_PROVISIONAL = 1u << 6
};
enum {
    OASR_MEMORY_HEALTHY = 0, OASR_MEMORY_DEGRADED = 1, OASR_MEMORY_QUARANTINED = 2, OASR_MEMORY_DEVICE_LOST = 3
};

typedef struct oasr_memory_domain_id_v1 {
    uint8_t physical_device_uuid[16];
    uint32_t heap_index;
    uint32_t kind;
} oasr_memory_domain_id_v1;

typedef struct oasr_memory_domain_v1 {
    uint32_t struct_size;
    uint32_t flags;
    oasr_memory_domain_id_v1 id;
    char name[48];
} oasr_memory_domain_v1;

typedef struct oasr_memory_request_v1 {
    uint32_t struct_size;
    uint32_t kind;
    uint32_t flags;
    uint32_t usage; /* ggml buffer usage: 1 WEIGHTS, 2 COMPUTE (ffi.rs:141-142) */
    uint64_t request_id;
    void *backend;
    void *peer_backend;
    void *buft;
    void *graph;
    const void *host_ptr;
    uint64_t requested_bytes;
    uint64_t currently_allocated_bytes;
    uint64_t max_tensor_bytes;
} oasr_memory_request_v1;

typedef struct oasr_memory_claim_v1 {
    uint32_t struct_size;
    uint32_t flags;
    uint64_t request_id;
    oasr_memory_domain_id_v1 domain;
    uint64_t payload_requested_bytes;
    uint64_t committed_before_bytes;
    uint64_t committed_after_upper_bytes;
    uint64_t commit_peak_extra_upper_bytes;
    uint64_t resident_after_upper_bytes;
    uint64_t retained_after_use_upper_bytes;
    uint64_t releasable_after_use_upper_bytes;
} oasr_memory_claim_v1;

typedef struct oasr_memory_quote_v1 {
    uint32_t struct_size;
    uint32_t flags;
    uint32_t residual_flags;
    uint32_t residual_request_count;
    uint64_t provisional_requested_upper_bytes;
    uint64_t stats_generation;
    uint64_t quote_token;
    uint64_t request_fingerprint;
} oasr_memory_quote_v1;

typedef struct oasr_memory_stats_v1 {
    uint32_t struct_size;
    uint32_t flags;
    oasr_memory_domain_id_v1 domain;
    uint64_t generation;
    uint64_t timestamp_monotonic_ns;
    uint64_t total_bytes;
    uint64_t budget_bytes;
    uint64_t device_used_bytes;
    uint64_t device_free_bytes;
    uint64_t backend_owned_live_bytes;
    uint64_t backend_owned_cached_bytes;
    uint64_t backend_owned_workspace_bytes;
    uint64_t backend_owned_high_water_bytes;
    uint64_t allocation_count;
    uint64_t allocation_failure_count;
    uint32_t health;
    int32_t last_ggml_status;
    int64_t last_native_error;
    uint64_t quarantine_generation;
} oasr_memory_stats_v1;

typedef struct oasr_memory_quarantine_v1 {
    uint32_t struct_size;
    uint32_t flags;
    uint32_t reason;
    int32_t ggml_status;
    int64_t native_error;
    char message[96];
} oasr_memory_quarantine_v1;

typedef struct oasr_memory_api_v1 {
    uint32_t struct_size;
    uint32_t abi_version;
    uint64_t capabilities;
    int (*get_domains)(void *dev, oasr_memory_domain_v1 *domains, uint32_t *count);
    int (*quote)(const oasr_memory_request_v1 *requests, uint32_t n, oasr_memory_quote_v1 *quote,
                 oasr_memory_claim_v1 *claims, uint32_t *n_claims);
    int (*reserve_private)(const oasr_memory_request_v1 *requests, uint32_t n, const oasr_memory_quote_v1 *quote,
                           oasr_memory_claim_v1 *claims, uint32_t *n_claims);
    int (*get_stats)(void *dev, void *backend, oasr_memory_stats_v1 *stats, uint32_t *count);
    int (*trim)(void *backend, uint64_t flags);
    int (*quarantine)(void *backend, const oasr_memory_quarantine_v1 *info);
} oasr_memory_api_v1;

/* ggml_backend_memory_get_api_v1 (GgmlBackendMemoryGetApiV1Fn, ffi.rs:331-332) */
const oasr_memory_api_v1 *oasr_b200_memory_get_api_v1(void);

/* ---- model drivers ------------------------------------------------------------------
 * The graphs openasr-core builds around the hot ops (layer map L2/L3), restated
 * natively so a whole encoder pass or decoder step runs on this device without
 * a host round trip per node.  Weights arrive as named host tensors in the
 * pack's ggml layouts (whisper.cpp / OpenAI tensor names). */
typedef struct oasr_named_tensor {
    const char *name;
    int32_t type;   /* enum oasr_type */
    int32_t _pad;
    int64_t ne[4];
    const void *data; /* host */
    uint64_t bytes;
} oasr_named_tensor;

typedef struct oasr_whisper_config {
    int32_t n_mels;        /* 80 | 128 */
    int32_t d_model;       /* n_heads * 64 */
    int32_t n_heads;
    int32_t n_enc_layers, n_dec_layers;
    int32_t n_vocab;
    int32_t n_audio_ctx;   /* 1500 encoder frames (30 s) */
    int32_t n_text_ctx;    /* 448 decoder positions */
    int32_t max_batch;     /* sequences decoded in lockstep, <= 8 (MAX_BATCH_LIMIT, batched_decode.rs:53) */
} oasr_whisper_config;

typedef struct oasr_whisper oasr_whisper;

/* Resident Whisper model (replaces the resident-weight session built by
 * models/whisper/ggml_executor.rs:3024-3137 + ggml_decoder_graph.rs:1777-1866). */
int oasr_b200_whisper_load(oasr_backend *be, const oasr_whisper_config *cfg, const oasr_named_tensor *tensors,
                           int32_t n_tensors, oasr_whisper **out);
int oasr_b200_whisper_free(oasr_whisper *m);
/* Log-mel frontend (whisper/mel.rs) of n_utts host PCM clips (16 kHz, concatenated,
 * n_samples[i] each; padded/trimmed to 30 s); mel_out (host, optional) gets
 * [n_utts][n_mels][3000]. */
int oasr_b200_whisper_mel(oasr_whisper *m, const float *pcm, const int64_t *n_samples, int32_t n_utts, float *mel_out);
/* Conv prelude + encoder + cross-attention K/V for n_utts utterances
 * (run_whisper_encoder_state, ggml_executor.rs:4020), from the device mel of the
 * last oasr_b200_whisper_mel call or from host mel [n_utts][n_mels][3000];
 * enc_out (host, optional) gets [n_utts][1500][d_model]. */
int oasr_b200_whisper_encode(oasr_whisper *m, const float *mel_host, int32_t n_utts, float *enc_out);
/* One batched decoder step at position pos (run_whisper_decoder_reused_batched_
 * incremental_step_ggml_v0, ggml_decoder_graph.rs:3299): tokens[n_utts] in,
 * logits [n_utts][n_vocab] (host, optional) and first-max next tokens out. */
int oasr_b200_whisper_decode_step(oasr_whisper *m, const int32_t *tokens, int32_t n_utts, int32_t pos, float *logits,
                                  int32_t *next);
/* The frontend from device-resident PCM (concatenated clips, n_samples host). */
int oasr_b200_whisper_mel_device(oasr_whisper *m, const float *pcm_dev, const int64_t *n_samples, int32_t n_utts);
/* Encoder + greedy decode from the device mel of the last whisper_mel* call;
 * tokens_out [n_utts][n_new] is a device pointer when tokens_on_device != 0
 * (then the call returns without waiting), else host memory. */
int oasr_b200_whisper_generate(oasr_whisper *m, int32_t n_utts, const int32_t *prompt, int32_t n_prompt, int32_t n_new,
                               int32_t eot, int32_t stop_at_eot, int32_t *tokens_out, int32_t tokens_on_device);
/* Whole greedy transcription (run_native_transcription, api/backend/
 * native_transcribe.rs:1005): mel -> encoder -> prompt -> n_new greedy tokens
 * (first-max argmax, seq2seq_greedy_decode.rs:418), decoder steps replayed from
 * one CUDA graph; tokens_out [n_utts][n_new].  With stop_at_eot the loop ends
 * once every sequence emitted `eot` (later entries are then undefined). */
int oasr_b200_whisper_transcribe(oasr_whisper *m, const float *pcm, const int64_t *n_samples, int32_t n_utts,
                                 const int32_t *prompt, int32_t n_prompt, int32_t n_new, int32_t eot,
                                 int32_t stop_at_eot, int32_t *tokens_out);

/* ---- serving: continuous batching (models/seq2seq_serve_batch.rs) ----------------
 * The serve-batch engine decodes a queue of requests in up to max_batch slots: a
 * finished slot is released and refilled from the queue (refill_free_slots,
 * seq2seq_serve_batch.rs:775), the running width follows the bucket rule below, and
 * it narrows with the active slots compacted to the front (try_shrink_active_slots,
 * :634) or widens while requests wait (try_rebucket_active_slots, :528).
 *
 * Bucket width (serve_batch_bucket_width, serve_batch_env.rs:317): `active` rounded
 * up to a power of two, capped at max_batch, never below `active`; 0 and 1 stay. */
int32_t oasr_b200_serve_batch_width(int32_t active, int32_t max_batch);
/* VRAM cap (serve_batch_vram_cap_decision_for_memory, serve_batch_env.rs:501):
 * requested > 1 becomes min(requested, (free - reserve) / slot_bytes), at least 1;
 * slot_bytes == 0 keeps the request.  oasr_b200_whisper_load applies it to
 * max_batch > 2 with the device's free memory after the weights and a reserve of
 * OASR_B200_SERVE_VRAM_RESERVE_MB (default 1024) MiB. */
int32_t oasr_b200_serve_batch_vram_cap(int32_t requested, uint64_t slot_bytes, uint64_t free_bytes,
                                       uint64_t reserve_bytes);
/* Slots a loaded Whisper model decodes at most (max_batch after the VRAM cap). */
int32_t oasr_b200_whisper_max_batch(oasr_whisper *m);

typedef struct oasr_serve_stats {
    int32_t steps;          /* decoder steps run (every slot of the width) */
    int32_t admissions;     /* admission groups (mel + encoder of the refilled slots) */
    int32_t width_changes;  /* re-bucketings: widen while requests wait, narrow with compaction */
    int32_t max_width;      /* widest batch run */
} oasr_serve_stats;

/* Serve n_utts utterances (host PCM, concatenated, n_samples[i] each) through the
 * continuous-batching loop: each slot is teacher-forced through `prompt`, then
 * decodes greedily until it emits `eot` (when stop_at_eot), its budget (budgets[i],
 * or max_new when budgets is NULL) or the context end.  tokens_out
 * [n_utts][max_new] gets each request's generated tokens (the `eot` included),
 * lengths_out[n_utts] their count.  max_width 0 = the model's max batch; the host
 * looks for finished slots every check_every steps, and at the step the earliest
 * budget ends (a slot that emits eot idles until the next look).  A slot's tokens do not depend on the batch it ran in: they equal a
 * serial oasr_b200_whisper_transcribe of the same utterance.  The abort callback is
 * polled before each group of steps. */
int oasr_b200_whisper_serve(oasr_whisper *m, const float *pcm, const int64_t *n_samples, int32_t n_utts,
                            const int32_t *prompt, int32_t n_prompt, const int32_t *budgets, int32_t max_new,
                            int32_t eot, int32_t stop_at_eot, int32_t max_width, int32_t check_every,
                            int32_t *tokens_out, int32_t *lengths_out, oasr_serve_stats *stats);

/* ---- Qwen3-ASR LLM decoder -------------------------------------------------------
 * The decoder-only LLM stack of models/qwen (Qwen3AsrLlmWholeDecoderGraphExecutor,
 * llm_transformer.rs; layer graph nn/decoder.rs:1850-2140): per layer RMSNorm ->
 * q|k|v -> per-head q_norm / k_norm RMSNorm -> RoPE NEOX -> set_rows f16 K/V ->
 * GQA flash_attn_ext -> attn_output -> residual -> RMSNorm -> silu(gate) * up ->
 * down -> residual; then RMSNorm -> lm_head -> first-max argmax
 * (build_fused_logits_top1, llm_transformer.rs:2096-2115).  Tensor names are the
 * GGUF names of the reference's qwen3 contract (decoder_contract.rs):
 * token_embd.weight (Q8_0), output_norm.weight, output.weight (optional: absent =
 * tied to token_embd), blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_q_norm,
 * attn_k_norm, attn_output, ffn_norm, ffn_gate, ffn_up, ffn_down}.weight; linear
 * weights Q8_0, Q4_0 or Q4_K, norms F32. */
typedef struct oasr_qwen_config {
    int32_t d_model;      /* 1024 */
    int32_t n_layers;     /* 28 */
    int32_t n_heads;      /* 16 query heads */
    int32_t n_kv_heads;   /* 8 (GQA) */
    int32_t head_dim;     /* 128 */
    int32_t ffn;          /* 3072 */
    int32_t n_vocab;      /* 151936 */
    int32_t max_pos;      /* KV positions per sequence (2048) */
    int32_t max_prefill;  /* prompt positions one prefill call may carry per sequence */
    int32_t max_batch;    /* sequences decoded in lockstep, <= 8 (batched_decode.rs:49) */
    float rope_theta;     /* 1e6 (llm_transformer.rs:489) */
    float rms_eps;        /* 1e-6 (logits_head.rs:23) */
} oasr_qwen_config;

typedef struct oasr_qwen oasr_qwen;

/* Resident decoder (replaces the resident arena + executor construction of
 * Qwen3AsrLlmWholeDecoderGraphExecutor and its KV arena,
 * allocate_zeroed_llm_resident_kv_arena, nn/decoder.rs:2339). */
int oasr_b200_qwen_load(oasr_backend *be, const oasr_qwen_config *cfg, const oasr_named_tensor *tensors,
                        int32_t n_tensors, oasr_qwen **out);
int oasr_b200_qwen_free(oasr_qwen *m);
/* The whole prompt as one causal pass (run_prefill, llm_transformer.rs:3859-3895):
 * emb [n_seq][n_tok][d_model] f32 prompt embeddings (host, or device when
 * emb_on_device) fill positions 0..n_tok-1 of each sequence's KV cache; the last
 * position's logits [n_seq][n_vocab] (host, optional) and first-max tokens
 * [n_seq] (host, optional) come back, and the decode state moves to position
 * n_tok with those tokens as the next inputs. */
int oasr_b200_qwen_prefill(oasr_qwen *m, const float *emb, int32_t emb_on_device, int32_t n_seq, int32_t n_tok,
                           float *logits, int32_t *next);
/* One batched decode step at position pos (run_step_reused_batched_top1,
 * llm_transformer.rs:4983): tokens [n_seq] (host; NULL = the tokens the previous
 * prefill or step selected) -> logits [n_seq][n_vocab] (host, optional) and
 * first-max tokens (host, optional). */
int oasr_b200_qwen_decode_step(oasr_qwen *m, const int32_t *tokens, int32_t n_seq, int32_t pos, float *logits,
                               int32_t *next);
/* Prefill + greedy decode of n_new tokens per sequence (the first from the
 * prompt's last logits), decode steps replayed from one CUDA graph
 * (decode_continuous_batch, batched_decode.rs:643).  tokens_out [n_seq][n_new]
 * is a device pointer when tokens_on_device != 0 (the call then returns without
 * waiting), else host memory.  With stop_at_eos the loop ends once every
 * sequence emitted `eos` (later entries are then undefined). */
int oasr_b200_qwen_generate(oasr_qwen *m, const float *emb, int32_t emb_on_device, int32_t n_seq, int32_t n_tok,
                            int32_t n_new, int32_t eos, int32_t stop_at_eos, int32_t *tokens_out,
                            int32_t tokens_on_device);
/* Copy positions [0, n_pos) of one layer's f16 K and V cache rows of sequence seq
 * to host [n_kv_heads][n_pos][head_dim] (either output may be NULL). */
int oasr_b200_qwen_read_kv(oasr_qwen *m, int32_t layer, int32_t seq, int32_t n_pos, uint16_t *k_out,
                           uint16_t *v_out);

/* ---- diagnostics (no reference counterpart) --------------------------------------
 * Runs the failure path of the bounded pipeline waits that every tensor-core kernel
 * uses: one CTA waits on an mbarrier that nobody arrives at, gives up after
 * limit_cycles (1 .. 2^31) SM clocks, records the timeout in the device error word and
 * returns.  The call returns what oasr_b200_synchronize then reports:
 * OASR_STATUS_EXECUTION_FAILED with a timeout message; the backend stays usable (a
 * timeout is not a device fault and does not poison it). */
int oasr_b200_selftest_bounded_wait(oasr_backend *be, int64_t limit_cycles);

/* ---- host-side helpers (no device work) --------------------------------------- */
/* ggml_row_size (ffi.rs:619) */
int64_t oasr_b200_row_size(int32_t type, int64_t ne0);
/* ggml_quantize_chunk (ffi.rs:623): quantize nrows rows of n_per_row floats
 * starting at row start_row into ggml blocks (Q8_0, Q4_0, Q4_K, F16). Returns
 * bytes written or a negative status.  Q8_0, Q4_0 and F16 are ggml's encoders
 * (quantize_row_*_ref, bit-exact against gguf-py); Q4_K is NOT ggml's
 * make_qkx2_quants search but a simple per-32 min/max encoder that writes valid
 * Q4_K blocks (for synthetic weights) -- decoding follows the format exactly, but
 * its bytes differ from ggml's Q4_K encoder for the same floats. */
int64_t oasr_b200_quantize_chunk(int32_t type, const float *src, void *dst, int64_t start_row, int64_t nrows,
                                 int64_t n_per_row);
/* Deterministic synthetic data: x[i] = mean + std * N(0,1) from SplitMix64
 * (state seed + (offset+i+1)*0x9E3779B97F4A7C15) and Box-Muller on pairs. */
int oasr_b200_synth_normal(uint64_t seed, uint64_t offset, float *x, int64_t n, float mean, float std);

#ifdef __cplusplus
}
#endif
#endif /* OASR_B200_H */
