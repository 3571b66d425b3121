// memory_api.cu -- the plugin ABI's optional memory API v1 table
// (ggml_backend_memory_get_api_v1; structs and constants of
// crates/openasr-core/src/ggml_runtime/ffi.rs:144-333, count protocol of
// backend_memory.rs:193-356) over this backend's own memory: resident weights,
// the activation scratch (the backend-private graph workspace), the split-KV
// tickets and tables, and the pinned weight-upload staging buffers.
//
// Domains: device-local HBM (heap 0) and host-pinned staging (heap 1), both
// named by the device's UUID.  Quotes are exact or conservative upper bounds
// computed from the same sizing rules the allocations use (scratch growth to
// max(1.25 x request, 2 x current), 2 MiB device granularity, repack copies
// of imported weights); a quote binds the request fingerprint and the memory
// generation, and reserve_private commits only the backend-private requests
// (GRAPH_PRIVATE: scratch, TRANSFER: staging) of the quote it was given.

#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <mutex>

#include "kernels.cuh"

namespace {

constexpr uint32_t kDomains = 2;
constexpr uint64_t kDeviceGranularity = 2ull << 20;

uint64_t round_up(uint64_t x, uint64_t g) { return (x + g - 1) / g * g; }

// device UUIDs, read once per ordinal
bool device_uuid(int device, uint8_t out[16]) {
    static std::mutex mu;
    static uint8_t cache[64][16];
    static bool have[64];
    if (device < 0 || device >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (!have[device]) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return false;
        memcpy(cache[device], prop.uuid.bytes, 16);
        have[device] = true;
    }
    memcpy(out, cache[device], 16);
    return true;
}

void domain_id(const oasr_backend *be, uint32_t kind, oasr_memory_domain_id_v1 *id) {
    memset(id, 0, sizeof *id);
    device_uuid(be->device, id->physical_device_uuid);
    id->heap_index = kind == OASR_MEMORY_DOMAIN_DEVICE_LOCAL ? 0 : 1;
    id->kind = kind;
}

uint64_t stage_bytes(const oasr_backend *be) {
    return (be->stage[0] ? kUploadStageBytes : 0) + (be->stage[1] ? kUploadStageBytes : 0);
}

// the count protocol: null array -> count; short array -> FAILED with the count needed
bool count_only(const void *items, uint32_t *count, uint32_t needed, int *status) {
    if (!items) {
        *count = needed;
        *status = OASR_STATUS_SUCCESS;
        return true;
    }
    if (*count < needed) {
        *count = needed;
        *status = OASR_STATUS_FAILED;
        return true;
    }
    return false;
}

uint64_t fnv1a(uint64_t h, const void *p, size_t n) {
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}

// every request names the same live backend; the fingerprint covers what a quote prices
int validate_requests(const oasr_memory_request_v1 *req, uint32_t n, oasr_backend **be_out, uint64_t *fp) {
    *be_out = nullptr;
    uint64_t h = 1469598103934665603ull;
    if (n > 0 && !req) return OASR_STATUS_FAILED;
    for (uint32_t i = 0; i < n; ++i) {
        const oasr_memory_request_v1 &r = req[i];
        if (r.struct_size < sizeof(oasr_memory_request_v1) || r.kind < OASR_MEMORY_REQUEST_BUFFER ||
            r.kind > OASR_MEMORY_REQUEST_TRANSFER || !r.backend)
            return OASR_STATUS_FAILED;
        if (*be_out && r.backend != *be_out) return OASR_STATUS_FAILED;
        *be_out = (oasr_backend *)r.backend;
        const uint64_t f[7] = {r.kind, r.flags, r.usage, r.request_id, r.requested_bytes, r.currently_allocated_bytes,
                               r.max_tensor_bytes};
        h = fnv1a(h, f, sizeof f);
    }
    *fp = h;
    return OASR_STATUS_SUCCESS;
}

uint32_t claims_of(const oasr_memory_request_v1 &r) { return r.kind == OASR_MEMORY_REQUEST_HOST_IMPORT ? 2 : 1; }

bool is_private(const oasr_memory_request_v1 &r) {
    return r.kind == OASR_MEMORY_REQUEST_GRAPH_PRIVATE || r.kind == OASR_MEMORY_REQUEST_TRANSFER;
}

void init_claim(oasr_memory_claim_v1 &c, const oasr_backend *be, const oasr_memory_request_v1 &r, uint32_t kind) {
    memset(&c, 0, sizeof c);
    c.struct_size = sizeof c;
    c.request_id = r.request_id;
    domain_id(be, kind, &c.domain);
    c.payload_requested_bytes = r.requested_bytes;
}

// quoted claims, per request and domain, running totals per domain in request order
uint32_t price(const oasr_backend *be, const oasr_memory_request_v1 *req, uint32_t n, oasr_memory_claim_v1 *out) {
    uint64_t dev = oasr_internal_owned_device_bytes(be), pin = stage_bytes(be);
    uint64_t scratch = be->scratch_bytes;
    bool staged = pin > 0;
    uint32_t k = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const oasr_memory_request_v1 &r = req[i];
        const uint64_t b = r.requested_bytes;
        if (r.kind == OASR_MEMORY_REQUEST_BUFFER || r.kind == OASR_MEMORY_REQUEST_HOST_IMPORT) {
            // an engine buffer: one allocation; an imported weight: its planes and the
            // copies the kernels read -- decode tiles and transposed f32 scales for Q8_0
            // (2.12 x the raw bytes), decode tiles for Q4_K (2.03 x), the int8 expansion
            // and transposed scales for Q4_0 (1 + 32/18 + 4/18 = 3.0 x) -- bounded by 3 x,
            // plus the raw copy the plane split reads while it runs
            const uint64_t resident = r.kind == OASR_MEMORY_REQUEST_BUFFER ? round_up(b, kDeviceGranularity)
                                                                            : round_up(3 * b, kDeviceGranularity);
            const uint64_t temp = r.kind == OASR_MEMORY_REQUEST_HOST_IMPORT ? round_up(b, kDeviceGranularity) : 0;
            oasr_memory_claim_v1 &c = out[k++];
            init_claim(c, be, r, OASR_MEMORY_DOMAIN_DEVICE_LOCAL);
            c.flags = OASR_MEMORY_CLAIM_CONSERVATIVE_UPPER;
            c.committed_before_bytes = dev;
            c.commit_peak_extra_upper_bytes = resident + temp;
            dev += resident;
            c.committed_after_upper_bytes = dev;
            c.resident_after_upper_bytes = dev;
            c.retained_after_use_upper_bytes = resident;
            c.releasable_after_use_upper_bytes = 0;
            if (r.kind == OASR_MEMORY_REQUEST_HOST_IMPORT) {
                oasr_memory_claim_v1 &h = out[k++];
                init_claim(h, be, r, OASR_MEMORY_DOMAIN_HOST_PINNED);
                h.flags = OASR_MEMORY_CLAIM_EXACT;
                h.committed_before_bytes = pin;
                const uint64_t add = staged ? 0 : 2 * (uint64_t)kUploadStageBytes;
                h.commit_peak_extra_upper_bytes = add;
                pin += add;
                staged = true;
                h.committed_after_upper_bytes = h.resident_after_upper_bytes = pin;
                h.retained_after_use_upper_bytes = h.releasable_after_use_upper_bytes = pin;
            }
        } else if (r.kind == OASR_MEMORY_REQUEST_GRAPH_PRIVATE) {
            // the size oasr_internal_scratch grows to for this request
            const uint64_t after = b <= scratch ? scratch : std::max<uint64_t>(b + (b >> 2), scratch * 2);
            oasr_memory_claim_v1 &c = out[k++];
            init_claim(c, be, r, OASR_MEMORY_DOMAIN_DEVICE_LOCAL);
            c.flags = OASR_MEMORY_CLAIM_EXACT;
            c.committed_before_bytes = dev;
            c.commit_peak_extra_upper_bytes = after - scratch;
            dev += after - scratch;
            scratch = after;
            c.committed_after_upper_bytes = c.resident_after_upper_bytes = dev;
            c.retained_after_use_upper_bytes = scratch;
            c.releasable_after_use_upper_bytes = scratch;  // trim releases the scratch
        } else {  // TRANSFER
            oasr_memory_claim_v1 &h = out[k++];
            init_claim(h, be, r, OASR_MEMORY_DOMAIN_HOST_PINNED);
            h.flags = OASR_MEMORY_CLAIM_EXACT;
            h.committed_before_bytes = pin;
            const uint64_t add = staged ? 0 : 2 * (uint64_t)kUploadStageBytes;
            h.commit_peak_extra_upper_bytes = add;
            pin += add;
            staged = true;
            h.committed_after_upper_bytes = h.resident_after_upper_bytes = pin;
            h.retained_after_use_upper_bytes = h.releasable_after_use_upper_bytes = pin;
        }
    }
    return k;
}

int mem_get_domains(void *dev, oasr_memory_domain_v1 *domains, uint32_t *count) {
    oasr_backend *be = (oasr_backend *)dev;
    if (!be || !count) return OASR_STATUS_FAILED;
    int st;
    if (count_only(domains, count, kDomains, &st)) return st;
    const uint32_t kinds[kDomains] = {OASR_MEMORY_DOMAIN_DEVICE_LOCAL, OASR_MEMORY_DOMAIN_HOST_PINNED};
    for (uint32_t i = 0; i < kDomains; ++i) {
        oasr_memory_domain_v1 &d = domains[i];
        memset(&d, 0, sizeof d);
        d.struct_size = sizeof d;
        domain_id(be, kinds[i], &d.id);
        snprintf(d.name, sizeof d.name, i == 0 ? "CUDA%d HBM" : "CUDA%d pinned upload staging", be->device);
    }
    *count = kDomains;
    return OASR_STATUS_SUCCESS;
}

int mem_get_stats(void *dev, void *backend, oasr_memory_stats_v1 *stats, uint32_t *count) {
    oasr_backend *be = (oasr_backend *)(backend ? backend : dev);
    if (!be || !count || (dev && backend && dev != backend)) return OASR_STATUS_FAILED;
    int st;
    if (count_only(stats, count, kDomains, &st)) return st;
    const uint64_t now =
        (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
            .count();
    const int p = be->poisoned.load();
    const uint32_t health = be->quarantined              ? OASR_MEMORY_QUARANTINED
                            : p == OASR_STATUS_DEVICE_LOST ? OASR_MEMORY_DEVICE_LOST
                            : p                          ? OASR_MEMORY_DEGRADED
                                                         : OASR_MEMORY_HEALTHY;
    for (uint32_t i = 0; i < kDomains; ++i) {
        oasr_memory_stats_v1 &s = stats[i];
        memset(&s, 0, sizeof s);
        s.struct_size = sizeof s;
        s.generation = be->mem_generation.load();
        s.timestamp_monotonic_ns = now;
        s.allocation_count = be->mem_alloc_count;
        s.allocation_failure_count = be->mem_alloc_failures;
        s.health = health;
        s.last_ggml_status = be->last_status;
        s.last_native_error = be->last_native_error;
        s.quarantine_generation = be->quarantine_generation;
        if (i == 0) {
            domain_id(be, OASR_MEMORY_DOMAIN_DEVICE_LOCAL, &s.domain);
            size_t fr = 0, tot = 0;
            if (cudaSetDevice(be->device) == cudaSuccess && cudaMemGetInfo(&fr, &tot) == cudaSuccess) {
                s.total_bytes = s.budget_bytes = tot;
                s.device_used_bytes = tot - fr;
                s.device_free_bytes = fr;
            } else {
                (void)cudaGetLastError();
                s.flags |= OASR_MEMORY_STATS_BUDGET_UNAVAILABLE;
            }
            s.backend_owned_live_bytes = be->weight_bytes + kBackendFixedBytes;
            s.backend_owned_workspace_bytes = be->scratch_bytes;
            s.backend_owned_high_water_bytes = std::max(be->mem_high_water, oasr_internal_owned_device_bytes(be));
        } else {
            domain_id(be, OASR_MEMORY_DOMAIN_HOST_PINNED, &s.domain);
            s.flags |= OASR_MEMORY_STATS_BUDGET_UNAVAILABLE;  // the host's pinned budget is not known here
            s.backend_owned_live_bytes = stage_bytes(be);
            s.backend_owned_high_water_bytes = stage_bytes(be);
        }
    }
    *count = kDomains;
    return OASR_STATUS_SUCCESS;
}

int mem_quote(const oasr_memory_request_v1 *requests, uint32_t n, oasr_memory_quote_v1 *quote,
              oasr_memory_claim_v1 *claims, uint32_t *n_claims) {
    if (!quote || !n_claims || quote->struct_size < sizeof(oasr_memory_quote_v1)) return OASR_STATUS_FAILED;
    oasr_backend *be;
    uint64_t fp;
    int st = validate_requests(requests, n, &be, &fp);
    if (st) return st;
    uint32_t needed = 0;
    for (uint32_t i = 0; i < n; ++i) needed += claims_of(requests[i]);
    memset(quote, 0, sizeof *quote);
    quote->struct_size = sizeof *quote;
    quote->request_fingerprint = fp;
    if (be) {
        quote->stats_generation = be->mem_generation.load();
        quote->quote_token = ++be->quote_token;
        be->quote_fingerprint = fp;
        be->quote_generation = quote->stats_generation;
    }
    if (count_only(claims, n_claims, needed, &st)) return st;
    *n_claims = be ? price(be, requests, n, claims) : 0;
    return OASR_STATUS_SUCCESS;
}

int mem_reserve_private(const oasr_memory_request_v1 *requests, uint32_t n, const oasr_memory_quote_v1 *quote,
                        oasr_memory_claim_v1 *claims, uint32_t *n_claims) {
    if (!quote || !n_claims || quote->struct_size < sizeof(oasr_memory_quote_v1)) return OASR_STATUS_FAILED;
    oasr_backend *be;
    uint64_t fp;
    int st = validate_requests(requests, n, &be, &fp);
    if (st) return st;
    uint32_t needed = 0;
    for (uint32_t i = 0; i < n; ++i) needed += is_private(requests[i]) ? 1 : 0;
    if (!be) {
        *n_claims = 0;
        return OASR_STATUS_SUCCESS;
    }
    if (quote->quote_token != be->quote_token || quote->request_fingerprint != fp || fp != be->quote_fingerprint ||
        quote->stats_generation != be->quote_generation || quote->stats_generation != be->mem_generation.load())
        return oasr_internal_fail(be, OASR_STATUS_FAILED,
                                  "memory reserve_private: the quote is stale or was issued for other requests");
    if (count_only(claims, n_claims, needed, &st)) return st;  // sizing query: nothing changes
    st = oasr_internal_precheck(be);
    if (st) return st;
    uint64_t scratch_req = 0;
    bool want_stage = false;
    for (uint32_t i = 0; i < n; ++i) {
        if (requests[i].kind == OASR_MEMORY_REQUEST_GRAPH_PRIVATE)
            scratch_req = std::max<uint64_t>(scratch_req, requests[i].requested_bytes);
        if (requests[i].kind == OASR_MEMORY_REQUEST_TRANSFER) want_stage = true;
    }
    const uint64_t dev_before = oasr_internal_owned_device_bytes(be), pin_before = stage_bytes(be);
    if (scratch_req) {
        oasr_internal_scratch(be, (size_t)scratch_req, &st);
        if (st) return st;
    }
    if (want_stage) {
        const cudaError_t e = oasr_internal_stage_alloc(be);
        if (e != cudaSuccess) return oasr_internal_cuda_fail(be, e, "memory reserve_private: staging", __LINE__);
    }
    uint32_t k = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const oasr_memory_request_v1 &r = requests[i];
        if (!is_private(r)) continue;
        oasr_memory_claim_v1 &c = claims[k++];
        const bool dev = r.kind == OASR_MEMORY_REQUEST_GRAPH_PRIVATE;
        init_claim(c, be, r, dev ? OASR_MEMORY_DOMAIN_DEVICE_LOCAL : OASR_MEMORY_DOMAIN_HOST_PINNED);
        c.flags = OASR_MEMORY_CLAIM_EXACT;
        c.committed_before_bytes = dev ? dev_before : pin_before;
        c.committed_after_upper_bytes = c.resident_after_upper_bytes =
            dev ? oasr_internal_owned_device_bytes(be) : stage_bytes(be);
        c.commit_peak_extra_upper_bytes = c.committed_after_upper_bytes - c.committed_before_bytes;
        c.retained_after_use_upper_bytes = c.releasable_after_use_upper_bytes =
            dev ? (uint64_t)be->scratch_bytes : stage_bytes(be);
    }
    *n_claims = k;
    be->mem_generation.fetch_add(1);  // the quote is spent
    return OASR_STATUS_SUCCESS;
}

int mem_trim(void *backend, uint64_t flags) {
    (void)flags;
    oasr_backend *be = (oasr_backend *)backend;
    if (!be) return OASR_STATUS_FAILED;
    // nothing is released on a device that cannot be made current or while the
    // backend's stream is being captured (the stream synchronize a release needs would
    // invalidate the host's capture): the call fails and changes nothing.  A quarantined
    // backend still releases (the host is taking its memory back).
    if (cudaSetDevice(be->device) != cudaSuccess) return OASR_STATUS_FAILED;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(be->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
        return OASR_STATUS_FAILED;
    oasr_internal_scratch_release(be);
    oasr_internal_stage_release(be);
    return OASR_STATUS_SUCCESS;
}

int mem_quarantine(void *backend, const oasr_memory_quarantine_v1 *info) {
    oasr_backend *be = (oasr_backend *)backend;
    if (!be) return OASR_STATUS_FAILED;
    if (info && info->struct_size < sizeof(oasr_memory_quarantine_v1)) return OASR_STATUS_FAILED;
    const int status = info && info->ggml_status == OASR_STATUS_DEVICE_LOST ? OASR_STATUS_DEVICE_LOST
                                                                           : OASR_STATUS_BACKEND_POISONED;
    int expected = 0;
    be->poisoned.compare_exchange_strong(expected, status);
    be->quarantined = 1;
    ++be->quarantine_generation;
    if (info) {
        char msg[97];
        memcpy(msg, info->message, 96);
        msg[96] = 0;
        be->last_native_error = info->native_error;
        be->last_error = std::string("quarantined by the host: ") + msg;
    } else {
        be->last_error = "quarantined by the host";
    }
    be->last_status = status;
    be->mem_generation.fetch_add(1);
    return OASR_STATUS_SUCCESS;
}

const oasr_memory_api_v1 kApi = {
    sizeof(oasr_memory_api_v1), OASR_MEMORY_ABI_V1, 0,  mem_get_domains, mem_quote, mem_reserve_private,
    mem_get_stats,              mem_trim,           mem_quarantine,
};

static_assert(sizeof(oasr_memory_domain_id_v1) == 24, "domain id layout");
static_assert(sizeof(oasr_memory_request_v1) == 88, "request layout");
static_assert(sizeof(oasr_memory_claim_v1) == 96, "claim layout");
static_assert(sizeof(oasr_memory_quote_v1) == 48, "quote layout");
static_assert(sizeof(oasr_memory_stats_v1) == 152, "stats layout");
static_assert(sizeof(oasr_memory_api_v1) == 64, "table layout");

}  // namespace

const oasr_memory_api_v1 *oasr_b200_memory_get_api_v1(void) { return &kApi; }
