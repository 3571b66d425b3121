// registry.cpp -- entry point lookup by name.
//
// The reference's loader resolves a plugin's optional entry points through
// ggml_backend_reg_get_proc_address(reg, name) (ffi.rs:599; the memory API in
// backend.rs:1290 is found as "ggml_backend_memory_get_api_v1").  A host that binds
// this library dynamically can do the same with oasr_b200_get_proc_address: the
// memory API under its ggml name, and every function of include/oasr_b200.h under
// its own name.
#include <string.h>

#include "oasr_b200.h"

namespace {

struct Entry {
    const char *name;
    void *fn;
};

#define OASR_ENTRY(f) {#f, reinterpret_cast<void *>(&f)}

const Entry kEntries[] = {
    {"ggml_backend_memory_get_api_v1", reinterpret_cast<void *>(&oasr_b200_memory_get_api_v1)},
    OASR_ENTRY(oasr_b200_act_bytes),
    OASR_ENTRY(oasr_b200_argmax_first),
    OASR_ENTRY(oasr_b200_device_count),
    OASR_ENTRY(oasr_b200_flash_attn_causal),
    OASR_ENTRY(oasr_b200_flash_attn_ext),
    OASR_ENTRY(oasr_b200_flash_attn_ext_static),
    OASR_ENTRY(oasr_b200_free),
    OASR_ENTRY(oasr_b200_get_proc_address),
    OASR_ENTRY(oasr_b200_get_stream),
    OASR_ENTRY(oasr_b200_init),
    OASR_ENTRY(oasr_b200_last_error),
    OASR_ENTRY(oasr_b200_mem_stats),
    OASR_ENTRY(oasr_b200_memory_get_api_v1),
    OASR_ENTRY(oasr_b200_mul_mat),
    OASR_ENTRY(oasr_b200_mul_mat_qact),
    OASR_ENTRY(oasr_b200_props),
    OASR_ENTRY(oasr_b200_quantize_act),
    OASR_ENTRY(oasr_b200_quantize_chunk),
    OASR_ENTRY(oasr_b200_qwen_decode_step),
    OASR_ENTRY(oasr_b200_qwen_free),
    OASR_ENTRY(oasr_b200_qwen_generate),
    OASR_ENTRY(oasr_b200_qwen_load),
    OASR_ENTRY(oasr_b200_qwen_prefill),
    OASR_ENTRY(oasr_b200_qwen_read_kv),
    OASR_ENTRY(oasr_b200_reserve_scratch),
    OASR_ENTRY(oasr_b200_row_size),
    OASR_ENTRY(oasr_b200_serve_batch_vram_cap),
    OASR_ENTRY(oasr_b200_serve_batch_width),
    OASR_ENTRY(oasr_b200_set_abort_callback),
    OASR_ENTRY(oasr_b200_selftest_bounded_wait),
    OASR_ENTRY(oasr_b200_set_rows),
    OASR_ENTRY(oasr_b200_set_stream),
    OASR_ENTRY(oasr_b200_supports_op),
    OASR_ENTRY(oasr_b200_synchronize),
    OASR_ENTRY(oasr_b200_synchronize_ex),
    OASR_ENTRY(oasr_b200_synth_normal),
    OASR_ENTRY(oasr_b200_weight_download),
    OASR_ENTRY(oasr_b200_weight_free),
    OASR_ENTRY(oasr_b200_weight_info),
    OASR_ENTRY(oasr_b200_weight_upload),
    OASR_ENTRY(oasr_b200_whisper_decode_step),
    OASR_ENTRY(oasr_b200_whisper_encode),
    OASR_ENTRY(oasr_b200_whisper_free),
    OASR_ENTRY(oasr_b200_whisper_generate),
    OASR_ENTRY(oasr_b200_whisper_load),
    OASR_ENTRY(oasr_b200_whisper_mel),
    OASR_ENTRY(oasr_b200_whisper_max_batch),
    OASR_ENTRY(oasr_b200_whisper_mel_device),
    OASR_ENTRY(oasr_b200_whisper_serve),
    OASR_ENTRY(oasr_b200_whisper_transcribe),
};

#undef OASR_ENTRY

}  // namespace

extern "C" void *oasr_b200_get_proc_address(const char *name) {
    if (!name) return nullptr;
    for (const Entry &e : kEntries)
        if (strcmp(e.name, name) == 0) return e.fn;
    return nullptr;
}
