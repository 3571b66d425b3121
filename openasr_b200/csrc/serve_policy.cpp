// serve_policy.cpp -- the serving scheduler's width rules (host only).
//
// The reference's serve-batch engine runs up to MAX_BATCH_LIMIT = 8 sequences per
// device.  Its width follows two rules, restated here:
//   * bucket width (serve_batch_bucket_width, models/serve_batch_env.rs:317-325): a
//     batch of `active` sequences runs at the next power of two, capped at the maximum,
//     so the set of decode graphs stays {1, 2, 4, 8};
//   * VRAM cap (serve_batch_vram_cap_decision_for_memory, serve_batch_env.rs:501-522):
//     a requested maximum above 1 is cut to the number of per-slot states that fit the
//     free device memory after a reserve, and never below 1.  The loader applies it only
//     to requests above 2, as serve_batch_vram_capped_max_batch (serve_batch_env.rs:
//     295-315) does; the reserve is 1024 MiB unless OASR_B200_SERVE_VRAM_RESERVE_MB says
//     otherwise (the reference's OPENASR_SERVE_BATCH_VRAM_RESERVE_MB).
#include <stdint.h>
#include <stdlib.h>

#include "oasr_b200.h"

extern "C" int32_t oasr_b200_serve_batch_width(int32_t active, int32_t max_batch) {
    if (active <= 1 || max_batch <= active) return active;
    int32_t w = 1;
    while (w < active) w <<= 1;
    if (w > max_batch) w = max_batch;
    return w < active ? active : w;
}

extern "C" int32_t oasr_b200_serve_batch_vram_cap(int32_t requested, uint64_t slot_bytes, uint64_t free_bytes,
                                                  uint64_t reserve_bytes) {
    if (requested <= 1 || slot_bytes == 0) return requested;
    const uint64_t usable = free_bytes > reserve_bytes ? free_bytes - reserve_bytes : 0;
    const uint64_t slots = usable / slot_bytes;
    if (slots >= (uint64_t)requested) return requested;
    return slots < 1 ? 1 : (int32_t)slots;
}

namespace oasr {

uint64_t serve_vram_reserve_bytes() {
    const char *env = getenv("OASR_B200_SERVE_VRAM_RESERVE_MB");
    uint64_t mb = 1024;
    if (env && *env) {
        char *end = nullptr;
        const unsigned long long v = strtoull(env, &end, 10);
        if (end && *end == 0 && v <= 1024ull * 1024ull) mb = v;
    }
    return mb << 20;
}

// device bytes one serving slot of a Whisper model holds: its self-attention K/V cache,
// its cross-attention K|V, its encoder activations and decode rows
uint64_t whisper_slot_bytes(const oasr_whisper_config *c) {
    const uint64_t d = (uint64_t)c->d_model, T = (uint64_t)c->n_audio_ctx, P = (uint64_t)c->n_text_ctx;
    const uint64_t L = (uint64_t)c->n_dec_layers;
    const uint64_t self_kv = L * 2 * P * d * 2;
    const uint64_t cross_kv = L * T * 2 * d * 2;
    const uint64_t frames = 3000, kpad = ((3 * d + 63) / 64) * 64;
    const uint64_t frontend = 480000 * 4 + frames * 201 * 4 + (uint64_t)c->n_mels * frames * 4 + frames * kpad * 2 +
                              frames * d * 4;
    const uint64_t encoder = T * d * 4 * 3 + T * 3 * d * 4 + T * 4 * d * 4 + T * 5 * d * 4;  // f32 rows + planes
    const uint64_t decode = P * 4 + (uint64_t)c->n_vocab * 4 + 16 * d * 4;
    return self_kv + cross_kv + frontend + encoder + decode;
}

}  // namespace oasr
