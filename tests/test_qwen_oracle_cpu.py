"""CPU checks of the Qwen3 decoder restatement in oracle/qwen_ref.py (no device).

The reference's own tests for this graph pin three properties that hold for any
weights, and the restatement is held to them here on a small seeded model:
  * a causal prefill of T positions equals T single-position decode steps
    (the prefill / decode split of run_prefill vs run_step,
    llm_transformer.rs:3203 and :3859);
  * native GQA attention equals attention over K/V heads expanded to the query
    heads (nn/decoder.rs:3860, expand_attention_kv :1799-1841);
  * the causal mask is build_causal_mask_f16_bits (nn/decoder.rs:766-790).
"""
import numpy as np

from openasr_b200 import models as om
from oracle import oracle as oo
from oracle import qwen_ref as qr

SMALL = om.QwenConfig(d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=128, ffn=512, n_vocab=300,
                      max_pos=64, max_prefill=32, max_batch=2)


def small_pack():
    return om.qwen_synthetic_pack(SMALL, seed=0x0A5A0003, synth=oo.synth_normal, quantize=oo.quantize)


def test_causal_mask_is_the_reference_layout():
    m = qr.causal_mask(4, 4).view(np.uint16)
    want = np.array([[0 if kv <= t else 0xFC00 for kv in range(4)] for t in range(4)], np.uint16)
    np.testing.assert_array_equal(m, want)


def test_prefill_equals_stepwise_decode():
    pack = small_pack()
    ref = qr.QwenRef(SMALL, pack)
    emb = om.qwen_synthetic_prefix(0x0A5A3000, 1, 9, SMALL.d_model)[0]
    c1 = ref.new_cache(1)
    last = ref.prefill(emb, c1)
    # the same prompt one position at a time: embedding row -> layers -> cache
    c2 = ref.new_cache(1)
    for t in range(emb.shape[0]):
        x = emb[t:t + 1]
        for l in range(SMALL.n_layers):
            x = ref.layer(x, l, c2, 0, t)
    np.testing.assert_array_equal(ref.head(x)[0], last)
    for (k1, v1), (k2, v2) in zip(c1, c2):
        np.testing.assert_array_equal(k1, k2)
        np.testing.assert_array_equal(v1, v2)


def test_native_gqa_equals_expanded_heads():
    rng = np.random.default_rng(5)
    H, HKV, NQ, NKV, D = 4, 2, 3, 17, 128
    q = rng.normal(0, 1, (1, H, NQ, D)).astype(np.float32)
    k = rng.normal(0, 1, (1, HKV, NKV, D)).astype(np.float16)
    v = rng.normal(0, 1, (1, HKV, NKV, D)).astype(np.float16)
    mask = qr.causal_mask(NQ, NKV, NKV - NQ)
    native = oo.flash_attn_ext(q, k, v, mask, 0.088, oo.FA_F32)
    # repeat_4d over [D, n_kv, 1, HKV] -> [D, n_kv, G, HKV]: query head h reads kv head h // G
    kx = np.ascontiguousarray(np.repeat(k, H // HKV, axis=1))
    vx = np.ascontiguousarray(np.repeat(v, H // HKV, axis=1))
    np.testing.assert_array_equal(native, oo.flash_attn_ext(q, kx, vx, mask, 0.088, oo.FA_F32))


def test_greedy_tokens_are_in_vocab_and_deterministic():
    pack = small_pack()
    ref = qr.QwenRef(SMALL, pack)
    emb = om.qwen_synthetic_prefix(0x0A5A3001, 1, 6, SMALL.d_model)[0]
    a, la = ref.greedy(emb, 4)
    b, lb = ref.greedy(emb, 4)
    np.testing.assert_array_equal(a, b)
    assert ((a >= 0) & (a < SMALL.n_vocab)).all()
    assert la.shape == (4, SMALL.n_vocab) and np.isfinite(la).all()
