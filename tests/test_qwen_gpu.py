"""Model-level parity of the Qwen3-ASR decoder driver (oasr_b200_qwen_*) against
the CPU restatement in oracle/qwen_ref.py, on seeded synthetic packs
(Qwen3-ASR-0.6B widths, at reduced depth and vocab
for the step-by-step checks and at full size for the prefill / smoke checks).

What is exact and what is not follows from ggml's arithmetic:
  * Layer 0's K/V cache rows of a prompt depend only on the embeddings, RMSNorm,
    the Q8_0 projections (integer block dots, in-order epilogue: bit-exact on
    the tensor cores), the per-head norms and RoPE (rotation table from the
    host's libm, like the CPU op): they equal the oracle's bit for bit.  A
    one-layer model agrees with the oracle to f32 noise (measured ~2e-7 of the
    largest logit) in prefill and in every decode step.
  * Past the first attention the f32 summation order differs (split-KV merges
    vs the oracle's sequential online softmax), so a value sitting on a q8_0
    rounding boundary flips one quantization step now and then, and the flips
    propagate through the layers (the same happens between ggml's own CPU
    builds).  Decode rows carry small N(0, 0.02) token embeddings, so their
    hidden state is mostly attention output and shows the noise most.  Measured
    on the seeded packs (max / median of |diff| / max |logit|): 2 layers,
    prefill 5e-3 / 1e-3, decode 1.1e-2 / 2e-3; 28 layers, prefill 2e-2 / 3e-3,
    decode 4e-2 / 6e-3.  The bounds below sit about 2x above those, and the
    greedy token must match wherever the oracle's top-2 margin exceeds the
    noise bound.
  * Same kernels on the same inputs give the same bits: the CUDA-graph greedy
    loop equals host-driven steps, and a batch equals its sequences run alone
    (the reference's batched == serial checks, batched_decode.rs); a decode
    step equals a prefill whose last row is that token's embedding up to the
    attention's split order.
"""
import numpy as np
import pytest

import openasr_b200 as ob
from openasr_b200 import models as om
from oracle import oracle as oo
from oracle import qwen_ref as qr
from tests.conftest import max_abs_rel

FLIP = 2e-2       # 2 layers: bound on quantization-flip noise in logits (relative to max |logit|)
FLIP_DEEP = 8e-2  # 28 layers
MID = om.QWEN3_ASR_0_6B.replace(n_layers=2, n_vocab=4096, max_pos=256, max_prefill=64, max_batch=4)
ONE = MID.replace(n_layers=1)


@pytest.fixture(scope="module")
def mid():
    return MID, om.qwen_synthetic_pack(MID, seed=0x0A5A0003)


@pytest.fixture(scope="module")
def mid_model(gpu_backend, mid):
    cfg, pack = mid
    m = om.QwenModel(gpu_backend, cfg, pack)
    yield m
    m.close()


def prefix(n, T, seed=0x0A5A3000, d=1024):
    return om.qwen_synthetic_prefix(seed, n, T, d)


def check_token(got, ref_logits, where, noise=FLIP):
    """greedy token: must match the oracle unless its top-2 margin is within the noise"""
    top2 = np.sort(ref_logits)[-2:]
    if top2[1] - top2[0] > noise * np.abs(ref_logits).max():
        assert got == oo.argmax_first(ref_logits)[0], where


def assert_mostly_exact(errs, exact=1e-5):
    """Steps agree to f32 noise unless one value landed on a q8_0 rounding boundary
    (measured: a single flip moves a one-layer decode row's logits by ~1.2e-2 of the
    largest logit); flips are a minority and stay within FLIP."""
    errs = np.asarray(errs)
    assert errs.max() < FLIP, errs
    assert (errs < exact).sum() * 2 > len(errs), errs


def rel_stats(got, ref):
    d = np.abs(np.asarray(got, np.float64) - ref) / np.abs(ref).max()
    return float(d.max()), float(np.median(d))


@pytest.mark.gpu
def test_one_layer_matches_reference_to_f32_noise(gpu_backend):
    pack = om.qwen_synthetic_pack(ONE, seed=0x0A5A0003)
    m = om.QwenModel(gpu_backend, ONE, pack)
    try:
        ref = qr.QwenRef(ONE, pack)
        emb = prefix(2, 30, seed=0x0A5A3050)
        logits, nxt = m.prefill(emb)
        for s in (1, 0):  # sequence 0 last: the decode steps below continue it
            cache = ref.new_cache(1)
            lr = ref.prefill(emb[s], cache)
            assert max_abs_rel(logits[s], lr) < 1e-5
            check_token(nxt[s], lr, f"prefill {s}", noise=1e-5)
            k, v = m.read_kv(0, s, 30)
            np.testing.assert_array_equal(k.view(np.uint16), cache[0][0][0, :, :30].view(np.uint16))
            np.testing.assert_array_equal(v.view(np.uint16), cache[0][1][0, :, :30].view(np.uint16))
        errs = []
        for i, tok in enumerate([5, 4095, 17, 2048, 3000, 1, 999, 123]):
            g, n1 = m.decode_step([tok], 30 + i)
            rr = ref.step([tok], 30 + i, cache)[0]
            errs.append(max_abs_rel(g[0], rr))
            check_token(n1[0], rr, f"step {i}")
        assert_mostly_exact(errs)
        # decode-step K/V rows: the GEMV sums blocks in another order, so f16 rows agree to one ulp
        k, v = m.read_kv(0, 0, 35)
        assert np.abs(k.astype(np.float32) - cache[0][0][0, :, :35]).max() <= 2e-3 * np.abs(k.astype(np.float32)).max()
        assert np.abs(v.astype(np.float32) - cache[0][1][0, :, :35]).max() <= 2e-3 * np.abs(v.astype(np.float32)).max()
    finally:
        m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("T", [64, 150, 257])
def test_one_layer_tensor_core_prompt_pass(gpu_backend, T):
    """Prompts of 64+ positions take the causal tcgen05 attention (fp16 operands and
    probabilities, 128-key tiles, the diagonal tile masked in the softmax); the oracle
    evaluates the same arithmetic (FA_TC128 with the causal mask)."""
    cfg = ONE.replace(max_prefill=T, max_pos=512)
    pack = om.qwen_synthetic_pack(cfg, seed=0x0A5A0003)
    m = om.QwenModel(gpu_backend, cfg, pack)
    try:
        ref = qr.QwenRef(cfg, pack)
        emb = prefix(2, T, seed=0x0A5A3060 + T)
        logits, nxt = m.prefill(emb)
        g, _ = m.decode_step([11, 22], T)  # decode steps continue from the tensor-core prompt pass
        for s, tok in ((0, 11), (1, 22)):
            cache = ref.new_cache(1)
            lr = ref.prefill(emb[s], cache)
            # the prompt's last row carries an N(0, 1) embedding: flips move it less than a
            # decode row (measured <= 3e-3); the attention itself is pinned op-level in
            # test_flash_attn_gpu.py::test_causal_tensor_core_attention
            mx, med = rel_stats(logits[s], lr)
            assert mx < 1e-2 and med < 2e-3, (T, s, mx, med)
            check_token(nxt[s], lr, f"T={T} seq {s}", noise=1e-2)
            k, v = m.read_kv(0, s, T)
            np.testing.assert_array_equal(k.view(np.uint16), cache[0][0][0, :, :T].view(np.uint16))
            np.testing.assert_array_equal(v.view(np.uint16), cache[0][1][0, :, :T].view(np.uint16))
            # one step: f32 noise, or a single rounding-boundary flip
            assert max_abs_rel(g[s], ref.step([tok], T, cache)[0]) < FLIP
    finally:
        m.close()


@pytest.mark.gpu
def test_prefill_layer0_kv_bit_exact_and_logits_match(mid_model, mid):
    cfg, pack = mid
    emb = prefix(2, 40)
    logits, nxt = mid_model.prefill(emb)
    ref = qr.QwenRef(cfg, pack)
    for s in range(2):
        cache = ref.new_cache(1)
        lr = ref.prefill(emb[s], cache)
        k0, v0 = mid_model.read_kv(0, s, 40)
        np.testing.assert_array_equal(k0.view(np.uint16), cache[0][0][0, :, :40].view(np.uint16))
        np.testing.assert_array_equal(v0.view(np.uint16), cache[0][1][0, :, :40].view(np.uint16))
        k1, v1 = mid_model.read_kv(1, s, 40)
        assert max_abs_rel(k1, cache[1][0][0, :, :40]) < FLIP
        assert max_abs_rel(v1, cache[1][1][0, :, :40]) < FLIP
        mx, med = rel_stats(logits[s], lr)
        assert mx < FLIP and med < 3e-3, (mx, med)
        check_token(nxt[s], lr, f"prefill seq {s}")


@pytest.mark.gpu
def test_decode_steps_match_reference_teacher_forced(mid_model, mid):
    cfg, pack = mid
    emb = prefix(1, 24, seed=0x0A5A3100)
    mid_model.prefill(emb)
    ref = qr.QwenRef(cfg, pack)
    cache = ref.new_cache(1)
    ref.prefill(emb[0], cache)
    errs = []
    for i, tok in enumerate([5, 4095, 17, 2048, 3000, 1, 0, 999, 123, 4000, 7, 77]):
        pos = 24 + i
        logits, nxt = mid_model.decode_step([tok], pos)
        lr = ref.step([tok], pos, cache)[0]
        errs.append(max_abs_rel(logits[0], lr))
        check_token(nxt[0], lr, f"step at {pos}")
    assert max(errs) < 2 * FLIP, errs
    assert np.median(errs) < FLIP, errs


@pytest.mark.gpu
def test_decode_step_equals_prefill_of_appended_row(mid_model, mid):
    cfg, pack = mid
    emb = prefix(1, 27, seed=0x0A5A3150)
    tok = 3210
    row = qr.QwenRef(cfg, pack).embed([tok])
    whole, _ = mid_model.prefill(np.concatenate([emb[0], row], 0)[None])
    mid_model.prefill(emb)
    step, _ = mid_model.decode_step([tok], 27)
    # the GEMV and the tensor-core GEMM give the same bits; the attention splits its KV
    # range differently (f32 noise), which q8_0 quantization absorbs unless a value sits
    # on a rounding boundary (measured: identical)
    assert max_abs_rel(step[0], whole[0]) < FLIP


@pytest.mark.gpu
def test_graph_generate_equals_host_steps(mid_model):
    emb = prefix(3, 33, seed=0x0A5A3200)
    n_new = 10
    got = mid_model.generate(emb, n_new)
    _, nxt = mid_model.prefill(emb)
    steps = [nxt]
    for i in range(n_new - 1):
        _, nxt = mid_model.decode_step(nxt, 33 + i)
        steps.append(nxt)
    np.testing.assert_array_equal(got, np.stack(steps, axis=1))


@pytest.mark.gpu
def test_batched_generate_equals_serial(mid_model):
    emb = prefix(4, 21, seed=0x0A5A3300)
    batched = mid_model.generate(emb, 9)
    for s in range(4):
        np.testing.assert_array_equal(mid_model.generate(emb[s:s + 1], 9)[0], batched[s], err_msg=f"sequence {s}")


@pytest.mark.gpu
def test_generate_after_scratch_growth_recaptures(mid_model, gpu_backend):
    """The step graph holds the backend scratch's address: growing the scratch after a
    capture must lead to a fresh capture, with unchanged tokens."""
    emb = prefix(2, 17, seed=0x0A5A3350)
    before = mid_model.generate(emb, 6)
    grown = gpu_backend.mem_stats()["scratch_bytes"] + (64 << 20)
    gpu_backend.reserve_scratch(grown)
    assert gpu_backend.mem_stats()["scratch_bytes"] >= grown
    np.testing.assert_array_equal(mid_model.generate(emb, 6), before)


@pytest.mark.gpu
def test_single_position_prompt_and_bounds(mid_model, mid):
    cfg, pack = mid
    emb = prefix(1, 1, seed=0x0A5A3400)
    logits, nxt = mid_model.prefill(emb)
    lr = qr.QwenRef(cfg, pack).prefill(emb[0], qr.QwenRef(cfg, pack).new_cache(1))
    assert max_abs_rel(logits[0], lr) < FLIP
    with pytest.raises(ob.GgmlBackendError):
        mid_model.prefill(prefix(1, cfg.max_prefill + 1))
    with pytest.raises(ob.GgmlBackendError):
        mid_model.generate(prefix(1, 8), cfg.max_pos)  # prompt + new tokens past max_pos
    # the model still works after the refusals
    again, nxt2 = mid_model.prefill(emb)
    np.testing.assert_array_equal(again, logits)


@pytest.fixture(scope="module")
def full(gpu_backend):
    cfg = om.QWEN3_ASR_0_6B.replace(max_batch=2, max_prefill=om.QWEN_PREFIX_FRAMES)
    pack = om.qwen_synthetic_pack(cfg)
    m = om.QwenModel(gpu_backend, cfg, pack)
    yield cfg, pack, m
    m.close()


@pytest.mark.gpu
def test_full_size_prefill_matches_reference(full):
    """configs[2] shape: 28 layers, vocab 151936, the 390-frame prompt."""
    cfg, pack, m = full
    emb = prefix(1, om.QWEN_PREFIX_FRAMES, seed=0x0A5A3500)
    logits, nxt = m.prefill(emb)
    ref = qr.QwenRef(cfg, pack)
    cache = ref.new_cache(1)
    lr = ref.prefill(emb[0], cache)
    k0, v0 = m.read_kv(0, 0, om.QWEN_PREFIX_FRAMES)
    np.testing.assert_array_equal(k0.view(np.uint16), cache[0][0][0, :, :om.QWEN_PREFIX_FRAMES].view(np.uint16))
    np.testing.assert_array_equal(v0.view(np.uint16), cache[0][1][0, :, :om.QWEN_PREFIX_FRAMES].view(np.uint16))
    mx, med = rel_stats(logits[0], lr)
    assert mx < FLIP_DEEP / 2 and med < 8e-3, (mx, med)
    check_token(nxt[0], lr, "full-size prefill", noise=FLIP_DEEP)
    # greedy decode steps on the oracle's tokens
    tok = int(oo.argmax_first(lr)[0])
    for i in range(3):
        l1, n1 = m.decode_step([tok], om.QWEN_PREFIX_FRAMES + i)
        r1 = ref.step([tok], om.QWEN_PREFIX_FRAMES + i, cache)[0]
        mx, med = rel_stats(l1[0], r1)
        assert mx < FLIP_DEEP and med < 1.5e-2, (i, mx, med)
        check_token(n1[0], r1, f"full-size step {i}", noise=FLIP_DEEP)
        tok = int(oo.argmax_first(r1)[0])


@pytest.mark.gpu
def test_full_size_batched_generate_equals_serial(full):
    cfg, pack, m = full
    emb = prefix(2, om.QWEN_PREFIX_FRAMES, seed=0x0A5A3600)
    batched = m.generate(emb, 16)
    assert ((batched >= 0) & (batched < cfg.n_vocab)).all()
    for s in range(2):
        np.testing.assert_array_equal(m.generate(emb[s:s + 1], 16)[0], batched[s])
