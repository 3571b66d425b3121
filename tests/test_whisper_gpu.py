"""Model-level parity of the Whisper driver (oasr_b200_whisper_*) against the
CPU reference graphs in oracle/whisper_ref.py, on seeded synthetic packs
(BASELINE.json configs[0] whisper-tiny shape, and the whisper-large-v3 shape at
reduced depth).

How the criteria follow from ggml's arithmetic: every mul_mat quantizes its
activations to q8_0 / q8_K first, so an element whose value lands within an
f32 ulp of a rounding boundary moves by a whole quantization step when the
f32 summation order differs (GPU reduction trees vs the oracle's sequential
sums; likewise between ggml's own AVX2 and AVX-512 builds).  Hence:
  * decoder steps fed the same encoder output must agree to 1e-5 (measured
    ~1e-7) and pick the same tokens;
  * the encoder agrees element-wise to 1e-6 in the median after one layer with
    isolated flip outliers <= 2e-3 (the op-level bar), and the flip noise
    grows with depth (bounded here at 2e-2 for 4 layers);
  * greedy transcripts are identical when both sides decode from the same
    encoder output, and end to end up to the first step whose reference top-2
    margin is below the encoder flip noise.
The encoder attention is compared with the oracle's tensor-core arithmetic
mode (fp16 operands), the rest with ggml CPU semantics."""
import numpy as np
import pytest

from openasr_b200 import models as om
from oracle import oracle as oo
from oracle import whisper_ref as wr
from tests.conftest import max_abs_rel


def rel_stats(a, b):
    d = np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))
    s = np.abs(b).max()
    return d.max() / s, float(np.median(d)) / s


@pytest.fixture(scope="module")
def tiny():
    cfg = om.WHISPER_TINY.replace(max_batch=4)
    return cfg, om.whisper_synthetic_pack(cfg, seed=0x0A5A0001)


@pytest.fixture(scope="module")
def tiny_model(gpu_backend, tiny):
    cfg, pack = tiny
    m = om.WhisperModel(gpu_backend, cfg, pack)
    yield m
    m.close()


def clips(n, seconds=(30.0, 7.5, 19.0, 5.0)):
    return [om.synthetic_audio(0x0A5A1000 + i, int(16000 * seconds[i % len(seconds)])) for i in range(n)]


@pytest.mark.gpu
def test_log_mel_frontend_matches_reference(tiny_model):
    cs = clips(2)
    got = tiny_model.mel(cs)
    for i, c in enumerate(cs):
        assert np.abs(got[i] - wr.log_mel(c, 80)).max() < 2e-4


@pytest.mark.gpu
def test_one_layer_encoder_matches_reference(gpu_backend):
    cfg = om.WHISPER_TINY.replace(n_enc_layers=1, n_dec_layers=1, max_batch=1)
    pack = om.whisper_synthetic_pack(cfg, seed=0x0A5A0001)
    m = om.WhisperModel(gpu_backend, cfg, pack)
    try:
        mel = wr.log_mel(clips(1)[0], 80)
        mx, med = rel_stats(m.encode(mel[None], 1)[0], wr.WhisperRef(cfg, pack).encode(mel))
        assert med < 1e-6 and mx < 2e-3, (mx, med)
    finally:
        m.close()


@pytest.mark.gpu
def test_tiny_encoder_flip_noise_is_bounded(tiny_model, tiny):
    cfg, pack = tiny
    mel = wr.log_mel(clips(1)[0], 80)
    mx, med = rel_stats(tiny_model.encode(mel[None], 1)[0], wr.WhisperRef(cfg, pack).encode(mel))
    assert mx < 2e-2 and med < 1e-3, (mx, med)


FLIP = 2e-2  # bound on one quantization flip's effect on a step's logits (relative to max |logit|)


@pytest.mark.gpu
def test_tiny_decoder_steps_match_reference_teacher_forced(tiny_model, tiny):
    cfg, pack = tiny
    mel = wr.log_mel(clips(1)[0], 80)
    enc = tiny_model.encode(mel[None], 1)[0]
    ref = wr.WhisperRef(cfg, pack)
    cross, state = ref.cross_kv(enc), ref.new_state()
    errs = []
    for pos, tok in enumerate(om.PROMPT[cfg.n_vocab] + [11, 2000, 51000, 7] + list(range(100, 2100, 100))):
        logits, nxt = tiny_model.decode_step([tok], pos)
        lr = ref.decode_step(tok, pos, cross, state)
        errs.append(max_abs_rel(logits[0], lr))
        top2 = np.sort(lr)[-2:]
        if top2[1] - top2[0] > FLIP * np.abs(lr).max():
            assert nxt[0] == oo.argmax_first(lr)[0], pos
    errs = np.array(errs)
    # steps agree to f32 noise until a quantization flip lands in the self-KV cache;
    # from then on the difference persists but stays within FLIP (where the first
    # flip lands depends on the f32 summation order; see the next test for rates)
    assert errs.max() < FLIP, errs


@pytest.mark.gpu
def test_tiny_decoder_first_step_is_exact_except_rare_flips(tiny_model, tiny):
    """30 fresh first steps (different prompt tokens) from the same encoder output:
    without a quantization flip a step agrees to f32 noise (~1e-7); flips are
    a minority (measured 1-7 in 30 on this 4-layer model, depending on the
    summation order) and bounded by FLIP.  A wrong kernel moves every step, so
    the median pins the arithmetic."""
    cfg, pack = tiny
    enc = tiny_model.encode(wr.log_mel(clips(1)[0], 80)[None], 1)[0]
    ref = wr.WhisperRef(cfg, pack)
    cross = ref.cross_kv(enc)
    errs = []
    for tok in range(50258, 50288):
        logits, _ = tiny_model.decode_step([tok], 0)
        errs.append(max_abs_rel(logits[0], ref.decode_step(tok, 0, cross, ref.new_state())))
    errs = np.array(errs)
    assert np.median(errs) < 1e-6, errs
    assert (errs < 1e-5).sum() >= 15 and errs.max() < FLIP, errs


def _agree_until_near_tie(got, toks, logits):
    """identical, or first divergence at a step whose reference top-2 margin is within the flip bound"""
    if np.array_equal(got, toks):
        return len(got)
    i = int(np.argmax(got != toks))
    top2 = np.sort(logits[i])[-2:]
    assert top2[1] - top2[0] <= FLIP * np.abs(logits[i]).max(), (i, got[i], toks[i], top2[1] - top2[0])
    return i


@pytest.mark.gpu
def test_tiny_greedy_224_matches_reference_from_same_encoder(tiny_model, tiny):
    """30 s of -20 dBFS noise, greedy 224 tokens, batch 1; both sides
    decode from the GPU encoder output."""
    cfg, pack = tiny
    c = clips(1)[0]
    got = tiny_model.transcribe([c], n_new=224)[0]
    enc = tiny_model.encode(wr.log_mel(c, 80)[None], 1)[0]
    ref = wr.WhisperRef(cfg, pack)
    toks, logits = ref.greedy(ref.cross_kv(enc), om.PROMPT[cfg.n_vocab], 224)
    _agree_until_near_tie(got, toks, logits)


@pytest.mark.gpu
def test_tiny_greedy_end_to_end_agrees_until_a_near_tie(tiny_model, tiny):
    cfg, pack = tiny
    c = clips(1)[0]
    got = tiny_model.transcribe([c], n_new=64)[0]
    ref = wr.WhisperRef(cfg, pack)
    toks, logits = ref.greedy(ref.cross_kv(ref.encode(wr.log_mel(c, 80))), om.PROMPT[cfg.n_vocab], 64)
    _agree_until_near_tie(got, toks, logits)


@pytest.mark.gpu
def test_batched_transcripts_equal_serial(tiny_model):
    cs = clips(4)
    batched = tiny_model.transcribe(cs, n_new=32)
    for i, c in enumerate(cs):
        np.testing.assert_array_equal(batched[i], tiny_model.transcribe([c], n_new=32)[0])


@pytest.mark.gpu
def test_large_v3_shape_q4k_reduced_depth(gpu_backend):
    """configs[3] shape (d 1280, 20 heads, 128 mels, Q4_K linears) at 1+2 layers:
    the tensor-core Q4_K GEMM, the fp16 conv GEMM and the tensor-core attention
    in the encoder; Q4_K GEMV, self- and cross-attention in the decoder."""
    cfg = om.WHISPER_LARGE_V3.replace(n_enc_layers=1, n_dec_layers=2, max_batch=2)
    pack = om.whisper_synthetic_pack(cfg, seed=0x0A5A0004)
    m = om.WhisperModel(gpu_backend, cfg, pack)
    try:
        c = clips(1)[0]
        mel = wr.log_mel(c, 128)
        enc = m.encode(mel[None], 1)[0]
        ref = wr.WhisperRef(cfg, pack)
        mx, med = rel_stats(enc, ref.encode(mel))
        # 1280-wide projections: tensor-core attention residuals (~1e-5) flip q8_K
        # activations in a large share of rows; bounded like the 4-layer tiny encoder
        assert mx < 2e-2 and med < 1e-3, (mx, med)
        cross, state = ref.cross_kv(enc), ref.new_state()
        errs = []
        for pos, tok in enumerate(om.PROMPT[cfg.n_vocab] + [440, 9, 123, 4567]):
            logits, nxt = m.decode_step([tok], pos)
            errs.append(max_abs_rel(logits[0], ref.decode_step(tok, pos, cross, state)))
        assert max(errs) < FLIP and np.median(errs) < 1e-5, errs
        toks = m.transcribe([c, clips(2)[1]], n_new=8)
        assert toks.shape == (2, 8) and np.all((toks >= 0) & (toks < cfg.n_vocab))
    finally:
        m.close()
