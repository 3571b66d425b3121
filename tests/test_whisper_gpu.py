"""Model-level parity of the Whisper driver (oasr_b200_whisper_*) against the
CPU reference graphs in oracle/whisper_ref.py, on seeded synthetic packs
(BASELINE.json configs[0] whisper-tiny shape, and the whisper-large-v3 shape at
reduced depth).  The encoder attention is checked against the oracle's
tensor-core arithmetic mode (fp16 operands), everything else against ggml CPU
semantics; op-level tolerance stays north_star's max-abs-rel 2e-3."""
import numpy as np
import pytest

import openasr_b200 as ob
from openasr_b200 import models as om
from oracle import oracle as oo
from oracle import whisper_ref as wr
from tests.conftest import max_abs_rel

TOL = 2e-3


@pytest.fixture(scope="module")
def tiny():
    cfg = om.WHISPER_TINY.replace(max_batch=4)
    pack = om.whisper_synthetic_pack(cfg, seed=0x0A5A0001)
    return cfg, pack


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
        ref = wr.log_mel(c, 80)
        assert np.abs(got[i] - ref).max() < 2e-4


@pytest.mark.gpu
def test_tiny_encoder_and_cross_kv_match_reference(tiny_model, tiny):
    cfg, pack = tiny
    mel = wr.log_mel(clips(1)[0], 80)
    enc = tiny_model.encode(mel[None], 1)[0]
    ref = wr.WhisperRef(cfg, pack)
    enc_ref = ref.encode(mel)
    assert max_abs_rel(enc, enc_ref) < TOL


@pytest.mark.gpu
def test_tiny_decoder_steps_match_reference_teacher_forced(tiny_model, tiny):
    cfg, pack = tiny
    mel = wr.log_mel(clips(1)[0], 80)
    enc = tiny_model.encode(mel[None], 1)[0]
    ref = wr.WhisperRef(cfg, pack)
    cross = ref.cross_kv(enc)  # same encoder output on both sides: isolates the decoder
    state = ref.new_state()
    tokens = om.PROMPT[cfg.n_vocab] + [11, 2000, 51000, 7]
    for pos, tok in enumerate(tokens):
        logits, nxt = tiny_model.decode_step([tok], pos)
        lr = ref.decode_step(tok, pos, cross, state)
        assert max_abs_rel(logits[0], lr) < 1e-4, pos
        top2 = np.sort(lr)[-2:]
        if top2[1] - top2[0] > 1e-3:
            assert nxt[0] == oo.argmax_first(lr)[0]


@pytest.mark.gpu
def test_tiny_greedy_transcript_matches_reference(tiny_model, tiny):
    """30 s of -20 dBFS noise, greedy 224 tokens, batch 1."""
    cfg, pack = tiny
    c = clips(1)[0]
    got = tiny_model.transcribe([c], n_new=224)[0]
    ref = wr.WhisperRef(cfg, pack)
    enc = ref.encode(wr.log_mel(c, 80))
    toks, logits = ref.greedy(ref.cross_kv(enc), om.PROMPT[cfg.n_vocab], 224)
    if not np.array_equal(got, toks):
        i = int(np.argmax(got != toks))
        top2 = np.sort(logits[i])[-2:]
        pytest.fail(f"first divergence at step {i}: gpu {got[i]} ref {toks[i]}, ref top-2 margin {top2[1]-top2[0]:.3g}")


@pytest.mark.gpu
def test_batched_transcripts_equal_serial(tiny_model):
    cs = clips(4)
    batched = tiny_model.transcribe(cs, n_new=32)
    for i, c in enumerate(cs):
        np.testing.assert_array_equal(batched[i], tiny_model.transcribe([c], n_new=32)[0])


@pytest.mark.gpu
def test_large_v3_shape_q4k_reduced_depth(gpu_backend):
    """configs[3] shape (d 1280, 20 heads, 128 mels, Q4_K linears) at 2+2 layers:
    exercises the tensor-core Q4_K GEMM, the fp16 conv GEMM and the tensor-core
    attention inside the encoder, and Q4_K GEMV decode."""
    cfg = om.WHISPER_LARGE_V3.replace(n_enc_layers=2, n_dec_layers=2, max_batch=2)
    pack = om.whisper_synthetic_pack(cfg, seed=0x0A5A0004)
    m = om.WhisperModel(gpu_backend, cfg, pack)
    try:
        c = clips(1)[0]
        mel = wr.log_mel(c, 128)
        enc = m.encode(mel[None], 1)[0]
        ref = wr.WhisperRef(cfg, pack)
        enc_ref = ref.encode(mel)
        assert max_abs_rel(enc, enc_ref) < TOL
        cross = ref.cross_kv(enc)
        state = ref.new_state()
        for pos, tok in enumerate(om.PROMPT[cfg.n_vocab] + [440, 9]):
            logits, _ = m.decode_step([tok], pos)
            assert max_abs_rel(logits[0], ref.decode_step(tok, pos, cross, state)) < 1e-4
        toks = m.transcribe([c, clips(2)[1]], n_new=8)
        assert toks.shape == (2, 8) and np.all((toks >= 0) & (toks < cfg.n_vocab))
    finally:
        m.close()
