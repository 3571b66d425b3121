"""The continuous-batching serve loop (oasr_b200_whisper_serve; the reference's
models/seq2seq_serve_batch.rs decode_continuous_batch) against serial
transcription: every request's tokens equal a batch-of-one
oasr_b200_whisper_transcribe of the same clip, cut at its budget or at its first
`eot`, through slot release and refill, power-of-two re-bucketing, compaction of
the active slots on a shrink, and a width cap.  A slot's decode never depends on
the batch it runs in (per-row block-order mul_mat, shape-only attention split
plans), so the comparison is exact."""
import numpy as np
import pytest

from openasr_b200 import models as om

SECONDS = (30.0, 7.5, 19.0, 5.0, 12.0, 26.0, 9.5, 2.0, 16.0)


@pytest.fixture(scope="module")
def model(gpu_backend):
    cfg = om.WHISPER_TINY.replace(max_batch=4)
    m = om.WhisperModel(gpu_backend, cfg, om.whisper_synthetic_pack(cfg, seed=0x0A5A0001))
    yield m
    m.close()


@pytest.fixture(scope="module")
def clips():
    return [om.synthetic_audio(0x0A5A2000 + i, int(16000 * s)) for i, s in enumerate(SECONDS)]


@pytest.fixture(scope="module")
def serial(model, clips):
    return [model.transcribe([c], n_new=40)[0] for c in clips]


def expected(serial, budgets, eot=None):
    out = []
    for s, b in zip(serial, budgets):
        t = s[:b]
        if eot is not None:
            hit = np.flatnonzero(t == eot)
            if hit.size:
                t = t[:hit[0] + 1]
        out.append(t)
    return out


def check(got, want):
    assert len(got) == len(want)
    for i, (g, w) in enumerate(zip(got, want)):
        np.testing.assert_array_equal(g, w, err_msg=f"request {i}")


@pytest.mark.gpu
def test_serve_equals_serial_with_refill_and_shrink(model, clips, serial):
    assert model.max_batch == 4
    budgets = [5, 40, 12, 20, 3, 27, 9, 33, 1]
    got, st = model.serve(clips, max_new=40, budgets=budgets, stop_at_eot=False, check_every=4)
    check(got, expected(serial, budgets))
    assert st.admissions > 1 and st.max_width == 4 and st.width_changes >= 1, (st.admissions, st.width_changes)


@pytest.mark.gpu
@pytest.mark.parametrize("check_every", [1, 3, 16])
def test_serve_independent_of_harvest_interval(model, clips, serial, check_every):
    budgets = [17, 2, 40, 8, 25, 11, 6, 30, 14]
    got, _ = model.serve(clips, max_new=40, budgets=budgets, stop_at_eot=False, check_every=check_every)
    check(got, expected(serial, budgets))


@pytest.mark.gpu
def test_serve_stops_at_eot(model, clips, serial):
    # a token the greedy path really emits stands in for the end-of-text id
    eot = int(serial[1][6])
    got, _ = model.serve(clips, max_new=40, stop_at_eot=True, eot=eot, check_every=2)
    want = expected(serial, [40] * len(clips), eot=eot)
    check(got, want)
    assert len(got[1]) <= 7 and got[1][-1] == eot


@pytest.mark.gpu
@pytest.mark.parametrize("max_width", [1, 2, 3])
def test_serve_width_cap(model, clips, serial, max_width):
    budgets = [9, 4, 15, 2, 11, 7, 13, 5, 8]
    got, st = model.serve(clips, max_new=40, budgets=budgets, stop_at_eot=False, max_width=max_width, check_every=2)
    check(got, expected(serial, budgets))
    assert st.max_width <= max_width


@pytest.mark.gpu
def test_serve_single_and_repeat(model, clips, serial):
    got, st = model.serve(clips[:1], max_new=40, stop_at_eot=False)
    check(got, [serial[0]])
    assert st.max_width == 1 and st.admissions == 1
    # a second call reuses the cached step graphs and starts from parked slots
    got, _ = model.serve(clips[3:6], max_new=40, budgets=[40, 3, 21], stop_at_eot=False)
    check(got, expected(serial[3:6], [40, 3, 21]))


@pytest.mark.gpu
def test_serve_rejects_bad_arguments(model, clips):
    from openasr_b200 import backend as bk

    with pytest.raises(bk.GgmlBackendError):
        model.serve(clips[:2], max_new=40, budgets=[0, 5])
    with pytest.raises(bk.GgmlBackendError):
        model.serve(clips[:2], max_new=448)


@pytest.mark.gpu
def test_serve_abort_between_steps_then_serve_again(gpu_backend, model, clips, serial):
    """The backend's abort callback (ggml_abort_callback) is polled before each group of
    serve steps: a predicate that turns true mid-serve ends the call with ABORTED, and
    the next serve call starts from parked slots and is exact."""
    from openasr_b200 import backend as bk

    calls = {"n": 0}

    def pred():
        calls["n"] += 1
        return calls["n"] >= 3  # the entry check and one group of steps pass

    gpu_backend.set_abort_callback(pred)
    try:
        with pytest.raises(bk.Aborted):
            model.serve(clips[:5], max_new=40, stop_at_eot=False, check_every=4)
    finally:
        gpu_backend.set_abort_callback(None)
    assert calls["n"] >= 3
    got, _ = model.serve(clips[:5], max_new=40, budgets=[7, 12, 3, 40, 9], stop_at_eot=False)
    check(got, expected(serial[:5], [7, 12, 3, 40, 9]))


@pytest.mark.gpu
def test_serve_large_v3_shape_equals_serial(gpu_backend):
    """The serve loop on the large-v3 shape (20 heads: the 4-head decode attention and the
    fused decoder GEMVs, Q4_K; 2 + 2 layers to keep it quick) at width 8 with refills and
    a shrink: every request equals its serial transcription."""
    cfg = om.WHISPER_LARGE_V3.replace(n_enc_layers=2, n_dec_layers=2, max_batch=8)
    m = om.WhisperModel(gpu_backend, cfg, om.whisper_synthetic_pack(cfg, seed=0x0A5A0004))
    try:
        cs = [om.synthetic_audio(0x0A5A2100 + i, int(16000 * (5 + 2.5 * i))) for i in range(11)]
        serial = [m.transcribe([c], n_new=24)[0] for c in cs]
        budgets = [24, 3, 17, 9, 24, 1, 12, 20, 6, 14, 24]
        got, st = m.serve(cs, max_new=24, budgets=budgets, stop_at_eot=False, check_every=4)
        check(got, expected(serial, budgets))
        assert st.max_width == 8 and st.admissions > 1
    finally:
        m.close()
