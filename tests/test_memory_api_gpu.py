"""The memory API v1 table on a device (ffi.rs:144-333; host protocol of
backend_memory.rs:193-390): domains, stats that follow the backend's own
allocations, quote -> reserve_private of the backend-private workspace and the
upload staging, stale-quote refusal, trim, and quarantine (host-side poisoning:
no device fault is involved)."""
import numpy as np
import pytest

import openasr_b200 as ob
from openasr_b200 import backend as bk
from oracle import oracle as oo


@pytest.fixture()
def fresh_backend():
    """A backend of its own (trim and quarantine change its state for good)."""
    import torch

    torch.cuda.init()
    be = ob.Backend(0)
    be.set_stream(torch.cuda.current_stream())
    yield be
    be.close()


def _stats(be):
    dev, pin = be.memory_stats()
    assert dev.domain.kind == bk.DOMAIN_DEVICE_LOCAL and pin.domain.kind == bk.DOMAIN_HOST_PINNED
    return dev, pin


@pytest.mark.gpu
def test_domains_name_the_device(fresh_backend):
    doms = fresh_backend.memory_domains()
    assert [d.id.kind for d in doms] == [bk.DOMAIN_DEVICE_LOCAL, bk.DOMAIN_HOST_PINNED]
    assert [d.id.heap_index for d in doms] == [0, 1]
    uuids = {bytes(d.id.physical_device_uuid) for d in doms}
    assert len(uuids) == 1 and uuids.pop() != bytes(16)
    assert all(d.struct_size == 80 and d.name for d in doms)


@pytest.mark.gpu
def test_stats_follow_uploads_and_frees(fresh_backend):
    be = fresh_backend
    dev0, pin0 = _stats(be)
    ms = be.mem_stats()
    assert dev0.total_bytes == ms["device_total"] and dev0.budget_bytes == dev0.total_bytes
    assert dev0.device_used_bytes + dev0.device_free_bytes == dev0.total_bytes
    assert pin0.flags & bk.STATS_BUDGET_UNAVAILABLE
    wq = oo.quantize(ob.Q8_0, oo.synth_normal(3, 512 * 1024, 0.0, 0.02).reshape(512, 1024))
    # the quote of this import bounds what the upload then adds to the device
    _, (dclaim, hclaim) = be.memory_quote([be.memory_request(bk.REQUEST_HOST_IMPORT, wq.nbytes, usage=1)])
    assert dclaim.domain.kind == bk.DOMAIN_DEVICE_LOCAL and hclaim.domain.kind == bk.DOMAIN_HOST_PINNED
    W = be.upload_weight(wq, ob.Q8_0, [1024, 512])
    dev1, pin1 = _stats(be)
    grown = dev1.backend_owned_live_bytes - dev0.backend_owned_live_bytes
    assert grown <= dclaim.retained_after_use_upper_bytes <= dclaim.commit_peak_extra_upper_bytes
    assert hclaim.committed_after_upper_bytes == pin1.backend_owned_live_bytes
    assert dev1.generation > dev0.generation
    assert dev1.allocation_count > dev0.allocation_count
    assert dev1.backend_owned_live_bytes - dev0.backend_owned_live_bytes == be.mem_stats()["weight_bytes"]
    assert pin1.backend_owned_live_bytes == 2 * (16 << 20)  # the staging buffers now exist
    assert dev1.backend_owned_high_water_bytes >= dev1.backend_owned_live_bytes + dev1.backend_owned_workspace_bytes
    W.free()
    dev2, _ = _stats(be)
    assert dev2.generation > dev1.generation and dev2.backend_owned_live_bytes == dev0.backend_owned_live_bytes
    assert dev2.health == bk.MEMORY_HEALTHY


@pytest.mark.gpu
def test_quote_then_reserve_private_grows_the_workspace(fresh_backend):
    be = fresh_backend
    dev0, _ = _stats(be)
    want = dev0.backend_owned_workspace_bytes + (96 << 20)
    reqs = [be.memory_request(bk.REQUEST_GRAPH_PRIVATE, want, request_id=11, usage=2),
            be.memory_request(bk.REQUEST_TRANSFER, 1 << 20, request_id=12),
            be.memory_request(bk.REQUEST_BUFFER, 5 << 20, request_id=13, usage=1)]
    q, claims = be.memory_quote(reqs)
    assert q.stats_generation == dev0.generation and q.quote_token > 0
    assert [c.request_id for c in claims] == [11, 12, 13]
    gp, tr, buf = claims
    assert gp.domain.kind == bk.DOMAIN_DEVICE_LOCAL and gp.commit_peak_extra_upper_bytes >= want - dev0.backend_owned_workspace_bytes
    assert tr.domain.kind == bk.DOMAIN_HOST_PINNED
    assert buf.flags & bk.CLAIM_CONSERVATIVE_UPPER and buf.commit_peak_extra_upper_bytes >= 5 << 20
    # the sizing query commits nothing
    assert be.memory_reserve_private(reqs, q, sizing_only=True) == 2
    assert _stats(be)[0].generation == dev0.generation
    actual = be.memory_reserve_private(reqs, q)
    assert [c.request_id for c in actual] == [11, 12] and all(c.flags & bk.CLAIM_EXACT for c in actual)
    dev1, pin1 = _stats(be)
    assert dev1.backend_owned_workspace_bytes >= want
    assert actual[0].committed_after_upper_bytes - actual[0].committed_before_bytes == \
        dev1.backend_owned_workspace_bytes - dev0.backend_owned_workspace_bytes
    assert pin1.backend_owned_live_bytes == 2 * (16 << 20)
    # a spent quote is refused, as is one made stale by an allocation in between
    with pytest.raises(ob.GgmlBackendError, match="stale"):
        be.memory_reserve_private(reqs, q)
    q2, _ = be.memory_quote(reqs[:1])
    W = be.upload_weight(oo.quantize(ob.Q8_0, oo.synth_normal(4, 64 * 256, 0.0, 0.02).reshape(64, 256)), ob.Q8_0,
                         [256, 64])
    with pytest.raises(ob.GgmlBackendError, match="stale"):
        be.memory_reserve_private(reqs[:1], q2)
    W.free()
    # a quote for other requests is refused too
    q3, _ = be.memory_quote(reqs[:1])
    with pytest.raises(ob.GgmlBackendError, match="stale"):
        be.memory_reserve_private(reqs[1:2], q3)


@pytest.mark.gpu
def test_trim_releases_workspace_and_staging_and_ops_still_run(fresh_backend):
    import torch

    be = fresh_backend
    be.reserve_scratch(64 << 20)
    K, N = 1024, 256
    wq = oo.quantize(ob.Q8_0, oo.synth_normal(5, N * K, 0.0, 0.02).reshape(N, K))
    W = be.upload_weight(wq, ob.Q8_0, [K, N])
    be.memory_trim()
    dev, pin = _stats(be)
    assert dev.backend_owned_workspace_bytes == 0 and pin.backend_owned_live_bytes == 0
    x = oo.synth_normal(6, 32 * K, 0.0, 1.0).reshape(32, K)
    out = torch.empty((32, N), dtype=torch.float32, device="cuda")
    be.mul_mat(W, torch.from_numpy(x).cuda(), out)
    be.synchronize()
    ref = oo.mul_mat(wq, ob.Q8_0, K, N, x)
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-5 * np.abs(ref).max()
    assert _stats(be)[0].backend_owned_workspace_bytes > 0  # the scratch grew back
    W.free()


@pytest.mark.gpu
def test_quarantine_poisons_the_backend(fresh_backend):
    be = fresh_backend
    be.memory_quarantine(bk.STATUS_EXECUTION_FAILED, "host saw a failed commit", native_error=77)
    dev, pin = _stats(be)
    assert dev.health == bk.MEMORY_QUARANTINED and dev.quarantine_generation == 1
    assert dev.last_ggml_status == bk.STATUS_BACKEND_POISONED and dev.last_native_error == 77
    with pytest.raises(ob.backend.BackendPoisoned):
        be.reserve_scratch(1 << 20)
    W = None
    with pytest.raises(ob.backend.BackendPoisoned):
        W = be.upload_weight(np.zeros((64, 272), np.uint8), ob.Q8_0, [256, 64])
    assert W is None
    # trim still releases memory on a quarantined backend
    be.memory_trim()


@pytest.mark.gpu
def test_model_drivers_recover_after_trim(fresh_backend):
    """trim releases the scratch that the drivers' captured decode steps point into:
    the next generation reserves it again before re-capturing (scratch cannot grow
    during a capture) and gives the same tokens."""
    from openasr_b200 import models as om

    be = fresh_backend
    wcfg = om.WHISPER_TINY.replace(max_batch=2)
    wm = om.WhisperModel(be, wcfg, om.whisper_synthetic_pack(wcfg, seed=0x0A5A0001))
    qcfg = om.QWEN3_ASR_0_6B.replace(n_layers=1, n_vocab=4096, max_pos=256, max_prefill=64, max_batch=2)
    qm = om.QwenModel(be, qcfg, om.qwen_synthetic_pack(qcfg, seed=0x0A5A0003))
    try:
        clip = [om.synthetic_audio(0x0A5A1000, 16000 * 8)]
        emb = om.qwen_synthetic_prefix(0x0A5A3000, 2, 40, qcfg.d_model)
        w_before, q_before = wm.transcribe(clip, n_new=12), qm.generate(emb, n_new=12)
        be.memory_trim()
        assert _stats(be)[0].backend_owned_workspace_bytes == 0
        w_after, q_after = wm.transcribe(clip, n_new=12), qm.generate(emb, n_new=12)
        np.testing.assert_array_equal(w_before, w_after)
        np.testing.assert_array_equal(q_before, q_after)
    finally:
        qm.close()
        wm.close()



@pytest.mark.gpu
def test_trim_during_stream_capture_is_refused(fresh_backend):
    """A trim while the backend's stream is being captured would synchronize inside the
    capture and invalidate it: it fails, releases nothing, and the capture completes."""
    import torch

    be = fresh_backend
    be.reserve_scratch(32 << 20)
    s = torch.cuda.Stream()
    be.set_stream(s)
    before = _stats(be)[0].backend_owned_workspace_bytes
    x = torch.zeros(16, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        x.add_(1.0)
        rc = bk.memory_api().trim(be.handle, 0)
    assert rc == bk.STATUS_FAILED
    g.replay()
    torch.cuda.synchronize()
    assert x[0].item() == 1.0
    assert _stats(be)[0].backend_owned_workspace_bytes == before
    be.set_stream(torch.cuda.current_stream())
