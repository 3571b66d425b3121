"""GPU parity of SET_ROWS (KV write) and the first-max argmax, plus the
backend's status/poison/abort behaviour (cpu_graph.rs:7893-7935, :8380-8405)."""
import numpy as np
import pytest

import openasr_b200 as ob
from oracle import oracle as oo


@pytest.mark.gpu
def test_reference_kat_kv_cache_set_rows(gpu_backend):
    import torch

    # cpu_graph.rs:13950-14030 (set_rows part)
    cache = torch.zeros((1, 1, 4, 2), dtype=torch.float16, device="cuda")
    src = torch.tensor([1, 2, 3, 4], dtype=torch.float32, device="cuda").reshape(1, 1, 2, 2)
    rows = torch.tensor([0, 3], dtype=torch.int32, device="cuda")
    gpu_backend.set_rows(cache, src, rows)
    gpu_backend.synchronize()
    np.testing.assert_array_equal(cache.float().cpu().numpy().ravel(), [1, 2, 0, 0, 0, 0, 3, 4])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_set_rows_matches_oracle(gpu_backend, dtype):
    import torch

    rng = np.random.default_rng(11)
    D, R, n, S = 1280, 448, 3, 8
    tdt, ndt = (torch.float16, np.float16) if dtype == "f16" else (torch.float32, np.float32)
    cache = np.zeros((1, S, R, D), ndt)
    src = rng.normal(0, 3, (1, S, n, D)).astype(np.float32)
    rows = np.array([5, 0, 447], np.int64)
    ct = torch.from_numpy(cache.copy()).cuda()
    gpu_backend.set_rows(ct, torch.from_numpy(src).cuda(), torch.from_numpy(rows).cuda())
    gpu_backend.synchronize()
    oo.set_rows(cache, src, rows)
    np.testing.assert_array_equal(ct.cpu().numpy(), cache)


@pytest.mark.gpu
def test_argmax_first_matches_oracle(gpu_backend):
    import torch

    rng = np.random.default_rng(12)
    x = rng.normal(0, 1, (8, 151936)).astype(np.float32)
    x[1, [7, 9000, 151935]] = 50.0          # ties -> lowest index
    x[2, :] = -np.inf; x[2, 77] = np.nan    # no finite value -> 0
    x[3, 10] = np.inf; x[3, 11] = 40.0      # non-finite ignored
    x[4, [4095, 4096]] = 60.0               # tie across a 4096-entry chunk edge
    x[5, [300, 301, 4000]] = 61.0           # ties inside one chunk
    x[6, 151935] = 62.0                     # max in the ragged last chunk
    x[7, :] = 1.0                           # all equal -> 0
    out = torch.empty(8, dtype=torch.int32, device="cuda")
    gpu_backend.argmax_first(torch.from_numpy(x).cuda(), out)
    gpu_backend.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oo.argmax_first(x))


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(3, 100), (2, 4096), (5, 4097), (1, 8191), (9, 51866), (2, 300000)])
def test_argmax_first_row_lengths(gpu_backend, shape):
    """Row lengths on both sides of the one-CTA / chunked boundary (4096 entries)."""
    import torch

    rng = np.random.default_rng(shape[1])
    x = rng.normal(0, 1, shape).astype(np.float32)
    x[:, rng.integers(0, shape[1], 4)] = 9.0  # shared ties in every row
    out = torch.empty(shape[0], dtype=torch.int32, device="cuda")
    gpu_backend.argmax_first(torch.from_numpy(x).cuda(), out)
    gpu_backend.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oo.argmax_first(x))


@pytest.mark.gpu
def test_out_of_range_row_index_is_an_execution_failure(gpu_backend):
    import torch

    cache = torch.zeros((1, 1, 4, 64), dtype=torch.float16, device="cuda")
    src = torch.ones((1, 1, 1, 64), dtype=torch.float32, device="cuda")
    bad = torch.tensor([4], dtype=torch.int32, device="cuda")  # checked in-kernel, no access
    gpu_backend.set_rows(cache, src, bad)
    with pytest.raises(ob.backend.ExecutionFailed):
        gpu_backend.synchronize()
    assert torch.count_nonzero(cache).item() == 0
    gpu_backend.synchronize()  # the error word is consumed; the backend stays usable


@pytest.mark.gpu
def test_abort_callback_returns_aborted(gpu_backend):
    import torch

    flag = {"abort": True}
    gpu_backend.set_abort_callback(lambda: flag["abort"])
    x = torch.zeros((8, 4), device="cuda")
    out = torch.zeros(8, dtype=torch.int32, device="cuda")
    with pytest.raises(ob.backend.Aborted):
        gpu_backend.argmax_first(x, out)
    flag["abort"] = False
    gpu_backend.argmax_first(x, out)
    gpu_backend.set_abort_callback(None)
    gpu_backend.synchronize()


@pytest.mark.gpu
def test_abort_predicate_is_the_references_bool_callback(gpu_backend):
    """ggml_abort_callback is extern "C" fn(*mut c_void) -> bool (ffi.rs:334-336): a
    callback of exactly that C type, passed straight to the C ABI, aborts the next
    enqueue while it returns true and lets it through once it returns false."""
    import ctypes

    import torch

    state = ctypes.c_bool(True)
    cb = ctypes.CFUNCTYPE(ctypes.c_bool, ctypes.c_void_p)(lambda data: ctypes.c_bool.from_address(data).value)
    L = ob.lib()
    assert L.oasr_b200_set_abort_callback(gpu_backend.handle, cb, ctypes.addressof(state)) == 0
    x = torch.zeros((4, 4), device="cuda")
    out = torch.zeros(4, dtype=torch.int32, device="cuda")
    tx, to = ob.describe(x), ob.describe(out)
    assert L.oasr_b200_argmax_first(gpu_backend.handle, ctypes.byref(tx), ctypes.byref(to)) == ob.backend.STATUS_ABORTED
    state.value = False
    assert L.oasr_b200_argmax_first(gpu_backend.handle, ctypes.byref(tx), ctypes.byref(to)) == 0
    assert L.oasr_b200_set_abort_callback(gpu_backend.handle, ob.backend.ABORT_CB(0), None) == 0
    gpu_backend.synchronize()


@pytest.mark.gpu
def test_synchronize_ex_reports_a_valid_cancel_capability(gpu_backend):
    """The merged status comes with the cancel-capability pair the reference host
    validates (cpu_graph.rs:7974-8002): native cancellation observed at submission
    checkpoints."""
    rc, cap = gpu_backend.synchronize_ex()
    assert rc == 0
    assert (cap.mechanism, cap.observation_granularity) == (ob.backend.CANCEL_NATIVE,
                                                           ob.backend.CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT)
    assert ob.backend.valid_cancel_capability(rc, cap)


@pytest.mark.gpu
def test_bounded_pipeline_wait_times_out_cleanly(gpu_backend):
    """A kernel whose mbarrier never completes gives up after its bound, records the
    timeout in the device error word and returns: the call reports EXECUTION_FAILED
    with a timeout message, and the backend keeps working (no device fault, no poison)."""
    import torch

    L = ob.lib()
    rc = L.oasr_b200_selftest_bounded_wait(gpu_backend.handle, 1 << 22)
    assert rc == ob.backend.STATUS_EXECUTION_FAILED
    assert "timed out" in L.oasr_b200_last_error(gpu_backend.handle).decode()
    rc, cap = gpu_backend.synchronize_ex()
    assert rc == 0 and ob.backend.valid_cancel_capability(rc, cap)
    x = torch.tensor([[1.0, 3.0, 3.0, 2.0]], device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    gpu_backend.argmax_first(x, out)
    gpu_backend.synchronize()
    assert out.item() == 1
    assert L.oasr_b200_selftest_bounded_wait(gpu_backend.handle, 0) == ob.backend.STATUS_FAILED  # bound out of range


@pytest.mark.gpu
def test_props_and_mem_stats(gpu_backend):
    p = gpu_backend.props()
    assert p["name"] == "CUDA0" and p["device_type"] == 1 and p["cc_major"] == 10
    assert p["sm_count"] >= 100
    s = gpu_backend.mem_stats()
    assert s["scratch_bytes"] > 0 and s["device_total"] > 100 * 2**30
