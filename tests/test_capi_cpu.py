"""CPU-only checks of the C-ABI library: it loads, exports every symbol that
include/oasr_b200.h declares, and its host-side helpers (ggml_quantize_chunk,
row sizes, synthetic data) agree bit-for-bit with the oracle and the gguf
golden vectors.  No device work."""
import os
import re

import numpy as np
import pytest

import openasr_b200 as ob
from openasr_b200 import backend as bk
from oracle import oracle as oo

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = np.load(os.path.join(ROOT, "tests", "golden", "blockfmt_gguf.npz"))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "oasr_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(oasr_b200_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = ob.lib()
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), f"liboasr_b200.so does not export {s}"
    # the Python binding declares a signature for each of them
    assert sorted(bk.SIGNATURES) == syms


def test_no_device_means_clean_failure():
    if ob.device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(ob.GgmlBackendError):
        ob.Backend(0)


@pytest.mark.parametrize("qt,name", [(ob.Q8_0, "q8_0"), (ob.Q4_0, "q4_0")])
def test_quantize_chunk_matches_gguf_golden(qt, name):
    np.testing.assert_array_equal(ob.quantize(qt, GOLD["x"]), GOLD[f"{name}_bytes"])


@pytest.mark.parametrize("qt", [ob.Q8_0, ob.Q4_0, ob.Q4_K, ob.F16])
def test_quantize_chunk_matches_oracle(qt):
    x = oo.synth_normal(0x0A5A0003, 6 * 2048, 0.0, 0.02).reshape(6, 2048)
    x[0, :256] = 0.0
    if qt == ob.F16:
        np.testing.assert_array_equal(ob.quantize(qt, x).view(np.float16), x.astype(np.float16))
    else:
        np.testing.assert_array_equal(ob.quantize(qt, x), oo.quantize(qt, x))


def test_row_size_matches_ggml_block_sizes():
    assert ob.row_size(ob.Q8_0, 1024) == 1088
    assert ob.row_size(ob.Q4_0, 1024) == 576
    assert ob.row_size(ob.Q4_K, 1024) == 576
    assert ob.row_size(ob.F16, 7) == 14
    assert ob.row_size(ob.Q4_K, 1000) == -1
    with pytest.raises(ob.GgmlBackendError):
        ob.quantize(ob.Q8_0, np.zeros((1, 33), np.float32))


def test_synth_normal_matches_oracle_stream():
    np.testing.assert_array_equal(ob.synth_normal(0x0A5A0001, 12345, 0.0, 0.02),
                                  oo.synth_normal(0x0A5A0001, 12345, 0.0, 0.02))
    np.testing.assert_array_equal(ob.synth_normal(3, 100, offset=77), oo.synth_normal(3, 177)[77:])


def test_proc_address_resolves_every_entry_point():
    """ggml_backend_reg_get_proc_address-style lookup (ffi.rs:599): each header function
    under its own name, the memory API under its ggml name, NULL otherwise."""
    import ctypes

    L = ob.lib()
    for s in header_symbols():
        addr = L.oasr_b200_get_proc_address(s.encode())
        assert addr and addr == ctypes.cast(getattr(L, s), ctypes.c_void_p).value, s
    assert L.oasr_b200_get_proc_address(b"ggml_backend_memory_get_api_v1") == \
        ctypes.cast(L.oasr_b200_memory_get_api_v1, ctypes.c_void_p).value
    assert not L.oasr_b200_get_proc_address(b"ggml_backend_no_such_entry")
    assert not L.oasr_b200_get_proc_address(None)


def test_abort_callback_has_the_references_bool_type():
    """ggml_abort_callback returns bool (ffi.rs:334-336); the binding passes exactly that type."""
    import ctypes

    text = open(os.path.join(ROOT, "include", "oasr_b200.h")).read()
    assert re.search(r"typedef\s+bool\s*\(\*oasr_abort_callback\)\(void \*data\);", text)
    assert bk.ABORT_CB._restype_ is ctypes.c_bool and bk.ABORT_CB._argtypes_ == (ctypes.c_void_p,)


def test_synchronize_ex_without_a_backend():
    """A NULL backend fails, reporting the DISABLED / NONE cancel pair, which the
    reference host accepts with a failure status (cpu_graph.rs:7974-8002)."""
    import ctypes

    cap = bk.CancelCapability(99, 99)
    rc = ob.lib().oasr_b200_synchronize_ex(None, ctypes.byref(cap))
    assert rc == bk.STATUS_FAILED
    assert (cap.mechanism, cap.observation_granularity) == (bk.CANCEL_DISABLED, bk.CANCEL_OBSERVATION_NONE)
    assert bk.valid_cancel_capability(rc, cap)
    # the validator itself follows the reference's table
    assert not bk.valid_cancel_capability(0, bk.CancelCapability(bk.CANCEL_DISABLED, bk.CANCEL_OBSERVATION_NONE))
    assert not bk.valid_cancel_capability(0, bk.CancelCapability(bk.CANCEL_NATIVE, bk.CANCEL_OBSERVATION_NONE))
    assert bk.valid_cancel_capability(0, bk.CancelCapability(bk.CANCEL_SEGMENTED, bk.CANCEL_OBSERVATION_GRAPH_COMPLETION))
