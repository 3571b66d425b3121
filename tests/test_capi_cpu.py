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
