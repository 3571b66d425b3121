"""CPU checks of the memory API v1 table (ggml_backend_memory_get_api_v1,
crates/openasr-core/src/ggml_runtime/ffi.rs:144-333): the fixed-width layouts the
reference's host asserts (backend_memory.rs:697-704), the table header, and the
argument validation that rejects bad handles and requests before touching any
backend.  No device work."""
import ctypes

import pytest

from openasr_b200 import backend as bk


def test_layouts_match_the_v1_fixed_width_contract():
    assert ctypes.sizeof(bk.MemDomainId) == 24
    assert ctypes.sizeof(bk.MemRequest) == 88
    assert ctypes.sizeof(bk.MemClaim) == 96
    assert ctypes.sizeof(bk.MemQuote) == 48
    assert ctypes.sizeof(bk.MemStats) == 152
    assert ctypes.sizeof(bk.MemoryApiV1) == 64


def test_table_header_and_entry_points():
    api = bk.memory_api()
    assert api.struct_size == 64 and api.abi_version == bk.MEMORY_ABI_V1
    for f in ("get_domains", "quote", "reserve_private", "get_stats", "trim", "quarantine"):
        assert getattr(api, f), f
    # a static table: the same address every call
    assert ctypes.addressof(bk.memory_api()) == ctypes.addressof(api)


def test_null_handles_fail_cleanly():
    api = bk.memory_api()
    n = ctypes.c_uint32(0)
    assert api.get_domains(None, None, ctypes.byref(n)) == bk.STATUS_FAILED
    assert api.get_stats(None, None, None, ctypes.byref(n)) == bk.STATUS_FAILED
    assert api.trim(None, 0) == bk.STATUS_FAILED
    assert api.quarantine(None, None) == bk.STATUS_FAILED


def _request(kind, backend, size=ctypes.sizeof(bk.MemRequest)):
    r = bk.MemRequest()
    r.struct_size, r.kind, r.backend, r.requested_bytes = size, kind, backend, 1 << 20
    return r


def _quote(requests):
    api = bk.memory_api()
    arr = (bk.MemRequest * max(len(requests), 1))(*requests)
    q = bk.MemQuote()
    q.struct_size = ctypes.sizeof(bk.MemQuote)
    n = ctypes.c_uint32(0)
    return api.quote(arr, len(requests), ctypes.byref(q), None, ctypes.byref(n)), q, n.value


def test_empty_quote_and_reservation():
    api = bk.memory_api()
    rc, q, n = _quote([])
    assert rc == bk.STATUS_SUCCESS and n == 0 and q.struct_size == 48
    m = ctypes.c_uint32(7)
    assert api.reserve_private(None, 0, ctypes.byref(q), None, ctypes.byref(m)) == bk.STATUS_SUCCESS
    assert m.value == 0


@pytest.mark.parametrize("case", ["short_struct", "bad_kind", "no_backend", "two_backends"])
def test_malformed_requests_are_refused_before_any_backend_access(case):
    # the backend addresses below are never dereferenced: validation fails first
    fake_a, fake_b = 0x1000, 0x2000
    reqs = {
        "short_struct": [_request(bk.REQUEST_GRAPH_PRIVATE, fake_a, size=40)],
        "bad_kind": [_request(9, fake_a)],
        "no_backend": [_request(bk.REQUEST_BUFFER, None)],
        "two_backends": [_request(bk.REQUEST_BUFFER, fake_a), _request(bk.REQUEST_BUFFER, fake_b)],
    }[case]
    rc, _, _ = _quote(reqs)
    assert rc == bk.STATUS_FAILED


def test_quote_needs_a_sized_quote_struct():
    api = bk.memory_api()
    q = bk.MemQuote()  # struct_size 0
    n = ctypes.c_uint32(0)
    assert api.quote(None, 0, ctypes.byref(q), None, ctypes.byref(n)) == bk.STATUS_FAILED
