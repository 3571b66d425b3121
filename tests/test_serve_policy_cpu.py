"""The serving scheduler's width rules through the C ABI (host-only functions, no
GPU): the power-of-two bucket width (serve_batch_bucket_width, models/
serve_batch_env.rs:317-325) and the VRAM cap (serve_batch_vram_cap_decision_for_
memory, serve_batch_env.rs:501-522), checked on the cases of the reference's own
unit tests (serve_batch_env.rs:961-969, 611-618, 846-856) and exhaustively against
a restatement of the rule."""
import pytest

from openasr_b200 import backend as bk

MIB = 1 << 20


@pytest.fixture(scope="module")
def lib():
    return bk.lib()


def test_bucket_width_reference_cases(lib):
    w = lib.oasr_b200_serve_batch_width
    assert [w(0, 8), w(1, 8), w(2, 8), w(3, 8), w(5, 8), w(3, 3), w(4, 3)] == [0, 1, 2, 4, 8, 3, 4]


def test_bucket_width_rule_exhaustive(lib):
    for mx in range(1, 17):
        for active in range(0, 18):
            if active <= 1 or mx <= active:
                want = active
            else:
                p = 1
                while p < active:
                    p <<= 1
                want = max(min(p, mx), active)
            assert lib.oasr_b200_serve_batch_width(active, mx) == want, (active, mx)
    # the widths a max batch of 8 ever runs: the graph set {1, 2, 4, 8}
    assert {lib.oasr_b200_serve_batch_width(a, 8) for a in range(1, 9)} == {1, 2, 4, 8}


def test_vram_cap_reference_cases(lib):
    cap = lib.oasr_b200_serve_batch_vram_cap
    assert cap(8, 512 * MIB, 1024 * MIB, 1024 * MIB) == 1  # nothing usable: never below one slot
    assert cap(8, 512, 4096, 1024) == 6
    assert cap(8, 512, 1500, 1024) == 1
    assert cap(2, 512, 1500, 1024) == 1


def test_vram_cap_rule(lib):
    cap = lib.oasr_b200_serve_batch_vram_cap
    assert cap(8, 0, 0, 0) == 8                   # no slot estimate: request kept
    assert cap(1, 1 << 40, 0, 0) == 1             # a single slot is never capped
    assert cap(8, 1 << 30, 100 << 30, 1 << 30) == 8
    for req in (2, 3, 8):
        for free in (0, 1000, 5000, 9000, 1 << 20):
            usable = max(free - 1024, 0)
            assert cap(req, 1000, free, 1024) == max(1, min(req, usable // 1000)), (req, free)
