"""oasr_b200_flash_attn_ext_static: the allocation-free attention entry point.

Hosts that reserve all device memory up front (or cannot afford a
synchronising cudaMalloc inside a real-time decode loop) call this variant: it
runs the split-KV kernels over a file-scope device array instead of the
backend's growable scratch.  Its results must equal oasr_b200_flash_attn_ext
bit for bit on the shapes that entry point also runs through the split-KV
kernels, on consecutive calls (the per-group tickets must be back at zero after
each call), and it must leave the backend's scratch untouched.  This file is
collected last so that it also runs after every other GPU test."""
import os
import subprocess
import sys

import numpy as np
import pytest

import openasr_b200 as ob
from tests.conftest import ROOT

STATIC_PARTIAL_BYTES = 4 << 20


def _inputs(seed, S, H, HKV, NQ, NKV, D, masked):
    import torch

    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.normal(0, 1, (S, H, NQ, D)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.normal(0, 1, (S, HKV, NKV, D)).astype(np.float16)).cuda()
    v = torch.from_numpy(rng.normal(0, 1, (S, HKV, NKV, D)).astype(np.float16)).cuda()
    mask = None
    if masked:
        m = np.zeros((S, 1, NQ, NKV), np.float16)
        for s in range(S):
            m[s, 0, :, rng.integers(1, NKV + 1):] = -np.inf
        mask = torch.from_numpy(m).cuda()
    return q, k, v, mask


def _out(S, H, NQ, D):
    import torch

    return torch.full((S, NQ, H, D), float("nan"), dtype=torch.float32, device="cuda")


# whisper decode self/cross attention, GQA decode with a causal mask, D = 128
SHAPES = [
    (8, 20, 20, 1, 1500, 64, False),
    (1, 20, 20, 1, 37, 64, False),
    (4, 16, 8, 1, 391, 128, True),
    (2, 16, 8, 3, 2048, 128, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES)
def test_static_equals_ext_on_consecutive_calls(gpu_backend, shape):
    S, H, HKV, NQ, NKV, D, masked = shape
    be = gpu_backend
    scale = 1.0 / np.sqrt(D)
    before = be.mem_stats()["scratch_bytes"]
    for call in range(2):
        q, k, v, mask = _inputs(7000 + 31 * call + NKV, S, H, HKV, NQ, NKV, D, masked)
        ref, got = _out(S, H, NQ, D), _out(S, H, NQ, D)
        be.flash_attn_ext(q, k, v, mask, scale, ref)
        be.flash_attn_ext_static(q, k, v, mask, scale, got)
        be.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}: non-finite output"
        assert np.array_equal(r.view(np.uint32), g.view(np.uint32)), \
            f"call {call}: max diff {np.abs(r - g).max()}"
    assert be.mem_stats()["scratch_bytes"] == before


@pytest.mark.gpu
def test_static_fresh_backend_never_grows_scratch():
    import torch

    be = ob.Backend(0)
    try:
        be.set_stream(torch.cuda.current_stream())
        before = be.mem_stats()["scratch_bytes"]
        q, k, v, _ = _inputs(11, 8, 20, 20, 1, 1500, 64, False)
        outs = [_out(8, 20, 1, 64) for _ in range(2)]
        for o in outs:
            be.flash_attn_ext_static(q, k, v, None, 0.125, o)
        be.synchronize()
        assert torch.equal(outs[0], outs[1])
        assert be.mem_stats()["scratch_bytes"] == before
    finally:
        be.close()


@pytest.mark.gpu
def test_static_rejects_oversize_split():
    """Largest split grid on this device: groups = 4 * SMs - 1 split in two at D = 128
    needs more partials than the static array holds; the call must fail cleanly and
    the backend must keep working."""
    import torch

    be = ob.Backend(0)
    try:
        be.set_stream(torch.cuda.current_stream())
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        groups = 4 * sms - 1
        H, D, NKV = 8, 128, 256
        NQ = groups  # one kv head, one sequence, 8 query rows per tile -> groups tiles
        need = 1 * H * NQ * 2 * (D + 2) * 4
        q, k, v, _ = _inputs(12, 1, H, 1, NQ, NKV, D, False)
        out = _out(1, H, NQ, D)
        if need > STATIC_PARTIAL_BYTES:
            with pytest.raises(ob.GgmlBackendError) as ei:
                be.flash_attn_ext_static(q, k, v, None, 0.088, out)
            assert "static scratch holds" in str(ei.value)
            assert torch.isnan(out).all()  # nothing was launched
        # the same backend still serves a shape that fits
        q2, k2, v2, _ = _inputs(13, 8, 20, 20, 1, 1500, 64, False)
        ref, got = _out(8, 20, 1, 64), _out(8, 20, 1, 64)
        be.flash_attn_ext(q2, k2, v2, None, 0.125, ref)
        be.flash_attn_ext_static(q2, k2, v2, None, 0.125, got)
        be.synchronize()
        assert torch.equal(ref, got)
    finally:
        be.close()


_CAPTURE_CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import openasr_b200 as ob
be = ob.Backend(0)
s = torch.cuda.Stream()
be.set_stream(s)
q = torch.randn(1, 20, 1, 64, device="cuda")
k = torch.randn(1, 20, 64, 64, device="cuda").half()
v = torch.randn(1, 20, 64, 64, device="cuda").half()
o = torch.empty(1, 1, 20, 64, device="cuda")
torch.cuda.synchronize()
g = torch.cuda.CUDAGraph()
refused = ""
with torch.cuda.graph(g, stream=s):
    try:
        be.flash_attn_ext_static(q, k, v, None, 0.125, o)
    except ob.GgmlBackendError as e:
        refused = str(e)
print("REFUSED" if "precede stream capture" in refused else "NOT REFUSED: " + refused)
be.close()
"""


@pytest.mark.gpu
def test_static_first_call_inside_capture_is_refused():
    """A fresh process whose first static call is made during stream capture gets a
    clear refusal instead of a symbol lookup inside the capture."""
    r = subprocess.run([sys.executable, "-c", _CAPTURE_CHILD, ROOT], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ))
    assert r.returncode == 0, r.stderr[-2000:]
    assert "REFUSED" in r.stdout and "NOT REFUSED" not in r.stdout, r.stdout + r.stderr[-2000:]
