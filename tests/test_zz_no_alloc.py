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


def _heads_inputs(seed, S, H, NKV):
    """Whisper decoder layout: one query per head, heads contiguous in a KV row ([seq][pos][H][64])
    -- the 4-head decode kernel"""
    import torch

    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.normal(0, 1, (S, H, 1, 64)).astype(np.float32)).cuda()
    kv = torch.from_numpy(rng.normal(0, 1, (S, NKV, 2, H, 64)).astype(np.float16)).cuda()
    return q, kv[:, :, 0].permute(0, 2, 1, 3), kv[:, :, 1].permute(0, 2, 1, 3), None


def _gqa_inputs(seed, S, H, HKV, NKV):
    """Qwen decoder layout: head-major f16 caches [seq][kv head][pos][128] viewed to the live
    prefix, one query row, no mask -- the GQA decode kernel"""
    import torch

    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.normal(0, 1, (S, H, 1, 128)).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.normal(0, 1, (S, HKV, 2048, 128)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.normal(0, 1, (S, HKV, 2048, 128)).astype(np.float16)).cuda()
    return q, kc[:, :, :NKV], vc[:, :, :NKV], None


def _out(S, H, NQ, D):
    import torch

    return torch.full((S, NQ, H, D), float("nan"), dtype=torch.float32, device="cuda")


# (layout, S, H, HKV, NQ, NKV, D, masked): the generic split-KV kernel (contiguous K/V,
# masks, query tiles), the 4-head kernel (Whisper self / cross caches) and the GQA kernel
# (Qwen caches, G = 1, 2, 4)
SHAPES = [
    ("split", 8, 20, 20, 1, 1500, 64, False),
    ("split", 1, 20, 20, 1, 37, 64, False),
    ("split", 4, 16, 8, 1, 391, 128, True),
    ("split", 2, 16, 8, 3, 2048, 128, True),
    ("heads", 8, 20, 20, 1, 1500, 64, False),
    ("heads", 3, 20, 20, 1, 448, 64, False),
    ("gqa", 8, 8, 8, 1, 646, 128, False),
    ("gqa", 4, 16, 8, 1, 391, 128, False),
    ("gqa", 2, 32, 8, 1, 2048, 128, False),
]


def _make(layout, seed, S, H, HKV, NQ, NKV, D, masked):
    if layout == "heads":
        return _heads_inputs(seed, S, H, NKV)
    if layout == "gqa":
        return _gqa_inputs(seed, S, H, HKV, NKV)
    return _inputs(seed, S, H, HKV, NQ, NKV, D, masked)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "-".join(map(str, s)))
def test_static_equals_ext_on_consecutive_calls(gpu_backend, shape):
    layout, S, H, HKV, NQ, NKV, D, masked = shape
    be = gpu_backend
    scale = 1.0 / np.sqrt(D)
    before = be.mem_stats()["scratch_bytes"]
    for call in range(2):
        q, k, v, mask = _make(layout, 7000 + 31 * call + NKV, S, H, HKV, NQ, NKV, D, masked)
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
@pytest.mark.parametrize("case", ["partials", "tickets"])
def test_static_rejects_oversize_split(case):
    """Split plans depend on the shapes only, so both limits are reached on any device:
    300 query rows of 8 heads at D = 128 over 256 keys split 4 ways need ~5 MB of
    partials (the array holds 4 MiB); 130 sequences of 8 kv heads in the GQA layout over
    128 keys are 1040 split groups (1024 tickets).  Each call must fail with the sizes
    named, launch nothing, and leave the backend working."""
    import torch

    be = ob.Backend(0)
    try:
        be.set_stream(torch.cuda.current_stream())
        if case == "partials":
            H, NQ, D = 8, 300, 128
            q, k, v, _ = _inputs(12, 1, H, 1, NQ, 256, D, False)
            out = _out(1, H, NQ, D)
        else:
            S, H, NQ, D = 130, 8, 1, 128
            g = torch.Generator(device="cuda").manual_seed(14)
            q = torch.randn((S, H, NQ, D), generator=g, device="cuda", dtype=torch.float32)
            k = torch.randn((S, H, 128, D), generator=g, device="cuda", dtype=torch.float32).half()
            v = torch.randn((S, H, 128, D), generator=g, device="cuda", dtype=torch.float32).half()
            out = _out(S, H, NQ, D)
        with pytest.raises(ob.GgmlBackendError) as ei:
            be.flash_attn_ext_static(q, k, v, None, 1.0 / np.sqrt(D), out)
        assert "static scratch holds" in str(ei.value)
        assert torch.isnan(out).all()  # nothing was launched
        # the regular entry point runs the same shape (growing its scratch)
        be.flash_attn_ext(q, k, v, None, 1.0 / np.sqrt(D), out)
        be.synchronize()
        assert torch.isfinite(out).all()
        # and the static entry still serves a shape that fits, bit-equal to the regular one
        q2, k2, v2, _ = _heads_inputs(13, 8, 20, 1500)
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
