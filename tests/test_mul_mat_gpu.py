"""GPU parity of GGML_OP_MUL_MAT (K1 decode GEMV, K2 GEMM) against the CPU
oracle on seeded synthetic inputs, through the C ABI.

Quantized weights: bit-exact.  Every kernel forms each per-block term as
ggml's CPU vec_dot does (same activation quantization, integer block dot, same
f32 scale products) and adds the terms in block order from zero -- the
oracle's order -- whichever kernel, warp count or device runs it.  The shapes
cover the dispatch boundaries: one unit per warp, several units per warp held
in registers, looping warps, and K long enough that the block terms are folded
in several shared-memory segments.  F16 / F32 weights: max-abs-rel 1e-5 (their
fp32 dot products are summed by lane trees and warp shuffles)."""
import numpy as np
import pytest

import openasr_b200 as ob
from oracle import oracle as oo
from tests.conftest import max_abs_rel


SHAPES = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (1280, 1280), (5120, 1280), (1280, 5120),
          (1152, 384), (384, 1536), (80, 4096), (48, 16384), (40, 33024)]
TYPES = [ob.Q8_0, ob.Q4_0, ob.Q4_K]


def _weights(N, K, qt, seed):
    w = oo.synth_normal(seed, N * K, 0.0, 0.02).reshape(N, K)
    return oo.quantize(qt, w)


def _run(be, wq, qt, N, K, x_np, prec=ob.PREC_DEFAULT):
    import torch

    W = be.upload_weight(wq, qt, [K, N])
    try:
        x = torch.from_numpy(x_np).cuda()
        out = torch.empty((x_np.shape[0], N), dtype=torch.float32, device="cuda")
        be.mul_mat(W, x, out, prec)
        be.synchronize()
        return out.cpu().numpy()
    finally:
        W.free()


@pytest.mark.gpu
@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 8])
def test_decode_gemv_matches_oracle(gpu_backend, qt, N, K, M):
    if qt == ob.Q4_K and K % 256:
        pytest.skip("Q4_K needs K % 256 == 0")
    seed = 0x0A5A0002 + N * 7 + K + qt
    wq = _weights(N, K, qt, seed)
    x = oo.synth_normal(seed ^ 0xFFFF, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, qt, N, K, x)
    ref = oo.mul_mat(wq, qt, K, N, x)
    np.testing.assert_array_equal(got, ref, err_msg=f"{qt} N={N} K={K} M={M}")


@pytest.mark.gpu
@pytest.mark.parametrize("qt", TYPES)
def test_lm_head_gemv_matches_oracle(gpu_backend, qt):
    N, K, M = 151936, 1024, 4
    wq = _weights(N, K, qt, 0x0A5A0005)
    x = oo.synth_normal(0x0A5A0006, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, qt, N, K, x)
    ref = oo.mul_mat(wq, qt, K, N, x)
    np.testing.assert_array_equal(got, ref)
    # greedy token identity on the logits (first-max)
    np.testing.assert_array_equal(oo.argmax_first(got), oo.argmax_first(ref))


@pytest.mark.gpu
@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("M", [9, 64, 512, 1500])
def test_prefill_encoder_gemm_matches_oracle(gpu_backend, qt, M):
    N, K = 1280, 1280
    wq = _weights(N, K, qt, 0x0A5A0007 + qt)
    x = oo.synth_normal(0x0A5A0008 + M, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, qt, N, K, x)
    ref = oo.mul_mat(wq, qt, K, N, x)
    np.testing.assert_array_equal(got, ref, err_msg=f"{qt} M={M}")


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 5, 8, 20])
def test_f16_and_f32_weights(gpu_backend, M):
    N, K = 96, 200
    w = oo.synth_normal(21, N * K, 0, 0.5).reshape(N, K)
    x = oo.synth_normal(22, M * K).reshape(M, K)
    w16 = w.astype(np.float16)
    got = _run(gpu_backend, w16.view(np.uint8).reshape(N, -1), ob.F16, N, K, x)
    ref = oo.mul_mat(w16.view(np.uint16), oo.F16, K, N, x)
    assert max_abs_rel(got, ref) <= 1e-5
    got32 = _run(gpu_backend, w.view(np.uint8).reshape(N, -1), ob.F32, N, K, x)
    ref32 = oo.mul_mat(w, oo.F32, K, N, x)
    assert max_abs_rel(got32, ref32) <= 1e-5
    # GGML_PREC_F32 keeps f32 activations against f16 weights
    got_p = _run(gpu_backend, w16.view(np.uint8).reshape(N, -1), ob.F16, N, K, x, prec=ob.PREC_F32)
    exact = x.astype(np.float64) @ w16.astype(np.float64).T
    assert max_abs_rel(got_p, exact) <= 1e-5


@pytest.mark.gpu
def test_reference_kat_tiny_graph_mul_mat_success(gpu_backend):
    # cpu_graph.rs:12827-12857 on the device: exact [17, 39, 23, 53]
    lhs = np.array([[1, 2], [3, 4]], np.float32)
    got = _run(gpu_backend, lhs.view(np.uint8).reshape(2, -1), ob.F32, 2, 2, np.array([[5, 6], [7, 8]], np.float32))
    np.testing.assert_array_equal(got.ravel(), [17, 39, 23, 53])
    w = np.array([0x3C00, 0, 0, 0x3C00], np.uint16).reshape(2, 2)  # :12860 identity f16
    got = _run(gpu_backend, w.view(np.uint8).reshape(2, -1), ob.F16, 2, 2, np.array([[2, 3]], np.float32))
    np.testing.assert_array_equal(got.ravel(), [2, 3])


@pytest.mark.gpu
def test_batched_broadcast_mul_mat(gpu_backend):
    import torch

    # weight [K, N, 2, 1] broadcast over rhs [K, M, 4, 1] (rhs.ne2 % lhs.ne2 == 0)
    K, N, M = 256, 64, 3
    w = oo.synth_normal(31, 2 * N * K, 0, 0.02).reshape(2 * N, K)
    wq = oo.quantize(oo.Q8_0, w)
    x = oo.synth_normal(32, 4 * M * K).reshape(4, M, K)
    W = gpu_backend.upload_weight(wq, ob.Q8_0, [K, N, 2, 1])
    xt = torch.from_numpy(x).cuda()
    out = torch.empty((4, M, N), dtype=torch.float32, device="cuda")
    gpu_backend.mul_mat(W, xt, out)
    gpu_backend.synchronize()
    W.free()
    ref = oo.mul_mat(wq.reshape(2, N, -1), oo.Q8_0, K, N, x[None], w_batch=(1, 2))[0]
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", TYPES)
def test_weight_upload_round_trip_is_bit_exact(gpu_backend, qt):
    K, N = 1024, 48
    wq = _weights(N, K, qt, 41)
    W = gpu_backend.upload_weight(wq, qt, [K, N])
    back = W.download()
    W.free()
    np.testing.assert_array_equal(back, wq)


@pytest.mark.gpu
@pytest.mark.parametrize("qt,N,K", [(ob.Q8_0, 4608, 4096), (ob.Q4_0, 8192, 4096), (ob.Q4_K, 8704, 4096),
                                    (ob.F16, 2176, 4096)])
def test_weight_upload_through_staging_is_bit_exact(gpu_backend, qt, N, K):
    """Weights larger than one 16 MiB staging buffer, with a ragged last chunk, cross
    through the pinned staging ring and (Q8_0 / Q4_0) are split into planes on the
    device; the download reassembles the raw blocks bit for bit, and a GEMV on the
    uploaded planes matches the oracle."""
    import torch

    if qt == ob.F16:
        wq = (oo.synth_normal(91, N * K, 0.0, 0.02).reshape(N, K)).astype(np.float16)
    else:
        wq = _weights(N, K, qt, 91)
    assert wq.nbytes > 16 << 20 and wq.nbytes % (16 << 20) != 0
    W = gpu_backend.upload_weight(wq, qt, [K, N])
    try:
        np.testing.assert_array_equal(W.download(), wq.view(np.uint8).reshape(N, -1))
        if qt != ob.F16:
            x = oo.synth_normal(92, 2 * K, 0.0, 1.0).reshape(2, K)
            out = torch.empty((2, N), dtype=torch.float32, device="cuda")
            gpu_backend.mul_mat(W, torch.from_numpy(x).cuda(), out)
            gpu_backend.synchronize()
            ref = oo.mul_mat(wq, qt, K, N, x)
            np.testing.assert_array_equal(out.cpu().numpy(), ref)
    finally:
        W.free()


@pytest.mark.gpu
def test_mul_mat_rejects_bad_shapes(gpu_backend):
    import torch

    wq = _weights(32, 256, ob.Q8_0, 1)
    W = gpu_backend.upload_weight(wq, ob.Q8_0, [256, 32])
    x = torch.zeros((2, 128), dtype=torch.float32, device="cuda")
    out = torch.zeros((2, 32), dtype=torch.float32, device="cuda")
    with pytest.raises(ob.backend.UnsupportedInputs, match="lhs.ne0 must equal rhs.ne0"):
        gpu_backend.mul_mat(W, x, out)
    W.free()
    # capability probe of backend.rs:295-323
    for t in (ob.Q4_0, ob.Q8_0, ob.Q4_K):
        assert gpu_backend.device_supports_matmul_for_type(t)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("M", [1, 8, 100])
def test_shared_activation_quantization(gpu_backend, qt, M):
    """quantize_act once, then mul_mat_qact on two weights == two plain mul_mats."""
    import torch

    K, N = 1024, 640
    x = oo.synth_normal(51 + M, M * K).reshape(M, K)
    xt = torch.from_numpy(x).cuda()
    qact = torch.empty(gpu_backend.act_bytes(qt, K, M), dtype=torch.uint8, device="cuda")
    gpu_backend.quantize_act(qt, xt, qact)
    for seed in (52, 53):
        wq = _weights(N, K, qt, seed)
        W = gpu_backend.upload_weight(wq, qt, [K, N])
        a = torch.empty((M, N), dtype=torch.float32, device="cuda")
        b = torch.empty((M, N), dtype=torch.float32, device="cuda")
        gpu_backend.mul_mat_qact(W, qact, M, a)
        gpu_backend.mul_mat(W, xt, b)
        gpu_backend.synchronize()
        W.free()
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
        np.testing.assert_array_equal(a.cpu().numpy(), oo.mul_mat(wq, qt, K, N, x))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(9, 128, 256), (128, 256, 1280), (300, 1280, 1280), (1500, 5120, 1280), (200, 1280, 5120), (77, 200, 512)])
def test_q4k_tensor_core_gemm_is_bit_exact(gpu_backend, M, N, K):
    """The tcgen05 Q4_K GEMM forms ggml's per-super-block term exactly and adds
    the super-blocks in order, so it must equal the oracle bit for bit."""
    wq = _weights(N, K, ob.Q4_K, 0x0A5A0009 + M)
    x = oo.synth_normal(0x0A5A000A + N, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, ob.Q4_K, N, K, x)
    ref = oo.mul_mat(wq, ob.Q4_K, K, N, x)
    np.testing.assert_array_equal(got, ref)


def _q4k_adversarial(N, K, seed):
    """raw Q4_K rows whose every sub-scale and min is 63 and quants 12..15: sc * q
    reaches 945 and a super-block's products all share one sign"""
    rng = np.random.default_rng(seed)
    nb = K // 256
    w = np.zeros((N, nb, 144), np.uint8)
    w[..., 0:2] = rng.uniform(1e-3, 2e-3, size=(N, nb)).astype(np.float16)[..., None].view(np.uint8)
    w[..., 2:4] = rng.uniform(1e-3, 2e-3, size=(N, nb)).astype(np.float16)[..., None].view(np.uint8)
    w[..., 4:16] = 0xFF
    q = rng.integers(12, 16, size=(N, nb, 4, 2, 32))  # chunk c: low nibbles then high nibbles
    w[..., 16:] = (q[..., 0, :] | (q[..., 1, :] << 4)).reshape(N, nb, 128).astype(np.uint8)
    return w.reshape(N, nb * 144)


@pytest.mark.gpu
@pytest.mark.parametrize("sign", [1.0, -1.0])
@pytest.mark.parametrize("M,N,K", [(128, 256, 1280), (300, 200, 2048), (9, 128, 256)])
def test_q4k_tensor_core_gemm_exact_beyond_2_24(gpu_backend, sign, M, N, K):
    """Adversarial Q4_K case: sub-scales 63 x quants 12..15 against activations of
    one sign near their block maximum (q8_K quants within a few steps of -+127), so
    a super-block's integer dot reaches 256 x 945 x 127 > 2^24 and one f32
    accumulation of its 256 products would round.  The GEMM accumulates each
    super-block as two exact 128-element halves; the result equals the oracle's
    integer arithmetic bit for bit."""
    wq = _q4k_adversarial(N, K, 0x0A5A0C00 + M)
    rng = np.random.default_rng(0x0A5A0C01 + N)
    x = (sign * (1.0 + 0.05 * rng.random((M, K)))).astype(np.float32)
    x[0, :256] = sign * 3.0  # a constant block: every quant -+127
    got = _run(gpu_backend, wq, ob.Q4_K, N, K, x)
    ref = oo.mul_mat(wq, ob.Q4_K, K, N, x)
    assert np.abs(ref).max() > 0
    np.testing.assert_array_equal(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", [ob.Q8_0, ob.Q4_K])
@pytest.mark.parametrize("N,K", [(17, 256), (100, 512), (51866, 1280), (40, 7680)])
@pytest.mark.parametrize("M", [1, 5, 8])
def test_decode_tiles_ragged_rows_and_depths(gpu_backend, qt, N, K, M):
    """The tensor-core GEMV reads 16-row decode tiles: a last tile with padding
    rows, one unit per row (K = 256), and rows longer than one unit per warp."""
    seed = 0x0A5A000B + N + K + M
    wq = _weights(N, K, qt, seed)
    x = oo.synth_normal(seed ^ 0x5A5A, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, qt, N, K, x)
    ref = oo.mul_mat(wq, qt, K, N, x)
    np.testing.assert_array_equal(got, ref, err_msg=f"{qt} N={N} K={K} M={M}")


_DP4A_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1])
import numpy as np, torch
import openasr_b200 as ob
from oracle import oracle as oo
be = ob.Backend(0)
mismatch = 0
for qt in (ob.Q8_0, ob.Q4_K):
    for (N, K, M) in ((1280, 1280, 8), (3840, 1280, 3), (1024, 3072, 1), (100, 384, 5), (64, 8192, 2)):
        if qt == ob.Q4_K and K % 256:
            continue
        w = oo.quantize(qt, oo.synth_normal(N + K + qt, N * K, 0.0, 0.02).reshape(N, K))
        x = oo.synth_normal(M + K, M * K).reshape(M, K)
        W = be.upload_weight(w, qt, [K, N])
        out = torch.empty((M, N), dtype=torch.float32, device="cuda")
        be.mul_mat(W, torch.from_numpy(x).cuda(), out)
        be.synchronize()
        W.free()
        mismatch += int((out.cpu().numpy() != oo.mul_mat(w, qt, K, N, x)).sum())
print("MISMATCH", mismatch)
be.close()
"""


@pytest.mark.gpu
def test_dp4a_decode_gemv_still_matches_oracle():
    """OASR_B200_DECODE_GEMV=dp4a keeps the CUDA-core GEMV for Q8_0 / Q4_K (the Q4_0
    path always uses it); it folds its block terms in block order too: bit-exact."""
    import os
    import subprocess
    import sys

    from tests.conftest import ROOT

    env = dict(os.environ, OASR_B200_DECODE_GEMV="dp4a")
    r = subprocess.run([sys.executable, "-c", _DP4A_CHILD, ROOT], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert int(r.stdout.split("MISMATCH")[1]) == 0, r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(9, 128, 128), (300, 1280, 1280), (1500, 1024, 3072), (77, 4096, 1024)])
def test_q4_0_tensor_core_gemm_is_bit_exact(gpu_backend, M, N, K):
    """Q4_0 at M > 8 runs the tcgen05 kind::i8 GEMM on its nibbles expanded to int8 at
    upload (q - 8, ggml's element order) with its own scales: ggml's Q4_0 x q8_0 block dot
    is that integer dot scaled like Q8_0's, so the result equals the oracle bit for bit."""
    wq = _weights(N, K, ob.Q4_0, 0x0A5A001C + M)
    x = oo.synth_normal(0x0A5A001D + N, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, ob.Q4_0, N, K, x)
    ref = oo.mul_mat(wq, ob.Q4_0, K, N, x)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(9, 128, 128), (128, 256, 384), (300, 1280, 1280), (1500, 1152, 384),
                                   (200, 200, 1536), (77, 4096, 1024)])
def test_q8_0_tensor_core_gemm_is_bit_exact(gpu_backend, M, N, K):
    """The tcgen05 kind::i8 Q8_0 GEMM forms each 32-block's integer dot exactly and adds
    the blocks' float terms in order with ggml's roundings, so it equals the oracle bit
    for bit (ragged M and N, K a multiple of 128)."""
    wq = _weights(N, K, ob.Q8_0, 0x0A5A000C + M)
    x = oo.synth_normal(0x0A5A000D + N, M * K).reshape(M, K)
    got = _run(gpu_backend, wq, ob.Q8_0, N, K, x)
    ref = oo.mul_mat(wq, ob.Q8_0, K, N, x)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("qt,N,K", [(ob.Q4_K, 1280, 5120), (ob.Q8_0, 4096, 1024)])
def test_tensor_core_gemm_repeatable(gpu_backend, qt, N, K):
    """1500 launches of the same tensor-core GEMM give the same bits every time: the
    kernels' shared-memory refills (weight metadata or scales read by the epilogue, then
    overwritten by an asynchronous copy) are ordered by proxy fences.  Without them the
    Q4_K GEMM computed a fragment from the next super-block's metadata about once per
    500 launches."""
    import torch

    M = 1500
    be = gpu_backend
    w = be.upload_weight(_weights(N, K, qt, 0x0A5A0D00 + N), qt, [K, N])
    try:
        x = torch.from_numpy(oo.synth_normal(0x0A5A0D01, M * K).reshape(M, K)).cuda()
        qa = torch.empty(be.act_bytes(qt, K, M), dtype=torch.uint8, device="cuda")
        be.quantize_act(qt, x, qa)
        ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
        y = torch.empty_like(ref)
        be.mul_mat_qact(w, qa, M, ref)
        bad = 0
        for _ in range(1500):
            be.mul_mat_qact(w, qa, M, y)
            bad += int(not torch.equal(y, ref))
        be.synchronize()
        assert bad == 0, f"{bad} of 1500 launches differed"
    finally:
        w.free()
