"""Pins the CPU oracle: block formats against the gguf package's numpy
restatements (tests/golden/blockfmt_gguf.npz) and op semantics against the
reference's own known-answer tests in crates/openasr-core/src/ggml_runtime/cpu_graph.rs."""
import os

import numpy as np
import pytest

from oracle import oracle as oo

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "blockfmt_gguf.npz"))


def test_f16_conversion_matches_numpy_rne():
    f = GOLD["f32_for_f16"]
    got = np.array([oo.lib().oo_f32_to_f16(float(v)) for v in f], np.uint16)
    np.testing.assert_array_equal(got, GOLD["f16_bits"])
    # every finite half round-trips exactly through f32
    bits = np.arange(65536, dtype=np.uint32)
    half = bits.astype(np.uint16).view(np.float16)
    finite = np.isfinite(half)
    back = np.array([oo.lib().oo_f16_to_f32(int(b)) for b in bits[finite]], np.float32)
    np.testing.assert_array_equal(back.view(np.uint32), half[finite].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name,qt", [("q8_0", oo.Q8_0), ("q4_0", oo.Q4_0)])
def test_quantize_bit_exact_vs_gguf(name, qt):
    q = oo.quantize(qt, GOLD["x"])
    np.testing.assert_array_equal(q, GOLD[f"{name}_bytes"])


@pytest.mark.parametrize("name,qt", [("q8_0", oo.Q8_0), ("q4_0", oo.Q4_0)])
def test_dequantize_bit_exact_vs_gguf(name, qt):
    d = oo.dequantize(qt, GOLD[f"{name}_bytes"], 256)
    np.testing.assert_array_equal(d.view(np.uint32), GOLD[f"{name}_deq"].astype(np.float32).view(np.uint32))


def test_q4_k_dequantize_bit_exact_vs_gguf():
    d = oo.dequantize(oo.Q4_K, GOLD["q4_k_bytes"], 256)
    np.testing.assert_array_equal(d.view(np.uint32), GOLD["q4_k_deq"].astype(np.float32).view(np.uint32))


def test_q4_k_quantizer_round_trip():
    x = oo.synth_normal(0x0A5A0002, 4 * 1024, 0.0, 0.02).reshape(4, 1024)
    q = oo.quantize(oo.Q4_K, x)
    assert q.shape == (4, 4 * 144)
    d = oo.dequantize(oo.Q4_K, q, 1024)
    # 4-bit affine per 32 with 6-bit sub-scales: error below one quantization step
    step = (x.reshape(-1, 32).max(1) - np.minimum(x.reshape(-1, 32).min(1), 0)) / 15
    err = np.abs(d - x).reshape(-1, 32).max(1)
    assert np.all(err <= step * 1.2 + 1e-6)


def test_synth_normal_is_deterministic_and_normal():
    a = oo.synth_normal(7, 100000)
    b = oo.synth_normal(7, 100000)
    np.testing.assert_array_equal(a, b)
    c = oo.synth_normal(7, 50, offset=1000)
    np.testing.assert_array_equal(c, a[1000:1050])
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1.0) < 0.02


# ---- reference known-answer tests (cpu_graph.rs) --------------------------------
def test_kat_tiny_graph_mul_mat_success():
    # cpu_graph.rs:12827-12857: lhs [2,2]=[1,2,3,4], rhs [2,2]=[5,6,7,8] -> [17,39,23,53]
    lhs = np.array([[1, 2], [3, 4]], np.float32)
    rhs = np.array([[5, 6], [7, 8]], np.float32)
    out = oo.mul_mat(lhs, oo.F32, 2, 2, rhs)
    np.testing.assert_array_equal(out.ravel(), [17, 39, 23, 53])


def test_kat_static_f16_weight_and_view():
    # cpu_graph.rs:12860 (identity f16 weight): [2,3] -> [2,3]
    w = np.array([0x3C00, 0, 0, 0x3C00], np.uint16).reshape(2, 2)
    out = oo.mul_mat(w, oo.F16, 2, 2, np.array([[2, 3]], np.float32))
    np.testing.assert_array_equal(out.ravel(), [2, 3])
    # cpu_graph.rs:12892: view_2d(ne0=2, ne1=2, nb1=4 B, offset=8 B) of [identity; 2*identity]
    base = np.array([0x3C00, 0, 0, 0x3C00, 0x4000, 0, 0, 0x4000], np.uint16).reshape(4, 2)
    view = np.ascontiguousarray(base.view(np.uint8).ravel()[8:16].view(np.uint16).reshape(2, 2))
    out = oo.mul_mat(view, oo.F16, 2, 2, np.array([[3, 4]], np.float32))
    np.testing.assert_array_equal(out.ravel(), [6, 8])
    # cpu_graph.rs:12941: f16 rhs input accepted
    out = oo.mul_mat(w, oo.F16, 2, 2, np.array([[2, 3]], np.float16).view(np.uint16), x_type=oo.F16)
    np.testing.assert_array_equal(out.ravel(), [2, 3])


def _ref_softmax(s):
    s = np.asarray(s, np.float32)
    w = np.exp(s - s.max())
    return w / w.sum()


def test_kat_qwen_decode_flash_attention_matches_reference():
    # cpu_graph.rs:13900-13948, tolerance 1e-4
    scale = np.float32(1 / np.sqrt(2))
    q = np.array([1, 0], np.float32).reshape(1, 1, 1, 2)
    k = np.array([1, 0, 0, 1], np.float32).reshape(1, 1, 2, 2)
    v = np.array([10, 20, 30, 40], np.float32).reshape(1, 1, 2, 2)
    out = oo.flash_attn_ext(q, k, v, None, float(scale)).ravel()
    w = _ref_softmax([scale, 0.0])
    exp = [w[0] * 10 + w[1] * 30, w[0] * 20 + w[1] * 40]
    np.testing.assert_allclose(out, exp, atol=1e-4, rtol=0)


def test_kat_batched_flash_attn_mask_planes_match_serial():
    # cpu_graph.rs:13471-13540
    scale = float(np.float32(1 / np.sqrt(2)))
    ninf, zero = np.float16(-np.inf).view(np.uint16), np.float16(0).view(np.uint16)
    q = np.array([1, 0, 0, 1], np.float32)
    k = np.array([1, 0, 0, 1, 1, 0, 0, 1], np.float32)
    v = np.array([10, 20, 30, 40, -5, -6, 50, 60], np.float32)
    mask = np.array([zero, ninf, ninf, zero], np.uint16)

    def run(n, qv, kv, vv, mv):
        return oo.flash_attn_ext(qv.reshape(n, 1, 1, 2), kv.reshape(n, 1, 2, 2), vv.reshape(n, 1, 2, 2),
                                 mv.reshape(n, 1, 1, 2), scale).ravel()

    batched = run(2, q, k, v, mask)
    np.testing.assert_allclose(batched[0:2], run(1, q[:2], k[:4], v[:4], mask[:2]), atol=1e-4)
    np.testing.assert_allclose(batched[2:4], run(1, q[2:], k[4:], v[4:], mask[2:]), atol=1e-4)
    # masked planes select exactly one kv row each
    np.testing.assert_allclose(batched, [10, 20, 50, 60], atol=1e-4)


def test_kat_kv_cache_set_rows():
    # cpu_graph.rs:13950-14030 (set_rows part): rows [0,3] of a zeroed f16 [2,4] cache
    cache = np.zeros((1, 1, 4, 2), np.float16)
    oo.set_rows(cache, np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 2, 2), np.array([0, 3]))
    np.testing.assert_array_equal(cache.astype(np.float32).ravel(), [1, 2, 0, 0, 0, 0, 3, 4])


def test_argmax_first_max_ties_and_nonfinite():
    # cpu_graph.rs:3750-3765: lowest column index whose finite value is maximal
    x = np.array([[1, 5, 5, 2], [np.nan, np.inf, 3, 3], [-1, -1, -1, -1]], np.float32)
    np.testing.assert_array_equal(oo.argmax_first(x), [1, 2, 0])


def test_flash_gqa_native_equals_expanded():
    # nn/decoder.rs:3860: native GQA (q heads share kv heads) == explicitly expanded kv
    rng = np.random.default_rng(3)
    q = rng.normal(size=(1, 4, 3, 32)).astype(np.float32)
    k = rng.normal(size=(1, 2, 10, 32)).astype(np.float16)
    v = rng.normal(size=(1, 2, 10, 32)).astype(np.float16)
    native = oo.flash_attn_ext(q, k, v, None, 0.2)
    kx, vx = np.repeat(k, 2, axis=1), np.repeat(v, 2, axis=1)
    expanded = oo.flash_attn_ext(q, kx, vx, None, 0.2)
    np.testing.assert_array_equal(native, expanded)


def test_quantized_mul_mat_close_to_dequantized_f32():
    K, N, M = 512, 16, 3
    w = oo.synth_normal(11, N * K, 0, 0.02).reshape(N, K)
    x = oo.synth_normal(12, M * K).reshape(M, K)
    for qt in (oo.Q8_0, oo.Q4_0, oo.Q4_K):
        wq = oo.quantize(qt, w)
        wd = oo.dequantize(qt, wq, K)
        got = oo.mul_mat(wq, qt, K, N, x)
        exact = x.astype(np.float64) @ wd.T.astype(np.float64)
        rel = np.abs(got - exact).max() / np.abs(exact).max()
        assert rel < 1.5e-2, (qt, rel)  # activation quantization error only


# ---- activation quantizers and block dots against an independent numpy restatement ----------
# tests/golden/gen_vecdot_golden.py restates ggml's q8_K quantizer and the Q4_K x q8_K,
# Q4_0 x q8_0 and Q8_0 x q8_0 block dots (with the canonical block-order f32 sum) in
# vectorised numpy, and takes the q8_0 activations from gguf's own quantizer.
VD = np.load(os.path.join(os.path.dirname(__file__), "golden", "vecdot_numpy.npz"))


def test_q8_k_quantizer_matches_independent_restatement():
    x = VD["q8k_x"]
    q = oo.quantize(oo.Q8_K, x).reshape(x.shape[0], -1, 292)
    d = q[..., 0:4].copy().view(np.float32)[..., 0]
    qs = q[..., 4:260].copy().view(np.int8).reshape(x.shape[0], -1)
    bs = q[..., 260:292].copy().view(np.int16).reshape(x.shape[0], -1)
    np.testing.assert_array_equal(d.view(np.uint32), VD["q8k_d"].view(np.uint32))
    np.testing.assert_array_equal(qs, VD["q8k_qs"])
    np.testing.assert_array_equal(bs, VD["q8k_bsums"])


@pytest.mark.parametrize("name,qt", [("q4k", oo.Q4_K), ("q8_0", oo.Q8_0), ("q4_0", oo.Q4_0)])
def test_block_dots_match_independent_restatement(name, qt):
    w, x, y = VD[f"{name}_w"], VD[f"{name}_x"], VD[f"{name}_y"]
    N, K = w.shape[0], x.shape[1]
    got = oo.mul_mat(np.ascontiguousarray(w), qt, K, N, x)
    np.testing.assert_array_equal(got.view(np.uint32), y.view(np.uint32))


def test_decode_exp_is_within_one_ulp():
    """oo_expf, the decode path's e^x (shared algorithm with the device's exp_f32)."""
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-87, 88, 20000), rng.normal(0, 1, 5000)]).astype(np.float32)
    got = oo.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert (np.abs(got - ref) / ulp).max() <= 1.0
    assert oo.expf(np.array([-np.inf, np.inf, -200.0, 0.0], np.float32)).tolist() == [0.0, np.inf, 0.0, 1.0]
