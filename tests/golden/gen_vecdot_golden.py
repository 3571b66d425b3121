"""Generate tests/golden/vecdot_numpy.npz: golden vectors for the activation
quantizers and block dot products of ggml's CPU mul_mat, from a vectorised numpy
restatement written here independently of oracle/oracle.c.

    python tests/golden/gen_vecdot_golden.py

Sources of each rule:
  * block geometry: gguf/constants.py GGML_QUANT_SIZES (gguf 0.19.0): Q8_0 (32, 34),
    Q4_0 (32, 18), Q4_K (256, 144), Q8_K (256, 292 = f32 d + 256 int8 + 16 int16 sums);
  * q8_0 activations: gguf/quants.py Q8_0.quantize_blocks (documented there as
    matching ggml-quants.c) -- called, not restated;
  * Q4_K scale / min unpacking: gguf/quants.py Q4_K.get_scale_min's bit layout;
  * q8_K activations (ggml's quantize_row_q8_K, which gguf-py does not implement):
    the scale of a 256-block is -127 / x_max with x_max the signed value of the
    first element of largest magnitude, quants nearest_int(iscale * x) clamped to
    127 (ties to even), d = 1 / iscale, 16-wide sums of the quants; an all-zero
    block has d = 0;
  * the per-block f32 terms: Q8_0 / Q4_0 (float)isum * (d_w * d_a); Q4_K
    (d_w * d_a) * isum - (dmin_w * d_a) * msum with isum = sum_j sc_j <q4_j, q8_j>
    and msum = sum_j m_j (sum of the 32 quants of sub-block j); the terms of a row
    summed in block order from zero in f32 -- the canonical order every
    mul_mat path of this repository uses.
Weights and activations come from numpy's own generator (not the oracle's
SplitMix64 stream).  Each row set includes edge cases: an all-zero block, a
constant block (every q8_K quant +-127), a block whose largest magnitudes tie
between a positive and a negative value, and rows spanning several decades.
"""
from __future__ import annotations

import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
F32 = np.float32


def f16_to_f32(u16: np.ndarray) -> np.ndarray:
    return np.asarray(u16, np.uint16).view(np.float16).astype(F32)


def q8k_quantize(x: np.ndarray):
    """x [R][K] f32 -> (d [R][K/256] f32, qs [R][K] int8, bsums [R][K/16] int16)"""
    R, K = x.shape
    xb = x.reshape(R, K // 256, 256).astype(F32)
    ax = np.abs(xb)
    first = np.argmax(ax, axis=-1)[..., None]                    # first element of largest |x|
    xmax = np.take_along_axis(xb, first, axis=-1)[..., 0]
    zero = ax.max(axis=-1) == 0
    with np.errstate(divide="ignore", invalid="ignore"):
        iscale = np.where(zero, F32(0), F32(-127.0) / np.where(zero, F32(1), xmax)).astype(F32)
    v = (iscale[..., None] * xb).astype(F32)                     # one f32 rounding
    q = np.minimum(np.rint(v), F32(127)).astype(np.int32)        # nearest, ties to even
    q[zero] = 0
    with np.errstate(divide="ignore"):
        d = np.where(zero, F32(0), F32(1.0) / np.where(zero, F32(1), iscale)).astype(F32)
    bsums = q.reshape(R, K // 16, 16).sum(axis=-1).astype(np.int16)
    return d, q.reshape(R, K).astype(np.int8), bsums


def q4k_scales(blocks: np.ndarray):
    """raw Q4_K blocks [..., 144] -> (sc [..., 8], m [..., 8]) int32 (get_scale_min layout)"""
    s = blocks[..., 4:16].astype(np.int32)
    sc = np.empty(blocks.shape[:-1] + (8,), np.int32)
    m = np.empty_like(sc)
    sc[..., :4] = s[..., 0:4] & 63
    m[..., :4] = s[..., 4:8] & 63
    sc[..., 4:] = (s[..., 8:12] & 0xF) | ((s[..., 0:4] >> 6) << 4)
    m[..., 4:] = (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 6) << 4)
    return sc, m


def q4k_quants(blocks: np.ndarray) -> np.ndarray:
    """raw Q4_K blocks [..., 144] -> 4-bit quants [..., 256] in element order"""
    qs = blocks[..., 16:144].reshape(blocks.shape[:-1] + (4, 32)).astype(np.int32)
    lo, hi = qs & 0xF, qs >> 4
    return np.stack([lo, hi], axis=-2).reshape(blocks.shape[:-1] + (256,))  # chunk c: 64c + l (lo), 64c + 32 + l (hi)


def dot_q4k(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """w [N][nb][144] raw Q4_K, x [M][K] f32 -> y [M][N] f32"""
    N, nb, _ = w.shape
    ad, aq, abs16 = q8k_quantize(x)
    M = x.shape[0]
    sc, mn = q4k_scales(w)                                       # [N][nb][8]
    q4 = q4k_quants(w)                                           # [N][nb][256]
    dw = f16_to_f32(w[..., 0:2].copy().view(np.uint16)[..., 0])
    dmw = f16_to_f32(w[..., 2:4].copy().view(np.uint16)[..., 0])
    a = aq.astype(np.int64).reshape(M, nb, 8, 32)
    q = (q4.astype(np.int64) * np.repeat(sc, 32, axis=-1)).reshape(N, nb, 8, 32)
    isum = np.einsum("nbjk,mbjk->mnb", q, a)                     # exact integers
    b32 = abs16.astype(np.int64).reshape(M, nb, 8, 2).sum(-1)    # sums of the 32 quants of sub-block j
    msum = np.einsum("nbj,mbj->mnb", mn.astype(np.int64), b32)
    y = np.zeros((M, N), F32)
    for b in range(nb):
        d = (dw[None, :, b] * ad[:, b, None]).astype(F32)
        dm = (dmw[None, :, b] * ad[:, b, None]).astype(F32)
        t = ((d * isum[..., b].astype(F32)).astype(F32) - (dm * msum[..., b].astype(F32)).astype(F32)).astype(F32)
        y = (y + t).astype(F32)
    return y


def dot_q8(wq: np.ndarray, qt, x: np.ndarray) -> np.ndarray:
    """wq [N][row bytes] raw Q8_0 / Q4_0 (gguf layout), x [M][K] f32 -> y [M][N] f32"""
    N, K = wq.shape[0], x.shape[1]
    nb = K // 32
    xa = quants.quantize(x, T.Q8_0).reshape(x.shape[0], nb, 34)
    ad = f16_to_f32(xa[..., 0:2].copy().view(np.uint16)[..., 0])
    aq = xa[..., 2:].view(np.int8).astype(np.int64)              # [M][nb][32]
    if qt == T.Q8_0:
        wb = wq.reshape(N, nb, 34)
        dw = f16_to_f32(wb[..., 0:2].copy().view(np.uint16)[..., 0])
        wv = wb[..., 2:].view(np.int8).astype(np.int64)
    else:
        wb = wq.reshape(N, nb, 18)
        dw = f16_to_f32(wb[..., 0:2].copy().view(np.uint16)[..., 0])
        b = wb[..., 2:].astype(np.int64)
        wv = np.concatenate([(b & 0xF) - 8, (b >> 4) - 8], axis=-1)  # element j | j + 16
    isum = np.einsum("nbk,mbk->mnb", wv, aq)
    y = np.zeros((x.shape[0], N), F32)
    for blk in range(nb):
        t = (isum[..., blk].astype(F32) * (dw[None, :, blk] * ad[:, blk, None]).astype(F32)).astype(F32)
        y = (y + t).astype(F32)
    return y


def activations(rng, M: int, K: int) -> np.ndarray:
    x = rng.normal(0.0, 1.0, size=(M, K)).astype(F32)
    x[0, :256] = 0.0                                   # all-zero super-block
    x[1, :256] = 3.5                                   # constant super-blocks: every q8_K quant is
    x[1, 256:512] = -0.75                              # -127 (iscale = -127 / x_max) or +127
    x[2, :256] = np.linspace(-2.0, 2.0, 256, dtype=F32)  # |max| ties between -2 and +2 (first wins)
    x[3] *= np.logspace(-3, 3, K, dtype=F32)           # several decades
    return x


def main() -> None:
    rng = np.random.default_rng(0x0A5A0011)
    out: dict[str, np.ndarray] = {}

    # q8_K quantizer
    xk = activations(rng, 6, 512)
    d, qs, bs = q8k_quantize(xk)
    out.update(q8k_x=xk, q8k_d=d, q8k_qs=qs, q8k_bsums=bs)

    # Q4_K x q8_K: random valid blocks (finite fp16 d / dmin), one block of maximal scales
    N, K, M = 24, 1024, 5
    w = rng.integers(0, 256, size=(N, K // 256, 144), dtype=np.uint8)
    w[..., 0:2] = rng.uniform(1e-4, 0.05, size=(N, K // 256)).astype(np.float16)[..., None].view(np.uint8)
    w[..., 2:4] = rng.uniform(0.0, 0.05, size=(N, K // 256)).astype(np.float16)[..., None].view(np.uint8)
    w[0, 0, 4:16] = 0xFF                               # all sub-scales and mins 63
    w[0, 0, 16:] = 0xFF                                # all quants 15
    x = activations(rng, M, K)
    out.update(q4k_w=w.reshape(N, -1), q4k_x=x, q4k_y=dot_q4k(w, x))

    # Q8_0 / Q4_0 x q8_0 (weights quantized by gguf's quantizers)
    for name, qt in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0)):
        N, K, M = 20, 512, 4
        wf = rng.normal(0.0, 0.02, size=(N, K)).astype(F32)
        wq = quants.quantize(wf, qt)
        x = activations(rng, M, K)
        out.update({f"{name}_w": wq, f"{name}_x": x, f"{name}_y": dot_q8(wq, qt, x)})

    path = os.path.join(HERE, "vecdot_numpy.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    main()
