"""Generate the committed golden fixtures for the block formats.

Run in a container that has the `gguf` Python package (0.19.0 was used):

    python tests/golden/gen_golden.py

The third-party `gguf` package (gguf/quants.py) holds numpy restatements of
ggml's Q8_0 / Q4_0 quantizers (documented there as bit-exact with
ggml-quants.c) and of the Q8_0 / Q4_0 / Q4_K dequantizers.  This script feeds
them seeded inputs from numpy's own generator (independent of the oracle's
SplitMix64 stream) and stores inputs and outputs, so the tests can pin the
oracle without importing gguf.
"""
from __future__ import annotations

import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    rng = np.random.default_rng(0x0A5A0001)
    out: dict[str, np.ndarray] = {}

    # Q8_0 / Q4_0: quantize + dequantize, with a few edge blocks (zeros, ties, huge range)
    x = rng.normal(0.0, 1.0, size=(8, 256)).astype(np.float32)
    x[0, :32] = 0.0                                   # all-zero block -> d = 0
    x[1, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    x[2, :32] = 127.0 * np.arange(32, dtype=np.float32) / 31.0  # exact .5 ties after scaling
    x[3, :32] *= 1e4
    x[4, :32] = -x[4, :32].__abs__()                  # all negative: Q4_0 max sign
    out["x"] = x
    for name, qt in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0)):
        q = quants.quantize(x, qt)
        out[f"{name}_bytes"] = q
        out[f"{name}_deq"] = quants.dequantize(q, qt)

    # Q4_K: gguf has no quantizer; dequantize random valid blocks (finite fp16 d/dmin)
    nblk = 64
    blocks = rng.integers(0, 256, size=(nblk, 144), dtype=np.uint8)
    d = rng.uniform(1e-4, 0.05, size=nblk).astype(np.float16)
    dmin = rng.uniform(0.0, 0.05, size=nblk).astype(np.float16)
    blocks[:, 0:2] = d.view(np.uint8).reshape(nblk, 2)
    blocks[:, 2:4] = dmin.view(np.uint8).reshape(nblk, 2)
    blocks[0, 4:] = 0                                  # zero scales / quants
    out["q4_k_bytes"] = blocks
    out["q4_k_deq"] = quants.dequantize(blocks.reshape(1, -1), T.Q4_K).reshape(nblk, 256)

    # fp16 conversions (numpy is IEEE round-to-nearest-even)
    f = np.concatenate([
        rng.normal(0, 1, 4096).astype(np.float32),
        rng.normal(0, 1e-5, 1024).astype(np.float32),   # subnormal range
        rng.normal(0, 3e4, 1024).astype(np.float32),    # near overflow
        np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 2.0**-25, 2.0**-24, np.inf, -np.inf], np.float32),
    ])
    out["f32_for_f16"] = f
    with np.errstate(over="ignore"):
        out["f16_bits"] = f.astype(np.float16).view(np.uint16)

    np.savez_compressed(os.path.join(HERE, "blockfmt_gguf.npz"), **out)
    print("wrote", os.path.join(HERE, "blockfmt_gguf.npz"))


if __name__ == "__main__":
    main()
