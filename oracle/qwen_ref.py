"""CPU reference of the Qwen3-ASR LLM decoder on the oracle's ggml-semantics ops.
TEST INFRASTRUCTURE ONLY (tests/, bench.py's cpu_baseline and reference arm):
restates the graph the reference builds per decoder layer,
  crates/openasr-core/src/nn/decoder.rs:1850-2140 (llm_layer)
    RMSNorm * attn_norm -> q, k, v projections -> per-head RMSNorm * q_norm /
    k_norm -> RoPE NEOX (ggml_rope_ext, cpu_graph.rs:1135-1155: freq_scale 1,
    ext_factor 0, attn_factor 1) -> set_rows f16 K/V -> flash_attn_ext(scale
    1/sqrt(head_dim), GQA) -> attn_output -> residual -> RMSNorm * ffn_norm ->
    silu(gate) * up -> down -> residual (nn/ffn.rs:64-91)
  models/qwen/llm_transformer.rs:2096-2115 (build_fused_logits_top1)
    RMSNorm * output_norm -> lm_head -> first-max argmax
with eps 1e-6 (logits_head.rs:23) and theta 1e6 (llm_transformer.rs:489).
The prompt runs as one causal pass (run_prefill, llm_transformer.rs:3859-3895,
causal f16 mask as build_causal_mask_f16_bits, nn/decoder.rs:766-790); each
decode step attends over the live prefix (run_step, llm_transformer.rs:3203).
Prompt attention of `tc_min_rows` or more positions is evaluated in the
oracle's tensor-core arithmetic mode (fp16 operands and probabilities, 128-key
blocks), the arithmetic the device's prompt pass is specified to use (ggml's
CUDA backend makes the same fp16 conversion); its accumulation inside the MMA
unit is the hardware's, so that op is checked against a bound.  Shorter prompts
and every decode step use the canonical summation orders of oracle.h (RMSNorm
trees, the split / GQA decode attention, the SiLU's e^x, block-order mul_mat):
a decode step from the same cache is the device's bit for bit.
Every elementwise op rounds to float32 separately, as ggml's f32 ops do.
"""
from __future__ import annotations

import numpy as np

from . import oracle as oo


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def causal_mask(n_q: int, n_kv: int, pos0: int = 0) -> np.ndarray:
    """f16 [n_q][n_kv]: query t (at position pos0 + t) sees kv <= pos0 + t."""
    m = np.zeros((n_q, n_kv), np.float16)
    for t in range(n_q):
        m[t, pos0 + t + 1:] = -np.inf
    return m


class QwenRef:
    """`cfg` carries d_model, n_layers, n_heads, n_kv_heads, head_dim, ffn, n_vocab,
    rope_theta, rms_eps, max_pos; `pack` is {name: (type, ne, data)} in the GGUF
    tensor names of the reference's qwen3 contract (decoder_contract.rs)."""

    def __init__(self, cfg, pack: dict, tc_min_rows: int = 64):
        self.cfg = cfg
        self.T = pack
        self.tc_min_rows = tc_min_rows
        self.out_name = "output.weight" if "output.weight" in pack else "token_embd.weight"

    def vec(self, name):
        return self.T[name][2]

    def lin(self, name, x):
        t, ne, data = self.T[name]
        return oo.mul_mat(data, t, ne[0], ne[1], np.ascontiguousarray(x, np.float32))

    def rms(self, x, w):
        """RMSNorm * w with the device's reduction tree: rows of d feed a Q8_0 mul_mat
        (q8_0 planes); per-head rows of 128 are one warp (qkv_post in model_qwen.cu)"""
        x = np.asarray(x, np.float32)
        n = x.shape[-1]
        layout = oo.norm_layout(n, oo.Q8_0) if n != self.cfg.head_dim else oo.NORM_E4
        return (oo.norm_dev(x, self.cfg.rms_eps, True, layout) * w).astype(np.float32)

    def new_cache(self, n_seq: int = 1, n_pos: int | None = None):
        """per layer (K, V) f16 [n_seq][n_kv_heads][n_pos (default max_pos)][head_dim]"""
        c = self.cfg
        shape = (n_seq, c.n_kv_heads, n_pos or c.max_pos, c.head_dim)
        return [(np.zeros(shape, np.float16), np.zeros(shape, np.float16)) for _ in range(c.n_layers)]

    def embed(self, tokens) -> np.ndarray:
        t, ne, data = self.T["token_embd.weight"]
        return np.stack([oo.dequantize(t, data[int(k):int(k) + 1], ne[0])[0] for k in tokens]).astype(np.float32)

    def layer(self, x: np.ndarray, l: int, cache, s: int, pos0: int, decode: bool = False):
        """x [T][d] = tokens at positions pos0..pos0+T-1 of sequence s; updates cache[l][:, s].
        decode: a decode step (one row attending over a cache of max_pos positions)."""
        c = self.cfg
        T, D, H, HKV = x.shape[0], c.head_dim, c.n_heads, c.n_kv_heads
        p = f"blk.{l}."
        h = self.rms(x, self.vec(p + "attn_norm.weight"))
        q = self.lin(p + "attn_q.weight", h).reshape(T, H, D)
        k = self.lin(p + "attn_k.weight", h).reshape(T, HKV, D)
        v = self.lin(p + "attn_v.weight", h).reshape(T, HKV, D)
        q = self.rms(q, self.vec(p + "attn_q_norm.weight"))
        k = self.rms(k, self.vec(p + "attn_k_norm.weight"))
        pos = np.arange(pos0, pos0 + T, dtype=np.int32)
        q = oo.rope_neox(q, pos, c.rope_theta)
        k = oo.rope_neox(k, pos, c.rope_theta)
        kc, vc = cache[l]
        kc[s, :, pos0:pos0 + T] = _f16(k.transpose(1, 0, 2))
        vc[s, :, pos0:pos0 + T] = _f16(v.transpose(1, 0, 2))
        n_kv = pos0 + T
        mask = causal_mask(T, n_kv, pos0) if T > 1 else None
        qh = np.ascontiguousarray(q.transpose(1, 0, 2))[None]
        kk, vv = np.ascontiguousarray(kc[s:s + 1, :, :n_kv]), np.ascontiguousarray(vc[s:s + 1, :, :n_kv])
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        if T >= self.tc_min_rows and pos0 == 0:
            a = oo.flash_attn_ext(qh, kk, vv, mask, scale, oo.FA_TC128)  # (1, T, H, D)
        elif T == 1:
            # one query row over head-major f16 rows of 256 bytes: the GQA decode kernel, its
            # split plan taken from the cache length (decode) or the prompt length (prefill)
            a = oo.fa_device(qh, kk, vv, None, scale, oo.FAK_GQA, c.max_pos if decode else n_kv)
        else:
            a = oo.fa_device(qh, kk, vv, mask, scale, oo.FAK_SPLIT, n_kv)
        x = (x + self.lin(p + "attn_output.weight", a.reshape(T, H * D))).astype(np.float32)
        h = self.rms(x, self.vec(p + "ffn_norm.weight"))
        g = self.lin(p + "ffn_gate.weight", h)
        u = self.lin(p + "ffn_up.weight", h)
        f = (oo.silu(g) * u).astype(np.float32)
        return (x + self.lin(p + "ffn_down.weight", f)).astype(np.float32)

    def head(self, x_last: np.ndarray) -> np.ndarray:
        """logits [rows][n_vocab] of final hidden rows"""
        h = self.rms(np.atleast_2d(x_last), self.vec("output_norm.weight"))
        return self.lin(self.out_name, h)

    def prefill(self, emb: np.ndarray, cache, s: int = 0) -> np.ndarray:
        """emb [T][d] prompt embeddings of sequence s -> logits of the last position"""
        x = np.ascontiguousarray(emb, np.float32)
        for l in range(self.cfg.n_layers):
            x = self.layer(x, l, cache, s, 0)
        return self.head(x[-1])[0]

    def step(self, tokens, pos: int, cache) -> np.ndarray:
        """one decode step: token of each sequence at position pos -> logits [n_seq][n_vocab]"""
        out = []
        for s, tok in enumerate(tokens):
            x = self.embed([tok])
            for l in range(self.cfg.n_layers):
                x = self.layer(x, l, cache, s, pos, decode=True)
            out.append(self.head(x)[0])
        return np.array(out)

    def greedy(self, emb: np.ndarray, n_new: int):
        """prefill + n_new greedy tokens (first from the prompt's last logits)"""
        cache = self.new_cache(1)
        logits = [self.prefill(emb, cache)]
        tokens = [int(oo.argmax_first(logits[-1])[0])]
        T = emb.shape[0]
        for i in range(n_new - 1):
            logits.append(self.step([tokens[-1]], T + i, cache)[0])
            tokens.append(int(oo.argmax_first(logits[-1])[0]))
        return np.array(tokens, np.int32), np.array(logits)
