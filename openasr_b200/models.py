"""Model-level host API: Whisper- and Qwen3-ASR-shaped configs, seeded synthetic
packs and the resident model handles over the C ABI (oasr_b200_whisper_*,
oasr_b200_qwen_*).

Synthetic packs follow BASELINE.json: linear weights N(0, 0.02) quantized to
the named ggml type (Q8_0 for whisper-tiny, Q4_K for whisper-large-v3), token
embedding / tied logits head Q8_0, conv stem F16, LayerNorm gains 1 and shifts
0, biases and learned positions N(0, 0.02), sinusoidal encoder positions.
Every tensor's stream is seeded from (pack seed, tensor name), so the GPU and
the CPU oracle consume byte-identical tensors.
"""
from __future__ import annotations

import ctypes
import dataclasses
import zlib

import numpy as np

from . import backend as bk


@dataclasses.dataclass(frozen=True)
class WhisperConfig:
    n_mels: int
    d_model: int
    n_heads: int
    n_enc_layers: int
    n_dec_layers: int
    n_vocab: int
    weight_type: int
    n_audio_ctx: int = 1500
    n_text_ctx: int = 448
    max_batch: int = 8

    @property
    def ffn(self) -> int:
        return 4 * self.d_model

    def replace(self, **kw) -> "WhisperConfig":
        return dataclasses.replace(self, **kw)


# BASELINE.json configs[0] and configs[3]
WHISPER_TINY = WhisperConfig(n_mels=80, d_model=384, n_heads=6, n_enc_layers=4, n_dec_layers=4, n_vocab=51865,
                             weight_type=bk.Q8_0)
WHISPER_LARGE_V3 = WhisperConfig(n_mels=128, d_model=1280, n_heads=20, n_enc_layers=32, n_dec_layers=32,
                                 n_vocab=51866, weight_type=bk.Q4_K)

# decoder prompt <|startoftranscript|><|en|><|transcribe|><|notimestamps|> and <|endoftext|>
PROMPT = {51865: [50258, 50259, 50359, 50363], 51866: [50258, 50259, 50360, 50364]}
EOT = 50257


def _seed(base: int, name: str) -> int:
    return (base * 0x9E3779B97F4A7C15 + zlib.crc32(name.encode())) & (2**64 - 1)


def _sinusoids(length: int, channels: int) -> np.ndarray:
    half = channels // 2
    inc = np.log(10000.0) / (half - 1)
    inv = np.exp(-inc * np.arange(half, dtype=np.float64))
    t = np.arange(length, dtype=np.float64)[:, None] * inv[None, :]
    return np.concatenate([np.sin(t), np.cos(t)], axis=1).astype(np.float32)


def whisper_synthetic_pack(cfg: WhisperConfig, seed: int = 0x0A5A0001, synth=None, quantize=None) -> dict:
    """{name: (ggml_type, ne[4], ndarray)} for a seeded random Whisper-shaped pack.
    `synth(seed, n, mean, std)` and `quantize(type, x2d)` default to this library's
    host helpers (the CPU oracle has bit-identical ones)."""
    synth = synth or bk.synth_normal
    quantize = quantize or bk.quantize
    d, f = cfg.d_model, cfg.ffn
    T: dict = {}

    def lin(name, K, N, qt):
        w = synth(_seed(seed, name), N * K, 0.0, 0.02).reshape(N, K)
        T[name] = (qt, [K, N, 1, 1], quantize(qt, w))

    def vec(name, n, kind):
        if kind == "one":
            v = np.ones(n, np.float32)
        elif kind == "zero":
            v = np.zeros(n, np.float32)
        else:
            v = synth(_seed(seed, name), n, 0.0, 0.02)
        T[name] = (bk.F32, [n, 1, 1, 1], v)

    def conv(name, IC, OC):
        w = synth(_seed(seed, name), OC * IC * 3, 0.0, 0.02).astype(np.float16)
        T[name] = (bk.F16, [3, IC, OC, 1], w.view(np.uint16))

    qt = cfg.weight_type
    conv("encoder.conv1.weight", cfg.n_mels, d)
    vec("encoder.conv1.bias", d, "rand")
    conv("encoder.conv2.weight", d, d)
    vec("encoder.conv2.bias", d, "rand")
    T["encoder.positional_embedding"] = (bk.F32, [d, cfg.n_audio_ctx, 1, 1], _sinusoids(cfg.n_audio_ctx, d))

    def block(p, cross):
        for ln in ["attn_ln", "mlp_ln"] + (["cross_attn_ln"] if cross else []):
            vec(p + ln + ".weight", d, "one")
            vec(p + ln + ".bias", d, "zero")
        for att in ["attn"] + (["cross_attn"] if cross else []):
            for proj in ("query", "key", "value", "out"):
                lin(f"{p}{att}.{proj}.weight", d, d, qt)
                if proj != "key":
                    vec(f"{p}{att}.{proj}.bias", d, "rand")
        lin(p + "mlp.0.weight", d, f, qt)
        vec(p + "mlp.0.bias", f, "rand")
        lin(p + "mlp.2.weight", f, d, qt)
        vec(p + "mlp.2.bias", d, "rand")

    for i in range(cfg.n_enc_layers):
        block(f"encoder.blocks.{i}.", False)
    vec("encoder.ln_post.weight", d, "one")
    vec("encoder.ln_post.bias", d, "zero")
    lin("decoder.token_embedding.weight", d, cfg.n_vocab, bk.Q8_0)
    pe = synth(_seed(seed, "decoder.positional_embedding"), cfg.n_text_ctx * d, 0.0, 0.02)
    T["decoder.positional_embedding"] = (bk.F32, [d, cfg.n_text_ctx, 1, 1], pe)
    for i in range(cfg.n_dec_layers):
        block(f"decoder.blocks.{i}.", True)
    vec("decoder.ln.weight", d, "one")
    vec("decoder.ln.bias", d, "zero")
    return T


def _named_tensors(pack: dict):
    """oasr_named_tensor array over a pack's host arrays (+ the objects to keep alive)"""
    arr = (bk.OasrNamedTensor * len(pack))()
    keep = []
    for i, (name, (t, ne, data)) in enumerate(pack.items()):
        data = np.ascontiguousarray(data)
        nm = name.encode()
        keep += [nm, data]
        arr[i].name = nm
        arr[i].type = t
        arr[i].ne[:] = list(ne) + [1] * (4 - len(ne))
        arr[i].data = data.ctypes.data
        arr[i].bytes = data.nbytes
    return arr, keep


def synthetic_audio(seed: int, n_samples: int, rms: float = 0.1) -> np.ndarray:
    """16 kHz Gaussian noise at -20 dBFS RMS (sigma 0.1)."""
    return bk.synth_normal(seed, n_samples, 0.0, rms)


class WhisperModel:
    """A resident Whisper model on one backend (oasr_b200_whisper_*)."""

    def __init__(self, backend: bk.Backend, cfg: WhisperConfig, pack: dict):
        self.backend = backend
        self.cfg = cfg
        c = bk.OasrWhisperConfig(cfg.n_mels, cfg.d_model, cfg.n_heads, cfg.n_enc_layers, cfg.n_dec_layers,
                                 cfg.n_vocab, cfg.n_audio_ctx, cfg.n_text_ctx, cfg.max_batch)
        arr, keep = _named_tensors(pack)
        h = ctypes.c_void_p()
        backend._check(bk.lib().oasr_b200_whisper_load(backend.handle, ctypes.byref(c), arr, len(pack), ctypes.byref(h)))
        self.handle = h
        del keep  # weights are resident now

    def close(self) -> None:
        if self.handle:
            bk.lib().oasr_b200_whisper_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    @staticmethod
    def _pcm(clips):
        pcm = np.ascontiguousarray(np.concatenate(clips).astype(np.float32))
        ns = np.array([len(c) for c in clips], np.int64)
        return pcm, ns

    def mel(self, clips) -> np.ndarray:
        pcm, ns = self._pcm(clips)
        out = np.empty((len(clips), self.cfg.n_mels, 3000), np.float32)
        self.backend._check(bk.lib().oasr_b200_whisper_mel(self.handle, pcm.ctypes.data, ns.ctypes.data, len(clips),
                                                           out.ctypes.data))
        return out

    def encode(self, mel: np.ndarray | None, n: int, want_output: bool = True) -> np.ndarray | None:
        out = np.empty((n, self.cfg.n_audio_ctx, self.cfg.d_model), np.float32) if want_output else None
        m = None if mel is None else np.ascontiguousarray(mel, np.float32)
        self.backend._check(bk.lib().oasr_b200_whisper_encode(self.handle, None if m is None else m.ctypes.data, n,
                                                              None if out is None else out.ctypes.data))
        return out

    def decode_step(self, tokens, pos: int):
        tk = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty((len(tk), self.cfg.n_vocab), np.float32)
        nxt = np.empty(len(tk), np.int32)
        self.backend._check(bk.lib().oasr_b200_whisper_decode_step(self.handle, tk.ctypes.data, len(tk), pos,
                                                                   logits.ctypes.data, nxt.ctypes.data))
        return logits, nxt

    def mel_device(self, pcm_dev, n_samples) -> None:
        """frontend from a device tensor of concatenated clips (torch, f32)"""
        ns = np.ascontiguousarray(n_samples, np.int64)
        self.backend._check(bk.lib().oasr_b200_whisper_mel_device(self.handle, pcm_dev.data_ptr(), ns.ctypes.data, len(ns)))

    def generate_device(self, n_utts: int, tokens_dev, n_new: int = 224, prompt=None) -> None:
        """encoder + greedy decode into a device int32 tensor [n_utts][n_new]; returns without waiting"""
        self._prompt = np.ascontiguousarray(prompt if prompt is not None else PROMPT[self.cfg.n_vocab], np.int32)
        self.backend._check(bk.lib().oasr_b200_whisper_generate(
            self.handle, n_utts, self._prompt.ctypes.data, len(self._prompt), n_new, EOT, 0, tokens_dev.data_ptr(), 1))

    def transcribe(self, clips, n_new: int = 224, prompt=None, stop_at_eot: bool = False) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt if prompt is not None else PROMPT[self.cfg.n_vocab], np.int32)
        pcm, ns = self._pcm(clips)
        out = np.empty((len(clips), n_new), np.int32)
        self.backend._check(bk.lib().oasr_b200_whisper_transcribe(
            self.handle, pcm.ctypes.data, ns.ctypes.data, len(clips), prompt.ctypes.data, len(prompt), n_new, EOT,
            1 if stop_at_eot else 0, out.ctypes.data))
        return out

    @property
    def max_batch(self) -> int:
        """serving slots after the load-time VRAM cap"""
        return int(bk.lib().oasr_b200_whisper_max_batch(self.handle))

    def serve(self, clips, max_new: int = 224, budgets=None, prompt=None, stop_at_eot: bool = True,
              max_width: int = 0, check_every: int = 8, eot: int = EOT):
        """Continuous-batching transcription of a queue of clips (models/seq2seq_serve_batch.rs
        decode_continuous_batch): finished slots are refilled from the queue and the batch
        re-bucketed to powers of two.  Returns ([generated tokens per clip], ServeStats)."""
        prompt = np.ascontiguousarray(prompt if prompt is not None else PROMPT[self.cfg.n_vocab], np.int32)
        pcm, ns = self._pcm(clips)
        n = len(clips)
        out = np.empty((n, max_new), np.int32)
        lens = np.zeros(n, np.int32)
        bud = None if budgets is None else np.ascontiguousarray(budgets, np.int32)
        st = bk.ServeStats()
        self.backend._check(bk.lib().oasr_b200_whisper_serve(
            self.handle, pcm.ctypes.data, ns.ctypes.data, n, prompt.ctypes.data, len(prompt),
            None if bud is None else bud.ctypes.data, max_new, eot, 1 if stop_at_eot else 0, max_width, check_every,
            out.ctypes.data, lens.ctypes.data, ctypes.byref(st)))
        return [out[i, :lens[i]].copy() for i in range(n)], st


# ---- Qwen3-ASR LLM decoder --------------------------------------------------------------
@dataclasses.dataclass(frozen=True)
class QwenConfig:
    d_model: int = 1024
    n_layers: int = 28
    n_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    n_vocab: int = 151936
    max_pos: int = 2048
    max_prefill: int = 512
    max_batch: int = 8
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    weight_type: int = bk.Q8_0

    def replace(self, **kw) -> "QwenConfig":
        return dataclasses.replace(self, **kw)


# Qwen3-ASR-0.6B-shaped decoder, seeded random Q8_0
QWEN3_ASR_0_6B = QwenConfig()
# The 390-frame prompt stands for 30 s of audio (13 audio embeddings per second).
QWEN_PREFIX_FRAMES = 390
QWEN_PREFIX_SECONDS = 30.0
QWEN_EOS = 151645  # <|im_end|>


def qwen_synthetic_pack(cfg: QwenConfig, seed: int = 0x0A5A0003, tied: bool = True, synth=None, quantize=None) -> dict:
    """{name: (ggml_type, ne[4], ndarray)} for a seeded random Qwen3-shaped decoder in the
    GGUF names of the reference's qwen3 contract.  Linear weights N(0, 0.02) quantized to
    cfg.weight_type, token embedding Q8_0 (also the logits head when `tied`, as in
    Qwen3-0.6B), RMSNorm gains N(1, 0.1) so that a missing or misplaced gain shows."""
    synth = synth or bk.synth_normal
    quantize = quantize or bk.quantize
    d, D, qt = cfg.d_model, cfg.head_dim, cfg.weight_type
    T: dict = {}

    def lin(name, K, N, t):
        w = synth(_seed(seed, name), N * K, 0.0, 0.02).reshape(N, K)
        T[name] = (t, [K, N, 1, 1], quantize(t, w))

    def gain(name, n):
        T[name] = (bk.F32, [n, 1, 1, 1], synth(_seed(seed, name), n, 1.0, 0.1))

    lin("token_embd.weight", d, cfg.n_vocab, bk.Q8_0)
    if not tied:
        lin("output.weight", d, cfg.n_vocab, bk.Q8_0)
    gain("output_norm.weight", d)
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        gain(p + "attn_norm.weight", d)
        lin(p + "attn_q.weight", d, cfg.n_heads * D, qt)
        lin(p + "attn_k.weight", d, cfg.n_kv_heads * D, qt)
        lin(p + "attn_v.weight", d, cfg.n_kv_heads * D, qt)
        gain(p + "attn_q_norm.weight", D)
        gain(p + "attn_k_norm.weight", D)
        lin(p + "attn_output.weight", cfg.n_heads * D, d, qt)
        gain(p + "ffn_norm.weight", d)
        lin(p + "ffn_gate.weight", d, cfg.ffn, qt)
        lin(p + "ffn_up.weight", d, cfg.ffn, qt)
        lin(p + "ffn_down.weight", cfg.ffn, d, qt)
    return T


def qwen_synthetic_prefix(seed: int, n_seq: int, n_tok: int, d: int) -> np.ndarray:
    """[n_seq][n_tok][d] audio-embedding frames drawn N(0, 1), one stream per sequence"""
    return np.stack([bk.synth_normal(_seed(seed, f"prefix.{s}"), n_tok * d).reshape(n_tok, d) for s in range(n_seq)])


class QwenModel:
    """A resident Qwen3-ASR LLM decoder on one backend (oasr_b200_qwen_*)."""

    def __init__(self, backend: bk.Backend, cfg: QwenConfig, pack: dict):
        self.backend = backend
        self.cfg = cfg
        c = bk.OasrQwenConfig(cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn,
                              cfg.n_vocab, cfg.max_pos, cfg.max_prefill, cfg.max_batch, cfg.rope_theta, cfg.rms_eps)
        arr, keep = _named_tensors(pack)
        h = ctypes.c_void_p()
        backend._check(bk.lib().oasr_b200_qwen_load(backend.handle, ctypes.byref(c), arr, len(pack), ctypes.byref(h)))
        self.handle = h
        del keep

    def close(self) -> None:
        if self.handle:
            bk.lib().oasr_b200_qwen_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    def prefill(self, emb: np.ndarray):
        """emb [n_seq][n_tok][d] -> (logits [n_seq][n_vocab], first tokens [n_seq])"""
        e = np.ascontiguousarray(emb, np.float32)
        n, T = e.shape[0], e.shape[1]
        logits = np.empty((n, self.cfg.n_vocab), np.float32)
        nxt = np.empty(n, np.int32)
        self.backend._check(bk.lib().oasr_b200_qwen_prefill(self.handle, e.ctypes.data, 0, n, T, logits.ctypes.data,
                                                            nxt.ctypes.data))
        return logits, nxt

    def decode_step(self, tokens, pos: int):
        tk = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty((len(tk), self.cfg.n_vocab), np.float32)
        nxt = np.empty(len(tk), np.int32)
        self.backend._check(bk.lib().oasr_b200_qwen_decode_step(self.handle, tk.ctypes.data, len(tk), pos,
                                                                logits.ctypes.data, nxt.ctypes.data))
        return logits, nxt

    def generate(self, emb: np.ndarray, n_new: int = 256, eos: int = QWEN_EOS, stop_at_eos: bool = False) -> np.ndarray:
        """prefill + n_new greedy tokens per sequence -> [n_seq][n_new]"""
        e = np.ascontiguousarray(emb, np.float32)
        n, T = e.shape[0], e.shape[1]
        out = np.empty((n, n_new), np.int32)
        self.backend._check(bk.lib().oasr_b200_qwen_generate(self.handle, e.ctypes.data, 0, n, T, n_new, eos,
                                                             1 if stop_at_eos else 0, out.ctypes.data, 0))
        return out

    def generate_device(self, emb_dev, n_seq: int, n_tok: int, tokens_dev, n_new: int = 256) -> None:
        """device embeddings (torch f32 [n_seq][n_tok][d]) -> device tokens; returns without waiting"""
        self.backend._check(bk.lib().oasr_b200_qwen_generate(self.handle, emb_dev.data_ptr(), 1, n_seq, n_tok, n_new,
                                                             QWEN_EOS, 0, tokens_dev.data_ptr(), 1))

    def read_kv(self, layer: int, seq: int, n_pos: int):
        """(K, V) f16 [n_kv_heads][n_pos][head_dim] of one layer and sequence"""
        c = self.cfg
        k = np.empty((c.n_kv_heads, n_pos, c.head_dim), np.float16)
        v = np.empty_like(k)
        self.backend._check(bk.lib().oasr_b200_qwen_read_kv(self.handle, layer, seq, n_pos, k.ctypes.data,
                                                            v.ctypes.data))
        return k, v
