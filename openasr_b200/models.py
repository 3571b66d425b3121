"""Model-level host API: Whisper-shaped configs, seeded synthetic packs and the
resident model handle over the C ABI (oasr_b200_whisper_*).

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
        arr = (bk.OasrNamedTensor * len(pack))()
        self._keep = []
        for i, (name, (t, ne, data)) in enumerate(pack.items()):
            data = np.ascontiguousarray(data)
            nm = name.encode()
            self._keep += [nm, data]
            arr[i].name = nm
            arr[i].type = t
            arr[i].ne[:] = list(ne) + [1] * (4 - len(ne))
            arr[i].data = data.ctypes.data
            arr[i].bytes = data.nbytes
        h = ctypes.c_void_p()
        backend._check(bk.lib().oasr_b200_whisper_load(backend.handle, ctypes.byref(c), arr, len(pack), ctypes.byref(h)))
        self.handle = h
        self._keep = None  # weights are resident now

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
