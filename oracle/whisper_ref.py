"""CPU reference of the Whisper graphs on the oracle's ggml-semantics ops.
TEST INFRASTRUCTURE ONLY (tests/, bench.py's cpu_baseline): restates the
reference's per-utterance graphs with float32 numpy for the elementwise glue
(every add/mul rounds separately, as ggml's f32 ops do):
  frontend   crates/openasr-core/src/models/whisper/mel.rs:120-262 and
             models/audio_frontend/{mod.rs:289-411, mel.rs:70-215}
  prelude    whisper/ggml_executor.rs:640-730 (ggml_conv_1d = im2col to f16 +
             F16 dot; + bias; GELU; positional add)
  encoder    whisper/ggml_executor.rs:1509-1810
  decoder    whisper/ggml_decoder_graph.rs:2840-3010
The DFT is evaluated in float64 (the reference uses rustfft; both round to
f32 power spectra).
The norms, the decode attentions and the matrix products follow the canonical
summation orders of oracle.h (the device's orders), so a decoder step given the
same encoder output is reproduced bit for bit.  The encoder's tensor-core ops
(the fp16 conv GEMM and the 1500-frame attention) accumulate inside the MMA
unit, whose f32 addition order is the hardware's; the encoder is therefore
checked against bounds, and decoding is compared from the device's encoder
output.
"""
from __future__ import annotations

import numpy as np

from . import oracle as oo

N_FFT, HOP = 400, 160
LN_EPS = np.float32(1e-5)


def hann_window(n: int = N_FFT) -> np.ndarray:
    scale = np.float32(np.float32(np.pi) * np.float32(2.0) / np.float32(n))
    i = np.arange(n, dtype=np.float32)
    return (np.float32(0.5) - np.float32(0.5) * np.cos(scale * i, dtype=np.float32)).astype(np.float32)


def _hz_to_mel(hz):
    f_sp = np.float32(200.0) / np.float32(3.0)
    min_log_mel = np.float32(1000.0) / f_sp
    logstep = np.float32(np.log(np.float32(6.4))) / np.float32(27.0)
    return min_log_mel + np.float32(np.log(np.float32(hz) / np.float32(1000.0))) / logstep if hz >= 1000.0 else np.float32(hz) / f_sp


def _mel_to_hz(mel):
    f_sp = np.float32(200.0) / np.float32(3.0)
    min_log_mel = np.float32(1000.0) / f_sp
    logstep = np.float32(np.log(np.float32(6.4))) / np.float32(27.0)
    if mel >= min_log_mel:
        return np.float32(1000.0) * np.float32(np.exp(np.float32(logstep * np.float32(mel - min_log_mel))))
    return f_sp * np.float32(mel)


def mel_filters(n_mels: int, n_fft: int = N_FFT, sr: float = 16000.0) -> np.ndarray:
    bins = n_fft // 2 + 1
    mmin, mmax = _hz_to_mel(0.0), _hz_to_mel(8000.0)
    hz = []
    for i in range(n_mels + 2):
        ratio = np.float32(i) / np.float32(n_mels + 1)
        hz.append(_mel_to_hz(np.float32(mmin + np.float32(ratio * np.float32(mmax - mmin)))))
    f = np.arange(bins, dtype=np.float32) * np.float32(sr) / np.float32(n_fft)
    out = np.zeros((n_mels, bins), np.float32)
    for m in range(n_mels):
        left, center, right = hz[m], hz[m + 1], hz[m + 2]
        lower = (f - left) / np.float32(center - left)
        upper = (right - f) / np.float32(right - center)
        out[m] = np.maximum(np.minimum(lower, upper), 0).astype(np.float32) * np.float32(np.float32(2.0) / np.float32(right - left))
    return out


def log_mel(pcm: np.ndarray, n_mels: int) -> np.ndarray:
    """[n_mels][3000] log-mel of one clip (pad/trim to 30 s)."""
    audio = np.zeros(480000, np.float32)
    take = min(len(pcm), 480000)
    audio[:take] = pcm[:take]
    pad = N_FFT // 2
    padded = np.concatenate([audio[1:pad + 1][::-1], audio, audio[-pad - 1:-1][::-1]])
    n_frames = 3000
    idx = np.arange(n_frames)[:, None] * HOP + np.arange(N_FFT)[None, :]
    frames = (padded[idx] * hann_window()[None, :]).astype(np.float32)
    spec = np.fft.rfft(frames.astype(np.float64), axis=1)
    power = (spec.real ** 2 + spec.imag ** 2).astype(np.float32)
    mel = (power @ mel_filters(n_mels).T).astype(np.float32)  # [frames][mels]
    mel = np.log10(np.maximum(mel, np.float32(1e-10))).astype(np.float32).T
    floor = np.float32(mel.max() - np.float32(8.0))
    return ((np.maximum(mel, floor) + np.float32(4.0)) / np.float32(4.0)).astype(np.float32)


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def layer_norm(x, g, b, family=None):
    """LayerNorm with the device's reduction tree for rows feeding a mul_mat of `family`"""
    x = np.asarray(x, np.float32)
    y = oo.norm_dev(x, float(LN_EPS), False, oo.norm_layout(x.shape[-1], family))
    return (y * g + b).astype(np.float32)


def act_family(wtype: int) -> int:
    """activation family (vec_dot type) of a weight type"""
    return oo.Q8_K if wtype == oo.Q4_K else oo.Q8_0


def conv1d(x_ct: np.ndarray, w_f16_bits: np.ndarray, ic: int, oc: int, stride: int, bias: np.ndarray):
    """ggml_conv_1d (k=3, pad 1): x [C][T] f32 -> [T_out][OC] f32, then + bias, GELU."""
    C, T = x_ct.shape
    T_out = (T + 2 - 3) // stride + 1
    xp = np.zeros((C, T + 2), np.float32)
    xp[:, 1:T + 1] = x_ct
    cols = np.stack([xp[:, t * stride:t * stride + 3] for t in range(T_out)])  # [T_out][C][3]
    im2col = _f16(cols.reshape(T_out, C * 3))
    w = w_f16_bits.reshape(oc, ic * 3)
    y = oo.mul_mat(w, oo.F16, ic * 3, oc, im2col.view(np.uint16), x_type=oo.F16)
    return oo.gelu((y + bias).astype(np.float32))


class WhisperRef:
    def __init__(self, cfg, pack: dict, enc_fa_mode: int = oo.FA_TC128):
        self.cfg = cfg
        self.T = pack
        self.enc_fa_mode = enc_fa_mode
        self.ef = act_family(pack["encoder.blocks.0.attn.query.weight"][0])
        self.df = act_family(pack["decoder.blocks.0.attn.query.weight"][0])
        # decode attention kernel: 4 heads per CTA when the head count allows it (fattn.cu)
        self.fak = oo.FAK_HEADS if cfg.n_heads % 4 == 0 else oo.FAK_SPLIT

    def w(self, name):
        return self.T[name]

    def lin(self, name, x, bias=None):
        t, ne, data = self.T[name + ".weight"]
        y = oo.mul_mat(data, t, ne[0], ne[1], np.ascontiguousarray(x, np.float32))
        if bias is not None or (name + ".bias") in self.T:
            b = self.T[name + ".bias"][2] if bias is None else bias
            y = (y + b).astype(np.float32)
        return y

    def vec(self, name):
        return self.T[name][2]

    # ---- encoder ---------------------------------------------------------------------
    def encode(self, mel: np.ndarray):
        c = self.cfg
        d, H = c.d_model, c.n_heads
        x = conv1d(mel, self.w("encoder.conv1.weight")[2], c.n_mels, d, 1, self.vec("encoder.conv1.bias"))
        x = conv1d(np.ascontiguousarray(x.T), self.w("encoder.conv2.weight")[2], d, d, 2, self.vec("encoder.conv2.bias"))
        x = (x + self.vec("encoder.positional_embedding").reshape(-1, d)).astype(np.float32)
        T = x.shape[0]
        for i in range(c.n_enc_layers):
            p = f"encoder.blocks.{i}."
            h = layer_norm(x, self.vec(p + "attn_ln.weight"), self.vec(p + "attn_ln.bias"), self.ef)
            q, k, v = self.lin(p + "attn.query", h), self.lin(p + "attn.key", h), self.lin(p + "attn.value", h)
            heads = lambda a: np.ascontiguousarray(a.reshape(T, H, 64).transpose(1, 0, 2))[None]
            a = oo.flash_attn_ext(heads(q), heads(k), heads(v), None, 0.125, self.enc_fa_mode)  # (1, T, H, 64)
            x = (x + self.lin(p + "attn.out", a.reshape(T, d))).astype(np.float32)
            h = layer_norm(x, self.vec(p + "mlp_ln.weight"), self.vec(p + "mlp_ln.bias"), self.ef)
            f = oo.gelu(self.lin(p + "mlp.0", h))
            x = (x + self.lin(p + "mlp.2", f)).astype(np.float32)
        return layer_norm(x, self.vec("encoder.ln_post.weight"), self.vec("encoder.ln_post.bias"), self.df)

    def cross_kv(self, enc: np.ndarray):
        """per decoder layer (K f16 [T][d], V f16 [T][d])"""
        out = []
        for i in range(self.cfg.n_dec_layers):
            p = f"decoder.blocks.{i}.cross_attn."
            out.append((_f16(self.lin(p + "key", enc)), _f16(self.lin(p + "value", enc))))
        return out

    # ---- decoder ---------------------------------------------------------------------
    def new_state(self):
        c = self.cfg
        return [(np.zeros((c.n_text_ctx, c.d_model), np.float16), np.zeros((c.n_text_ctx, c.d_model), np.float16))
                for _ in range(c.n_dec_layers)]

    def decode_step(self, token: int, pos: int, cross, self_kv):
        c = self.cfg
        d, H = c.d_model, c.n_heads
        t, ne, data = self.T["decoder.token_embedding.weight"]
        emb = oo.dequantize(t, data[token:token + 1], d)[0]
        x = (emb + self.vec("decoder.positional_embedding").reshape(-1, d)[pos]).astype(np.float32)[None]
        for i in range(c.n_dec_layers):
            p = f"decoder.blocks.{i}."
            h = layer_norm(x, self.vec(p + "attn_ln.weight"), self.vec(p + "attn_ln.bias"), self.df)
            q, k, v = self.lin(p + "attn.query", h), self.lin(p + "attn.key", h), self.lin(p + "attn.value", h)
            kc, vc = self_kv[i]
            kc[pos], vc[pos] = _f16(k[0]), _f16(v[0])
            kk = np.ascontiguousarray(kc[:pos + 1].reshape(pos + 1, H, 64).transpose(1, 0, 2))[None]
            vv = np.ascontiguousarray(vc[:pos + 1].reshape(pos + 1, H, 64).transpose(1, 0, 2))[None]
            a = oo.fa_device(q.reshape(1, H, 1, 64).copy(), kk, vv, None, 0.125, self.fak, c.n_text_ctx)
            x = (x + self.lin(p + "attn.out", a.reshape(1, d))).astype(np.float32)
            h = layer_norm(x, self.vec(p + "cross_attn_ln.weight"), self.vec(p + "cross_attn_ln.bias"), self.df)
            q = self.lin(p + "cross_attn.query", h)
            ck, cv = cross[i]
            Tn = ck.shape[0]
            kk = np.ascontiguousarray(ck.reshape(Tn, H, 64).transpose(1, 0, 2))[None]
            vv = np.ascontiguousarray(cv.reshape(Tn, H, 64).transpose(1, 0, 2))[None]
            a = oo.fa_device(q.reshape(1, H, 1, 64).copy(), kk, vv, None, 0.125, self.fak, Tn)
            x = (x + self.lin(p + "cross_attn.out", a.reshape(1, d))).astype(np.float32)
            h = layer_norm(x, self.vec(p + "mlp_ln.weight"), self.vec(p + "mlp_ln.bias"), self.df)
            x = (x + self.lin(p + "mlp.2", oo.gelu(self.lin(p + "mlp.0", h)))).astype(np.float32)
        h = layer_norm(x, self.vec("decoder.ln.weight"), self.vec("decoder.ln.bias"), oo.Q8_0)
        logits = oo.mul_mat(data, t, ne[0], ne[1], h)[0]
        return logits

    def greedy(self, cross, prompt, n_new):
        state = self.new_state()
        tokens = list(prompt)
        logits_all = []
        for pos in range(len(prompt) + n_new - 1):
            logits = self.decode_step(tokens[pos], pos, cross, state)
            if pos >= len(prompt) - 1:
                logits_all.append(logits)
                tokens.append(int(oo.argmax_first(logits)[0]))
        return np.array(tokens[len(prompt):], np.int32), np.array(logits_all)
