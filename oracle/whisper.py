"""Whisper pieces around the attention calls, restated in numpy (float32).

TEST INFRASTRUCTURE ONLY: produces real attention inputs for the parity tests and pins
the attention restatement end to end against the reference binary (the `mel` and `logits`
commands of src/main.zig:173-191).

- `synth_audio`: the seeded synthetic recording the configs describe (harmonic tone with a
  drifting F0, 8 harmonics at 1/k, 4 Hz amplitude modulation, -30 dB noise, 0.5 s of
  silence every 3 s), 16 kHz int16.
- `mel_filters`: a Slaney-style mel filterbank (the published librosa construction) for
  the synthetic model file; the forward pass reads whatever filters the file holds.
- `log_mel`: src/mel.zig:103-157 (reflect pad 200, 30 s zero tail, 400-point periodic
  Hann, hop 160, power spectrum, filters in float64 sums, log10 floor 1e-10,
  clamp to max - 8, (x + 4) / 4).
- `write_ggml` / `synth_model`: the ggml file layout of src/model.zig:1-13 with tensor
  names from src/encoder.zig:72-95 and src/decoder.zig:94-126.
- `encode`: src/encoder.zig:118-179; `Decoder`: src/decoder.zig:144-218 with Q8 weights
  quantized as src/gemm.zig:208-230.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import numpy as np

from . import attention as A

SAMPLE_RATE = 16000
N_FFT = 400
HOP = 160
N_BINS = N_FFT // 2 + 1
GGML_MAGIC = 0x67676D6C
SOT = 50257  # src/model.zig:38


# ---- synthetic input ---------------------------------------------------------------------

def synth_audio(seconds: float = 30.0, seed: int = 0) -> np.ndarray:
    """int16 samples. F0 follows a triangle wave between 100 and 250 Hz with a 60 s
    period; harmonics k = 1..8 at amplitude 1/k; 4 Hz AM between 0.2 and 1; white noise
    30 dB below the tone's RMS; the tone is muted for the last 0.5 s of every 3 s."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * SAMPLE_RATE))
    t = np.arange(n, dtype=np.float64) / SAMPLE_RATE
    phase_in_period = (t / 60.0) % 1.0
    tri = 1.0 - np.abs(2.0 * phase_in_period - 1.0)  # 0 -> 1 -> 0
    f0 = 100.0 + 150.0 * tri
    phase = 2.0 * np.pi * np.cumsum(f0) / SAMPLE_RATE
    tone = np.zeros(n)
    for k in range(1, 9):
        tone += np.sin(k * phase) / k
    tone *= 0.6 + 0.4 * np.sin(2.0 * np.pi * 4.0 * t)
    tone[(t % 3.0) >= 2.5] = 0.0
    rms = np.sqrt(np.mean(tone[tone != 0] ** 2))
    x = tone + rng.standard_normal(n) * rms * 10 ** (-30 / 20)
    x *= 0.5 / np.max(np.abs(x))
    return np.round(x * 32767).astype(np.int16)


def write_wav(path: str, samples: np.ndarray) -> None:
    s = np.asarray(samples, np.int16)
    data = s.tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE"
    hdr += b"fmt " + struct.pack("<IHHIIHH", 16, 1, 1, SAMPLE_RATE, SAMPLE_RATE * 2, 2, 16)
    hdr += b"data" + struct.pack("<I", len(data))
    with open(path, "wb") as f:
        f.write(hdr + data)


def pcm_to_f32(samples: np.ndarray) -> np.ndarray:
    """s / 32768, as src/wav.zig:37-40."""
    return (np.asarray(samples, np.int16).astype(np.float32) / np.float32(32768.0)).astype(np.float32)


def mel_filters(n_mels: int = 80) -> np.ndarray:
    """Slaney mel filterbank [n_mels][201] (librosa's published construction, f32)."""
    def hz_to_mel(f):
        f = np.asarray(f, np.float64)
        lin = f * 3.0 / 200.0
        logstep = np.log(6.4) / 27.0
        return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-10) / 1000.0) / logstep, lin)

    def mel_to_hz(m):
        m = np.asarray(m, np.float64)
        logstep = np.log(6.4) / 27.0
        return np.where(m >= 15.0, 1000.0 * np.exp(logstep * (m - 15.0)), 200.0 * m / 3.0)

    fft_f = np.linspace(0, SAMPLE_RATE / 2, N_BINS)
    mel_f = mel_to_hz(np.linspace(hz_to_mel(0.0), hz_to_mel(SAMPLE_RATE / 2), n_mels + 2))
    fdiff = np.diff(mel_f)
    ramps = mel_f[:, None] - fft_f[None, :]
    w = np.zeros((n_mels, N_BINS))
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        w[i] = np.maximum(0, np.minimum(lower, upper))
    w *= (2.0 / (mel_f[2:n_mels + 2] - mel_f[:n_mels]))[:, None]
    return w.astype(np.float32)


def log_mel(samples_f32: np.ndarray, filters: np.ndarray) -> np.ndarray:
    """src/mel.zig:103-157. Returns [n_mel][n_len] float32."""
    x = np.asarray(samples_f32, np.float32)
    n_mel = filters.shape[0]
    pad_front = N_FFT // 2
    pad_tail = SAMPLE_RATE * 30
    padded = np.zeros(len(x) + pad_tail + 2 * pad_front, np.float32)
    padded[pad_front:pad_front + len(x)] = x
    for i in range(pad_front):
        padded[i] = x[pad_front - i] if i + 1 < len(x) else 0.0
    n_len = (len(padded) - N_FFT) // HOP
    n_real = len(x) + pad_front
    n_frames_real = min(n_real // HOP + 1, n_len)
    j = np.arange(N_FFT)
    hann = (0.5 - 0.5 * np.cos(2.0 * np.pi * j / N_FFT)).astype(np.float32)
    out = np.full((n_mel, n_len), np.float32(np.log10(1e-10)), np.float32)
    frames = np.zeros((n_frames_real, N_FFT), np.float32)
    for i in range(n_frames_real):
        off = i * HOP
        avail = min(N_FFT, n_real - off)
        frames[i, :avail] = hann[:avail] * padded[off:off + avail]
    spec = np.fft.rfft(frames.astype(np.float64), axis=1)
    power = (spec.real ** 2 + spec.imag ** 2).astype(np.float32)
    sums = power.astype(np.float64) @ filters.astype(np.float64).T  # [frames][n_mel], f64 sums
    out[:, :n_frames_real] = np.log10(np.maximum(sums, 1e-10)).astype(np.float32).T
    mmax = np.float64(out.max()) - 8.0
    o = out.astype(np.float64)
    o = np.where(o < mmax, mmax, o).astype(np.float32)
    return ((o + np.float32(4.0)) / np.float32(4.0)).astype(np.float32)


# ---- model file --------------------------------------------------------------------------

@dataclass
class Hparams:
    n_vocab: int = 51864
    n_audio_ctx: int = 1500
    n_audio_state: int = 384
    n_audio_head: int = 6
    n_audio_layer: int = 4
    n_text_ctx: int = 448
    n_text_state: int = 384
    n_text_head: int = 6
    n_text_layer: int = 4
    n_mels: int = 80
    ftype: int = 1


TINY_EN = Hparams()
BASE_EN = Hparams(n_audio_state=512, n_audio_head=8, n_audio_layer=6, n_text_state=512, n_text_head=8,
                  n_text_layer=6)
SMALL_EN = Hparams(n_audio_state=768, n_audio_head=12, n_audio_layer=12, n_text_state=768, n_text_head=12,
                   n_text_layer=12)


def sinusoids(length: int, channels: int) -> np.ndarray:
    """Whisper's sinusoidal encoder positions (sin half, cos half; timescale 10000)."""
    inc = np.log(10000.0) / (channels // 2 - 1)
    inv = np.exp(-inc * np.arange(channels // 2))
    st = np.arange(length)[:, None] * inv[None, :]
    return np.concatenate([np.sin(st), np.cos(st)], axis=1).astype(np.float32)


@dataclass
class Tensor:
    name: str
    data: np.ndarray  # logical [outer..inner] numpy shape; ggml ne is the reverse
    f16: bool


def synth_model(hp: Hparams, seed: int = 0, encoder_only: bool = False) -> List[Tensor]:
    """Random-init weights N(0, 0.02^2) (f16 2-d weights, linear biases), LayerNorm gains 1
    and biases 0, sinusoidal encoder positions, N(0, 0.02^2) decoder positions."""
    rng = np.random.default_rng(seed)
    T: List[Tensor] = []

    def w(name, *shape):
        T.append(Tensor(name, (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float16), True))

    def b(name, n):
        T.append(Tensor(name, (rng.standard_normal(n, dtype=np.float32) * 0.02).astype(np.float32), False))

    def ln(prefix, n):
        T.append(Tensor(prefix + ".weight", np.ones(n, np.float32), False))
        T.append(Tensor(prefix + ".bias", np.zeros(n, np.float32), False))

    ns = hp.n_audio_state
    w("encoder.conv1.weight", ns, hp.n_mels, 3)
    b("encoder.conv1.bias", ns)
    w("encoder.conv2.weight", ns, ns, 3)
    b("encoder.conv2.bias", ns)
    T.append(Tensor("encoder.positional_embedding", sinusoids(hp.n_audio_ctx, ns), False))
    for i in range(hp.n_audio_layer):
        p = f"encoder.blocks.{i}"
        ln(p + ".attn_ln", ns)
        w(p + ".attn.query.weight", ns, ns); b(p + ".attn.query.bias", ns)
        w(p + ".attn.key.weight", ns, ns)
        w(p + ".attn.value.weight", ns, ns); b(p + ".attn.value.bias", ns)
        w(p + ".attn.out.weight", ns, ns); b(p + ".attn.out.bias", ns)
        ln(p + ".mlp_ln", ns)
        w(p + ".mlp.0.weight", 4 * ns, ns); b(p + ".mlp.0.bias", 4 * ns)
        w(p + ".mlp.2.weight", ns, 4 * ns); b(p + ".mlp.2.bias", ns)
    ln("encoder.ln_post", ns)
    if encoder_only:
        return T
    nt = hp.n_text_state
    w("decoder.token_embedding.weight", hp.n_vocab, nt)
    T.append(Tensor("decoder.positional_embedding",
                    (rng.standard_normal((hp.n_text_ctx, nt), dtype=np.float32) * 0.02).astype(np.float32), False))
    for i in range(hp.n_text_layer):
        p = f"decoder.blocks.{i}"
        ln(p + ".attn_ln", nt)
        w(p + ".attn.query.weight", nt, nt); b(p + ".attn.query.bias", nt)
        w(p + ".attn.key.weight", nt, nt)
        w(p + ".attn.value.weight", nt, nt); b(p + ".attn.value.bias", nt)
        w(p + ".attn.out.weight", nt, nt); b(p + ".attn.out.bias", nt)
        ln(p + ".cross_attn_ln", nt)
        w(p + ".cross_attn.query.weight", nt, nt); b(p + ".cross_attn.query.bias", nt)
        w(p + ".cross_attn.key.weight", nt, nt)
        w(p + ".cross_attn.value.weight", nt, nt); b(p + ".cross_attn.value.bias", nt)
        w(p + ".cross_attn.out.weight", nt, nt); b(p + ".cross_attn.out.bias", nt)
        ln(p + ".mlp_ln", nt)
        w(p + ".mlp.0.weight", 4 * nt, nt); b(p + ".mlp.0.bias", 4 * nt)
        w(p + ".mlp.2.weight", nt, 4 * nt); b(p + ".mlp.2.bias", nt)
    ln("decoder.ln", nt)
    return T


def write_ggml(path: str, hp: Hparams, tensors: List[Tensor], filters: np.ndarray, n_vocab_file: int = 50257):
    """src/model.zig:1-13: magic, 11 hparams, filters, vocab, tensors (ne[0] innermost)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<I", GGML_MAGIC))
        f.write(struct.pack("<11i", hp.n_vocab, hp.n_audio_ctx, hp.n_audio_state, hp.n_audio_head,
                            hp.n_audio_layer, hp.n_text_ctx, hp.n_text_state, hp.n_text_head, hp.n_text_layer,
                            hp.n_mels, hp.ftype))
        f.write(struct.pack("<ii", filters.shape[0], filters.shape[1]))
        f.write(np.ascontiguousarray(filters, np.float32).tobytes())
        f.write(struct.pack("<i", n_vocab_file))
        for i in range(n_vocab_file):
            tok = b" " if i == 220 else f"<{i}>".encode()
            f.write(struct.pack("<I", len(tok)) + tok)
        for t in tensors:
            ne = list(reversed(t.data.shape))
            name = t.name.encode()
            f.write(struct.pack("<iii", len(ne), len(name), 1 if t.f16 else 0))
            f.write(struct.pack(f"<{len(ne)}i", *ne))
            f.write(name)
            f.write(np.ascontiguousarray(t.data, np.float16 if t.f16 else np.float32).tobytes())


# ---- forward passes ----------------------------------------------------------------------

def layer_norm(x, w, b, eps=1e-5):
    """src/ops.zig:371-398 (population variance, eps 1e-5)."""
    x = x.astype(np.float32)
    mean = x.mean(-1, keepdims=True, dtype=np.float32)
    d = x - mean
    var = (d * d).mean(-1, keepdims=True, dtype=np.float32)
    return (d * (np.float32(1.0) / np.sqrt(var + np.float32(eps))) * w + b).astype(np.float32)


def gelu(x):
    """ggml's tanh GELU (src/ops.zig:312-316)."""
    x = x.astype(np.float32)
    c = np.float32(0.7978845608028654)
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * (x + np.float32(0.044715) * x * x * x)))).astype(np.float32)


def linear(x, w, b=None):
    y = x.astype(np.float32) @ w.astype(np.float32).T
    if b is not None:
        y = y + b
    return y.astype(np.float32)


def q8_quantize(w16: np.ndarray):
    """gemm.Q8.quantize (src/gemm.zig:208-230): blocks of 32, scale = absmax / 127,
    round half away from zero of v * (127 / absmax), clamp to +-127."""
    w = w16.astype(np.float32)
    n, k = w.shape
    blk = w.reshape(n, k // 32, 32)
    amax = np.abs(blk).max(-1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    inv = np.where(amax > 0, np.float32(127.0) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    r = (blk * inv[..., None]).astype(np.float32)
    r = np.sign(r) * np.floor(np.abs(r) + np.float32(0.5))
    q = np.clip(r, -127, 127).astype(np.int8)
    return q.reshape(n, k), scale


def q8_dequant(q, scale):
    n, k = q.shape
    return (q.reshape(n, k // 32, 32).astype(np.float32) * scale[..., None]).reshape(n, k).astype(np.float32)


AttnFn = Callable[..., np.ndarray]


def _oracle_attention(q, k, v, n_q, n_kv, n_state, n_head, causal):
    return A.attention(q.reshape(-1), k.reshape(-1), v.reshape(-1), n_q, n_kv, n_state, n_head, causal).reshape(n_q, n_state)


def encode(W: Dict[str, np.ndarray], hp: Hparams, mel: np.ndarray, offset: int = 0,
           attention: AttnFn = _oracle_attention, record: Optional[list] = None) -> np.ndarray:
    """src/encoder.zig:118-179 for the window of 2 * n_ctx frames at `offset`.
    `record`, when given, receives (q, k, v, attn_out) of every layer."""
    n_ctx, ns, H = hp.n_audio_ctx, hp.n_audio_state, hp.n_audio_head
    T = 2 * n_ctx
    n_len = mel.shape[1]
    # conv1: col[t][c*3+k] = mel[c][offset + t + k - 1], zero outside [0, T) and past n_len
    col = np.zeros((T, hp.n_mels, 3), np.float32)
    for kk in range(3):
        ti = np.arange(T) + kk - 1
        fi = offset + ti
        ok = (ti >= 0) & (ti < T) & (fi < n_len)
        col[ok, :, kk] = mel[:, fi[ok]].T
    x = gelu(linear(col.reshape(T, -1), W["encoder.conv1.weight"].reshape(ns, -1), W["encoder.conv1.bias"]))
    col2 = np.zeros((n_ctx, ns, 3), np.float32)
    for kk in range(3):
        ti = 2 * np.arange(n_ctx) + kk - 1
        ok = (ti >= 0) & (ti < T)
        col2[ok, :, kk] = x[ti[ok]]
    x = gelu(linear(col2.reshape(n_ctx, -1), W["encoder.conv2.weight"].reshape(ns, -1), W["encoder.conv2.bias"]))
    x = (x + W["encoder.positional_embedding"][:n_ctx]).astype(np.float32)
    for i in range(hp.n_audio_layer):
        p = f"encoder.blocks.{i}."
        h = layer_norm(x, W[p + "attn_ln.weight"], W[p + "attn_ln.bias"])
        q = linear(h, W[p + "attn.query.weight"], W[p + "attn.query.bias"])
        k = linear(h, W[p + "attn.key.weight"])
        v = linear(h, W[p + "attn.value.weight"], W[p + "attn.value.bias"])
        a = attention(q, k, v, n_ctx, n_ctx, ns, H, False)
        if record is not None:
            record.append((q, k, v, a))
        x = (x + linear(a, W[p + "attn.out.weight"], W[p + "attn.out.bias"])).astype(np.float32)
        h = layer_norm(x, W[p + "mlp_ln.weight"], W[p + "mlp_ln.bias"])
        h = gelu(linear(h, W[p + "mlp.0.weight"], W[p + "mlp.0.bias"]))
        x = (x + linear(h, W[p + "mlp.2.weight"], W[p + "mlp.2.bias"])).astype(np.float32)
    return layer_norm(x, W["encoder.ln_post.weight"], W["encoder.ln_post.bias"])


@dataclass
class Decoder:
    """src/decoder.zig: f32 KV cache, cross K/V per window. `weights="q8"` quantizes the
    decoder matrices as the current source does (src/decoder.zig:220-229); `"f16"` widens
    the file's f16 matrices instead, which is what the shipped reference binary (an older
    build) computes: its logits agree with this variant to about 1e-6."""

    W: Dict[str, np.ndarray]
    hp: Hparams
    attention: AttnFn = _oracle_attention
    weights: str = "q8"
    q8: Dict[str, np.ndarray] = field(default_factory=dict)
    n_past: int = 0

    def __post_init__(self):
        hp = self.hp
        assert self.weights in ("q8", "f16")
        for name, w in self.W.items():
            if name.startswith("decoder.") and w.ndim == 2 and name.endswith("weight") and "positional" not in name:
                if self.weights == "q8":
                    q, s = q8_quantize(w)
                    self.q8[name] = q8_dequant(q, s)
                else:
                    self.q8[name] = w.astype(np.float32)
        nt = hp.n_text_state
        self.cache_k = np.zeros((hp.n_text_layer, hp.n_text_ctx, nt), np.float32)
        self.cache_v = np.zeros_like(self.cache_k)

    def set_audio(self, enc: np.ndarray):
        """setAudio (src/decoder.zig:144-153)."""
        self.cross_k, self.cross_v = [], []
        for i in range(self.hp.n_text_layer):
            p = f"decoder.blocks.{i}.cross_attn."
            self.cross_k.append(linear(enc, self.q8[p + "key.weight"]))
            self.cross_v.append(linear(enc, self.q8[p + "value.weight"], self.W[p + "value.bias"]))
        self.n_past = 0

    def forward(self, tokens: List[int]) -> np.ndarray:
        """forward (src/decoder.zig:160-218): logits of the last token."""
        hp, W, Q = self.hp, self.W, self.q8
        nt, H = hp.n_text_state, hp.n_text_head
        n = len(tokens)
        x = (Q["decoder.token_embedding.weight"][tokens] + W["decoder.positional_embedding"][self.n_past:self.n_past + n]).astype(np.float32)
        n_kv = self.n_past + n
        for i in range(hp.n_text_layer):
            p = f"decoder.blocks.{i}."
            h = layer_norm(x, W[p + "attn_ln.weight"], W[p + "attn_ln.bias"])
            q = linear(h, Q[p + "attn.query.weight"], W[p + "attn.query.bias"])
            self.cache_k[i, self.n_past:n_kv] = linear(h, Q[p + "attn.key.weight"])
            self.cache_v[i, self.n_past:n_kv] = linear(h, Q[p + "attn.value.weight"], W[p + "attn.value.bias"])
            a = self.attention(q, self.cache_k[i, :n_kv], self.cache_v[i, :n_kv], n, n_kv, nt, H, True)
            x = (x + linear(a, Q[p + "attn.out.weight"], W[p + "attn.out.bias"])).astype(np.float32)
            h = layer_norm(x, W[p + "cross_attn_ln.weight"], W[p + "cross_attn_ln.bias"])
            q = linear(h, Q[p + "cross_attn.query.weight"], W[p + "cross_attn.query.bias"])
            a = self.attention(q, self.cross_k[i], self.cross_v[i], n, hp.n_audio_ctx, nt, H, False)
            x = (x + linear(a, Q[p + "cross_attn.out.weight"], W[p + "cross_attn.out.bias"])).astype(np.float32)
            h = layer_norm(x, W[p + "mlp_ln.weight"], W[p + "mlp_ln.bias"])
            h = gelu(linear(h, Q[p + "mlp.0.weight"], W[p + "mlp.0.bias"]))
            x = (x + linear(h, Q[p + "mlp.2.weight"], W[p + "mlp.2.bias"])).astype(np.float32)
        self.n_past += n
        last = layer_norm(x[-1:], W["decoder.ln.weight"], W["decoder.ln.bias"])
        return linear(last, Q["decoder.token_embedding.weight"])[0]


def weights_dict(tensors: List[Tensor]) -> Dict[str, np.ndarray]:
    """Weights as the reference loads them: f16 matrices widened to f32 for the encoder
    (src/encoder.zig:181-187), f16 kept for Q8 quantization of the decoder."""
    out = {}
    for t in tensors:
        out[t.name] = t.data if t.name.startswith("decoder.") and t.f16 else t.data.astype(np.float32)
    return out
