"""CPU restatement of the reference audio tower -- TEST INFRASTRUCTURE ONLY.

Follows cnmoro/fast-moss-diarization:
  * `WhisperEncoder` (`crates/fmd-core/src/model/whisper_encoder.rs`):
    conv1 (k3 s1 p1) + erf-GELU, conv2 (k3 s2 p1) + erf-GELU, learned
    positions, pre-LN layers with q and k both scaled by head_dim^-1/4, dense
    bidirectional attention, final LayerNorm (eps 1e-5);
  * `VqAdaptor` (`crates/fmd-core/src/model/adaptor.rs`): time merge by
    `merge_size` frames, Linear -> SiLU -> Linear -> LayerNorm;
  * `MossModel::encode_audio` (`crates/fmd-core/src/model/mod.rs:82-126`):
    batched encoder passes, per-chunk trim to `tokens * merge` frames,
    per-file concatenation, then the adaptor.
Tensors are torch f32 on the CPU. With `act="bf16"` / `"f16"` every op output
is rounded through that dtype where the reference stores one (candle ops in
the activation dtype), which shows how far the reference itself sits from
f32; `act=None` is the f32 restatement the GPU path is checked against.

Parity status: the encoder restatement is pinned against the independent
Whisper encoder of `transformers` (tests/golden/make_whisper_golden.py,
tests/golden/whisper_tiny.npz); `time_merge` against the reference's own unit
tests (adaptor.rs:88-128, restated in tests/test_audio_oracle.py). The
adaptor's projections are pinned only through torch's own ops.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

LN_EPS = 1e-5  # whisper_encoder.rs:14


@dataclass
class AudioConfig:
    """`AudioConfig` (config.rs:61-75) + the adaptor fields of `ModelConfig`."""
    num_mel_bins: int = 80
    d_model: int = 1024
    encoder_layers: int = 24
    encoder_attention_heads: int = 16
    encoder_ffn_dim: int = 4096
    max_source_positions: int = 1500
    audio_merge_size: int = 4
    adaptor_input_dim: int = 4096
    hidden_size: int = 1024
    adaptor_norm_eps: float = 1e-6

    @property
    def head_dim(self) -> int:  # config.rs:72-74
        return self.d_model // self.encoder_attention_heads


def _t(a) -> torch.Tensor:
    return torch.as_tensor(np.asarray(a, dtype=np.float32))


class WhisperRef:
    def __init__(self, cfg: AudioConfig, weights: dict, act: str | None = None):
        self.cfg = cfg
        self.dt = {None: None, "bf16": torch.bfloat16, "f16": torch.float16}[act]
        w = weights
        self.conv1_w, self.conv1_b = _t(w["conv1_w"]), _t(w["conv1_b"])
        self.conv2_w, self.conv2_b = _t(w["conv2_w"]), _t(w["conv2_b"])
        self.pos = _t(w["positions"])
        self.layers = [{k: _t(v) for k, v in lw.items()} for lw in w["layers"]]
        self.ln_w, self.ln_b = _t(w["ln_w"]), _t(w["ln_b"])
        self.ad = {k: _t(w[k]) for k in ("ad1_w", "ad1_b", "ad2_w", "ad2_b", "adn_w", "adn_b")}

    def r(self, x: torch.Tensor) -> torch.Tensor:
        return x if self.dt is None else x.to(self.dt).to(torch.float32)

    # ---- ops (linear.rs:29-65, :306-330) ----
    def linear(self, x, w, b=None):
        y = self.r(x @ w.T)
        return y if b is None else self.r(y + self.r(b))

    def layer_norm(self, x, w, b, eps):
        mean = x.mean(-1, keepdim=True)
        var = ((x - mean) ** 2).mean(-1, keepdim=True)
        return self.r((x - mean) / torch.sqrt(var + eps) * w + b)

    def gelu(self, x):
        return self.r(0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0))))

    def conv1d(self, x, w, b, stride):
        y = self.r(torch.nn.functional.conv1d(x, w, None, stride=stride, padding=1))
        return self.r(y + self.r(b)[None, :, None])

    # ---- encoder (whisper_encoder.rs:45-64, :88-100, :142-163) ----
    def attention(self, x, L):
        b, t, d = x.shape
        H, hd = self.cfg.encoder_attention_heads, self.cfg.head_dim
        scale = hd ** -0.25
        q = self.r(self.linear(x, L["q_w"], L["q_b"]) * scale)
        k = self.r(self.linear(x, L["k_w"]) * scale)
        v = self.linear(x, L["v_w"], L["v_b"])
        split = lambda z: z.reshape(b, t, H, hd).transpose(1, 2)
        s = self.r(split(q) @ split(k).transpose(-1, -2))
        p = self.r(torch.softmax(s, dim=-1))
        ctx = self.r(p @ split(v)).transpose(1, 2).reshape(b, t, d)
        return self.linear(ctx, L["o_w"], L["o_b"])

    def layer(self, x, L):
        x = self.r(x + self.attention(self.layer_norm(x, L["ln1_w"], L["ln1_b"], LN_EPS), L))
        h = self.layer_norm(x, L["ln2_w"], L["ln2_b"], LN_EPS)
        h = self.linear(self.gelu(self.linear(h, L["fc1_w"], L["fc1_b"])), L["fc2_w"], L["fc2_b"])
        return self.r(x + h)

    def forward(self, mel) -> torch.Tensor:
        """(batch, n_mels, 2 x frames) log-mel -> (batch, frames, d_model)."""
        x = self.r(_t(mel))
        x = self.gelu(self.conv1d(x, self.conv1_w, self.conv1_b, 1))
        x = self.gelu(self.conv1d(x, self.conv2_w, self.conv2_b, 2))
        x = x.transpose(1, 2)
        x = self.r(x + self.r(self.pos[: x.shape[1]]))
        for L in self.layers:
            x = self.layer(x, L)
        return self.layer_norm(x, self.ln_w, self.ln_b, LN_EPS)

    # ---- adaptor (adaptor.rs:41-64) ----
    def time_merge(self, x) -> torch.Tensor:
        b, t, d = x.shape
        m = self.cfg.audio_merge_size
        g = t // m
        return x[:, : g * m].reshape(b, g, d * m)

    def adaptor(self, merged) -> torch.Tensor:
        a = self.ad
        h = self.linear(merged, a["ad1_w"], a["ad1_b"])
        h = self.r(h * torch.sigmoid(h))
        h = self.linear(h, a["ad2_w"], a["ad2_b"])
        return self.layer_norm(h, a["adn_w"], a["adn_b"], self.cfg.adaptor_norm_eps)

    # ---- MossModel::encode_audio (model/mod.rs:82-126) ----
    def encode_audio(self, mel, chunk_token_lengths, chunk_mapping, num_audios, encoder_batch=16):
        mel = _t(mel)
        n = mel.shape[0]
        frames = []
        start = 0
        while start < n:
            take = min(max(encoder_batch, 1), n - start)
            enc = self.forward(mel[start:start + take])
            frames.extend(enc[i:i + 1] for i in range(take))
            start += take
        merge = self.cfg.audio_merge_size
        per_audio = [[] for _ in range(num_audios)]
        for idx, chunk in enumerate(frames):
            keep = chunk_token_lengths[idx] * merge
            per_audio[chunk_mapping[idx]].append(chunk[:, : min(keep, chunk.shape[1])])
        out = []
        for parts in per_audio:
            if not parts:
                raise ValueError("an audio without chunks cannot be joined")
            joined = parts[0] if len(parts) == 1 else torch.cat(parts, 1)
            out.append(self.adaptor(self.time_merge(joined))[0])
        return out


def random_audio_weights(cfg: AudioConfig, seed: int, w_std: float = 0.5) -> dict:
    """Seeded weights of the audio tower's shape (numpy f32). Projection
    weights ~ N(0, w_std^2 / fan_in) keep activations O(1) through the layers;
    norm gains ~ 1 + N(0, 0.1^2); biases ~ N(0, 0.05^2)."""
    rng = np.random.default_rng(seed)
    D, FF, M = cfg.d_model, cfg.encoder_ffn_dim, cfg.num_mel_bins
    hid, K = cfg.hidden_size, cfg.adaptor_input_dim

    def lin(o, i):
        return (rng.standard_normal((o, i), dtype=np.float32) * (w_std / math.sqrt(i))).astype(np.float32)

    def vec(n, s=0.05):
        return (rng.standard_normal(n, dtype=np.float32) * s).astype(np.float32)

    def gain(n):
        return (1.0 + rng.standard_normal(n, dtype=np.float32) * 0.1).astype(np.float32)

    w = {
        "conv1_w": (rng.standard_normal((D, M, 3), dtype=np.float32) * (1.0 / math.sqrt(3 * M))).astype(np.float32),
        "conv1_b": vec(D),
        "conv2_w": (rng.standard_normal((D, D, 3), dtype=np.float32) * (1.0 / math.sqrt(3 * D))).astype(np.float32),
        "conv2_b": vec(D),
        "positions": (rng.standard_normal((cfg.max_source_positions, D), dtype=np.float32) * 0.3).astype(np.float32),
        "layers": [],
    }
    for _ in range(cfg.encoder_layers):
        w["layers"].append({
            "q_w": lin(D, D), "q_b": vec(D), "k_w": lin(D, D), "v_w": lin(D, D), "v_b": vec(D),
            "o_w": lin(D, D), "o_b": vec(D), "ln1_w": gain(D), "ln1_b": vec(D),
            "fc1_w": lin(FF, D), "fc1_b": vec(FF), "fc2_w": lin(D, FF), "fc2_b": vec(D),
            "ln2_w": gain(D), "ln2_b": vec(D),
        })
    w.update({"ln_w": gain(D), "ln_b": vec(D), "ad1_w": lin(hid, K), "ad1_b": vec(hid), "ad2_w": lin(hid, hid),
              "ad2_b": vec(hid), "adn_w": gain(hid), "adn_b": vec(hid)})
    return w


def round_weights(weights: dict, act: str) -> dict:
    """The same weights rounded through the activation dtype (as the GPU stores them)."""
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[act]

    def rd(a):
        return torch.as_tensor(a).to(dt).to(torch.float32).numpy()

    out = {k: rd(v) for k, v in weights.items() if k != "layers"}
    out["layers"] = [{k: rd(v) for k, v in lw.items()} for lw in weights["layers"]]
    return out
