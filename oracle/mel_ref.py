"""CPU restatement of the reference log-mel frontend -- TEST INFRASTRUCTURE ONLY.

Follows cnmoro/fast-moss-diarization `crates/fmd-core/src/audio/mel.rs`
(`MelFrontend::log_mel`, :84-133; `reflect_index`, :141-156; `hann_periodic`,
:158-165; Slaney `hz_to_mel` / `mel_to_hz`, :167-181; `mel_filter_bank`,
:183-240) and the chunk planning of `extract_features`
(`crates/fmd-core/src/audio/mod.rs:47-116`, `audio_token_length`,
`config.rs:210-223`). The window and the filterbank are built in f32 as the
reference builds them; the transform and the power spectrum are evaluated in
f64 (numpy's FFT), the log tail in f32.

Parity: pinned against `transformers.WhisperFeatureExtractor` (the reference's
own parity target, mel.rs:339-375) through tests/golden/make_mel_golden.py ->
tests/golden/mel_1s.npz, and against the reference's unit tests
(mel.rs:243-337, audio/mod.rs:137-196) restated in tests/test_mel_oracle.py.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

WHISPER_ENCODER_STRIDE = 2  # config.rs:210


@dataclass
class FeatureConfig:
    """`FeatureConfig` defaults (config.rs:121-166)."""
    feature_size: int = 80
    sampling_rate: int = 16_000
    hop_length: int = 160
    n_fft: int = 400
    n_samples: int = 480_000
    nb_max_frames: int = 3_000


def reflect_index(idx: int, length: int) -> int:
    """np.pad(mode="reflect") indexing (mel.rs:141-156)."""
    if length <= 1:
        return 0
    period = 2 * (length - 1)
    i = idx % period
    return period - i if i >= length else i


def hann_periodic(n: int) -> np.ndarray:
    """Periodic Hann in f64, stored as f32 (mel.rs:158-165)."""
    x = 2.0 * np.pi * np.arange(n, dtype=np.float64) / n
    return (0.5 - 0.5 * np.cos(x)).astype(np.float32)


_F32 = np.float32


def hz_to_mel(freq) -> np.float32:
    f_sp, min_log_hz = _F32(200.0) / _F32(3.0), _F32(1000.0)
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(_F32(6.4)) / _F32(27.0)
    freq = _F32(freq)
    return _F32(min_log_mel + np.log(freq / min_log_hz) / logstep) if freq >= min_log_hz else _F32(freq / f_sp)


def mel_to_hz(mel) -> np.float32:
    f_sp, min_log_hz = _F32(200.0) / _F32(3.0), _F32(1000.0)
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(_F32(6.4)) / _F32(27.0)
    mel = _F32(mel)
    return _F32(min_log_hz * np.exp(logstep * (mel - min_log_mel))) if mel >= min_log_mel else _F32(f_sp * mel)


def mel_filter_bank(n_freq: int, n_mels: int, f_min: float, f_max: float, sample_rate: float) -> np.ndarray:
    """Dense (n_mels, n_freq) Slaney-normalised triangles; each filter keeps its
    first contiguous run of positive weights (mel.rs:183-240)."""
    fft_freqs = [_F32(_F32(i) * (_F32(sample_rate) / _F32(2.0)) / _F32(n_freq - 1)) for i in range(n_freq)]
    mel_min, mel_max = hz_to_mel(f_min), hz_to_mel(f_max)
    pts = [mel_to_hz(mel_min + (mel_max - mel_min) * _F32(i) / _F32(n_mels + 1)) for i in range(n_mels + 2)]
    fb = np.zeros((n_mels, n_freq), dtype=np.float32)
    for m in range(n_mels):
        left, center, right = pts[m], pts[m + 1], pts[m + 2]
        enorm = _F32(2.0) / (right - left)
        started = False
        for k, f in enumerate(fft_freqs):
            lower = (f - left) / (center - left)
            upper = (right - f) / (right - center)
            w = _F32(max(min(lower, upper), _F32(0.0)) * enorm)
            if w > 0:
                started = True
                fb[m, k] = w
            elif started:
                break
    return fb


class MelRef:
    def __init__(self, cfg: FeatureConfig = FeatureConfig()):
        self.cfg = cfg
        self.n_freq = cfg.n_fft // 2 + 1
        self.window = hann_periodic(cfg.n_fft)
        self.filters = mel_filter_bank(self.n_freq, cfg.feature_size, 0.0, cfg.sampling_rate / 2.0,
                                       float(cfg.sampling_rate))

    def num_frames(self, n: int) -> int:  # mel.rs:76-82
        return n // self.cfg.hop_length

    def log_mel(self, samples) -> np.ndarray:
        """(n_mels, frames) f32 (mel.rs:84-133)."""
        x = np.asarray(samples, dtype=np.float32)
        n, N, hop = x.size, self.cfg.n_fft, self.cfg.hop_length
        frames = self.num_frames(n)
        half = N // 2
        origin = np.arange(frames)[:, None] * hop - half + np.arange(N)[None, :]
        if n <= 1:
            idx = np.zeros_like(origin)
        else:
            period = 2 * (n - 1)
            idx = np.mod(origin, period)
            idx = np.where(idx >= n, period - idx, idx)
        fr = x[idx].astype(np.float64) * self.window.astype(np.float64)[None, :]
        spec = np.fft.rfft(fr, n=N, axis=1)
        power = spec.real ** 2 + spec.imag ** 2
        mel = (power @ self.filters.T.astype(np.float64)).T.astype(np.float32)  # (n_mels, frames)
        logv = np.log10(np.maximum(mel, np.float32(1e-10))).astype(np.float32)
        floor = logv.max() - np.float32(8.0)
        return ((np.maximum(logv, floor) + np.float32(4.0)) / np.float32(4.0)).astype(np.float32)


def audio_token_length(num_samples: int, hop_length: int, merge_size: int) -> int:
    """config.rs:212-223."""
    if num_samples == 0:
        return 0
    stride = hop_length * WHISPER_ENCODER_STRIDE * merge_size
    return (num_samples - 1) // stride + 1


def plan_chunks(lengths, cfg: FeatureConfig, merge_size: int):
    """Chunk layout of `extract_features` (audio/mod.rs:57-82): for every waveform
    of `lengths[i]` samples, 30 s windows (an empty waveform still yields one
    empty window). Returns (chunks as (audio, start, end), chunk_token_lengths,
    chunk_mapping, tokens_per_audio)."""
    chunks, tokens, mapping, per_audio = [], [], [], [0] * len(lengths)
    for a, n in enumerate(lengths):
        total, start = max(n, 1), 0
        while start < total:
            end = min(start + cfg.n_samples, n)
            t = audio_token_length(end - start, cfg.hop_length, merge_size)
            per_audio[a] += t
            chunks.append((a, start, end))
            tokens.append(t)
            mapping.append(a)
            start += cfg.n_samples
    return chunks, tokens, mapping, per_audio


def extract_features(waveforms, cfg: FeatureConfig = FeatureConfig(), merge_size: int = 4):
    """(mel (n_chunks, n_mels, frames), chunk_token_lengths, chunk_mapping,
    tokens_per_audio), every chunk zero-padded to the full window
    (audio/mod.rs:84-116)."""
    ref = MelRef(cfg)
    chunks, tokens, mapping, per_audio = plan_chunks([len(w) for w in waveforms], cfg, merge_size)
    mel = np.zeros((len(chunks), cfg.feature_size, cfg.nb_max_frames), dtype=np.float32)
    for i, (a, s, e) in enumerate(chunks):
        padded = np.zeros(cfg.n_samples, dtype=np.float32)
        padded[: e - s] = np.asarray(waveforms[a], dtype=np.float32)[s:e]
        mel[i] = ref.log_mel(padded)
    return mel, tokens, mapping, per_audio
