"""Generate tests/golden/mel_1s.npz: the log-mel spectrogram that the
independent `transformers.WhisperFeatureExtractor` (the reference frontend's
own parity target, crates/fmd-core/src/audio/mel.rs:339-375) computes for a
seeded 1 s test signal, used to pin oracle/mel_ref.py.

A 1 s window (chunk_length=1: 16,000 samples, 100 frames) keeps the fixture
small; the frontend's maths does not depend on the window length.

Run from the repository root:  python tests/golden/make_mel_golden.py
"""

from __future__ import annotations

from pathlib import Path

import numpy as np

SEED = 5
N_SAMPLES = 16_000


def test_signal(seed: int = SEED, n: int = N_SAMPLES) -> np.ndarray:
    """Two tones, a chirp and seeded noise, then 0.2 s of silence at the end."""
    t = np.arange(n, dtype=np.float64) / 16_000.0
    x = 0.3 * np.sin(2 * np.pi * 440.0 * t) + 0.1 * np.sin(2 * np.pi * 3_100.0 * t)
    x += 0.05 * np.sin(2 * np.pi * (200.0 + 2_000.0 * t) * t)
    x += 0.01 * np.random.default_rng(seed).standard_normal(n)
    x[-3_200:] = 0.0
    return x.astype(np.float32)


def main() -> None:
    from transformers import WhisperFeatureExtractor

    fe = WhisperFeatureExtractor(feature_size=80, sampling_rate=16_000, hop_length=160, chunk_length=1, n_fft=400)
    x = test_signal()
    out = fe(x, sampling_rate=16_000, return_tensors="np")["input_features"][0].astype(np.float32)
    np.savez_compressed(Path(__file__).with_name("mel_1s.npz"), mel=out, seed=SEED)
    print("wrote mel_1s.npz", out.shape, float(out.min()), float(out.max()))


if __name__ == "__main__":
    main()
