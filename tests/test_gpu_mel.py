"""The log-mel frontend on the GPU (`fmd_mel_log_mel`, the analogue of
`MelFrontend::log_mel`, crates/fmd-core/src/audio/mel.rs:84-133) against the
oracle (oracle/mel_ref.py, pinned to transformers' WhisperFeatureExtractor).

Tolerance: 1e-3 absolute on the rescaled log-mel values (the reference's own
bar against transformers is 2e-3, mel.rs:367). The GPU evaluates the DFT in
f64 and the log tail in f32; observed differences are ~1e-5.
"""

from __future__ import annotations

import importlib.util

import numpy as np
import pytest

from conftest import PKG, ROOT
from oracle import mel_ref as M
from oracle.whisper_ref import AudioConfig as RefConfig
from oracle.whisper_ref import WhisperRef, random_audio_weights, round_weights

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _signal():
    spec = importlib.util.spec_from_file_location("make_mel_golden", ROOT / "tests" / "golden" / "make_mel_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.test_signal()


def _waves(seed, seconds):
    rng = np.random.default_rng(seed)
    out = []
    for s in seconds:
        n = int(16_000 * s)
        t = np.arange(n) / 16_000.0
        f = rng.uniform(100, 4000)
        x = 0.2 * np.sin(2 * np.pi * f * t) + 0.02 * rng.standard_normal(n)
        out.append(x.astype(np.float32))
    return out


def test_full_windows_match_the_oracle():
    import torch

    waves = _waves(1, [30.0, 12.5, 0.3])
    windows = np.zeros((3, 480_000), np.float32)
    for i, w in enumerate(waves):
        windows[i, : w.size] = w
    ref = M.MelRef()
    with PKG.MelFrontend() as fe:
        got = fe.log_mel_device(windows)
        same = fe.log_mel_device(torch.from_numpy(windows).cuda())  # device-resident samples
    assert torch.equal(got, same)
    got = got.cpu().numpy()
    assert got.shape == (3, 80, 3000)
    for i in range(3):
        assert np.abs(got[i] - ref.log_mel(windows[i])).max() < TOL


def test_golden_window_and_properties():
    cfg = PKG.FeatureConfig(n_samples=16_000, nb_max_frames=100)
    g = np.load(ROOT / "tests" / "golden" / "mel_1s.npz")["mel"]
    with PKG.MelFrontend(cfg) as fe:
        got = fe.log_mel(_signal())
        assert np.abs(got - g).max() < TOL
        tone = (np.sin(np.arange(16_000, dtype=np.float32) * 440.0 * 2 * np.pi / 16_000) * 0.1).astype(np.float32)
        a, b = fe.log_mel(tone), fe.log_mel(tone * 10)
        assert np.abs(b - a - 0.5).max() < 1e-3          # gain shift (mel.rs:313-329)
        assert abs(a.max() - a.min() - 2.0) < 1e-4        # 80 dB span (mel.rs:301-311)
        silent = fe.log_mel(np.zeros(16_000, np.float32))
        assert np.abs(silent - silent.flat[0]).max() < 1e-6 and abs(silent.flat[0] + 1.5) < 1e-6


def test_extract_features_feeds_encode_audio():
    """Waveforms -> chunk plan + GPU log-mel -> GPU encoder + adaptor, against the
    oracle chain, with the encoder's window shortened to 2 s (200 mel frames)."""
    fcfg = PKG.FeatureConfig(n_samples=32_000, nb_max_frames=200)
    acfg = PKG.AudioConfig(num_mel_bins=80, d_model=256, encoder_layers=2, encoder_attention_heads=4,
                           encoder_ffn_dim=512, max_source_positions=100, audio_merge_size=4, adaptor_input_dim=1024,
                           hidden_size=256)
    w = round_weights(random_audio_weights(RefConfig(**acfg.oracle_kwargs()), 81), "bf16")
    waves = _waves(2, [2.5, 1.0, 0.0])
    with PKG.MelFrontend(fcfg) as fe, PKG.AudioEncoder(acfg, w, "bf16", max_batch=4) as enc:
        feats = PKG.extract_features(waves, fcfg, fe, acfg.audio_merge_size)
        assert feats.chunk_mapping == [0, 0, 1, 2] and feats.chunk_token_lengths == [25, 7, 13, 0]
        got = enc.encode_audio(feats.mel, feats.chunk_token_lengths, feats.chunk_mapping, 3)
    mel, tokens, mapping, per_audio = M.extract_features(waves, M.FeatureConfig(n_samples=32_000, nb_max_frames=200), 4)
    assert tokens == feats.chunk_token_lengths and per_audio == feats.tokens_per_audio
    assert np.abs(feats.mel.cpu().numpy() - mel).max() < TOL
    want = WhisperRef(RefConfig(**acfg.oracle_kwargs()), w).encode_audio(mel, tokens, mapping, 3)
    assert [g.shape[0] for g in got] == [32, 13, 0]
    for g, r in zip(got[:2], want[:2]):
        r = r.numpy()
        e2 = np.linalg.norm(g - r) / np.linalg.norm(r)
        assert e2 < 1e-2, e2
