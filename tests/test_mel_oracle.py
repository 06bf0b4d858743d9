"""The log-mel oracle (oracle/mel_ref.py) against its pins, and the host-side
parts of the GPU frontend that need no device.

* the `transformers` WhisperFeatureExtractor output on a seeded 1 s signal
  (tests/golden/mel_1s.npz, made by tests/golden/make_mel_golden.py);
* the reference's own unit tests (crates/fmd-core/src/audio/mel.rs:243-337 and
  audio/mod.rs:137-196), restated;
* the library's filterbank builder (`fmd_mel_filters`) against the oracle's.
"""

from __future__ import annotations

import ctypes as C
import importlib.util

import numpy as np

from conftest import PKG, ROOT
from oracle import mel_ref as M

GOLDEN = ROOT / "tests" / "golden"


def _signal():
    spec = importlib.util.spec_from_file_location("make_mel_golden", GOLDEN / "make_mel_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.test_signal()


def tone(seconds, amp=0.3, hz=440.0):
    n = int(16_000 * seconds)
    return (np.sin(np.arange(n, dtype=np.float32) * hz * 2 * np.pi / 16_000) * amp).astype(np.float32)


def test_matches_the_transformers_feature_extractor():
    g = np.load(GOLDEN / "mel_1s.npz")["mel"]
    got = M.MelRef(M.FeatureConfig(n_samples=16_000, nb_max_frames=100)).log_mel(_signal())
    assert got.shape == g.shape == (80, 100)
    assert np.abs(got - g).max() < 1e-4  # the reference's own bar against transformers is 2e-3 (mel.rs:367)


def test_mel_scale_round_trips_and_is_continuous():  # mel.rs:247-263
    for hz in [0.0, 100.0, 999.0, 1000.0, 4000.0, 8000.0]:
        assert abs(M.mel_to_hz(M.hz_to_mel(hz)) - hz) < 1e-2
    assert abs(M.hz_to_mel(1000.0) - 15.0) < 1e-4
    assert abs(M.hz_to_mel(999.999) - M.hz_to_mel(1000.0)) < 1e-3


def test_reflect_padding_and_periodic_hann():  # mel.rs:265-285
    assert [M.reflect_index(i, 5) for i in (-2, -1, 0, 4, 5, 6)] == [2, 1, 0, 4, 3, 2]
    np.testing.assert_allclose(M.hann_periodic(4), [0.0, 0.5, 1.0, 0.5], atol=1e-6)


def test_filterbank_shape_and_support():  # mel.rs:287-299
    fb = M.mel_filter_bank(201, 80, 0.0, 8000.0, 16000.0)
    assert fb.shape == (80, 201)
    starts = [int(np.nonzero(r)[0][0]) for r in fb]
    assert all(len(np.nonzero(r)[0]) > 0 for r in fb)
    assert starts == sorted(starts)
    for r in fb:  # one contiguous run per filter
        nz = np.nonzero(r)[0]
        assert nz[-1] - nz[0] + 1 == nz.size


def test_frame_count_bounds_gain_and_silence():  # mel.rs:301-337, :377-385
    ref = M.MelRef()
    assert ref.num_frames(480_000) == 3000
    short = M.MelRef(M.FeatureConfig(n_samples=16_000, nb_max_frames=100))
    mel = short.log_mel(tone(1.0, 0.5))
    assert mel.shape == (80, 100) and np.isfinite(mel).all()
    assert abs(mel.max() - mel.min() - 2.0) < 1e-4
    a, b = short.log_mel(tone(1.0, 0.1)), short.log_mel(tone(1.0, 1.0))
    assert np.abs(b - a - 2.0 * np.log10(10.0) / 4.0).max() < 1e-3
    silent = short.log_mel(np.zeros(16_000, np.float32))
    assert np.abs(silent - silent.flat[0]).max() < 1e-6


def test_extract_features_chunk_planning():  # audio/mod.rs:137-196
    cfg = M.FeatureConfig()
    _, tokens, mapping, per_audio = M.plan_chunks([3 * 16_000], cfg, 4)
    assert tokens == [38] and per_audio == [38] and mapping == [0]
    _, tokens, mapping, per_audio = M.plan_chunks([70 * 16_000], cfg, 4)
    assert tokens == [375, 375, 125] and per_audio == [875] and mapping == [0, 0, 0]
    _, tokens, mapping, per_audio = M.plan_chunks([35 * 16_000, 5 * 16_000, 31 * 16_000], cfg, 4)
    assert mapping == [0, 0, 1, 2, 2] and per_audio[0] == 375 + 63
    _, tokens, mapping, _ = M.plan_chunks([0], cfg, 4)  # an empty waveform is one empty window
    assert tokens == [0] and mapping == [0]
    # the package's planner is the same
    assert PKG.audio.plan_chunks([35 * 16_000, 5 * 16_000, 0], PKG.FeatureConfig(), 4) == \
        M.plan_chunks([35 * 16_000, 5 * 16_000, 0], cfg, 4)


def test_chunk_boundaries_do_not_bleed_between_files():  # audio/mod.rs:178-195
    cfg = M.FeatureConfig(n_samples=16_000, nb_max_frames=100)
    mel, *_ = M.extract_features([tone(1.0), np.zeros(16_000, np.float32)], cfg, 4)
    assert np.abs(mel[1] - mel[1].flat[0]).max() < 1e-6
    assert np.abs(mel[0] - mel[0].flat[0]).max() > 1e-3


def test_library_filterbank_matches_the_oracle_and_rejects_bad_shapes():
    fb = PKG.audio.mel_filters()
    want = M.MelRef().filters
    np.testing.assert_allclose(fb, want, rtol=1e-5, atol=1e-7)  # f32 ln/exp of two libraries: ulps
    lib = PKG.load_library()
    h = C.c_void_p()
    bad = PKG.FeatureConfig(nb_max_frames=2999)
    assert lib.fmd_mel_create(C.byref(bad.to_c()), 0, C.byref(h)) == PKG._lib.FMD_EINVAL and not h
    wide = PKG.FeatureConfig(n_fft=1024)  # 513 frequency bins: more than one CTA's threads
    assert lib.fmd_mel_create(C.byref(wide.to_c()), 0, C.byref(h)) == PKG._lib.FMD_ENOTSUP and not h


def test_chunk_planning_matches_the_oracle_on_random_lengths():
    rng = np.random.default_rng(7)
    cfg_o, cfg_p = M.FeatureConfig(), PKG.FeatureConfig()
    for _ in range(200):
        lengths = [int(x) for x in rng.integers(0, 5 * 480_000, size=int(rng.integers(1, 6)))]
        for merge in (1, 2, 4):
            assert PKG.audio.plan_chunks(lengths, cfg_p, merge) == M.plan_chunks(lengths, cfg_o, merge)
            _, tokens, _, per_audio = M.plan_chunks(lengths, cfg_o, merge)
            # every full window is the reference's 480000 / (160 x 2 x merge) tokens
            assert max(tokens) <= 480_000 // (160 * 2 * merge) + 1
            assert sum(per_audio) == sum(tokens)
