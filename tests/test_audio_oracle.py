"""The audio-tower oracle (oracle/whisper_ref.py) against its pins, and the
host-side checks of the audio C ABI that need no GPU.

* encoder: the independent `transformers` Whisper encoder's output on seeded
  weights and mel (tests/golden/whisper_tiny.npz, made by
  tests/golden/make_whisper_golden.py);
* time merge: the reference's own unit tests (adaptor.rs:88-128);
* encode_audio: trimming, per-file concatenation in chunk order, batch-size
  invariance and the failure on an audio without chunks (model/mod.rs:82-126).
"""

from __future__ import annotations

import ctypes as C
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import PKG, ROOT
from oracle.whisper_ref import AudioConfig, WhisperRef, random_audio_weights

GOLDEN = ROOT / "tests" / "golden"


def _golden_cfg():
    spec = importlib.util.spec_from_file_location("make_whisper_golden", GOLDEN / "make_whisper_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.CFG


def test_encoder_matches_the_transformers_whisper_encoder():
    g = np.load(GOLDEN / "whisper_tiny.npz")
    cfg = _golden_cfg()
    ref = WhisperRef(cfg, random_audio_weights(cfg, int(g["weight_seed"])))
    out = ref.forward(g["mel"]).numpy()
    assert out.shape == g["out"].shape == (2, cfg.max_source_positions, cfg.d_model)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=2e-5 * float(np.abs(g["out"]).max()))


def _merge_only(merge):
    cfg = AudioConfig(d_model=2, audio_merge_size=merge)
    ref = WhisperRef.__new__(WhisperRef)
    ref.cfg = cfg
    return ref


def test_time_merge_folds_frames_into_features():  # adaptor.rs:100-113
    xs = torch.arange(8, dtype=torch.float32).reshape(1, 4, 2)
    merged = _merge_only(4).time_merge(xs)
    assert tuple(merged.shape) == (1, 1, 8)
    assert merged.flatten().tolist() == list(range(8))


def test_time_merge_full_chunk_and_partial_group():  # adaptor.rs:115-128
    ref = _merge_only(4)
    assert tuple(ref.time_merge(torch.zeros(2, 1500, 16)).shape) == (2, 375, 64)
    assert tuple(ref.time_merge(torch.zeros(1, 7, 2)).shape) == (1, 1, 8)


def _small_cfg():
    return AudioConfig(num_mel_bins=80, d_model=64, encoder_layers=1, encoder_attention_heads=1, encoder_ffn_dim=128,
                       max_source_positions=16, audio_merge_size=4, adaptor_input_dim=256, hidden_size=32)


def test_encode_audio_trims_and_joins_in_chunk_order():
    cfg = _small_cfg()
    ref = WhisperRef(cfg, random_audio_weights(cfg, 3))
    mel = np.random.default_rng(4).standard_normal((5, 80, 32), dtype=np.float32)
    tokens, mapping = [4, 2, 4, 1, 3], [0, 0, 1, 2, 2]
    out = ref.encode_audio(mel, tokens, mapping, 3, encoder_batch=2)
    assert [o.shape[0] for o in out] == [6, 4, 4]
    # audio 0 = chunk 0 (4 tokens) then chunk 1 (2 tokens), each the adaptor of its own frames
    frames = ref.forward(mel)
    merged = ref.time_merge(frames)
    proj = ref.adaptor(merged)
    want0 = torch.cat([proj[0, :4], proj[1, :2]])
    assert torch.allclose(out[0], want0, atol=1e-5)
    assert torch.allclose(out[2], torch.cat([proj[3, :1], proj[4, :3]]), atol=1e-5)
    # batch-size invariance (mod.rs:95-105)
    again = ref.encode_audio(mel, tokens, mapping, 3, encoder_batch=16)
    for a, b in zip(out, again):
        assert torch.allclose(a, b, atol=1e-5)
    # tokens beyond a chunk's frames keep only the chunk's frames (mod.rs:110-116)
    capped = ref.encode_audio(mel[:1], [99], [0], 1)
    assert capped[0].shape[0] == cfg.max_source_positions // cfg.audio_merge_size
    with pytest.raises(ValueError):
        ref.encode_audio(mel[:1], [4], [0], 2)


def test_bf16_reference_numerics_stay_close_to_f32():
    """How far the reference's own bf16 op-by-op rounding sits from f32 on the
    golden case: the scale of the tolerance the GPU path is held to."""
    g = np.load(GOLDEN / "whisper_tiny.npz")
    cfg = _golden_cfg()
    w = random_audio_weights(cfg, int(g["weight_seed"]))
    out = WhisperRef(cfg, w, act="bf16").forward(g["mel"]).numpy()
    rel = np.linalg.norm(out - g["out"]) / np.linalg.norm(g["out"])
    assert rel < 2e-2


def test_audio_create_rejects_unsupported_shapes_without_a_device():
    lib = PKG.load_library()
    _lib = PKG._lib
    cfg = PKG.AudioConfig(d_model=1000)
    h = C.c_void_p()
    w = _lib.AudioWeights()
    st = lib.fmd_audio_create(C.byref(cfg.to_c()), C.byref(w), _lib.PREC_BF16, 0, 1, C.byref(h))
    assert st == _lib.FMD_ENOTSUP and not h
    st = lib.fmd_audio_create(C.byref(PKG.AudioConfig().to_c()), C.byref(w), _lib.PREC_F32, 0, 1, C.byref(h))
    assert st == _lib.FMD_ENOTSUP and not h
    bad_heads = PKG.AudioConfig(encoder_attention_heads=8)  # head_dim 128: not supported
    st = lib.fmd_audio_create(C.byref(bad_heads.to_c()), C.byref(w), _lib.PREC_BF16, 0, 1, C.byref(h))
    assert st == _lib.FMD_ENOTSUP and not h
    st = lib.fmd_audio_create(C.byref(PKG.AudioConfig().to_c()), C.byref(w), _lib.PREC_BF16, 0, 0, C.byref(h))
    assert st == _lib.FMD_EINVAL and not h


def test_package_config_matches_the_oracle_config():
    assert PKG.AudioConfig().oracle_kwargs() == AudioConfig().__dict__
    doc = {"audio_config": {"num_mel_bins": 80, "d_model": 1024, "encoder_layers": 24,
                            "encoder_attention_heads": 16, "encoder_ffn_dim": 4096, "max_source_positions": 1500},
           "text_config": {"hidden_size": 1024, "rms_norm_eps": 1e-6}, "audio_merge_size": 4,
           "adaptor_input_dim": 4096}
    assert PKG.AudioConfig.from_model_config(doc) == PKG.AudioConfig()


def test_token_offsets_match_the_oracle_layout():
    """The library's host-only layout of encode_audio's output
    (fmd_audio_token_offsets) against the row counts of the oracle's
    encode_audio (trim to min(tokens, frames / merge), join in chunk order)."""
    cfg = _small_cfg()
    ref = WhisperRef(cfg, random_audio_weights(cfg, 5))
    mel = np.random.default_rng(6).standard_normal((6, 80, 32), dtype=np.float32)
    pcfg = PKG.AudioConfig(**cfg.__dict__)
    rng = np.random.default_rng(8)
    for _ in range(5):
        tokens = [int(t) for t in rng.integers(0, 7, 6)]  # up to past the 4 rows a chunk holds
        mapping = sorted(int(m) for m in rng.integers(0, 3, 6))
        mapping[:3] = [0, 1, 2]
        mapping.sort()
        out = ref.encode_audio(mel, tokens, mapping, 3, encoder_batch=4)
        off = PKG.audio.token_offsets(pcfg, tokens, mapping, 3)
        assert np.diff(off).tolist() == [o.shape[0] for o in out]
    with pytest.raises(PKG.FmdError):
        PKG.audio.token_offsets(pcfg, [1, 2], [0, 0], 2)  # audio 1 has no chunks
    with pytest.raises(PKG.FmdError):
        PKG.audio.token_offsets(pcfg, [1, -2], [0, 1], 2)
