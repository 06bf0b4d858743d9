"""The audio tower on the GPU (include/fmd_audio.h) against the f32 oracle
(oracle/whisper_ref.py, pinned to the `transformers` Whisper encoder).

Tolerance: the GPU computes in the activation dtype with f32 accumulation and
an f32 residual stream; the oracle is f32 on the same (activation-dtype
rounded) weights. Relative L2 error of the output < 1e-2 and max abs error <
3 % of the output's max abs value. The reference's own op-by-op bf16 rounding
sits at ~0.6 % relative L2 from f32 on the 2-layer full-width case.
Batching is exact: every row after the encoder is independent, so outputs do
not depend on the encoder batch size (bit-for-bit).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import PKG
from oracle.whisper_ref import AudioConfig as RefConfig
from oracle.whisper_ref import WhisperRef, random_audio_weights, round_weights

pytestmark = pytest.mark.gpu
_lib = PKG._lib


def _close(got, want, rel_l2=1e-2, rel_max=3e-2):
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    e2 = np.linalg.norm(got - want) / np.linalg.norm(want)
    em = np.abs(got - want).max() / np.abs(want).max()
    assert e2 < rel_l2 and em < rel_max, f"rel l2 {e2:.3e}, rel max {em:.3e}"


def _setup(cfg_kw, seed, act):
    cfg = PKG.AudioConfig(**cfg_kw)
    w = round_weights(random_audio_weights(RefConfig(**cfg.oracle_kwargs()), seed), act)
    return cfg, w, WhisperRef(RefConfig(**cfg.oracle_kwargs()), w)


def _mel(n, cfg, seed):
    return np.random.default_rng(seed).standard_normal((n, cfg.num_mel_bins, cfg.mel_frames), dtype=np.float32)


@pytest.mark.parametrize("precision,act", [("bf16", "bf16"), ("int8", "f16")])
def test_encoder_full_width_two_layers(precision, act):
    cfg, w, ref = _setup(dict(encoder_layers=2), 31, act)
    mel = _mel(3, cfg, 32)
    with PKG.AudioEncoder(cfg, w, precision, max_batch=2) as enc:  # two encoder batches: 2 + 1 chunks
        got = enc.forward(mel)
        ms, kernels = enc.last_timing()
    assert kernels > 0 and ms > 0
    _close(got, ref.forward(mel).numpy())


def test_encoder_full_model_one_chunk():
    """All 24 layers at the BASELINE shapes (one 30 s chunk)."""
    cfg, w, ref = _setup({}, 41, "bf16")
    mel = _mel(1, cfg, 42)
    with PKG.AudioEncoder(cfg, w, "bf16", max_batch=1) as enc:
        got = enc.forward(mel)
    _close(got, ref.forward(mel).numpy(), rel_l2=2e-2, rel_max=5e-2)


SMALL = dict(num_mel_bins=80, d_model=256, encoder_layers=2, encoder_attention_heads=4, encoder_ffn_dim=512,
             max_source_positions=100, audio_merge_size=4, adaptor_input_dim=1024, hidden_size=256)


def test_encode_audio_matches_oracle_and_is_batch_invariant():
    import torch

    cfg, w, ref = _setup(SMALL, 51, "bf16")
    mel = _mel(5, cfg, 52)
    tokens, mapping = [25, 7, 25, 1, 13], [0, 0, 1, 2, 2]
    want = ref.encode_audio(mel, tokens, mapping, 3)
    with PKG.AudioEncoder(cfg, w, "bf16", max_batch=4) as enc:
        off = enc.audio_offsets(5, tokens, mapping, 3)
        assert off.tolist() == [0, 32, 57, 71]
        got = enc.encode_audio(mel, tokens, mapping, 3, encoder_batch=2)
        for g, r in zip(got, want):
            _close(g, r.numpy())
        dev1, _ = enc.encode_audio_device(mel, tokens, mapping, 3, encoder_batch=1)
        dev4, _ = enc.encode_audio_device(mel, tokens, mapping, 3, encoder_batch=16)  # capped at max_batch
        assert torch.equal(dev1, dev4)
        # device-resident mel (f32 and the activation dtype) gives the same rows as host mel
        mel_dev = torch.from_numpy(mel).cuda()
        dev_f32, _ = enc.encode_audio_device(mel_dev, tokens, mapping, 3, encoder_batch=2)
        assert torch.equal(dev_f32, dev1)
        dev_bf, _ = enc.encode_audio_device(mel_dev.to(torch.bfloat16), tokens, mapping, 3)
        ref_bf = WhisperRef(RefConfig(**cfg.oracle_kwargs()), w).encode_audio(
            mel_dev.to(torch.bfloat16).float().cpu().numpy(), tokens, mapping, 3)
        _close(dev_bf.float().cpu().numpy(), torch.cat(ref_bf).numpy())


def test_encode_audio_errors_follow_the_reference():
    cfg, w, _ = _setup(SMALL, 61, "bf16")
    mel = _mel(2, cfg, 62)
    with PKG.AudioEncoder(cfg, w, "bf16", max_batch=2) as enc:
        with pytest.raises(PKG.FmdError) as e:
            enc.encode_audio(mel, [3, 3], [0, 0], 2)  # audio 1 has no chunks (mod.rs:118-125)
        assert e.value.status == _lib.FMD_EINVAL
        with pytest.raises(PKG.FmdError) as e:
            enc.encode_audio(mel, [3, 3], [0, 2], 2)
        assert e.value.status == _lib.FMD_EINVAL
        with pytest.raises(PKG.FmdError) as e:
            enc.encode_audio(mel, [3, -1], [0, 1], 2)
        assert e.value.status == _lib.FMD_EINVAL
        # the handle stays usable after a rejected call
        out = enc.encode_audio(mel, [3, 3], [0, 1], 2)
        assert [o.shape for o in out] == [(3, 256), (3, 256)]


def test_encode_audio_feeds_the_prompt_splice():
    """Adaptor output (device, activation dtype) goes straight into
    fmd_splice_audio, as `Engine::transcribe` chains them (engine.rs:338-360)."""
    import torch

    from conftest import tiny_config

    syn = __import__("fmd_b200.synthetic", fromlist=["make_weights"])
    tcfg = tiny_config()
    cfg, w, ref = _setup(dict(SMALL, hidden_size=tcfg.hidden_size), 71, "bf16")
    mel = _mel(2, cfg, 72)
    with PKG.AudioEncoder(cfg, w, "bf16", max_batch=2) as enc:
        audio, off = enc.encode_audio_device(mel, [25, 10], [0, 0], 1)
    n_audio = int(off[-1])
    ids = [5, 6] + [1000] * n_audio + [7]
    with PKG.Qwen3Decoder(tcfg, "bf16") as dec:
        dec.load_weights(syn.make_weights(tcfg, seed=3))
        out = torch.empty((len(ids), tcfg.hidden_size), dtype=torch.bfloat16, device="cuda")
        dec.splice_audio(ids, audio.data_ptr(), n_audio, "bf16", 1000, out.data_ptr())
        torch.cuda.synchronize()
    assert torch.equal(out[2:2 + n_audio], audio)
