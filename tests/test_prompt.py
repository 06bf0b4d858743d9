"""Audio-span layout (prompt.rs:89-124) and the oracle's prompt splice
(model/mod.rs:134-180), on CPU. The span tests restate the reference's own
`prompt.rs` unit tests (:175-293) with its synthetic ids: placeholder 999,
digits 100..109."""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import oracle_model, tiny_config

prompt = importlib.import_module("fmd_b200.prompt")
syn = importlib.import_module("fmd_b200.synthetic")

AUDIO = 999
DIGITS = list(range(100, 110))


def span(n, cfg=prompt.ProcessorConfig()):
    return prompt.audio_span_ids(n, AUDIO, DIGITS, cfg)


def test_markers_appear_every_five_seconds():  # prompt.rs:175-189
    ids = span(375)  # exactly 30 s at 12.5 tokens/s
    assert sum(1 for i in ids if i == AUDIO) == 375
    assert [i for i in ids if i != AUDIO] == [105, 101, 100, 101, 105, 102, 100, 102, 105, 103, 100]


def test_first_marker_sits_after_the_first_62_tokens():  # prompt.rs:191-196
    ids = span(375)
    assert all(i == AUDIO for i in ids[:62])
    assert ids[62] == 105


def test_short_audio_gets_no_markers():  # prompt.rs:199-204
    assert span(50) == [AUDIO] * 50


def test_disabling_markers_yields_a_flat_span():  # prompt.rs:207-213
    assert span(400, prompt.ProcessorConfig(enable_time_marker=False)) == [AUDIO] * 400


def test_empty_audio_yields_an_empty_span():  # prompt.rs:216-220
    assert span(0) == []


def test_ten_minutes_keeps_every_audio_token():  # prompt.rs:286-293
    ids = span(7500)
    assert sum(1 for i in ids if i == AUDIO) == 7500
    assert 7500 < len(ids) < 7500 + 400


def test_build_wraps_the_span_in_the_template_halves():  # prompt.rs:139-150
    ids = prompt.build_prompt_ids([1, 2, 3], 130, [7, 8], AUDIO, DIGITS)
    assert ids.dtype == np.int32
    assert list(ids[:3]) == [1, 2, 3] and list(ids[-2:]) == [7, 8]
    assert list(ids[3:-2]) == span(130)


def test_oracle_splice_follows_the_runs():
    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=4)
    m = oracle_model(cfg, w, "bf16", max_len=256)
    ids = prompt.build_prompt_ids([5, 6], 130, [9], AUDIO, DIGITS)
    rng = np.random.default_rng(0)
    audio = rng.standard_normal((130, cfg.hidden_size), dtype=np.float32)
    got = ref_splice(m, ids, audio)
    assert got.shape == (len(ids), cfg.hidden_size)
    k = 0
    for p, i in enumerate(ids):
        if i == AUDIO:
            want = m.act.r(__import__("torch").from_numpy(audio[k]))
            k += 1
        else:
            want = m.embed([int(i)])[0]
        assert (got[p] == want).all()
    # no audio: a plain embedding lookup; a count mismatch is an error (mod.rs:143-150)
    assert (ref_splice(m, [1, 2, 3], np.zeros((0, cfg.hidden_size), np.float32)) == m.embed([1, 2, 3])).all()
    with pytest.raises(ValueError, match="audio placeholders"):
        ref_splice(m, ids, audio[:-1])


def ref_splice(m, ids, audio):
    from oracle import qwen3_ref as ref

    return ref.splice_audio(m, ids, audio, AUDIO)
