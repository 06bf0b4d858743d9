"""Prompt assembly on the GPU (`fmd_splice_audio`, the analogue of
`MossModel::splice_audio`, model/mod.rs:134-180) against the oracle's splice:
bit-exact, since every row is a copy (text) or a round-to-nearest conversion
(f32 audio) into the activation dtype. Then the spliced device arena feeds the
engine directly and must give the same tokens as the host-arena path."""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import PKG, oracle_model, tiny_config

prompt = importlib.import_module("fmd_b200.prompt")
syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu

AUDIO = 1000  # a vocabulary id of the tiny config used as the placeholder
DIGITS = list(range(10, 20))


def _bits_to_f32(t):
    import torch

    return t.view(torch.int16).to(torch.int32).bitwise_left_shift(16).view(torch.float32)


@pytest.mark.parametrize("audio_dtype", ["f32", "bf16"])
def test_splice_matches_oracle(audio_dtype):
    import torch

    from oracle import qwen3_ref as ref

    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=8)
    m = oracle_model(cfg, w, "bf16", max_len=256)
    rng = np.random.default_rng(1)
    cases = [([3, 4, 5], 130, [6, 7]), ([1], 0, [2, 3, 4]), ([], 64, [])]
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(w)
        for before, n_audio, after in cases:
            ids = prompt.build_prompt_ids(before, n_audio, after, AUDIO, DIGITS)
            audio = rng.standard_normal((max(n_audio, 1), cfg.hidden_size), dtype=np.float32)[:n_audio]
            want = ref.splice_audio(m, ids, audio, AUDIO).numpy()
            a_dev = torch.from_numpy(audio).to("cuda")
            if audio_dtype == "bf16":
                a_dev = a_dev.to(torch.bfloat16)
            out = torch.empty((len(ids), cfg.hidden_size), dtype=torch.bfloat16, device="cuda")
            for _ in range(2):  # the second call reuses the index buffer
                dec.splice_audio(ids, a_dev.data_ptr() if n_audio else 0, n_audio, audio_dtype, AUDIO,
                                 out.data_ptr())
                got = _bits_to_f32(out.cpu()).numpy()
                assert np.array_equal(got, want)


def test_splice_errors():
    import torch

    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=8)
    ids = prompt.build_prompt_ids([3], 20, [4], AUDIO, DIGITS)
    audio = torch.zeros((20, cfg.hidden_size), dtype=torch.float32, device="cuda")
    out = torch.empty((len(ids), cfg.hidden_size), dtype=torch.bfloat16, device="cuda")
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(w)
        with pytest.raises(PKG.FmdError, match="audio placeholders") as e:  # mod.rs:143-150
            dec.splice_audio(ids, audio.data_ptr(), 19, "f32", AUDIO, out.data_ptr())
        assert e.value.status == PKG._lib.FMD_EINVAL
        host_out = np.empty((len(ids), cfg.hidden_size), dtype=np.uint16)
        with pytest.raises(PKG.FmdError, match="device memory"):
            dec.splice_audio(ids, audio.data_ptr(), 20, "f32", AUDIO, host_out.ctypes.data)
        with pytest.raises(PKG.FmdError, match="out of range"):
            dec.splice_audio([cfg.vocab_size + 5], 0, 0, "f32", AUDIO, out.data_ptr())
        # the handle stays usable
        dec.splice_audio(ids, audio.data_ptr(), 20, "f32", AUDIO, out.data_ptr())


def test_spliced_device_arena_feeds_the_engine():
    import torch

    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=9, norm_jitter=0.2)
    rng = np.random.default_rng(2)
    layout = [([3, 4], 90, [5]), ([7], 40, [8, 9]), ([2], 150, [])]
    ids = [prompt.build_prompt_ids(b, n, a, AUDIO, DIGITS) for b, n, a in layout]
    audio = [rng.standard_normal((n, cfg.hidden_size), dtype=np.float32) for _, n, _ in layout]
    lens = [len(x) for x in ids]
    max_new, forced = [5, 7, 4], [-1, 3, -1]
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=2, max_tokens=2048, max_rows=256)
        arena = torch.empty((sum(lens), cfg.hidden_size), dtype=torch.bfloat16, device="cuda")
        row = 0
        for x, a in zip(ids, audio):
            dev_rows = arena[row:row + len(x)]
            dec.splice_audio(x, torch.from_numpy(a).cuda().data_ptr(), len(a), "f32", AUDIO, dev_rows.data_ptr())
            row += len(x)
        host = arena.cpu().view(torch.int16).numpy().view(np.uint16)
        eng = PKG.Engine(dec)
        eng.load_device(lens, max_new, forced, arena.data_ptr(), arena.shape[0])
        eng.run(max_batch=2, prefill_chunk=64)
        got = eng.fetch()
        want, _ = eng.generate(lens, max_new, forced, host, max_batch=2, prefill_chunk=64)
    assert [g.tokens for g in got] == [x.tokens for x in want]
    assert [g.finish_reason for g in got] == [x.finish_reason for x in want]
