"""GPU continuous-batching engine (on-GPU scheduler, slot refill, chunked
prefill) against the oracle's greedy loop (engine.rs:505-538)."""

from __future__ import annotations

import dataclasses
import importlib

import numpy as np
import pytest

from conftest import PKG, check_greedy_stream, gpu_teacher_forced, oracle_model, tiny_config

syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu


def _check_streams(dec, m, prompts, out, budgets, forced, eos_id):
    """Every pick of the engine's free-running streams against the oracle fed
    the same streams (near-ties may flip only within twice the observed logit
    error, measured on the operator path over the same streams). Returns the
    number of picks compared."""
    from oracle import qwen3_ref as ref

    streams = [o.tokens for o in out]
    got = gpu_teacher_forced(dec, prompts, streams)
    want = ref.teacher_forced_logits(m, prompts, streams)
    compared = 0
    for i in range(len(prompts)):
        err = max(float(np.abs(g - r.numpy()).max()) for g, r in zip(got[i], want[i]))
        res = check_greedy_stream(streams[i], out[i].finish_reason, want[i], 2.0 * err + 1e-6, budgets[i], eos_id,
                                  forced[i])
        compared += res["compared"]
    return compared


def _setup(seed=11):
    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=seed, norm_jitter=0.2)
    return cfg, w


def test_engine_refill_matches_oracle():
    cfg, w = _setup()
    rng = np.random.default_rng(7)
    lens = [30, 100, 64, 1, 250, 77]
    max_new = [6, 4, 10, 3, 5, 0]
    forced = [-1, 2, -1, -1, -1, -1]
    prompts = [rng.standard_normal((n, cfg.hidden_size), dtype=np.float32) for n in lens]
    arena = np.concatenate(prompts)
    m = oracle_model(cfg, w, "bf16")
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=6, max_tokens=2048, max_rows=256)
        eng = PKG.Engine(dec)
        out, stats = eng.generate(lens, max_new, forced, arena, max_batch=2, prefill_chunk=64)
        out1, _ = eng.generate(lens, max_new, forced, arena, max_batch=1, prefill_chunk=100)
        assert stats.requests == len(lens)
        assert stats.prefill_tokens == sum(lens)
        assert stats.generated_tokens == sum(len(o.tokens) for o in out)
        n = _check_streams(dec, m, prompts, out, max_new, forced, cfg.eos_token_id)
        n1 = _check_streams(dec, m, prompts, out1, max_new, forced, cfg.eos_token_id)
    # every emitted token (and every EOS stop) was compared: 6 + 2 + 10 + 3 + 5 + 0
    assert n >= 26 and n1 >= 26, (n, n1)
    assert out[1].finish_reason == "stop" and len(out[1].tokens) == 2
    assert out[5].tokens == [] and out[5].finish_reason == "length"


def test_engine_eos_ends_a_sequence():
    """EOS is not emitted and ends the sequence with reason "stop"
    (engine.rs:513-516). The EOS id is set to the oracle's first pick of a
    prompt whose top-2 margin is clear, so the assertion always applies."""
    from oracle import qwen3_ref as ref

    cfg, w = _setup(seed=12)
    m = oracle_model(cfg, w, "bf16")
    rng = np.random.default_rng(8)
    for _ in range(20):
        prompt = rng.standard_normal((40, cfg.hidden_size), dtype=np.float32)
        first = ref.teacher_forced_logits(m, [prompt], [[]])[0][0].numpy()
        top2 = np.sort(first)[-2:]
        if top2[1] - top2[0] > 0.05:
            break
    else:
        pytest.fail("no prompt with a clear first pick in 20 draws")
    cfg_eos = dataclasses.replace(cfg, eos_token_id=int(np.argmax(first)))
    with PKG.Qwen3Decoder(cfg_eos, "bf16") as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=2, max_tokens=1024, max_rows=128)
        out, stats = PKG.Engine(dec).generate([40], [8], None, prompt, max_batch=2, prefill_chunk=64)
    assert out[0].tokens == [] and out[0].finish_reason == "stop"
    assert stats.generated_tokens == 0 and stats.requests == 1


def test_engine_many_requests_page_recycling():
    """A queue longer than the slots, with a KV pool that only fits a few
    sequences at once: pages are recycled on the device and every request
    completes with its full budget."""
    cfg, w = _setup(seed=13)
    rng = np.random.default_rng(9)
    n = 24
    lens = rng.integers(1, 300, n)
    max_new = rng.integers(1, 40, n)
    arena = rng.standard_normal((int(lens.sum()), cfg.hidden_size), dtype=np.float32)
    with PKG.Qwen3Decoder(cfg, "int8_bf16") as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=4, max_tokens=1400, max_rows=256)
        out, stats = PKG.Engine(dec).generate(lens, max_new, None, arena, max_batch=4, prefill_chunk=128)
    assert stats.requests == n and stats.device_status == 0
    for i in range(n):
        assert out[i].finish_reason == "length"
        assert len(out[i].tokens) == max_new[i]
        assert all(0 <= t < cfg.vocab_size for t in out[i].tokens)


@pytest.mark.parametrize("prec", ["int8_bf16", "bf16"])
def test_split_decode_steps_are_bit_identical(prec, monkeypatch):
    """Decode-only steps split over two streams (FMD_DECODE_SPLIT=1: rows
    [0, 8) and [8, 16) of a 16-slot batch each run the layer loop on their
    own stream, the lm_head over all rows after the join) give the same
    tokens and logits as one pass over all rows: every kernel of the loop
    treats rows independently. Requests outnumber slots, so the halves see
    refills, uneven row counts and an empty second half at the queue's end."""
    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=13, norm_jitter=0.2)
    rng = np.random.default_rng(21)
    n = 24
    lens = [int(x) for x in rng.integers(1, 200, n)]
    max_new = [int(x) for x in rng.integers(1, 40, n)]
    forced = [-1] * n
    prompts = [rng.standard_normal((k, cfg.hidden_size), dtype=np.float32) for k in lens]
    arena = np.concatenate(prompts)
    step_ids = [int(t) for t in rng.integers(0, 50, 13)]
    got = {}
    for split in ("1", "0"):
        monkeypatch.setenv("FMD_DECODE_SPLIT", split)
        with PKG.Qwen3Decoder(cfg, prec) as dec:
            dec.load_weights(w)
            dec.reserve(max_slots=16, max_tokens=16 * 256, max_rows=16 + 128)
            assert dec.debug_paths()["decode_split"] == (split == "1")
            eng = PKG.Engine(dec)
            out, _ = eng.generate(lens, max_new, forced, arena, max_batch=16, prefill_chunk=128)
            got[split] = [list(o.tokens) for o in out]
            # the operator path too: one decode step over 13 rows (halves of 8 and 5)
            for s in range(13):
                dec.open_slot(s, lens[s] + 2)
            dec.prefill(list(range(13)), prompts[:13], want_logits=False)
            got[split + "op"] = dec.decode_step(list(range(13)), step_ids)
    assert got["1"] == got["0"]
    assert sum(len(t) for t in got["1"]) > n
    assert np.array_equal(got["1op"][0], got["0op"][0]) and np.array_equal(got["1op"][1], got["0op"][1])
