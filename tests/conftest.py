"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

PKG = __graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


@pytest.fixture(scope="session")
def pkg():
    return PKG


def tiny_config(**kw):
    """A small Qwen3-shaped config: same head_dim/GQA ratio as the real model."""
    base = dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=8192)
    base.update(kw)
    return PKG.TextConfig(**base)


def mid_config(**kw):
    """The BASELINE model's layer shapes (hidden 1024, 16/8 heads, FFN 3072,
    vocab 151936) with fewer layers, so the CPU oracle finishes in seconds."""
    base = dict(num_hidden_layers=2, max_position_embeddings=8192)
    base.update(kw)
    return PKG.TextConfig(**base)


def oracle_model(cfg, weights, precision, max_len=8192):
    from oracle import qwen3_ref as ref

    return ref.Qwen3Ref(ref.TextConfig(**cfg.oracle_kwargs()), weights, precision, max_len=max_len)


def rel_err(got, want) -> float:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def gpu_teacher_forced(dec, prompts, streams):
    """GPU logits of the operator path (`fmd_prefill` + `fmd_decode_step` over a
    ragged batch) fed the given token streams, laid out as
    `oracle.qwen3_ref.teacher_forced_logits`: `out[i][s]` are sequence i's f32
    logits before its s-th pick, `len(streams[i]) + 1` entries. Uses slots
    0..n-1 and releases them."""
    n = len(prompts)
    for i in range(n):
        dec.open_slot(i, len(prompts[i]) + len(streams[i]) + 1)
    lg, _ = dec.prefill(list(range(n)), prompts)
    out = [[lg[i].copy()] for i in range(n)]
    for s in range(max((len(t) for t in streams), default=0)):
        live = [i for i in range(n) if s < len(streams[i])]
        lg, _ = dec.decode_step(live, [int(streams[i][s]) for i in live])
        for j, i in enumerate(live):
            out[i].append(lg[j].copy())
    for i in range(n):
        dec.release_slot(i)
    return out


def check_greedy_stream(tokens, finish_reason, ref_logits, tol, budget, eos_id, forced_stop=-1):
    """Every pick of a free-running GPU greedy stream against the oracle fed
    the same stream (`ref_logits[s]`: the oracle's logits before pick s).

    Each emitted token must be the oracle's argmax, except at a near-tie
    (top-2 margin <= `tol`, twice the observed logit error), where it must
    still be a maximiser up to `tol`. The stop must agree too: EOS as the pick
    after the last token ("stop", engine.rs:513-516), the forced stop step, or
    the budget ("length"). Returns a dict with the number of picks compared,
    the exact matches and every near-tie flip with its margin, so a caller can
    report them; nothing is skipped."""
    flips = []
    exact = 0
    for s, tok in enumerate(tokens):
        lg = np.asarray(ref_logits[s], dtype=np.float64)
        top2 = np.partition(lg, -2)[-2:]
        best = int(np.argmax(lg))
        assert tok != eos_id, f"step {s}: EOS was emitted"
        if tok == best:
            exact += 1
            continue
        margin = float(top2[1] - top2[0])
        assert lg[tok] >= lg.max() - tol, (s, tok, best, float(lg.max() - lg[tok]), tol)
        assert margin <= tol, f"step {s}: picked {tok}, oracle {best} with a clear margin {margin} > {tol}"
        flips.append((s, int(tok), best, margin))
    compared = len(tokens)
    if finish_reason == "length":
        assert len(tokens) == budget, (len(tokens), budget)
    else:
        assert finish_reason == "stop", finish_reason
        if forced_stop >= 0 and len(tokens) == forced_stop:
            pass  # the forced end-of-turn step
        else:
            lg = np.asarray(ref_logits[len(tokens)], dtype=np.float64)
            assert lg[eos_id] >= lg.max() - tol, "stopped without EOS being a maximiser"
            compared += 1
    return {"compared": compared, "exact": exact, "flips": flips}
