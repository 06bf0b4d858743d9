"""The greedy pick that allocates nothing (`fmd_greedy_pick_noalloc`).

It exists for callers that can't let a library call cudaMalloc or cudaFree,
such as a host engine that owns every device byte itself, or code that must
not stall behind the synchronisation those calls can imply. Its scratch is a
fixed array compiled into the library. This test checks that, called twice
in a row on device logits, it returns the same greedy ids as the existing
`fmd_decode_step` entry point produced for those logits. Tie-break and ids
must match exactly. The file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes as C
import importlib

import numpy as np
import pytest

from conftest import PKG, tiny_config

pytestmark = pytest.mark.gpu


def _pick(lib, logits_dev, n, vocab, ids_dev, stream):
    return lib.fmd_greedy_pick_noalloc(C.c_void_p(logits_dev.data_ptr()), n, vocab, C.c_void_p(ids_dev.data_ptr()),
                                       C.c_void_p(stream))


def test_noalloc_greedy_pick_matches_decode_step():
    import torch

    syn = importlib.import_module("fmd_b200.synthetic")
    cfg = tiny_config(vocab_size=151_936)  # the full vocabulary: 38 candidate CTAs per row
    w = syn.make_weights(cfg, seed=31, norm_jitter=0.2)
    rng = np.random.default_rng(31)
    lib = PKG.load_library()
    steps = []
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=4, max_tokens=1024, max_rows=256)
        slots = [0, 1, 2]
        for s in slots:
            dec.open_slot(s, 200)
        dec.prefill(slots, [rng.standard_normal((n, cfg.hidden_size), dtype=np.float32) for n in (5, 70, 130)])
        for _ in range(2):
            logits, ids = dec.decode_step(slots, rng.integers(0, cfg.vocab_size, len(slots)))
            steps.append((logits, ids))

    stream = torch.cuda.current_stream().cuda_stream
    for logits, ids in steps:  # two calls in a row, each on fresh logits
        dev = torch.from_numpy(logits).to("cuda")
        out = torch.full((len(ids),), -1, dtype=torch.int32, device="cuda")
        assert _pick(lib, dev, len(ids), cfg.vocab_size, out, stream) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got, ids), (got, ids)
        assert np.array_equal(got, np.argmax(logits, axis=1))


def test_noalloc_greedy_pick_ties_and_limits():
    import torch

    lib = PKG.load_library()
    vocab = 100_000
    x = np.full((2, vocab), -3.0, dtype=np.float32)
    x[0, [99_999, 4_100, 70_000]] = 2.5          # equal maxima in three different candidate CTAs
    x[1, 12] = 1.0
    x[1, 8_191] = 1.0
    dev = torch.from_numpy(x).to("cuda")
    out = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        assert _pick(lib, dev, 2, vocab, out, stream) == 0
        torch.cuda.synchronize()
        assert out.cpu().tolist() == [4_100, 12]
    # sizes beyond the stated maximum are refused before any launch
    assert _pick(lib, dev, 65, vocab, out, stream) == PKG._lib.FMD_EINVAL
    assert _pick(lib, dev, 2, (1 << 20) + 1, out, stream) == PKG._lib.FMD_EINVAL


def test_noalloc_greedy_pick_rows_without_a_finite_logit():
    """A row of -inf logits picks its first column (np.argmax's answer); a
    row of NaNs gets the documented sentinel -1 instead of an id outside the
    vocabulary; NaNs next to finite values are skipped. Run twice: the second
    call reuses the scratch the first one left behind."""
    import torch

    lib = PKG.load_library()
    vocab = 151_936
    x = np.zeros((4, vocab), dtype=np.float32)
    x[0] = -np.inf
    x[1] = np.nan
    x[2] = np.nan
    x[2, 77_777] = -5.0                         # the only non-NaN value of the row
    x[3] = -np.inf
    x[3, 150_000] = np.nan
    x[3, 9_000] = -1.0
    dev = torch.from_numpy(x).to("cuda")
    out = torch.full((4,), -7, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        assert _pick(lib, dev, 4, vocab, out, stream) == 0
        torch.cuda.synchronize()
        assert out.cpu().tolist() == [0, -1, 77_777, 9_000]
    assert int(np.argmax(x[0])) == 0
