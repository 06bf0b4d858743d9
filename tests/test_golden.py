"""Golden fixtures (tests/golden/tiny_decoder.npz, made by make_golden.py).

CPU: the oracle still reproduces its frozen outputs. GPU: the CUDA path
matches them within the north-star tolerance (2e-2 relative on logits)."""

from __future__ import annotations

import importlib
from pathlib import Path

import numpy as np
import pytest

from conftest import PKG, oracle_model, rel_err

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load():
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden
    return make_golden, np.load(GOLDEN / "tiny_decoder.npz")


def _setup():
    mg, data = _load()
    syn = importlib.import_module("fmd_b200.synthetic")
    cfg = PKG.TextConfig(**mg.CFG)
    w = syn.make_weights(cfg, seed=mg.WEIGHT_SEED, norm_jitter=0.2)
    assert abs(mg.weight_checksum(w) - float(data["checksum"])) < 1e-3 * float(data["checksum"])
    prompts = [data[f"prompt{i}"] for i in range(len(data["lens"]))]
    return mg, data, cfg, w, prompts


@pytest.mark.parametrize("prec", ["bf16", "int8"])
def test_oracle_reproduces_golden(prec):
    mg, data, cfg, w, prompts = _setup()
    m = oracle_model(cfg, w, prec, max_len=512)
    for i, p in enumerate(prompts):
        caches = m.new_caches(1, 128)
        got = [m.logits(m.prefill(p[None], caches))[0, 0].numpy()]
        for t in data["tokens"][i]:
            got.append(m.decode_step(int(t), caches).numpy())
        assert rel_err(np.stack(got), data[f"logits_{prec}_{i}"]) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("prec", ["bf16", "f16", "int8", "int8_bf16"])
def test_gpu_matches_golden(prec):
    mg, data, cfg, w, prompts = _setup()
    with PKG.Qwen3Decoder(cfg, prec) as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=2, max_tokens=512, max_rows=128)
        dec.open_slot(0, 128)
        dec.open_slot(1, 128)
        lg, _ = dec.prefill([0, 1], prompts)
        got = [[lg[0]], [lg[1]]]
        for s in range(data["tokens"].shape[1]):
            lg, _ = dec.decode_step([0, 1], data["tokens"][:, s])
            got[0].append(lg[0])
            got[1].append(lg[1])
    for i in range(2):
        want = data[f"logits_{prec}_{i}"]
        for s in range(want.shape[0]):
            assert rel_err(got[i][s], want[s]) < 2e-2, (i, s)
