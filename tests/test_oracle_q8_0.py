"""Pin the Q8_0 restatement (oracle/q8_0.py) to gguf-py 0.19.0, an
independent implementation of GGML's Q8_0 (the format candle-core 0.11.0's
`QTensor::quantize(.., GgmlDType::Q8_0)` produces, linear.rs:197)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import q8_0

gguf = pytest.importorskip("gguf")


def _gguf_blocks(w: np.ndarray) -> np.ndarray:
    return gguf.quants.Q8_0.quantize_blocks(w.reshape(-1, 32).astype(np.float32))


@pytest.mark.parametrize("seed,scale", [(0, 0.02), (1, 1.0), (2, 1e-4), (3, 300.0)])
def test_quantise_matches_gguf_bit_for_bit(seed, scale):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((48, 512)) * scale).astype(np.float32)
    qs, d = q8_0.quantize(w)
    ours = q8_0.to_blocks(qs, d).reshape(-1, 34)
    assert np.array_equal(ours, _gguf_blocks(w))


def test_edge_blocks():
    w = np.zeros((4, 64), dtype=np.float32)
    w[1, :32] = np.linspace(-127, 127, 32)          # integral after scaling
    w[2, :32] = (np.arange(32) - 15.5) * 0.5        # halves -> round away from zero
    w[3, 32:] = np.float32(1e-38)                   # subnormal scale
    w[3, 40] = -3.0e38                              # huge magnitude
    qs, d = q8_0.quantize(w)
    assert np.array_equal(q8_0.to_blocks(qs, d).reshape(-1, 34), _gguf_blocks(w))
    assert not qs[0].any() and not d[0].any()       # all-zero block: d = 0, q = 0
    assert qs.min() >= -127 and qs.max() <= 127


def test_dequantise_matches_gguf_and_is_exact():
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((16, 256)) * 0.05).astype(np.float32)
    qs, d = q8_0.quantize(w)
    ours = q8_0.dequantize(qs, d)
    theirs = gguf.quants.Q8_0.dequantize_blocks(q8_0.to_blocks(qs, d).reshape(-1, 34)).reshape(16, 256)
    assert np.array_equal(ours, theirs)
    # q * f32(f16 d) is exact in f32: the f64 product rounds to the same value
    exact = qs.astype(np.float64).reshape(16, 8, 32) * d.astype(np.float64).reshape(16, 8, 1)
    assert np.array_equal(ours.astype(np.float64), exact.reshape(16, 256))
    # the error is half a step plus the f16 rounding of the scale (2^-11
    # relative) times |q| <= 127
    step = d.astype(np.float32).repeat(32, axis=1)
    assert np.all(np.abs(ours - w) <= 0.5 * step + 127 * step * 2.0 ** -11 + 1e-12)


def test_block_round_trip():
    rng = np.random.default_rng(5)
    qs = rng.integers(-127, 128, (8, 128), dtype=np.int8)
    d = np.abs(rng.standard_normal((8, 4)) * 0.002).astype(np.float16)
    qs2, d2 = q8_0.from_blocks(q8_0.to_blocks(qs, d), 8, 128)
    assert np.array_equal(qs, qs2) and np.array_equal(d.view(np.uint16), d2.view(np.uint16))
