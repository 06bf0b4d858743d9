"""GGML Q8_0 block format, restated in numpy -- TEST INFRASTRUCTURE ONLY.

The reference quantises every large projection with
`QTensor::quantize(&w, GgmlDType::Q8_0)` from an f32 view of the checkpoint
(`crates/fmd-core/src/model/linear.rs:194-202`, `:239-251`; tied head
`crates/fmd-core/src/model/qwen3.rs:566-578`). That code lives in the
third-party crate candle-core 0.11.0 (`Cargo.lock:321-324`), which is not
vendored under the reference tree. The format is GGML's published Q8_0:

  * blocks of 32 consecutive values along the INPUT axis of a row-major
    `(out, in)` weight;
  * per block: `d = amax / 127` (f32), stored as an IEEE f16;
    `id = 1/d` (0 when d == 0); `q[j] = roundf(x[j] * id)` with round half
    away from zero, stored as int8;
  * on-disk/in-memory block = 34 bytes: `{f16 d; int8 qs[32]}`;
  * dequantisation: `x' = f32(q) * f32(f16 d)`, which is exact in f32
    (an 8-bit integer times an 11-bit significand fits in 24 bits).

gguf-py 0.19.0 (`gguf.quants.Q8_0`) is an independent implementation of the same
format; `tests/test_oracle_q8_0.py` pins this restatement to it bit for bit.
"""

from __future__ import annotations

import numpy as np

QK8_0 = 32
BLOCK_BYTES = 2 + QK8_0


def _roundf(x: np.ndarray) -> np.ndarray:
    """C `roundf`: nearest integer, halves away from zero."""
    return np.sign(x) * np.floor(np.abs(x) + np.float32(0.5))


def quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Quantise a row-major `(rows, cols)` f32 matrix.

    Returns `(qs, d)`: `qs` int8 `(rows, cols)` and `d` float16
    `(rows, cols // 32)`, i.e. the structure-of-arrays form of the 34-byte
    blocks.
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % QK8_0:
        raise ValueError(f"Q8_0 needs the input width to be a multiple of 32, got {cols}")
    blocks = w.reshape(rows, cols // QK8_0, QK8_0)
    amax = np.abs(blocks).max(axis=2, keepdims=True)
    d = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _roundf((blocks * inv).astype(np.float32))
    qs = q.astype(np.int8).reshape(rows, cols)
    return qs, d.reshape(rows, cols // QK8_0).astype(np.float16)


def dequantize(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """Exact f32 dequantisation of `(qs, d)` from :func:`quantize`."""
    rows, cols = qs.shape
    scale = d.astype(np.float32).reshape(rows, cols // QK8_0, 1)
    return (qs.astype(np.float32).reshape(rows, cols // QK8_0, QK8_0) * scale).reshape(rows, cols)


def to_blocks(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """Pack `(qs, d)` into GGML's 34-byte `{f16 d; int8 qs[32]}` blocks.

    Returns a uint8 array of shape `(rows, cols // 32, 34)`.
    """
    rows, cols = qs.shape
    nb = cols // QK8_0
    out = np.empty((rows, nb, BLOCK_BYTES), dtype=np.uint8)
    out[:, :, :2] = np.ascontiguousarray(d.astype(np.float16)).view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = qs.view(np.uint8).reshape(rows, nb, QK8_0)
    return out


def from_blocks(blocks: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of :func:`to_blocks`."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(rows, cols // QK8_0, BLOCK_BYTES)
    d = np.ascontiguousarray(b[:, :, :2]).view(np.float16).reshape(rows, cols // QK8_0)
    qs = np.ascontiguousarray(b[:, :, 2:]).view(np.int8).reshape(rows, cols)
    return qs, d
