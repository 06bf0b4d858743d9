"""The f16 operand rule of the lm_head kernels (fmd_gemv.cu k_lm_head with
F16, fmd_lm_head_tc.cu): a staged row, already rounded to bf16, is scaled by
2^sh with sh = 14 - e (e the exponent of the row's largest |value|, clamped to
[-126, 126]) and converted to f16; the logits are scaled back by 2^-sh. Checked
here in numpy on the same steps: every value of the row that is at least 2^-31
of the row's largest converts exactly (bf16 has 8 significant bits, f16 11, and
f16 is normal from 2^-14), the largest lands in [2^14, 2^15), nothing
overflows, and a Q8_0 block dot product through the scaled operands equals the
unscaled one exactly in f64 (the products and their sums over 32 values are
exact there), so the MMA's f32 sums see the same operands up to the common
power of two."""

from __future__ import annotations

import numpy as np
import pytest


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (nearest even) and back to f32."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def row_shift(row: np.ndarray) -> int:
    m = np.float32(np.abs(row).max())
    if m == 0:
        return 0
    e = int((m.view(np.uint32) >> 23) & 0xFF) - 127
    return max(-126, min(126, 14 - e))


@pytest.mark.parametrize("seed", range(20))
@pytest.mark.parametrize("spread", [1.0, 8.0, 24.0])
def test_scaled_bf16_rows_convert_exactly_to_f16(seed, spread):
    rng = np.random.default_rng(seed)
    # log-uniform magnitudes over 2^spread, random signs, one row scale
    base = np.float32(2.0 ** rng.uniform(-20, 20))
    row = to_bf16(base * np.exp2(rng.uniform(-spread, 0, 1024)).astype(np.float32)
                  * rng.choice([-1, 1], 1024).astype(np.float32))
    sh = row_shift(row)
    scaled = row.astype(np.float64) * 2.0 ** sh
    assert np.abs(scaled).max() < 2.0 ** 15 and np.abs(scaled).max() >= 2.0 ** 14
    f16 = scaled.astype(np.float16)
    big = np.abs(row) >= np.abs(row).max() * 2.0 ** -31
    assert np.array_equal(f16[big].astype(np.float64), scaled[big])
    # a Q8_0 block dot product, exact in f64 either way
    q = rng.integers(-127, 128, 1024).astype(np.float64)
    for b in range(0, 1024, 32):
        if big[b:b + 32].all():
            assert np.dot(q[b:b + 32], f16[b:b + 32].astype(np.float64)) * 2.0 ** -sh == \
                np.dot(q[b:b + 32], row[b:b + 32].astype(np.float64))


def test_zero_and_extreme_rows():
    assert row_shift(np.zeros(8, np.float32)) == 0
    tiny = to_bf16(np.full(8, 2.0 ** -120, np.float32))
    assert row_shift(tiny) == 126  # clamped: 2^-120 * 2^126 = 2^6, still exact in f16
    assert np.array_equal((tiny.astype(np.float64) * 2.0 ** 126).astype(np.float16).astype(np.float64),
                          tiny.astype(np.float64) * 2.0 ** 126)
    huge = to_bf16(np.full(8, 2.0 ** 100, np.float32))
    sh = row_shift(huge)
    assert sh == -86 and (huge.astype(np.float64) * 2.0 ** sh).max() == 2.0 ** 14
