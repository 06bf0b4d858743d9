"""tcgen05.mma issue cost through fmd_debug_mma_issue: one CTA issues 4,096
MMAs of M 128 x N x K 16 in a bare loop, from a lone thread of a diverged warp
(form 0) or from the elected lane of a converged warp (form 1, the form of
every tensor-core kernel in the library, fmd_common.cuh elect_one). Whatever
the form, an MMA costs a fixed number of cycles up to N 128 (the floor the
lm_head's 32-row and attention's 64-key MMAs run into), and at N 256 the
converged form reaches the tensor peak: 128 cycles per MMA of 524,288
multiply-adds, 4,096 per cycle per SM. Which form is cheaper on a bare loop
depends on the code the compiler makes of it; inside the library's kernels
the converged form measured faster (prefill attention 161 -> 143 us per
captured launch, the tensor-core lm_head 119 -> 107 us)."""

from __future__ import annotations

import importlib

import pytest

from conftest import PKG, tiny_config

syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu


def test_small_mmas_cost_a_fixed_issue_time_and_n256_reaches_the_tensor_peak():
    cfg = tiny_config()
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(syn.make_weights(cfg, seed=3))
        dec.reserve(max_slots=2, max_tokens=256, max_rows=64)
        rows = []
        for n in (32, 64, 128, 256):
            diverged, converged = dec.debug_mma_issue(0, n), dec.debug_mma_issue(1, n)
            rows.append((n, diverged, converged))
            assert converged > 0 and diverged > 0
        print("\nN, cycles per MMA (diverged thread, converged warp + elected lane):",
              [(n, round(a, 1), round(b, 1)) for n, a, b in rows])
        # up to N 128 a fixed cost per MMA: N 32 costs as much as N 128
        for form in (1, 2):
            assert abs(rows[0][form] - rows[2][form]) <= 0.1 * rows[2][form], rows
        # N 256, converged: within 25 % of the tensor peak (128 cycles per MMA)
        assert rows[-1][2] < 160.0, rows[-1]
        with pytest.raises(PKG.FmdError) as e:
            dec.debug_mma_issue(2, 64)
        assert e.value.status == PKG._lib.FMD_EINVAL
