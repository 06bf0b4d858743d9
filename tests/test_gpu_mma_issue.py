"""The issue form of tcgen05.mma that every tensor-core kernel of the library
uses (fmd_common.cuh elect_one: the MMA warp runs its issue loop converged and
one elected lane issues) against one thread of a diverged warp issuing alone
(`if (threadIdx.x == 0)`), through fmd_debug_mma_issue: one CTA, 4,096 MMAs of
M 128 x N x K 16. On B200 the converged form runs small MMAs several times
faster and reaches the tensor peak at N = 256 (128 cycles per MMA of 524,288
multiply-adds = 4,096 per cycle per SM); the diverged form costs about 300
cycles per MMA whatever N."""

from __future__ import annotations

import importlib

import pytest

from conftest import PKG, tiny_config

syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu


def test_converged_issue_is_faster_and_reaches_the_tensor_peak():
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
        for n, diverged, converged in rows:
            # small MMAs: the converged form at least twice as fast
            if n <= 64:
                assert converged * 2 <= diverged, (n, diverged, converged)
        # N = 256: within 25 % of the tensor peak (128 cycles per MMA)
        assert rows[-1][2] < 160.0, rows[-1]
        with pytest.raises(PKG.FmdError) as e:
            dec.debug_mma_issue(2, 64)
        assert e.value.status == PKG._lib.FMD_EINVAL
