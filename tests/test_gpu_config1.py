"""BASELINE config 1 at full depth: greedy ids and logits of the whole model.

The 28-layer Qwen3 shape (hidden 1024, 16/8 heads, FFN 3072, vocab 151,936)
with random-init N(0, 0.02) weights and norm gains 1, four ragged prompts of
412 / 797 / 1,190 / 1,500 rows (75 % an N(0, 1) span standing in for the audio
adaptor output, the rest embedding rows of uniform text ids), 64 greedy steps.

* The engine (`fmd_generate`: on-GPU scheduler, chunked prefill, fused decode
  step) runs the four requests free: its token streams are the product.
* The oracle (the CPU restatement of qwen3.rs / engine.rs) is fed the same
  streams, so every one of the 4 x 64 picks is compared, not only those before
  a first divergence: each pick must be the oracle's argmax wherever the
  oracle's top-2 margin exceeds twice the observed logit error, and a
  maximiser up to that error at a near-tie.
* The operator path (`fmd_prefill` + `fmd_decode_step` on a ragged batch) is
  fed the same streams and its logits must stay within 2e-2 relative error
  (max |gpu - ref| / max |ref|) of the oracle's at every step -- or within
  2.5 x the noise floor where that floor is above 2e-2.

The noise floor: the oracle against itself with every matmul accumulated in
f64 instead of f32 (same rounding points, so an equally valid evaluation).
Through 28 layers of bf16 rounding the two drift 2.3 % apart on this
workload, above the 2e-2 bar; with f16 activations they stay 0.3 % apart. A
second implementation of the same arithmetic cannot be held closer to the
oracle than the oracle is to itself, so bf16 at full depth is held to
2.5 x the floor measured in the test, and int8 to 2e-2 (the 2-layer
full-shape tests of test_gpu_decoder.py hold bf16 to 2e-2).

The reference's `Int8` precision is Q8_0 weights with f16 activations
(precision.rs:32-41); `bf16` is the dense path.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import PKG, check_greedy_stream, gpu_teacher_forced, rel_err

syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu

LOGIT_RTOL = 2e-2
STEPS = 64


@pytest.fixture(scope="module")
def config1():
    cfg = PKG.TextConfig(max_position_embeddings=8192)
    w = syn.make_weights(cfg, seed=0)  # N(0, 0.02), norm gains 1
    prompts = syn.config1_prompts(cfg, w["embed"], seed=0)
    return cfg, w, prompts


@pytest.mark.parametrize("prec", ["int8", "bf16"])
def test_config1_free_running_greedy_matches_oracle(prec, config1):
    from oracle import qwen3_ref as ref

    cfg, w, prompts = config1
    lens = [p.shape[0] for p in prompts]
    assert lens == [412, 797, 1190, 1500]
    with PKG.Qwen3Decoder(cfg, prec) as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=4, max_tokens=8192, max_rows=2112)
        out, stats = PKG.Engine(dec).generate(lens, STEPS, None, np.concatenate(prompts), max_batch=4,
                                              prefill_chunk=2048)
        assert stats.device_status == 0 and stats.requests == 4
        streams = [o.tokens for o in out]
        got = gpu_teacher_forced(dec, prompts, streams)

    rcfg = ref.TextConfig(**cfg.oracle_kwargs())
    m = ref.Qwen3Ref(rcfg, w, prec, max_len=2048)
    want = ref.teacher_forced_logits(m, prompts, streams)
    # noise floor on the first prompt's prefill logits
    m64 = ref.Qwen3Ref(rcfg, w, prec, max_len=2048, accumulate="f64")
    c64 = m64.new_caches(1, lens[0] + 1)
    floor = rel_err(m64.logits(m64.prefill(prompts[0][None], c64))[0, 0].numpy(), want[0][0].numpy())
    del m64, c64
    bound = max(LOGIT_RTOL, 2.5 * floor)

    report = []
    for i in range(4):
        assert len(got[i]) == len(want[i]) == len(streams[i]) + 1
        errs = [rel_err(g, r.numpy()) for g, r in zip(got[i], want[i])]
        assert max(errs) < bound, (i, int(np.argmax(errs)), max(errs), floor)
        abs_err = max(float(np.abs(g - r.numpy()).max()) for g, r in zip(got[i], want[i]))
        tol = 2.0 * abs_err + 1e-6
        res = check_greedy_stream(streams[i], out[i].finish_reason, want[i], tol, STEPS, cfg.eos_token_id)
        first_flip = res["flips"][0][0] if res["flips"] else len(streams[i])
        report.append((lens[i], res["compared"], res["exact"], first_flip, round(max(errs), 5), round(tol, 4),
                       res["flips"]))
    print(f"\nconfig 1 [{prec}] noise floor (oracle f32 vs f64 accumulation) {floor:.4f}, logit bound {bound:.4f}")
    print(f"config 1 [{prec}] per sequence: (prompt, picks compared, exact, ids identical for the first N, "
          f"max logit rel err, tie tolerance, near-tie flips (step, gpu, oracle, margin))")
    for r in report:
        print("   ", r)
    assert sum(r[1] for r in report) >= 4 * STEPS
