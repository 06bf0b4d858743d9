"""Failure detection on the GPU without a GPU fault.

Every ring kernel of the library waits on mbarriers with an iteration limit;
a wait that runs out sets the device status word, drains nothing it has not
issued and returns, and the host reports FMD_ETIMEDOUT. Here one such wait is
made to run out on a barrier that nothing arrives on (no copy in flight), and
the handle must then serve a normal prefill and decode step whose logits
match the oracle. KV overflow and bad arguments are covered in
test_gpu_decoder.py; the engine's host-side no-progress detector in
test_watchdog.py.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import PKG, oracle_model, rel_err, tiny_config

syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_reports_etimedout_and_the_handle_stays_usable():
    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=21, norm_jitter=0.2)
    m = oracle_model(cfg, w, "bf16")
    rng = np.random.default_rng(21)
    prompt = rng.standard_normal((70, cfg.hidden_size), dtype=np.float32)
    with PKG.Qwen3Decoder(cfg, "bf16") as dec:
        dec.load_weights(w)
        dec.reserve(max_slots=2, max_tokens=512, max_rows=128)
        dec.open_slot(0, 128)
        for _ in range(2):  # twice: the status word is cleared after it is reported
            with pytest.raises(PKG.FmdError) as e:
                dec.debug_wait_timeout(1000)
            assert e.value.status == PKG._lib.FMD_ETIMEDOUT
            assert "wait gave up in k_wait_probe" in str(e.value)
        lg, _ = dec.prefill([0], [prompt])
        caches = m.new_caches(1, 128)
        want = m.logits(m.prefill(prompt[None], caches))[0, 0].numpy()
        assert rel_err(lg[0], want) < 2e-2
        tok = int(np.argmax(want))
        lg, _ = dec.decode_step([0], [tok])
        assert rel_err(lg[0], m.decode_step(tok, caches).numpy()) < 2e-2
        with pytest.raises(PKG.FmdError) as e:
            dec.debug_wait_timeout(0)
        assert e.value.status == PKG._lib.FMD_EINVAL
