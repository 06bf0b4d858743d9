"""GPU parity of the decoder-forward operator surface against the CPU oracle.

Tolerances: logits within 2e-2 relative (max-abs error
over max-abs logit) for bf16, f16 and Q8_0; Q8_0 dequantisation bit-exact;
greedy ids equal wherever the oracle's top-2 margin exceeds the observed
logit error (near-ties may flip under a different reduction order, as the
reference itself concedes in python/tests/test_engine.py:155-159).
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import PKG, mid_config, oracle_model, rel_err, tiny_config

syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu

LOGIT_RTOL = 2e-2
PRECS = ["bf16", "f16", "int8", "int8_bf16"]


@pytest.fixture(scope="module")
def tiny_w():
    return syn.make_weights(tiny_config(), seed=11, norm_jitter=0.2)


def make_decoder(cfg, w, prec, slots=4, tokens=4096, rows=128):
    d = PKG.Qwen3Decoder(cfg, prec, device=0)
    d.load_weights(w)
    d.reserve(slots, tokens, rows)
    return d


def check_pick(gpu_id: int, gpu_logits: np.ndarray, want: np.ndarray) -> None:
    """The device argmax is the lowest-index max of the returned logits, and
    it is a maximiser of the oracle logits up to the observed error."""
    assert gpu_id == int(np.argmax(gpu_logits))
    tol = 2.0 * float(np.abs(gpu_logits - want).max()) + 1e-6
    assert want[gpu_id] >= want.max() - tol, (gpu_id, int(np.argmax(want)))


@pytest.mark.parametrize("prec", PRECS)
def test_prefill_then_teacher_forced_decode(prec, tiny_w):
    cfg = tiny_config()
    m = oracle_model(cfg, tiny_w, prec)
    rng = np.random.default_rng(0)
    prompt = rng.standard_normal((300, cfg.hidden_size), dtype=np.float32)  # > max_rows: 3 passes
    with make_decoder(cfg, tiny_w, prec) as dec:
        dec.open_slot(0, 400)
        lg, ids = dec.prefill([0], [prompt])
        caches = m.new_caches(1, 400)
        want = m.logits(m.prefill(prompt[None], caches))[0, 0].numpy()
        assert rel_err(lg[0], want) < LOGIT_RTOL
        check_pick(int(ids[0]), lg[0], want)
        for t in rng.integers(0, cfg.vocab_size, 24):
            lg, nxt = dec.decode_step([0], [int(t)])
            want = m.decode_step(int(t), caches).numpy()
            assert rel_err(lg[0], want) < LOGIT_RTOL
            check_pick(int(nxt[0]), lg[0], want)
        assert dec.slot_len(0) == 324


@pytest.mark.parametrize("prec", ["bf16", "int8"])
def test_ragged_batch_matches_solo(prec, tiny_w):
    """One prefill + decode over sequences of very different lengths (1, 63,
    64, 200 positions: page edges and a single-token prompt) equals each
    sequence run alone -- the guarantee the reference tests with a padded
    short clip (python/tests/test_engine.py:176-200)."""
    cfg = tiny_config()
    m = oracle_model(cfg, tiny_w, prec)
    rng = np.random.default_rng(1)
    lens = [1, 63, 64, 200]
    prompts = [rng.standard_normal((n, cfg.hidden_size), dtype=np.float32) for n in lens]
    with make_decoder(cfg, tiny_w, prec, rows=512) as dec:
        slots = [3, 0, 2, 1]
        for s in slots:
            dec.open_slot(s, 260)
        lg, ids = dec.prefill(slots, prompts)
        caches = [m.new_caches(1, 260) for _ in lens]
        for i, p in enumerate(prompts):
            want = m.logits(m.prefill(p[None], caches[i]))[0, 0].numpy()
            assert rel_err(lg[i], want) < LOGIT_RTOL, i
        for _ in range(12):
            toks = rng.integers(0, cfg.vocab_size, len(lens))
            lg, nxt = dec.decode_step(slots, toks)
            for i in range(len(lens)):
                want = m.decode_step(int(toks[i]), caches[i]).numpy()
                assert rel_err(lg[i], want) < LOGIT_RTOL, i
                check_pick(int(nxt[i]), lg[i], want)


def test_chunked_prefill_equals_single_pass(tiny_w):
    """Appending a prompt in pieces (chunked prefill, qwen3.rs:475-496) gives
    the same cache and logits as one call."""
    cfg = tiny_config()
    rng = np.random.default_rng(2)
    prompt = rng.standard_normal((230, cfg.hidden_size), dtype=np.float32)
    with make_decoder(cfg, tiny_w, "bf16", rows=512) as dec:
        dec.open_slot(0, 300)
        dec.open_slot(1, 300)
        la, _ = dec.prefill([0], [prompt])
        dec.prefill([1], [prompt[:97]])
        dec.prefill([1], [prompt[97:200]])
        lb, _ = dec.prefill([1], [prompt[200:]])
        assert rel_err(lb[0], la[0]) < 1e-2
        ka, va = dec.debug_kv(0, 1, 0, 230)
        kb, vb = dec.debug_kv(1, 1, 0, 230)
        assert rel_err(kb, ka) < 1e-2 and rel_err(vb, va) < 1e-2


@pytest.mark.parametrize("prec", ["bf16", "int8_bf16"])
def test_kv_cache_contents(prec, tiny_w):
    """K after q/k-norm + RoPE and V, as written to the paged cache
    (qwen3.rs:218-227), match the oracle's dense cache."""
    cfg = tiny_config()
    m = oracle_model(cfg, tiny_w, prec)
    rng = np.random.default_rng(3)
    prompt = rng.standard_normal((130, cfg.hidden_size), dtype=np.float32)
    with make_decoder(cfg, tiny_w, prec) as dec:
        dec.open_slot(0, 140)
        dec.prefill([0], [prompt])
        caches = m.new_caches(1, 140)
        m.prefill(prompt[None], caches)
        for layer in range(cfg.num_hidden_layers):
            k, v = dec.debug_kv(0, layer, 0, 130)
            wk = caches[layer].k[0, :, :130].numpy().transpose(1, 0, 2)
            wv = caches[layer].v[0, :, :130].numpy().transpose(1, 0, 2)
            assert rel_err(k, wk) < 2e-2 and rel_err(v, wv) < 2e-2


def test_q8_0_dequantisation_is_bit_exact(pkg):
    """Device Q8_0 storage dequantises to exactly q * f32(f16 d) for weights
    quantised on load from f32 (linear.rs:194-202) and for pre-quantised
    blocks (including the tied lm_head, qwen3.rs:566-578)."""
    from oracle import q8_0

    cfg = tiny_config()
    for pre in (False, True):
        w = syn.make_weights(cfg, seed=5, prequantized=pre)
        m = oracle_model(cfg, w, "int8")
        with make_decoder(cfg, w, "int8") as dec:
            for layer in range(cfg.num_hidden_layers):
                for name in ("qkv", "o", "gate_up", "down"):
                    got = dec.debug_weight(layer, name)
                    want = getattr(m.layers[layer], name).numpy()
                    assert np.array_equal(got, want), (pre, layer, name)
            assert np.array_equal(dec.debug_weight(0, "lm_head"), m.lm_head.numpy())
    # and it is the GGML format: identical to quantise->dequantise in numpy
    w = syn.make_weights(cfg, seed=6)
    with make_decoder(cfg, w, "int8") as dec:
        qs, d = q8_0.quantize(w["layers"][1]["down"])
        assert np.array_equal(dec.debug_weight(1, "down"), q8_0.dequantize(qs, d))


def test_dense_weights_are_activation_dtype_views(pkg):
    cfg = tiny_config()
    w = syn.make_weights(cfg, seed=7)
    with make_decoder(cfg, w, "bf16") as dec:
        got = dec.debug_weight(0, "gate_up")
        want = syn.bf16_bits_to_f32(syn.f32_to_bf16_bits(np.concatenate([w["layers"][0]["gate"],
                                                                         w["layers"][0]["up"]])))
        assert np.array_equal(got, want)


def test_embed_lookup(tiny_w):
    cfg = tiny_config()
    m = oracle_model(cfg, tiny_w, "bf16")
    with make_decoder(cfg, tiny_w, "bf16") as dec:
        ids = [0, 5, 1023, 5]
        assert np.array_equal(dec.embed(ids), m.embed([ids])[0].numpy())


def test_errors_are_reported_not_fatal(tiny_w):
    """KV overflow, closed slots and pool exhaustion come back as status codes
    (qwen3.rs:88-94, engine.rs:414-421) and the handle keeps working."""
    cfg = tiny_config()
    rng = np.random.default_rng(4)
    with make_decoder(cfg, tiny_w, "bf16", slots=2, tokens=256) as dec:
        dec.open_slot(0, 10)
        with pytest.raises(PKG.FmdError) as e:
            dec.prefill([0], [rng.standard_normal((11, cfg.hidden_size), dtype=np.float32)])
        assert e.value.status == PKG._lib.FMD_EOVERFLOW
        dec.prefill([0], [rng.standard_normal((10, cfg.hidden_size), dtype=np.float32)])
        with pytest.raises(PKG.FmdError) as e:
            dec.decode_step([0], [1])
        assert e.value.status == PKG._lib.FMD_EOVERFLOW
        with pytest.raises(PKG.FmdError) as e:
            dec.decode_step([1], [1])
        assert e.value.status == PKG._lib.FMD_EINVAL
        with pytest.raises(PKG.FmdError) as e:
            dec.open_slot(1, 100_000)
        assert e.value.status in (PKG._lib.FMD_ENOMEM, PKG._lib.FMD_EOVERFLOW)
        dec.release_slot(0)
        dec.open_slot(0, 64)
        lg, _ = dec.prefill([0], [rng.standard_normal((5, cfg.hidden_size), dtype=np.float32)])
        assert np.isfinite(lg).all()


@pytest.mark.parametrize("prec", ["bf16", "int8_bf16"])
def test_full_layer_shapes(prec):
    """The BASELINE layer shapes (hidden 1024, 16/8 heads, FFN 3072, vocab
    151936), two layers."""
    cfg = mid_config()
    w = syn.make_weights(cfg, seed=21)
    m = oracle_model(cfg, w, prec)
    rng = np.random.default_rng(5)
    prompt = rng.standard_normal((700, cfg.hidden_size), dtype=np.float32)
    with make_decoder(cfg, w, prec, slots=2, tokens=2048, rows=512) as dec:
        dec.open_slot(0, 720)
        lg, ids = dec.prefill([0], [prompt])
        caches = m.new_caches(1, 720)
        want = m.logits(m.prefill(prompt[None], caches))[0, 0].numpy()
        assert rel_err(lg[0], want) < LOGIT_RTOL
        check_pick(int(ids[0]), lg[0], want)
        for t in rng.integers(0, cfg.vocab_size, 6):
            lg, nxt = dec.decode_step([0], [int(t)])
            want = m.decode_step(int(t), caches).numpy()
            assert rel_err(lg[0], want) < LOGIT_RTOL
            check_pick(int(nxt[0]), lg[0], want)


@pytest.mark.parametrize("proj", ["1", "0"])
@pytest.mark.parametrize("prec", ["bf16", "int8_bf16"])
def test_long_chunked_prefill_full_shapes(prec, proj, monkeypatch):
    """Chunked prefill at the BASELINE head shapes with histories past 2k
    positions (qwen3.rs:475-496): two sequences prefilled together in chunks of
    up to 1000 rows (tens of 64-row attention blocks per chunk, up to 41 key
    pages per block), then a decode step; logits against the oracle. Both
    mixed-step GEMM paths: the persistent projection GEMM with fused qkv and
    SwiGLU epilogues (default) and k_gemm_tc with the split-K epilogue kernels
    (FMD_PROJ_TC=0), dense and Q8_0 weights."""
    monkeypatch.setenv("FMD_PROJ_TC", proj)
    cfg = mid_config(num_hidden_layers=1)
    w = syn.make_weights(cfg, seed=23)
    m = oracle_model(cfg, w, prec, max_len=4096)
    rng = np.random.default_rng(9)
    lens = [2600, 1333]
    prompts = [rng.standard_normal((n, cfg.hidden_size), dtype=np.float32) for n in lens]
    with make_decoder(cfg, w, prec, slots=2, tokens=8192, rows=2048) as dec:
        for s, n in enumerate(lens):
            dec.open_slot(s, n + 8)
        done = [0, 0]
        last = [None, None]
        while min(d - n for d, n in zip(done, lens)) < 0:
            slots, parts = [], []
            for s, n in enumerate(lens):
                if done[s] < n:
                    take = min(1000, n - done[s])
                    slots.append(s)
                    parts.append(prompts[s][done[s]:done[s] + take])
                    done[s] += take
            lg, _ = dec.prefill(slots, parts)
            for i, s in enumerate(slots):
                last[s] = lg[i]
        for s, n in enumerate(lens):
            caches = m.new_caches(1, n + 8)
            want = m.logits(m.prefill(prompts[s][None], caches))[0, 0].numpy()
            assert rel_err(last[s], want) < LOGIT_RTOL, s
            tok = int(np.argmax(want))
            lg, _ = dec.decode_step([s], [tok])
            want = m.decode_step(tok, caches).numpy()
            assert rel_err(lg[0], want) < LOGIT_RTOL, s


@pytest.mark.parametrize("prec", ["int8_bf16", "int8"])
def test_decode_batch_of_32_full_shapes(prec):
    """A decode step of 32 sequences at the BASELINE shapes (two layers), the
    batch size of config 3: four 8-row n-tiles in every decode GEMV. Every
    row's logits and greedy id against the oracle's solo run of that
    sequence."""
    cfg = mid_config()
    w = syn.make_weights(cfg, seed=27)
    m = oracle_model(cfg, w, prec)
    rng = np.random.default_rng(13)
    n = 32
    lens = rng.integers(1, 40, n)
    prompts = [rng.standard_normal((int(k), cfg.hidden_size), dtype=np.float32) for k in lens]
    with make_decoder(cfg, w, prec, slots=n, tokens=n * 128, rows=2048) as dec:
        for s in range(n):
            dec.open_slot(s, int(lens[s]) + 4)
        dec.prefill(list(range(n)), prompts)
        caches = []
        for s in range(n):
            cs = m.new_caches(1, int(lens[s]) + 4)
            m.prefill(prompts[s][None], cs)
            caches.append(cs)
        for _ in range(2):
            toks = rng.integers(0, cfg.vocab_size, n)
            lg, ids = dec.decode_step(list(range(n)), toks)
            for s in range(n):
                want = m.decode_step(int(toks[s]), caches[s]).numpy()
                assert rel_err(lg[s], want) < LOGIT_RTOL, s
                check_pick(int(ids[s]), lg[s], want)


@pytest.mark.parametrize("prec,n", [("int8_bf16", 5), ("int8_bf16", 32), ("int8", 32), ("int8_bf16", 48),
                                    ("int8", 64)])
def test_lm_head_on_the_tensor_cores(prec, n, monkeypatch):
    """The Q8_0 lm_head on tcgen05 (fmd_lm_head_tc.cu: the exact int8 values
    through the MMA, one tensor-memory accumulator per 32-wide block, the f16
    block scale applied in f32) against the mma.sync kernel it replaces
    (FMD_LM_HEAD_TC=0) and the oracle, for 1-32 rows (N = 32) and 33-64
    rows (N = 64): the same arithmetic up to the f32 summation order, so the
    two kernels' rounded logits differ by at most one unit in the last place
    of the activation type, and each pick is the row's lowest-index maximum."""
    cfg = mid_config(num_hidden_layers=1)
    w = syn.make_weights(cfg, seed=29)
    m = oracle_model(cfg, w, prec)
    rng = np.random.default_rng(n)
    lens = rng.integers(1, 30, n)
    prompts = [rng.standard_normal((int(k), cfg.hidden_size), dtype=np.float32) for k in lens]
    toks = rng.integers(0, cfg.vocab_size, n)
    got = {}
    for tc in ("1", "0"):
        monkeypatch.setenv("FMD_LM_HEAD_TC", tc)
        with make_decoder(cfg, w, prec, slots=n, tokens=n * 64, rows=1024) as dec:
            for s in range(n):
                dec.open_slot(s, int(lens[s]) + 2)
            dec.prefill(list(range(n)), prompts, want_logits=False)
            got[tc] = dec.decode_step(list(range(n)), toks)
            assert dec.debug_paths()["lm_head_tc"] == (tc == "1")  # the kernel that ran
    lg_tc, ids_tc = got["1"]
    lg_ref, _ = got["0"]
    worst = (0.0, None)
    for s in range(n):
        cs = m.new_caches(1, int(lens[s]) + 2)
        m.prefill(prompts[s][None], cs)
        want = m.decode_step(int(toks[s]), cs).numpy()
        e_tc, e_ref = rel_err(lg_tc[s], want), rel_err(lg_ref[s], want)
        # the two kernels differ by the f32 summation order inside a block
        # and across blocks: elementwise within one unit in the last place
        # of the activation type at the row's largest logit
        scale = float(np.abs(want).max())
        d = np.abs(lg_tc[s] - lg_ref[s])
        j = int(np.argmax(d))
        if d[j] / scale > worst[0]:
            worst = (float(d[j] / scale), (s, j, float(lg_tc[s][j]), float(lg_ref[s][j]), float(want[j])))
        assert e_tc < LOGIT_RTOL, s
        assert e_tc <= 1.25 * e_ref + 1e-4, (s, e_tc, e_ref)
        check_pick(int(ids_tc[s]), lg_tc[s], want)
    print(f"\nlm_head tc [{prec}, {n} rows]: largest difference to the mma.sync kernel {worst[0]:.3g} of the row "
          f"max (row, col, tc, mma.sync, oracle) = {worst[1]}")
    assert worst[0] <= 2.0 ** (-7 if prec == "int8_bf16" else -10), worst


@pytest.mark.parametrize("n", [5, 32, 48])
def test_lm_head_f16_operands_are_bit_identical(n, monkeypatch):
    """The mma.sync lm_head for Q8_0 weights and bf16 rows takes f16 MMA
    operands (fmd_gemv.cu k_lm_head, F16): each staged row, rounded to bf16,
    is scaled by a power of two into f16 and the logits are scaled back. The
    scaling is exact and the products are exact either way, so the logits
    and picks equal those of the bf16-operand kernel (FMD_LM_HEAD_F16=0)
    bit for bit, and match the oracle; 5 and 32 rows (one 32-row tile, two
    consumer groups) and 48 rows (64-row tiles)."""
    cfg = mid_config(num_hidden_layers=1)
    w = syn.make_weights(cfg, seed=37)
    m = oracle_model(cfg, w, "int8_bf16")
    rng = np.random.default_rng(100 + n)
    lens = rng.integers(1, 30, n)
    prompts = [rng.standard_normal((int(k), cfg.hidden_size), dtype=np.float32) for k in lens]
    toks = rng.integers(0, cfg.vocab_size, n)
    got = {}
    monkeypatch.setenv("FMD_LM_HEAD_TC", "0")
    for f16 in ("1", "0"):
        monkeypatch.setenv("FMD_LM_HEAD_F16", f16)
        with make_decoder(cfg, w, "int8_bf16", slots=n, tokens=n * 64, rows=1024) as dec:
            for s in range(n):
                dec.open_slot(s, int(lens[s]) + 2)
            dec.prefill(list(range(n)), prompts, want_logits=False)
            got[f16] = dec.decode_step(list(range(n)), toks)
            assert not dec.debug_paths()["lm_head_tc"]
    (lg_a, ids_a), (lg_b, ids_b) = got["1"], got["0"]
    diff = int(np.count_nonzero(lg_a != lg_b))
    assert diff == 0, f"{diff} logits differ between f16 and bf16 operands"
    assert np.array_equal(ids_a, ids_b)
    for s in range(n):
        cs = m.new_caches(1, int(lens[s]) + 2)
        m.prefill(prompts[s][None], cs)
        want = m.decode_step(int(toks[s]), cs).numpy()
        assert rel_err(lg_a[s], want) < LOGIT_RTOL, s
        check_pick(int(ids_a[s]), lg_a[s], want)


@pytest.mark.parametrize("prec", ["bf16", "int8"])
def test_prefill_attention_persistent_two_tile_is_bit_identical(prec, monkeypatch):
    """Prefill attention on persistent CTAs with two query tiles each
    (k_attn_prefill_pp: pairs of consecutive 64-row blocks of a sequence per
    kv head, the snake work order, S / P / PV counts carried across a CTA's
    items) computes exactly what the one-CTA-per-block kernel does (the same
    MMAs, softmax and lazy rescale per tile): the logits of both paths are
    bit-identical, and match the oracle. Sequences with an even and an odd
    number of blocks, a lone block, a one-row block and histories across
    chunks."""
    cfg = mid_config(num_hidden_layers=1)
    w = syn.make_weights(cfg, seed=31)
    m = oracle_model(cfg, w, prec, max_len=4096)
    rng = np.random.default_rng(17)
    lens = [2600, 1333, 64, 65, 1, 700]
    prompts = [rng.standard_normal((n, cfg.hidden_size), dtype=np.float32) for n in lens]
    got = {}
    for pp in ("1", "0"):
        monkeypatch.setenv("FMD_PREFILL_PP", pp)
        with make_decoder(cfg, w, prec, slots=len(lens), tokens=8192, rows=2048) as dec:
            assert dec.debug_paths()["prefill_pp"] == (pp == "1")
            for s, n in enumerate(lens):
                dec.open_slot(s, n + 8)
            done = [0] * len(lens)
            last = [None] * len(lens)
            while any(d < n for d, n in zip(done, lens)):
                slots, parts, budget = [], [], 2000
                for s, n in enumerate(lens):
                    take = min(1000, n - done[s], budget)
                    if take > 0:
                        slots.append(s)
                        parts.append(prompts[s][done[s]:done[s] + take])
                        done[s] += take
                        budget -= take
                lg, _ = dec.prefill(slots, parts)
                for i, s in enumerate(slots):
                    last[s] = lg[i]
            got[pp] = np.stack(last)
    assert np.array_equal(got["1"], got["0"])
    for s, n in enumerate(lens):
        caches = m.new_caches(1, n + 8)
        want = m.logits(m.prefill(prompts[s][None], caches))[0, 0].numpy()
        assert rel_err(got["1"][s], want) < LOGIT_RTOL, s
