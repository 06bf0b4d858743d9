"""The reference's own hot-path unit tests, restated against the oracle.

These are the only known answers the reference holds for decoder semantics:
crates/fmd-core/src/model/qwen3.rs:601-820, linear.rs:337-364 and
engine.rs:601-615. Each test cites the one it restates.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import qwen3_ref as ref


def _act(name="f32"):
    return ref._Act(ref.ACT_DTYPES[name])


def test_cache_appends_and_reports_length():  # qwen3.rs:601-617
    c = ref.KvCache(torch.zeros(2, 2, 8, 4), torch.zeros(2, 2, 8, 4))
    assert c.len == 0
    k = torch.ones(2, 2, 3, 4)
    k_all, v_all = c.append(k, k)
    assert c.len == 3 and tuple(k_all.shape) == (2, 2, 3, 4) and tuple(v_all.shape) == (2, 2, 3, 4)
    k_all, _ = c.append(k, k)
    assert c.len == 6 and tuple(k_all.shape) == (2, 2, 6, 4)


def test_cache_refuses_to_overflow():  # qwen3.rs:619-626
    c = ref.KvCache(torch.zeros(1, 1, 4, 2), torch.zeros(1, 1, 4, 2))
    with pytest.raises(ValueError, match="overflow"):
        c.append(torch.zeros(1, 1, 5, 2), torch.zeros(1, 1, 5, 2))


def test_cache_bytes_match_the_allocation():  # qwen3.rs:628-633
    assert ref.KvCache.bytes_per_layer(4, 8, 1000, 128, 2) == 2 * 4 * 8 * 1000 * 128 * 2


def test_repeat_kv_expands_grouped_heads():  # qwen3.rs:635-648
    xs = torch.tensor([1.0, 2.0, 3.0, 4.0]).reshape(1, 2, 1, 2)
    out = ref.repeat_kv(xs, 2)
    assert tuple(out.shape) == (1, 4, 1, 2)
    assert out.flatten().tolist() == [1.0, 2.0, 1.0, 2.0, 3.0, 4.0, 3.0, 4.0]
    assert ref.repeat_kv(xs, 1).shape == xs.shape


def test_rope_is_shift_invariant():  # qwen3.rs:650-673
    a = _act()
    cos, sin = ref.rope_tables(4, 10_000.0, 32, a)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 1, 1, 4, generator=g)
    k = torch.randn(1, 1, 1, 4, generator=g)

    def score(qp, kp):
        qr = ref.rope_apply(q, cos[qp:qp + 1], sin[qp:qp + 1], a)
        kr = ref.rope_apply(k, cos[kp:kp + 1], sin[kp:kp + 1], a)
        return float((qr @ kr.transpose(2, 3)).flatten()[0])

    assert abs(score(5, 2) - score(20, 17)) < 1e-4


def test_grouped_attention_matches_expanded_attention():  # qwen3.rs:675-714
    a = _act()
    b, kv_heads, repeat, t, l, d = 2, 3, 2, 4, 7, 5
    heads = kv_heads * repeat
    g = torch.Generator().manual_seed(1)
    q = torch.randn(b, heads, t, d, generator=g)
    k = torch.randn(b, kv_heads, l, d, generator=g)
    v = torch.randn(b, kv_heads, l, d, generator=g)
    expected = (torch.softmax(q @ ref.repeat_kv(k, repeat).transpose(-1, -2), -1) @ ref.repeat_kv(v, repeat))
    expected = expected.transpose(1, 2).reshape(b, t, heads * d)
    got = ref._grouped_attention(q, k, v, None, repeat, 1.0, a)
    assert got.shape == expected.shape
    assert float((got - expected).abs().max()) < 1e-5


def _cfg_mask(batch, q_offset, q_len, kv_len, pads):
    # cfg() of qwen3.rs:584-599 has 4 query heads over 2 kv heads: repeat = 2
    return ref.build_mask(batch, q_offset, q_len, kv_len, pads, 2)


def test_no_query_row_is_fully_masked():  # qwen3.rs:716-748
    m = _cfg_mask(2, 0, 6, 6, [4, 0])[:, 0]
    for bi in range(2):
        for ri in range(m.shape[1]):
            assert torch.isfinite(m[bi, ri]).any(), (bi, ri)
    assert torch.isinf(m[0, 4, :4]).all()
    assert float(m[0, 4, 4]) == 0.0
    assert torch.isinf(m[0, 4, 5])


def test_softmax_over_the_mask_never_produces_nan():  # qwen3.rs:750-761
    mask = _cfg_mask(2, 0, 6, 6, [4, 0])
    probs = torch.softmax(torch.zeros(2, 1, 12, 6) + mask, dim=-1)
    assert torch.isfinite(probs.sum())


def test_mask_is_tiled_for_the_regrouped_queries():  # qwen3.rs:763-777
    mask = _cfg_mask(1, 0, 3, 3, [0])
    assert tuple(mask.shape) == (1, 1, 6, 3)
    m = mask[0, 0]
    for q in range(3):
        assert torch.equal(m[q], m[3 + q])


def test_mask_blocks_future_and_padding():  # qwen3.rs:799-820
    m = _cfg_mask(2, 0, 4, 4, [2, 0])[:, 0]
    assert torch.isinf(m[0, 2, 0]) and torch.isinf(m[0, 2, 1])
    assert float(m[0, 2, 2]) == 0.0
    assert torch.isinf(m[0, 2, 3])
    assert float(m[1, 2, 0]) == 0.0 and float(m[1, 2, 1]) == 0.0 and float(m[1, 2, 2]) == 0.0
    assert torch.isinf(m[1, 2, 3])


def test_dense_linear_matches_a_hand_computed_product():  # linear.rs:337-351
    w = torch.tensor([[1.0, 2.0], [3.0, 4.0]])
    b = torch.tensor([10.0, 20.0])
    x = torch.tensor([[1.0, 1.0]])
    assert (x @ w.T + b).tolist() == [[13.0, 27.0]]


def test_argmax_picks_the_largest_logit_per_row():  # engine.rs:601-615
    assert ref.argmax_rows(torch.tensor([[0.1, 0.9, 0.2], [5.0, 1.0, 2.0]])) == [1, 0]
    assert ref.argmax_rows(torch.tensor([[[9.0, 0.0, 0.0], [0.0, 0.0, 7.0]]])) == [2]
    # ties resolve to the lowest index
    assert ref.argmax_rows(torch.tensor([[1.0, 3.0, 3.0]])) == [1]


def test_int8_runs_activations_in_f16():  # precision.rs:117-122
    assert ref.ACT_DTYPES["int8"] == torch.float16
    assert ref.is_quantized("int8") and not ref.is_quantized("bf16")


def test_left_padded_batch_equals_solo_runs():
    """The equivalence the reference's batching relies on (qwen3.rs:10-14,
    python/tests/test_engine.py:148-200): a left-padded, shared-position batch
    gives each sequence the logits of its solo run, including a short prompt
    padded next to a much longer one."""
    cfg = ref.TextConfig(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                         num_attention_heads=2, num_key_value_heads=1, head_dim=64)
    rng = np.random.default_rng(0)

    def n(*s):
        return (rng.standard_normal(s) * 0.05).astype(np.float32)

    w = {"embed": n(256, 128), "norm": np.ones(128, np.float32), "layers": [
        {"input_norm": np.ones(128, np.float32), "post_norm": np.ones(128, np.float32),
         "q_norm": np.ones(64, np.float32), "k_norm": np.ones(64, np.float32), "q": n(128, 128), "k": n(64, 128),
         "v": n(64, 128), "o": n(128, 128), "gate": n(256, 128), "up": n(256, 128), "down": n(128, 256)}
        for _ in range(2)]}
    m = ref.Qwen3Ref(cfg, w, "f32", max_len=128)
    prompts = [rng.standard_normal((3, 128)).astype(np.float32), rng.standard_normal((60, 128)).astype(np.float32)]
    caches = m.new_caches(2, 70)
    hl, pads = m.prefill_padded(prompts, caches, block=16)
    batched = m.logits(hl)[:, 0]
    step = m.decode_step_padded([5, 9], caches, pads)
    for i, p in enumerate(prompts):
        c = m.new_caches(1, 70)
        solo = m.logits(m.prefill(p[None], c))[0, 0]
        assert float((batched[i] - solo).abs().max()) < 1e-4
        solo_step = m.decode_step([5, 9][i], c)
        assert float((step[i] - solo_step).abs().max()) < 1e-4
