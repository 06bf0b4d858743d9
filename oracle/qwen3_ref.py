"""CPU restatement of the reference Qwen3 decoder -- TEST INFRASTRUCTURE ONLY.

Follows cnmoro/fast-moss-diarization `crates/fmd-core/src/model/qwen3.rs` and
`crates/fmd-core/src/model/linear.rs` (file:line cited per function). Tensors
are held as torch f32 on the CPU; every place where the reference stores a
result in the activation dtype (bf16 / f16) is emulated by rounding through
that dtype (`_Act.r`). Matmuls accumulate in f32 and round once, which is the
cuBLAS/candle contract for half-precision GEMMs.

Two execution modes:
  * solo / ragged (`Qwen3Ref.prefill` + `decode_step` on one sequence):
    positions 0..len for every sequence. This is what the CUDA path computes.
  * left-padded batch (`prefill_padded` / `decode_step_padded`): the
    reference's own batching, shared positions plus the additive mask of
    `qwen3.rs:523-562`. The reference relies on RoPE shift invariance to make
    the two agree (`qwen3.rs:10-14`, `:650-673`, `python/tests/test_engine.py:148-173`).

Parity status: pinned by the reference's known-answer tests (restated in
`tests/test_oracle_pins.py`); end-to-end logits/ids are parity unpinned (the
reference ships no golden outputs and cannot be built here).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import q8_0

PREFILL_BLOCK = 256  # qwen3.rs:26
EOS_TOKEN_ID = 151_645  # config.rs:110-116, engine.rs:246


@dataclass
class TextConfig:
    """`TextConfig` (config.rs:8-58) with the BASELINE model's values as defaults."""

    vocab_size: int = 151_936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 131_072

    @property
    def q_dim(self) -> int:  # config.rs:45-47
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:  # config.rs:50-52
        return self.num_key_value_heads * self.head_dim

    @property
    def kv_repeat(self) -> int:  # config.rs:55-57
        return self.num_attention_heads // self.num_key_value_heads


# precision name -> activation dtype (precision.rs:32-41). "int8" keeps the
# reference's f16 activations; "int8_bf16" is the BASELINE Q8_0 + bf16 variant.
ACT_DTYPES = {
    "f32": torch.float32,
    "bf16": torch.bfloat16,
    "f16": torch.float16,
    "int8": torch.float16,
    "int8_bf16": torch.bfloat16,
}


def is_quantized(precision: str) -> bool:  # precision.rs:43-45
    return precision.startswith("int8")


class _Act:
    """Rounding through the activation dtype."""

    def __init__(self, dtype: torch.dtype):
        self.dtype = dtype

    def r(self, x: torch.Tensor) -> torch.Tensor:
        if self.dtype == torch.float32:
            return x.to(torch.float32)
        return x.to(self.dtype).to(torch.float32)


def rope_tables(head_dim: int, theta: float, max_len: int, act: _Act) -> tuple[torch.Tensor, torch.Tensor]:
    """`Rope::new` (qwen3.rs:116-136).

    inv_freq is computed in f64 and cast to f32; `pos * inv_freq` is an f32
    product (the `(L,1)x(1,D/2)` matmul has a single term); cos/sin are taken
    in f32 and then stored in the activation dtype (`:133-134`).
    """
    inv = np.array(
        [1.0 / theta ** (2.0 * i / head_dim) for i in range(head_dim // 2)], dtype=np.float64
    ).astype(np.float32)
    pos = np.arange(max_len, dtype=np.float32).reshape(max_len, 1)
    freqs = torch.from_numpy(pos * inv.reshape(1, -1))
    return act.r(torch.cos(freqs)), act.r(torch.sin(freqs))


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, act: _Act) -> torch.Tensor:
    """candle `rotary_emb::rope` as called by `Rope::apply` (qwen3.rs:139-144).

    Non-interleaved half split: for i < D/2,
      out[i]       = x[i]*cos[i] - x[i+D/2]*sin[i]
      out[i+D/2]   = x[i]*sin[i] + x[i+D/2]*cos[i]
    `x` is `(..., t, D)`, `cos`/`sin` are `(t, D/2)`.
    """
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return act.r(torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1))


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, act: _Act) -> torch.Tensor:
    """`RmsNorm::forward` (linear.rs:293-302): f32 sum of squares over the last
    dim, `x * rsqrt(mean + eps) * w`, stored in the activation dtype."""
    ms = (x * x).mean(dim=-1, keepdim=True)
    return act.r(x * torch.rsqrt(ms + eps) * w)


def repeat_kv(xs: torch.Tensor, repeat: int) -> torch.Tensor:
    """`repeat_kv` (qwen3.rs:153-162): `(b, kv, t, d) -> (b, kv*repeat, t, d)`,
    each kv head duplicated in place (kv-major)."""
    if repeat == 1:
        return xs
    b, kv, t, d = xs.shape
    return xs.unsqueeze(2).expand(b, kv, repeat, t, d).reshape(b, kv * repeat, t, d)


def build_mask(
    batch: int, q_offset: int, q_len: int, kv_len: int, pad_lengths: list[int], repeat: int
) -> torch.Tensor:
    """`Qwen3::build_mask` (qwen3.rs:523-562): additive `(b, 1, repeat*q_len, kv_len)`.

    Key `ki` is masked for query at absolute `abs_q` when it is in the future,
    or when it is padding and the query itself is not (pad query rows fall back
    to plain causal masking so no row is fully masked, `:539-548`). The q_len
    rows are tiled `repeat` times for the regrouped queries.
    """
    rows = repeat * q_len
    m = torch.zeros(batch, rows, kv_len, dtype=torch.float32)
    ki = torch.arange(kv_len)
    for bi in range(batch):
        pad = pad_lengths[bi]
        for qi in range(q_len):
            abs_q = q_offset + qi
            masked = ki > abs_q
            if abs_q >= pad:
                masked = masked | (ki < pad)
            row = torch.where(masked, torch.tensor(float("-inf")), torch.tensor(0.0))
            for r in range(repeat):
                m[bi, r * q_len + qi] = row
    return m.unsqueeze(1)


def _mm32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return a @ b


def _mm64(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """The same product accumulated in f64 (then stored as f32): an equally
    valid evaluation order, used to measure how far two correct
    implementations drift apart through the rounding points."""
    return (a.double() @ b.double()).float()


def _grouped_attention(
    q: torch.Tensor, k_all: torch.Tensor, v_all: torch.Tensor, mask: torch.Tensor | None,
    repeat: int, scale: float, act: _Act, mm=_mm32,
) -> torch.Tensor:
    """Grouped-query attention core of `Attention::forward` (qwen3.rs:240-257).

    q `(b, heads, t, d)`; k_all/v_all `(b, kv_heads, L, d)`; mask broadcastable to
    `(b, 1, repeat*t, L)`. Returns `(b, t, heads*d)`.
    """
    b, heads, t, d = q.shape
    kv_heads = heads // repeat
    grouped = q.reshape(b, kv_heads, repeat * t, d)
    scores = act.r(act.r(mm(grouped, k_all.transpose(-1, -2))) * scale)
    if mask is not None:
        scores = scores + mask
    probs = act.r(torch.softmax(scores, dim=-1))
    ctx = act.r(mm(probs, v_all))
    return ctx.reshape(b, kv_heads, repeat, t, d).permute(0, 3, 1, 2, 4).reshape(b, t, heads * d)


@dataclass
class LayerWeights:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    qkv: torch.Tensor  # (q_dim + 2*kv_dim, hidden), f32 holding the stored values
    o: torch.Tensor  # (hidden, q_dim)
    gate_up: torch.Tensor  # (2*intermediate, hidden)
    down: torch.Tensor  # (hidden, intermediate)


@dataclass
class KvCache:
    """Dense per-layer cache `(b, kv_heads, capacity, d)` (qwen3.rs:33-108)."""

    k: torch.Tensor
    v: torch.Tensor
    len: int = 0

    @property
    def capacity(self) -> int:
        return self.k.shape[2]

    def append(self, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """`KvCache::append` (qwen3.rs:86-102); overflow is an error (`:88-94`)."""
        t = k.shape[2]
        if self.len + t > self.capacity:
            raise ValueError(
                f"kv cache overflow: {self.len} + {t} exceeds capacity {self.capacity}"
            )
        self.k[:, :, self.len:self.len + t] = k
        self.v[:, :, self.len:self.len + t] = v
        self.len += t
        return self.k[:, :, :self.len], self.v[:, :, :self.len]

    @staticmethod
    def bytes_per_layer(batch: int, kv_heads: int, capacity: int, head_dim: int, elem_bytes: int) -> int:
        """`KvCache::bytes_per_layer` (qwen3.rs:70-78)."""
        return 2 * batch * kv_heads * capacity * head_dim * elem_bytes


def _fused_q8(parts: list[np.ndarray]) -> torch.Tensor:
    """Concatenate along the output axis, then quantise (linear.rs:239-251)."""
    joined = np.concatenate([np.asarray(p, dtype=np.float32) for p in parts], axis=0)
    qs, d = q8_0.quantize(joined)
    return torch.from_numpy(q8_0.dequantize(qs, d))


class Qwen3Ref:
    """Restated `Qwen3` (qwen3.rs:342-563).

    `weights` is the host weight dictionary produced by the synthetic
    generator (f32 "checkpoint" values, plus optional pre-quantised Q8_0
    `(qs, d)` tensors under `weights["q8"]`). `accumulate="f64"` evaluates
    every matmul in f64 (same rounding points): the distance between the two
    variants is the noise floor that any second implementation of the same
    arithmetic inherits.
    """

    def __init__(self, cfg: TextConfig, weights: dict, precision: str = "bf16", max_len: int = 65_536,
                 accumulate: str = "f32"):
        if precision not in ACT_DTYPES:
            raise ValueError(f"unknown precision {precision!r}")
        self.mm = {"f32": _mm32, "f64": _mm64}[accumulate]
        self.cfg = cfg
        self.precision = precision
        self.act = _Act(ACT_DTYPES[precision])
        a = self.act
        quant = is_quantized(precision)
        pre = weights.get("q8") if quant else None

        def dense(x):  # the activation-dtype view of the checkpoint (linear.rs:124-125)
            return a.r(torch.from_numpy(np.asarray(x, dtype=np.float32)))

        def proj(parts, keys, i):
            if quant:
                if pre is not None:  # pre-quantised parts, stacked along the output axis
                    return torch.cat([torch.from_numpy(q8_0.dequantize(*pre["layers"][i][k])) for k in keys], 0)
                return _fused_q8(parts)
            return dense(np.concatenate([np.asarray(p, dtype=np.float32) for p in parts], axis=0))

        self.layers: list[LayerWeights] = []
        for i, lw in enumerate(weights["layers"]):
            self.layers.append(LayerWeights(
                input_norm=dense(lw["input_norm"]),
                post_norm=dense(lw["post_norm"]),
                q_norm=dense(lw["q_norm"]),
                k_norm=dense(lw["k_norm"]),
                qkv=proj([lw["q"], lw["k"], lw["v"]] if "q" in lw else None, ("q", "k", "v"), i),
                o=proj([lw["o"]] if "o" in lw else None, ("o",), i),
                gate_up=proj([lw["gate"], lw["up"]] if "gate" in lw else None, ("gate", "up"), i),
                down=proj([lw["down"]] if "down" in lw else None, ("down",), i),
            ))
        # The embedding lookup stays dense even in int8 (qwen3.rs:360); the
        # tied head is quantised from the f32 source in int8 (qwen3.rs:566-578).
        self.embed_table = dense(weights["embed"])
        if quant:
            if pre is not None and "lm_head" in pre:
                qs, d = pre["lm_head"]
                self.lm_head = torch.from_numpy(q8_0.dequantize(qs, d))
            else:
                self.lm_head = _fused_q8([weights.get("lm_head", weights["embed"])])
        else:
            self.lm_head = dense(weights.get("lm_head", weights["embed"]))
        self.norm = dense(weights["norm"])
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.rope_theta, max_len, a)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)  # qwen3.rs:198

    # --- model surface -------------------------------------------------------------

    def embed(self, ids) -> torch.Tensor:
        """`Qwen3::embed` (qwen3.rs:405-412): `(b, t)` ids -> `(b, t, hidden)`."""
        ids = torch.as_tensor(np.asarray(ids, dtype=np.int64))
        return self.embed_table[ids.reshape(-1)].reshape(*ids.shape, self.cfg.hidden_size)

    def new_caches(self, batch: int, capacity: int) -> list[KvCache]:
        """`Qwen3::new_caches` (qwen3.rs:415-428)."""
        c = self.cfg
        return [
            KvCache(
                torch.zeros(batch, c.num_key_value_heads, capacity, c.head_dim),
                torch.zeros(batch, c.num_key_value_heads, capacity, c.head_dim),
            )
            for _ in range(c.num_hidden_layers)
        ]

    def cache_bytes(self, batch: int, capacity: int) -> int:
        """`Qwen3::cache_bytes` (qwen3.rs:431-440)."""
        c = self.cfg
        elem = 4 if self.act.dtype == torch.float32 else 2
        return c.num_hidden_layers * KvCache.bytes_per_layer(
            batch, c.num_key_value_heads, capacity, c.head_dim, elem)

    def _attention(self, lw: LayerWeights, xs, cache: KvCache, offset: int, mask) -> torch.Tensor:
        """`Attention::forward` (qwen3.rs:203-259)."""
        qkv = self.act.r(self.mm(xs, lw.qkv.T))  # FusedLinear::forward (linear.rs:85-95)
        return self.act.r(self.mm(self._context(lw, qkv, cache, offset, mask), lw.o.T))

    def _context(self, lw: LayerWeights, qkv, cache: KvCache, offset: int, mask) -> torch.Tensor:
        """The part of `Attention::forward` between the fused QKV projection and
        the output projection (qwen3.rs:211-257): split, per-head q/k norm,
        RoPE at `offset`, cache append, grouped attention."""
        a, c = self.act, self.cfg
        b, t, _ = qkv.shape
        q = qkv[..., :c.q_dim].reshape(b, t, c.num_attention_heads, c.head_dim)
        k = qkv[..., c.q_dim:c.q_dim + c.kv_dim].reshape(b, t, c.num_key_value_heads, c.head_dim)
        v = qkv[..., c.q_dim + c.kv_dim:].reshape(b, t, c.num_key_value_heads, c.head_dim)
        # head-wise norm before the transpose (qwen3.rs:218-222)
        q = rms_norm(q, lw.q_norm, c.rms_norm_eps, a).transpose(1, 2)
        k = rms_norm(k, lw.k_norm, c.rms_norm_eps, a).transpose(1, 2)
        v = v.transpose(1, 2)
        cos, sin = self.cos[offset:offset + t], self.sin[offset:offset + t]
        q = rope_apply(q, cos, sin, a)
        k = rope_apply(k, cos, sin, a)
        k_all, v_all = cache.append(k, v)
        return _grouped_attention(q, k_all, v_all, mask, c.kv_repeat, self.scale, a, self.mm)

    def _mlp(self, lw: LayerWeights, xs) -> torch.Tensor:
        """`Mlp::forward` (qwen3.rs:288-292): down(silu(gate) * up)."""
        a, i = self.act, self.cfg.intermediate_size
        gu = a.r(self.mm(xs, lw.gate_up.T))
        gated = a.r(torch.nn.functional.silu(gu[..., :i]))
        return a.r(self.mm(a.r(gated * gu[..., i:]), lw.down.T))

    def forward_embeds(self, embeds, caches: list[KvCache], offset: int, mask) -> torch.Tensor:
        """`Qwen3::forward_embeds` + `Layer::forward` (qwen3.rs:444-456, :322-339)."""
        a, c = self.act, self.cfg
        xs = embeds
        for lw, cache in zip(self.layers, caches):
            h = self._attention(lw, rms_norm(xs, lw.input_norm, c.rms_norm_eps, a), cache, offset, mask)
            xs = a.r(xs + h)
            h = self._mlp(lw, rms_norm(xs, lw.post_norm, c.rms_norm_eps, a))
            xs = a.r(xs + h)
        return rms_norm(xs, self.norm, c.rms_norm_eps, a)

    def logits(self, hidden) -> torch.Tensor:
        """`Qwen3::logits` (qwen3.rs:459-463): lm_head in the activation dtype, then f32."""
        return self.act.r(self.mm(hidden, self.lm_head.T))

    # --- solo (ragged) mode: one sequence, positions 0..len ---------------------

    def _causal(self, q_offset: int, q_len: int, kv_len: int) -> torch.Tensor:
        return build_mask(1, q_offset, q_len, kv_len, [0], self.cfg.kv_repeat)

    def prefill(self, embeds, caches: list[KvCache], block: int = PREFILL_BLOCK) -> torch.Tensor:
        """`Qwen3::prefill` (qwen3.rs:475-496) for `(1, T, hidden)` embeds with no
        padding. Returns the final-norm hidden state of the last position."""
        embeds = torch.as_tensor(embeds, dtype=torch.float32)
        embeds = self.act.r(embeds)
        if embeds.dim() == 2:
            embeds = embeds.unsqueeze(0)
        total = embeds.shape[1]
        if total == 0:
            raise ValueError("empty prompt")
        start, last = caches[0].len, None
        end = start + total
        pos = start
        while pos < end:
            n = min(block, end - pos)
            blk = embeds[:, pos - start:pos - start + n]
            last = self.forward_embeds(blk, caches, pos, self._causal(pos, n, pos + n))
            pos += n
        return last[:, -1:]

    def decode_step(self, token: int, caches: list[KvCache]) -> torch.Tensor:
        """`Qwen3::decode_step` (qwen3.rs:499-511) for one sequence: returns f32
        logits `(vocab,)`."""
        off = caches[0].len
        emb = self.embed([[token]])
        hidden = self.forward_embeds(emb, caches, off, self._causal(off, 1, off + 1))
        return self.logits(hidden)[0, 0]

    def decode_step_ragged(self, tokens, caches: list[list[KvCache]]) -> torch.Tensor:
        """Solo-mode decode of several sequences in one pass: row i is
        `decode_step(tokens[i], caches[i])` (each sequence at its own position,
        with its own caches). The projections run over all rows at once, the
        attention per sequence. Returns f32 logits `(len(tokens), vocab)`."""
        a, c = self.act, self.cfg
        xs = self.embed([[int(t)] for t in tokens])
        for li, lw in enumerate(self.layers):
            qkv = a.r(self.mm(rms_norm(xs, lw.input_norm, c.rms_norm_eps, a), lw.qkv.T))
            ctx = torch.cat([self._context(lw, qkv[i:i + 1], caches[i][li], caches[i][li].len, None)
                             for i in range(len(tokens))], 0)
            xs = a.r(xs + a.r(self.mm(ctx, lw.o.T)))
            xs = a.r(xs + self._mlp(lw, rms_norm(xs, lw.post_norm, c.rms_norm_eps, a)))
        return self.logits(rms_norm(xs, self.norm, c.rms_norm_eps, a))[:, 0]

    # --- left-padded batch mode: the reference's own batching ----------------------

    def prefill_padded(self, embeds: list, caches: list[KvCache], block: int = PREFILL_BLOCK):
        """`Engine::generate_batch` padding (engine.rs:476-491) + `Qwen3::prefill`
        (qwen3.rs:475-496). Returns `(hidden_last (b,1,h), pad_lengths)`."""
        a, h = self.act, self.cfg.hidden_size
        lens = [int(e.shape[-2]) for e in embeds]
        tmax = max(lens)
        pads = [tmax - n for n in lens]
        rows = []
        for e, pad in zip(embeds, pads):
            e = a.r(torch.as_tensor(e, dtype=torch.float32).reshape(-1, h))
            rows.append(torch.cat([torch.zeros(pad, h), e], 0))
        batched = torch.stack(rows)
        b = len(embeds)
        last, start = None, 0
        while start < tmax:
            n = min(block, tmax - start)
            mask = build_mask(b, start, n, start + n, pads, self.cfg.kv_repeat)
            last = self.forward_embeds(batched[:, start:start + n], caches, start, mask)
            start += n
        return last[:, -1:], pads

    def decode_step_padded(self, ids: list[int], caches: list[KvCache], pads: list[int]) -> torch.Tensor:
        """`Qwen3::decode_step` (qwen3.rs:499-511) on the left-padded batch."""
        off = caches[0].len
        emb = self.embed([[t] for t in ids])
        mask = build_mask(len(ids), off, 1, off + 1, pads, self.cfg.kv_repeat)
        return self.logits(self.forward_embeds(emb, caches, off, mask))[:, 0]


def argmax_rows(logits) -> list[int]:
    """`argmax_rows` (engine.rs:550-559): per-row argmax of `(b, v)` or the last
    position of `(b, t, v)`; ties resolve to the lowest index."""
    x = torch.as_tensor(logits)
    if x.dim() == 3:
        x = x[:, -1]
    return [int(i) for i in torch.argmax(x.to(torch.float32), dim=-1)]


@dataclass
class Generated:
    tokens: list[int] = field(default_factory=list)
    finish_reason: str = "length"


def generate(model: Qwen3Ref, embeds, budget: int, eos_id: int = EOS_TOKEN_ID,
             forced_stop: int | None = None, record_logits: bool = False):
    """Greedy loop of `Engine::generate_batch` (engine.rs:505-538) for one
    sequence in solo mode.

    Each step takes the argmax of the current logits; EOS ends the sequence
    with reason "stop" and is not emitted; otherwise the token is emitted and
    fed back; at most `budget` tokens are emitted ("length").
    `forced_stop=n` treats the n-th generated token (0-based) as EOS, the
    synthetic end-of-turn of the BASELINE configs.
    Returns `(Generated, [logits per step])`.
    """
    embeds = torch.as_tensor(embeds, dtype=torch.float32)
    n = embeds.shape[-2]
    caches = model.new_caches(1, n + budget)
    logits = model.logits(model.prefill(embeds.reshape(1, n, -1), caches))[0, 0]
    out, hist = Generated(), []
    for step in range(budget):
        if record_logits:
            hist.append(logits.clone())
        tok = argmax_rows(logits.reshape(1, -1))[0]
        if tok == eos_id or (forced_stop is not None and step == forced_stop):
            out.finish_reason = "stop"
            break
        out.tokens.append(tok)
        if step + 1 == budget:
            break
        logits = model.decode_step(tok, caches)
    return out, hist


def teacher_forced_logits(model: Qwen3Ref, prompts, streams) -> list[list[torch.Tensor]]:
    """The logits the greedy loop of `Engine::generate_batch` (engine.rs:505-538)
    sees at every step when it is fed the given token streams instead of its
    own picks: `out[i][s]` are sequence i's f32 logits before its s-th pick
    (the prefill's last position for s = 0, then one decode step per token of
    `streams[i]`), so `out[i]` has `len(streams[i]) + 1` entries. Sequences run
    in solo mode (positions from 0), batched per step with
    `decode_step_ragged`."""
    caches, out = [], []
    for p, toks in zip(prompts, streams):
        p = torch.as_tensor(np.asarray(p, dtype=np.float32))
        n = p.shape[-2]
        cs = model.new_caches(1, n + len(toks) + 1)
        caches.append(cs)
        out.append([model.logits(model.prefill(p.reshape(1, n, -1), cs))[0, 0]])
    for s in range(max((len(t) for t in streams), default=0)):
        live = [i for i, t in enumerate(streams) if s < len(t)]
        lg = model.decode_step_ragged([streams[i][s] for i in live], [caches[i] for i in live])
        for j, i in enumerate(live):
            out[i].append(lg[j])
    return out


def splice_audio(model: Qwen3Ref, token_ids, audio_embeds, audio_token_id: int) -> torch.Tensor:
    """`MossModel::splice_audio` (model/mod.rs:134-180): the prompt embedding of
    one sequence. The ids are walked as alternating runs of text and audio
    placeholders; text runs are embedded, audio runs are taken in order from
    `audio_embeds` (converted to the activation dtype, mod.rs:141), and the
    parts are concatenated. A placeholder count different from the number of
    audio rows is an error (mod.rs:143-150). Returns `(len(ids), hidden)`."""
    ids = [int(i) for i in np.asarray(token_ids).reshape(-1)]
    audio = model.act.r(torch.as_tensor(np.asarray(audio_embeds, dtype=np.float32)).reshape(-1, model.cfg.hidden_size))
    n_slots = sum(1 for i in ids if i == audio_token_id)
    if n_slots != audio.shape[0]:
        raise ValueError(f"prompt has {n_slots} audio placeholders but the encoder produced "
                         f"{audio.shape[0]} embeddings")
    if n_slots == 0:
        return model.embed(ids)
    parts, used, i = [], 0, 0
    while i < len(ids):
        is_audio = ids[i] == audio_token_id
        j = i
        while j < len(ids) and (ids[j] == audio_token_id) == is_audio:
            j += 1
        if is_audio:
            parts.append(audio[used:used + (j - i)])
            used += j - i
        else:
            parts.append(model.embed(ids[i:j]))
        i = j
    return torch.cat(parts, 0)
