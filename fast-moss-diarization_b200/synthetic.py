"""Seeded synthetic weights and workloads for the BASELINE configurations.

There is no checkpoint and no network here, so every weight and prompt is
generated from a seed. Shapes follow the reference's Qwen3 backbone; the
workloads follow the five BASELINE configs: random-init N(0, 0.02) weights
(norm gains 1), prompts whose first 75 % is an N(0, 1) embedding span standing
in for the audio adaptor output and the rest uniform text ids; Q8_0 weights
drawn directly as int8 uniform in [-127, 127] with |N(0, 0.002)| f16 scales.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .config import TextConfig

QK = 32


def _normal(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def make_weights(cfg: TextConfig, seed: int = 0, std: float = 0.02, norm_jitter: float = 0.0,
                 prequantized: bool = False, q8_scale_std: float = 0.002) -> dict:
    """Host weight dictionary.

    Dense mode: f32 "checkpoint" values for every projection (the reference
    converts them to the activation dtype, or quantises them to Q8_0 from f32
    in int8 mode). `prequantized=True`: projections are generated directly as
    Q8_0 `(qs int8, d f16)` pairs under `w["q8"]`, and the tied lm_head is the
    Q8_0 quantisation of the embedding (as the reference builds it).
    """
    rng = np.random.default_rng(seed)
    h, i, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.q_dim, cfg.kv_dim

    def gain(n):
        if norm_jitter == 0.0:
            return np.ones(n, dtype=np.float32)
        return (1.0 + rng.uniform(-norm_jitter, norm_jitter, n)).astype(np.float32)

    def q8(rows, cols):
        qs = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
        d = np.abs(rng.standard_normal((rows, cols // QK), dtype=np.float32) * np.float32(q8_scale_std))
        return qs, d.astype(np.float16)

    w: dict = {"embed": _normal(rng, (cfg.vocab_size, h), std), "norm": gain(h), "layers": []}
    q8layers = []
    for _ in range(cfg.num_hidden_layers):
        lw = {"input_norm": gain(h), "post_norm": gain(h), "q_norm": gain(cfg.head_dim),
              "k_norm": gain(cfg.head_dim)}
        if prequantized:
            q8layers.append({"q": q8(qd, h), "k": q8(kvd, h), "v": q8(kvd, h), "o": q8(h, qd),
                             "gate": q8(i, h), "up": q8(i, h), "down": q8(h, i)})
        else:
            lw.update(q=_normal(rng, (qd, h), std), k=_normal(rng, (kvd, h), std), v=_normal(rng, (kvd, h), std),
                      o=_normal(rng, (h, qd), std), gate=_normal(rng, (i, h), std), up=_normal(rng, (i, h), std),
                      down=_normal(rng, (h, i), std))
        w["layers"].append(lw)
    if prequantized:
        w["q8"] = {"layers": q8layers}
    return w


def log_uniform_lengths(rng: np.random.Generator, n: int, lo: int, hi: int) -> np.ndarray:
    return np.exp(rng.uniform(np.log(lo), np.log(hi), n)).astype(np.int64).clip(lo, hi)


@dataclass
class Workload:
    """A request queue: per-request prompt lengths, budgets, forced stops, and
    a seed-derived embedding arena (rows back to back, f32 or bf16 bits)."""

    name: str
    prompt_lens: np.ndarray
    max_new: np.ndarray
    forced_stop: np.ndarray
    max_batch: int
    prefill_chunk: int
    precision: str
    arena: np.ndarray | None = None          # (rows, hidden) float32 or uint16 (bf16 bits)
    arena_dtype: str = "f32"
    meta: dict = field(default_factory=dict)

    def subset(self, idx) -> "Workload":
        """The requests `idx` (in that order) as their own queue, without an
        arena (build one with `build_prompt_arena` for the subset)."""
        idx = np.asarray(idx, dtype=np.int64)
        return Workload(self.name, self.prompt_lens[idx], self.max_new[idx], self.forced_stop[idx], self.max_batch,
                        self.prefill_chunk, self.precision, None, self.arena_dtype, dict(self.meta))

    @property
    def embed_rows(self) -> np.ndarray:
        off = np.zeros(len(self.prompt_lens), dtype=np.int64)
        off[1:] = np.cumsum(self.prompt_lens)[:-1]
        return off


def build_prompt_arena(cfg: TextConfig, embed: np.ndarray, lens, seed: int, span_frac: float = 0.75,
                       pool_rows: int = 65536, out_bf16: bool = False) -> np.ndarray:
    """Prompt embeddings, back to back: the first `span_frac` of each prompt are
    N(0,1) rows (the audio-span stand-in; drawn from a seeded pool of rows to
    keep generation cheap for long queues), the rest are embedding-table rows of
    uniform random text ids."""
    rng_span = np.random.default_rng(seed + 1)
    rng_txt = np.random.default_rng(seed + 2)
    h = cfg.hidden_size
    total = int(np.sum(lens))
    pool = rng_span.standard_normal((min(pool_rows, max(total, 1)), h), dtype=np.float32)
    out = np.empty((total, h), dtype=np.uint16 if out_bf16 else np.float32)
    r = 0
    for n in lens:
        n = int(n)
        n_span = int(round(span_frac * n))
        span = pool[rng_span.integers(0, pool.shape[0], n_span)] if n_span else np.empty((0, h), np.float32)
        ids = rng_txt.integers(0, cfg.vocab_size, n - n_span)
        rows = np.concatenate([span, embed[ids]], axis=0)
        out[r:r + n] = f32_to_bf16_bits(rows) if out_bf16 else rows
        r += n
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (NaN-free inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def config1_prompts(cfg: TextConfig, embed: np.ndarray, seed: int = 0):
    """4 ragged prompts of 412/797/1190/1500 tokens, greedy 64."""
    lens = [412, 797, 1190, 1500]
    arena = build_prompt_arena(cfg, embed, lens, seed)
    out, r = [], 0
    for n in lens:
        out.append(arena[r:r + n])
        r += n
    return out


def workload(config: int, cfg: TextConfig, embed: np.ndarray, seed: int = 0, n_requests: int | None = None,
             out_bf16: bool = True, with_arena: bool = True) -> Workload:
    """Request queues of BASELINE configs 2 to 5;
    `with_arena=False` leaves the prompt embeddings out (lengths only)."""
    rng = np.random.default_rng(seed + 100 * config)
    if config == 2:
        n = n_requests or 8
        lens = log_uniform_lengths(rng, n, 1200, 5000)
        forced = rng.integers(256, 513, n)
        max_new = np.full(n, 4096)
        wl = Workload("bf16_b8_forced_eot", lens, max_new, forced, max_batch=8, prefill_chunk=2048,
                      precision="bf16")
    elif config == 3:
        n = n_requests or 256
        lens = log_uniform_lengths(rng, n, 300, 8000)
        stops = np.minimum(rng.geometric(1.0 / 600, n), 4096)
        wl = Workload("q8_0_b32_continuous", lens, np.full(n, 4096), stops, max_batch=32, prefill_chunk=2048,
                      precision="int8_bf16")
    elif config == 4:
        # 24 decoders first (contexts log-uniform 1k-8k, decoding throughout),
        # then 8 prompts of 16k tokens prefilled in 2048-row chunks while the
        # 24 decode (FIFO admission puts the long prompts behind them)
        n_dec = 24
        dec_lens = log_uniform_lengths(rng, n_dec, 1000, 8000)
        lens = np.concatenate([dec_lens, np.full(8, 16384, dtype=np.int64)])
        max_new = np.concatenate([np.full(n_dec, 4096), np.full(8, 16)])
        forced = np.full(n_dec + 8, -1)
        wl = Workload("chunked_prefill_mixed", lens, max_new, forced, max_batch=32, prefill_chunk=2048,
                      precision="int8_bf16", meta={"n_decoders": n_dec})
    elif config == 5:
        n = n_requests or 2048
        lens = log_uniform_lengths(rng, n, 300, 16000)
        stops = np.minimum(rng.geometric(1.0 / 800, n), 4096)
        wl = Workload("q8_0_b64_dp", lens, np.full(n, 4096), stops, max_batch=64, prefill_chunk=2048,
                      precision="int8_bf16")
    else:
        raise ValueError(f"no request-queue workload for config {config}")
    # the forced stop is the n-th generated token; geometric draws are >= 1
    wl.arena_dtype = "bf16" if out_bf16 else "f32"
    if with_arena:
        wl.arena = build_prompt_arena(cfg, embed, wl.prompt_lens, seed + 7 * config, out_bf16=out_bf16)
    return wl
