"""Continuous-batching generation over prompt embeddings.

Mirrors the decode half of `Engine::transcribe` (crates/fmd-core/src/
engine.rs:382-424) and `Engine::generate_batch` (engine.rs:463-541): requests
are length-sorted (engine.rs:385), decoded greedily with EOS 151645 ending a
sequence (not emitted), at most `max_new_tokens` tokens each. Unlike the
reference's static micro-batches, finished slots are refilled on the GPU from
the queue, and prompt prefill is chunked into decode steps.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .decoder import Qwen3Decoder


@dataclass
class Generated:
    """`Generated` (engine.rs:544-547)."""

    tokens: list[int] = field(default_factory=list)
    finish_reason: str = "length"


@dataclass
class BatchStats:
    """The decode-side fields of `BatchStats` (engine.rs:151-174), plus the
    device-timed window of the last `run`/`step` call."""

    requests: int = 0
    generate_seconds: float = 0.0
    generated_tokens: int = 0
    prefill_tokens: int = 0
    steps: int = 0
    device_status: int = 0
    window_steps: int = 0
    window_tokens: int = 0
    window_device_ms: float = 0.0
    attn_decode_ms: float = 0.0
    attn_kv_tokens: int = 0
    attn_rows: int = 0
    window_mixed_steps: int = 0
    graph_kernels_mixed: int = 0
    graph_kernels_decode: int = 0
    lm_head_ms: float = 0.0

    @classmethod
    def from_c(cls, st) -> "BatchStats":
        return cls(requests=int(st.requests_done), generate_seconds=st.generate_seconds,
                   generated_tokens=int(st.generated_tokens), prefill_tokens=int(st.prefill_tokens),
                   steps=int(st.steps), device_status=int(st.device_status), window_steps=int(st.window_steps),
                   window_tokens=int(st.window_tokens), window_device_ms=float(st.window_device_ms),
                   attn_decode_ms=float(st.attn_decode_ms), attn_kv_tokens=int(st.attn_kv_tokens),
                   attn_rows=int(st.attn_rows), window_mixed_steps=int(st.window_mixed_steps),
                   graph_kernels_mixed=int(st.graph_kernels_mixed), graph_kernels_decode=int(st.graph_kernels_decode),
                   lm_head_ms=float(st.lm_head_ms))

    @property
    def decode_tokens_per_second(self) -> float:
        return self.generated_tokens / self.generate_seconds if self.generate_seconds > 0 else 0.0


_REASONS = {_lib.FINISH_STOP: "stop", _lib.FINISH_LENGTH: "length", _lib.FINISH_ERROR: "error"}


class Engine:
    def __init__(self, decoder: Qwen3Decoder):
        self.dec = decoder
        self.lib = decoder.lib
        self.n = 0
        self.order = None

    def load(self, prompt_lens, max_new_tokens, forced_stop, arena: np.ndarray, embed_rows=None,
             sort_by_length: bool = True) -> None:
        """Queue requests. `arena` holds all prompt rows (f32, or uint16 bits of
        the activation dtype); request i reads `prompt_lens[i]` rows from
        `embed_rows[i]` (default: back to back)."""
        if arena.dtype == np.uint16:
            dt = _lib.DT_BF16 if self.dec.act == "bf16" else _lib.DT_F16
        else:
            arena = np.ascontiguousarray(arena, dtype=np.float32)
            dt = _lib.DT_F32
        arena = np.ascontiguousarray(arena)
        self._load(prompt_lens, max_new_tokens, forced_stop, arena.ctypes.data, arena.shape[0], dt, embed_rows,
                   sort_by_length)

    def load_device(self, prompt_lens, max_new_tokens, forced_stop, arena_ptr: int, arena_rows: int,
                    embed_rows=None, sort_by_length: bool = True) -> None:
        """`load` from an arena already in device memory (activation dtype,
        `arena_rows` x hidden at device address `arena_ptr`), such as the rows
        `Qwen3Decoder.splice_audio` writes: no host round trip."""
        dt = _lib.DT_BF16 if self.dec.act == "bf16" else _lib.DT_F16
        self._load(prompt_lens, max_new_tokens, forced_stop, arena_ptr, arena_rows, dt, embed_rows, sort_by_length)

    def _load(self, prompt_lens, max_new_tokens, forced_stop, arena_ptr, arena_rows, dt, embed_rows,
              sort_by_length) -> None:
        lens = np.asarray(prompt_lens, dtype=np.int64)
        n = len(lens)
        if embed_rows is None:
            embed_rows = np.zeros(n, dtype=np.int64)
            embed_rows[1:] = np.cumsum(lens)[:-1]
        mx = np.broadcast_to(np.asarray(max_new_tokens, dtype=np.int64), (n,))
        fs = np.broadcast_to(np.asarray(-1 if forced_stop is None else forced_stop, dtype=np.int64), (n,))
        order = np.argsort(lens, kind="stable") if sort_by_length else np.arange(n)
        reqs = (_lib.Request * n)()
        for j, i in enumerate(order):
            reqs[j].prompt_len = int(lens[i])
            reqs[j].max_new_tokens = int(mx[i])
            reqs[j].forced_stop = int(fs[i])
            reqs[j].embed_row = int(embed_rows[i])
        self.lib_check(self.lib.fmd_engine_load(self.dec.handle, reqs, n, C.c_void_p(arena_ptr), arena_rows, dt))
        self.n = n
        self.order = order
        self.max_new = int(mx.max()) if n else 0

    def lib_check(self, st: int) -> None:
        _lib.check(st, self.dec.handle)

    def run(self, max_batch: int, prefill_chunk: int = 2048, max_steps: int = 1 << 40) -> BatchStats:
        st = _lib.Stats()
        self.lib_check(self.lib.fmd_engine_run(self.dec.handle, max_batch, prefill_chunk, max_steps, C.byref(st)))
        return BatchStats.from_c(st)

    def start(self, max_batch: int, prefill_chunk: int = 2048) -> None:
        """Reset onto the loaded queue and build the step graph."""
        self.lib_check(self.lib.fmd_engine_start(self.dec.handle, max_batch, prefill_chunk))

    def step(self, max_steps: int) -> BatchStats:
        """Advance the started engine by up to `max_steps` device steps."""
        st = _lib.Stats()
        self.lib_check(self.lib.fmd_engine_step(self.dec.handle, max_steps, C.byref(st)))
        return BatchStats.from_c(st)

    @property
    def done(self) -> bool:
        st = _lib.Stats()
        self.lib_check(self.lib.fmd_engine_step(self.dec.handle, 0, C.byref(st)))
        return st.requests_done >= self.n

    def fetch(self) -> list[Generated]:
        stride = max(self.max_new, 1)
        toks = np.zeros((self.n, stride), dtype=np.int32)
        res = (_lib.Result * self.n)()
        self.lib_check(self.lib.fmd_engine_fetch(self.dec.handle, toks.ctypes.data_as(C.POINTER(C.c_int32)),
                                                 stride, res))
        out: list[Generated | None] = [None] * self.n
        for j, i in enumerate(self.order):
            r = res[j]
            out[i] = Generated(tokens=toks[j, :r.n_tokens].tolist(), finish_reason=_REASONS.get(r.finish_reason, "?"))
        return out

    def generate(self, prompt_lens, max_new_tokens, forced_stop, arena, max_batch: int, prefill_chunk: int = 2048):
        self.load(prompt_lens, max_new_tokens, forced_stop, arena)
        stats = self.run(max_batch, prefill_chunk)
        return self.fetch(), stats
