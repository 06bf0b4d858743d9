"""Prompt layout of the audio span and its assembly into prefill rows.

`audio_span_ids` restates `PromptBuilder::audio_span_ids`
(crates/fmd-core/src/prompt.rs:89-124): the audio span is a run of
placeholder ids with the elapsed second count written as digit tokens every
`time_marker_every_seconds`, including the reference's quirk that the marker
for second `s` lands at audio index `(s / every) * tokens_per_marker`.
`build_prompt_ids` is `PromptBuilder::build` (prompt.rs:139-150) with the
tokenised chat-template halves passed in (the tokenizer is not on this path).

The prompt rows themselves are assembled on the GPU by
`Qwen3Decoder.splice_audio` (`fmd_splice_audio`, the analogue of
`MossModel::splice_audio`, model/mod.rs:134-180).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ProcessorConfig:
    """`ProcessorConfig` defaults (crates/fmd-core/src/config.rs:170-202)."""

    audio_tokens_per_second: float = 12.5
    audio_merge_size: int = 4
    time_marker_every_seconds: int = 5
    enable_time_marker: bool = True


def audio_span_ids(audio_tokens: int, audio_token_id: int, digit_ids, cfg: ProcessorConfig = ProcessorConfig()):
    """Placeholder ids for `audio_tokens` audio embeddings, with digit time
    markers (prompt.rs:89-124). `digit_ids[d]` is the token of digit d."""
    every = cfg.time_marker_every_seconds
    if not cfg.enable_time_marker or audio_tokens == 0 or every == 0:
        return [audio_token_id] * audio_tokens
    tokens_per_marker = int(cfg.audio_tokens_per_second * every)  # `as usize` truncates
    if tokens_per_marker == 0:
        return [audio_token_id] * audio_tokens
    duration = audio_tokens / cfg.audio_tokens_per_second
    out: list[int] = []
    consumed = 0
    sec = every
    while sec <= int(duration):
        pos = (sec // every) * tokens_per_marker
        if pos > consumed:
            out.extend([audio_token_id] * (pos - consumed))
            consumed = pos
        out.extend(int(digit_ids[int(ch)]) for ch in str(sec))
        sec += every
    if audio_tokens > consumed:
        out.extend([audio_token_id] * (audio_tokens - consumed))
    return out


def build_prompt_ids(before_ids, audio_tokens: int, after_ids, audio_token_id: int, digit_ids,
                     cfg: ProcessorConfig = ProcessorConfig()) -> np.ndarray:
    """`PromptBuilder::build` (prompt.rs:139-150): the tokenised text before the
    audio, the audio span, the tokenised text after it."""
    ids = list(before_ids) + audio_span_ids(audio_tokens, audio_token_id, digit_ids, cfg) + list(after_ids)
    return np.asarray(ids, dtype=np.int32)
