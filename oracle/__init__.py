"""CPU oracle for the batched Qwen3 decoder step -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference decoder
(`crates/fmd-core/src/model/qwen3.rs`, `crates/fmd-core/src/model/linear.rs`,
`crates/fmd-core/src/engine.rs` of cnmoro/fast-moss-diarization). It exists to
check the CUDA path, never to run in its place: only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` may import it.

Pinning status:
  * Q8_0 quantise/dequantise is pinned against gguf-py 0.19.0's independent
    implementation of the same GGML format (`tests/test_oracle_q8_0.py`).
  * The decoder restatement is pinned against every known-answer test the
    reference holds for this path (`qwen3.rs:601-820`, `linear.rs:337-364`,
    `engine.rs:601-615`), restated in `tests/test_oracle_pins.py`.
  * End-to-end logits and greedy ids are PARITY UNPINNED: the reference ships
    no golden logits or token ids, and it cannot be built here (pure Rust on
    candle 0.11.0; no Rust toolchain). `tests/golden/` freezes this oracle's own
    outputs so later changes to it are caught.
"""
