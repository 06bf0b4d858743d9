"""Generate the golden fixtures in this directory from the CPU oracle.

The reference ships no golden logits or ids for its decoder and cannot be run
here (pure Rust on candle 0.11.0, no Rust toolchain), so these fixtures freeze
the oracle's own outputs on a small seeded Qwen3-shaped model. They pin the
oracle against accidental change (tests/test_golden.py, CPU) and give the GPU
path a fixed target (same file, `gpu` marker).

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

PKG = __graft_entry__.load_package()
from fmd_b200 import synthetic  # noqa: E402
from oracle import qwen3_ref as ref  # noqa: E402

OUT = Path(__file__).resolve().parent / "tiny_decoder.npz"
CFG = dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
           num_key_value_heads=2, max_position_embeddings=8192)
WEIGHT_SEED = 11
PRECISIONS = ["bf16", "f16", "int8", "int8_bf16"]
LENS = [37, 70]
STEPS = 6


def weight_checksum(w: dict) -> float:
    s = float(np.abs(w["embed"]).sum())
    for lw in w["layers"]:
        for k in sorted(lw):
            s += float(np.abs(lw[k]).sum())
    return s


def generate() -> dict:
    cfg = PKG.TextConfig(**CFG)
    w = synthetic.make_weights(cfg, seed=WEIGHT_SEED, norm_jitter=0.2)
    rng = np.random.default_rng(1234)
    prompts = [rng.standard_normal((n, cfg.hidden_size)).astype(np.float32) for n in LENS]
    tokens = rng.integers(0, cfg.vocab_size, (len(LENS), STEPS)).astype(np.int32)
    out = {"checksum": np.array(weight_checksum(w)), "tokens": tokens, "lens": np.array(LENS)}
    for i, p in enumerate(prompts):
        out[f"prompt{i}"] = p
    for prec in PRECISIONS:
        m = ref.Qwen3Ref(ref.TextConfig(**cfg.oracle_kwargs()), w, prec, max_len=512)
        for i, p in enumerate(prompts):
            caches = m.new_caches(1, 128)
            rows = [m.logits(m.prefill(p[None], caches))[0, 0].numpy()]
            for t in tokens[i]:
                rows.append(m.decode_step(int(t), caches).numpy())
            out[f"logits_{prec}_{i}"] = np.stack(rows).astype(np.float32)
    return out


if __name__ == "__main__":
    data = generate()
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")
