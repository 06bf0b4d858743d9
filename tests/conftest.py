"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

PKG = __graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


@pytest.fixture(scope="session")
def pkg():
    return PKG


def tiny_config(**kw):
    """A small Qwen3-shaped config: same head_dim/GQA ratio as the real model."""
    base = dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=8192)
    base.update(kw)
    return PKG.TextConfig(**base)


def mid_config(**kw):
    """The BASELINE model's layer shapes (hidden 1024, 16/8 heads, FFN 3072,
    vocab 151936) with fewer layers, so the CPU oracle finishes in seconds."""
    base = dict(num_hidden_layers=2, max_position_embeddings=8192)
    base.update(kw)
    return PKG.TextConfig(**base)


def oracle_model(cfg, weights, precision, max_len=8192):
    from oracle import qwen3_ref as ref

    return ref.Qwen3Ref(ref.TextConfig(**cfg.oracle_kwargs()), weights, precision, max_len=max_len)


def rel_err(got, want) -> float:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))
