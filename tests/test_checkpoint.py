"""Checkpoint loading (safetensors, the reference's tensor names and shard
index; qwen3.rs:354-390, hub.rs:166-214, config.rs:8-58), on CPU."""

from __future__ import annotations

import importlib
import json

import numpy as np
import pytest

from conftest import tiny_config

ckpt = importlib.import_module("fmd_b200.checkpoint")
syn = importlib.import_module("fmd_b200.synthetic")

P = "model.language_model"


def _names(w):
    """The reference's name for every tensor of a weight dictionary."""
    out = {f"{P}.embed_tokens.weight": w["embed"], f"{P}.norm.weight": w["norm"]}
    for i, lw in enumerate(w["layers"]):
        p = f"{P}.layers.{i}."
        out.update({p + "input_layernorm.weight": lw["input_norm"], p + "post_attention_layernorm.weight": lw["post_norm"],
                    p + "self_attn.q_norm.weight": lw["q_norm"], p + "self_attn.k_norm.weight": lw["k_norm"],
                    p + "self_attn.q_proj.weight": lw["q"], p + "self_attn.k_proj.weight": lw["k"],
                    p + "self_attn.v_proj.weight": lw["v"], p + "self_attn.o_proj.weight": lw["o"],
                    p + "mlp.gate_proj.weight": lw["gate"], p + "mlp.up_proj.weight": lw["up"],
                    p + "mlp.down_proj.weight": lw["down"]})
    return out


def write_checkpoint(d, cfg, w, shards=1, bf16=True, extra=None):
    """A Moss-style checkpoint directory: config.json with `text_config`, the
    backbone tensors (projections and embedding as bf16 bits when `bf16`),
    split over `shards` files with an index when there is more than one."""
    tensors = {}
    for k, v in _names(w).items():
        v = np.asarray(v, dtype=np.float32)
        tensors[k] = syn.f32_to_bf16_bits(v) if bf16 and v.ndim == 2 else v
    tensors.update(extra or {})
    text = {k: getattr(cfg, k) for k in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                                          "num_attention_heads", "num_key_value_heads", "head_dim", "rms_norm_eps",
                                          "rope_theta", "max_position_embeddings")}
    (d / "config.json").write_text(json.dumps({"text_config": text, "audio_token_id": 151654}))
    names = list(tensors)
    if shards == 1:
        ckpt.write_safetensors(d / "model.safetensors", tensors)
        return tensors
    weight_map = {}
    for s in range(shards):
        part = {n: tensors[n] for n in names[s::shards]}
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        ckpt.write_safetensors(d / fname, part)
        weight_map.update({n: fname for n in part})
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    return tensors


@pytest.mark.parametrize("shards", [1, 3])
def test_load_checkpoint_round_trip(tmp_path, shards):
    cfg = tiny_config(max_position_embeddings=4096)
    w = syn.make_weights(cfg, seed=2, norm_jitter=0.1)
    stored = write_checkpoint(tmp_path, cfg, w, shards=shards)
    got_cfg, got = ckpt.load_checkpoint(tmp_path)
    assert got_cfg == cfg
    assert "lm_head" not in got  # tied to the embedding (qwen3.rs:366-372)
    for k, v in _names(got).items():
        assert v.dtype == stored[k].dtype and np.array_equal(v, stored[k]), k


def test_untied_head_and_errors(tmp_path):
    cfg = tiny_config(max_position_embeddings=4096)
    w = syn.make_weights(cfg, seed=3)
    head = np.random.default_rng(0).standard_normal((cfg.vocab_size, cfg.hidden_size)).astype(np.float32)
    write_checkpoint(tmp_path, cfg, w, extra={"lm_head.weight": head})
    _, got = ckpt.load_checkpoint(tmp_path)
    assert np.array_equal(got["lm_head"], head)
    # a missing tensor is named in the error
    t = ckpt.read_safetensors(tmp_path / "model.safetensors")
    del t[f"{P}.layers.1.mlp.up_proj.weight"]
    ckpt.write_safetensors(tmp_path / "model.safetensors", t)
    with pytest.raises(KeyError, match="layers.1.mlp.up_proj"):
        ckpt.load_checkpoint(tmp_path)
    # attention biases have no kernel here
    doc = json.loads((tmp_path / "config.json").read_text())
    doc["text_config"]["attention_bias"] = True
    (tmp_path / "config.json").write_text(json.dumps(doc))
    with pytest.raises(ValueError, match="attention_bias"):
        ckpt.text_config(tmp_path)


def test_safetensors_dtypes(tmp_path):
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    b = np.arange(6, dtype=np.float16)
    c = syn.f32_to_bf16_bits(np.linspace(-2, 2, 8, dtype=np.float32))
    ckpt.write_safetensors(tmp_path / "x.safetensors", {"a": a, "b": b, "c": c})
    got = ckpt.read_safetensors(tmp_path / "x.safetensors")
    assert np.array_equal(got["a"], a) and np.array_equal(got["b"], b) and np.array_equal(got["c"], c)
    assert got["c"].dtype == np.uint16


def test_interop_with_the_safetensors_package(tmp_path):
    """Files written here load with the `safetensors` package and vice versa."""
    st = pytest.importorskip("safetensors.numpy")
    a = np.random.default_rng(1).standard_normal((5, 7)).astype(np.float32)
    b = np.random.default_rng(2).standard_normal(9).astype(np.float16)
    ckpt.write_safetensors(tmp_path / "mine.safetensors", {"a": a, "b": b})
    theirs = st.load_file(str(tmp_path / "mine.safetensors"))
    assert np.array_equal(theirs["a"], a) and np.array_equal(theirs["b"], b)
    st.save_file({"a": a, "b": b}, str(tmp_path / "theirs.safetensors"))
    mine = ckpt.read_safetensors(tmp_path / "theirs.safetensors")
    assert np.array_equal(mine["a"], a) and np.array_equal(mine["b"], b)


# ---- the audio tower (whisper_encoder.rs:28-41, :74-83, :115-131; adaptor.rs:18-36) ----
_ENC_LAYER = {"q_w": "self_attn.q_proj.weight", "q_b": "self_attn.q_proj.bias", "k_w": "self_attn.k_proj.weight",
              "v_w": "self_attn.v_proj.weight", "v_b": "self_attn.v_proj.bias", "o_w": "self_attn.out_proj.weight",
              "o_b": "self_attn.out_proj.bias", "ln1_w": "self_attn_layer_norm.weight",
              "ln1_b": "self_attn_layer_norm.bias", "fc1_w": "fc1.weight", "fc1_b": "fc1.bias", "fc2_w": "fc2.weight",
              "fc2_b": "fc2.bias", "ln2_w": "final_layer_norm.weight", "ln2_b": "final_layer_norm.bias"}
_ENC_TOP = {"conv1_w": "conv1.weight", "conv1_b": "conv1.bias", "conv2_w": "conv2.weight", "conv2_b": "conv2.bias",
            "positions": "embed_positions.weight", "ln_w": "layer_norm.weight", "ln_b": "layer_norm.bias"}
_ADAPTOR = {"ad1_w": "layers.0.weight", "ad1_b": "layers.0.bias", "ad2_w": "layers.2.weight",
            "ad2_b": "layers.2.bias", "adn_w": "layers.3.weight", "adn_b": "layers.3.bias"}


def audio_tensors(w):
    out = {f"model.whisper_encoder.{n}": w[k] for k, n in _ENC_TOP.items()}
    for i, lw in enumerate(w["layers"]):
        out.update({f"model.whisper_encoder.layers.{i}.{n}": lw[k] for k, n in _ENC_LAYER.items()})
    out.update({f"model.vq_adaptor.{n}": w[k] for k, n in _ADAPTOR.items()})
    return out


def write_audio_checkpoint(d, acfg, w, bf16=True):
    """A Moss-style checkpoint directory holding the audio tower (matrices as
    bf16 bits when `bf16`) and a config.json with `audio_config`."""
    tensors = {k: (syn.f32_to_bf16_bits(np.asarray(v, np.float32)) if bf16 and np.ndim(v) >= 2
                   else np.asarray(v, np.float32)) for k, v in audio_tensors(w).items()}
    doc = {"audio_config": {k: getattr(acfg, k) for k in ("num_mel_bins", "d_model", "encoder_layers",
                                                           "encoder_attention_heads", "encoder_ffn_dim",
                                                           "max_source_positions")},
           "text_config": {"hidden_size": acfg.hidden_size, "rms_norm_eps": acfg.adaptor_norm_eps},
           "audio_merge_size": acfg.audio_merge_size, "adaptor_input_dim": acfg.adaptor_input_dim,
           "audio_token_id": 151654}
    (d / "config.json").write_text(json.dumps(doc))
    ckpt.write_safetensors(d / "model.safetensors", tensors)
    return tensors


def _small_audio():
    from conftest import PKG
    from oracle.whisper_ref import AudioConfig as RefConfig
    from oracle.whisper_ref import random_audio_weights

    acfg = PKG.AudioConfig(d_model=256, encoder_layers=2, encoder_attention_heads=4, encoder_ffn_dim=512,
                           max_source_positions=100, adaptor_input_dim=1024, hidden_size=256)
    return acfg, random_audio_weights(RefConfig(**acfg.oracle_kwargs()), 91)


def test_audio_checkpoint_round_trip(tmp_path):
    acfg, w = _small_audio()
    written = write_audio_checkpoint(tmp_path, acfg, w)
    cfg, got = ckpt.load_audio_checkpoint(tmp_path)
    assert cfg == acfg
    for k in _ENC_TOP:
        assert np.array_equal(np.asarray(got[k]), written[f"model.whisper_encoder.{_ENC_TOP[k]}"]), k
    for i in range(acfg.encoder_layers):
        for k, n in _ENC_LAYER.items():
            assert np.array_equal(np.asarray(got["layers"][i][k]),
                                  written[f"model.whisper_encoder.layers.{i}.{n}"]), (i, k)
    for k, n in _ADAPTOR.items():
        assert np.array_equal(np.asarray(got[k]), written[f"model.vq_adaptor.{n}"]), k


def test_audio_checkpoint_errors(tmp_path):
    acfg, w = _small_audio()
    written = write_audio_checkpoint(tmp_path, acfg, w)
    written.pop("model.whisper_encoder.layers.1.fc2.bias")
    ckpt.write_safetensors(tmp_path / "model.safetensors", written)
    with pytest.raises(KeyError, match="layers.1.fc2.bias"):
        ckpt.load_audio_checkpoint(tmp_path)
    written["model.whisper_encoder.layers.1.fc2.bias"] = np.zeros(7, np.float32)
    ckpt.write_safetensors(tmp_path / "model.safetensors", written)
    with pytest.raises(ValueError, match="shape"):
        ckpt.load_audio_checkpoint(tmp_path)
