"""Checkpoint loading: safetensors shards under the reference's tensor names.

`load_checkpoint(directory)` returns the `TextConfig` and the host weight
dictionary that `Qwen3Decoder.load_weights` takes, read the way the
reference reads a Moss checkpoint:

* shard discovery as in `crates/fmd-core/src/hub.rs:166-214`: the shards named
  by `model.safetensors.index.json` (`weight_map`), else every `*.safetensors`
  file of the directory;
* the text backbone's shape from `config.json` (`text_config`,
  `crates/fmd-core/src/config.rs:8-58, 79-86`);
* tensor names of `Qwen3::load` / `Layer::load` / `Attention::load`
  (`crates/fmd-core/src/model/qwen3.rs:177-193, 268-318, 354-390`) under the
  `model.language_model` prefix, with the lm_head taken from
  `model.language_model.lm_head.weight`, else `lm_head.weight`, else tied to
  the embedding (`qwen3.rs:366-372`).

Tensors stay memory-mapped in their stored dtype (bf16 as uint16 bit
patterns, f16, f32); the library converts them and, in the int8 precisions,
quantises the projections from their f32 values (`linear.rs:104-107`).
`write_safetensors` writes the same format (used by the tests).

`load_audio_checkpoint(directory)` reads the audio tower the same way: the
Whisper encoder under `model.whisper_encoder` (whisper_encoder.rs:28-41,
:74-83, :115-131: `conv1`, `conv2`, `embed_positions`,
`layers.{i}.self_attn.{q,k,v,out}_proj` (k without bias),
`self_attn_layer_norm`, `fc1`, `fc2`, `final_layer_norm`, `layer_norm`) and the
adaptor under `model.vq_adaptor` (adaptor.rs:18-36: `layers.0`, `layers.2`, the
`layers.3` norm), with `AudioConfig` from config.json (`audio_config`,
`audio_merge_size`, `adaptor_input_dim`, the text width; config.rs:61-90).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from .config import TextConfig

PREFIX = "model.language_model"
_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16}
_NAMES = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.uint16): "BF16"}


def read_safetensors(path) -> dict:
    """name -> read-only array view of one safetensors file (bf16 as uint16 bits)."""
    path = Path(path)
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        if meta["dtype"] not in _DTYPES:
            raise ValueError(f"{path.name}: tensor {name} has unsupported dtype {meta['dtype']}")
        lo, hi = meta["data_offsets"]
        out[name] = data[lo:hi].view(_DTYPES[meta["dtype"]]).reshape(meta["shape"])
    return out


def write_safetensors(path, tensors: dict) -> None:
    """Write `tensors` (f32, f16, or uint16 bf16 bits) as one safetensors file."""
    header, off, blobs = {}, 0, []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        if arr.dtype not in _NAMES:
            raise ValueError(f"tensor {name}: dtype {arr.dtype} has no safetensors name here")
        b = arr.tobytes()
        header[name] = {"dtype": _NAMES[arr.dtype], "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    raw = json.dumps(header).encode()
    raw += b" " * (-len(raw) % 8)  # the data section starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)


def shard_files(directory) -> list[Path]:
    """Shards in index order (hub.rs:166-214)."""
    d = Path(directory)
    index = d / "model.safetensors.index.json"
    if index.exists():
        weight_map = json.loads(index.read_text())["weight_map"]
        names = []
        for shard in weight_map.values():
            if shard not in names:
                names.append(shard)
        return [d / n for n in names]
    files = sorted(d.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors weights found in {d}")
    return files


def text_config(directory) -> TextConfig:
    """`TextConfig` from config.json (its `text_config` section when present)."""
    doc = json.loads((Path(directory) / "config.json").read_text())
    tc = doc.get("text_config", doc)
    if tc.get("attention_bias", False):
        raise ValueError("attention_bias checkpoints are not supported by these kernels")
    fields = TextConfig.__dataclass_fields__
    return TextConfig(**{k: tc[k] for k in fields if k in tc})


def load_checkpoint(directory, prefix: str = PREFIX):
    """(TextConfig, weights) of the text backbone of a checkpoint directory."""
    cfg = text_config(directory)
    tensors: dict = {}
    for shard in shard_files(directory):
        tensors.update(read_safetensors(shard))

    def get(name, shape):
        key = f"{prefix}.{name}"
        if key not in tensors:
            raise KeyError(f"checkpoint has no tensor {key}")
        arr = tensors[key]
        if tuple(arr.shape) != tuple(shape):
            raise ValueError(f"{key}: shape {tuple(arr.shape)}, expected {tuple(shape)}")
        return arr

    h, i, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    qd, kvd = cfg.q_dim, cfg.kv_dim
    layers = []
    for li in range(cfg.num_hidden_layers):
        p = f"layers.{li}."
        layers.append({
            "input_norm": get(p + "input_layernorm.weight", (h,)),
            "post_norm": get(p + "post_attention_layernorm.weight", (h,)),
            "q_norm": get(p + "self_attn.q_norm.weight", (hd,)),
            "k_norm": get(p + "self_attn.k_norm.weight", (hd,)),
            "q": get(p + "self_attn.q_proj.weight", (qd, h)),
            "k": get(p + "self_attn.k_proj.weight", (kvd, h)),
            "v": get(p + "self_attn.v_proj.weight", (kvd, h)),
            "o": get(p + "self_attn.o_proj.weight", (h, qd)),
            "gate": get(p + "mlp.gate_proj.weight", (i, h)),
            "up": get(p + "mlp.up_proj.weight", (i, h)),
            "down": get(p + "mlp.down_proj.weight", (h, i)),
        })
    w = {"embed": get("embed_tokens.weight", (cfg.vocab_size, h)), "norm": get("norm.weight", (h,)),
         "layers": layers}
    for key in (f"{prefix}.lm_head.weight", "lm_head.weight"):  # qwen3.rs:366-372
        if key in tensors:
            w["lm_head"] = tensors[key]
            break
    return cfg, w


ENCODER_PREFIX = "model.whisper_encoder"
ADAPTOR_PREFIX = "model.vq_adaptor"


def audio_config(directory):
    """`AudioConfig` of the audio tower from config.json."""
    from .audio import AudioConfig

    return AudioConfig.from_model_config(json.loads((Path(directory) / "config.json").read_text()))


def load_audio_checkpoint(directory, encoder_prefix: str = ENCODER_PREFIX, adaptor_prefix: str = ADAPTOR_PREFIX):
    """(AudioConfig, weights) of the audio tower, the dictionary `AudioEncoder` takes."""
    cfg = audio_config(directory)
    tensors: dict = {}
    for shard in shard_files(directory):
        tensors.update(read_safetensors(shard))

    def get(prefix, name, shape):
        key = f"{prefix}.{name}"
        if key not in tensors:
            raise KeyError(f"checkpoint has no tensor {key}")
        arr = tensors[key]
        if tuple(arr.shape) != tuple(shape):
            raise ValueError(f"{key}: shape {tuple(arr.shape)}, expected {tuple(shape)}")
        return arr

    D, FF, M = cfg.d_model, cfg.encoder_ffn_dim, cfg.num_mel_bins
    e = lambda name, shape: get(encoder_prefix, name, shape)  # noqa: E731
    w = {"conv1_w": e("conv1.weight", (D, M, 3)), "conv1_b": e("conv1.bias", (D,)),
         "conv2_w": e("conv2.weight", (D, D, 3)), "conv2_b": e("conv2.bias", (D,)),
         "positions": e("embed_positions.weight", (cfg.max_source_positions, D)),
         "ln_w": e("layer_norm.weight", (D,)), "ln_b": e("layer_norm.bias", (D,)), "layers": []}
    for i in range(cfg.encoder_layers):
        p = f"layers.{i}."
        w["layers"].append({
            "q_w": e(p + "self_attn.q_proj.weight", (D, D)), "q_b": e(p + "self_attn.q_proj.bias", (D,)),
            "k_w": e(p + "self_attn.k_proj.weight", (D, D)),
            "v_w": e(p + "self_attn.v_proj.weight", (D, D)), "v_b": e(p + "self_attn.v_proj.bias", (D,)),
            "o_w": e(p + "self_attn.out_proj.weight", (D, D)), "o_b": e(p + "self_attn.out_proj.bias", (D,)),
            "ln1_w": e(p + "self_attn_layer_norm.weight", (D,)), "ln1_b": e(p + "self_attn_layer_norm.bias", (D,)),
            "fc1_w": e(p + "fc1.weight", (FF, D)), "fc1_b": e(p + "fc1.bias", (FF,)),
            "fc2_w": e(p + "fc2.weight", (D, FF)), "fc2_b": e(p + "fc2.bias", (D,)),
            "ln2_w": e(p + "final_layer_norm.weight", (D,)), "ln2_b": e(p + "final_layer_norm.bias", (D,)),
        })
    hid, K = cfg.hidden_size, cfg.adaptor_input_dim
    a = lambda name, shape: get(adaptor_prefix, name, shape)  # noqa: E731
    w.update({"ad1_w": a("layers.0.weight", (hid, K)), "ad1_b": a("layers.0.bias", (hid,)),
              "ad2_w": a("layers.2.weight", (hid, hid)), "ad2_b": a("layers.2.bias", (hid,)),
              "adn_w": a("layers.3.weight", (hid,)), "adn_b": a("layers.3.bias", (hid,))})
    return cfg, w
