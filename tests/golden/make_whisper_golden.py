"""Generate tests/golden/whisper_tiny.npz: the output of the independent
Whisper encoder in `transformers` (WhisperEncoder, f32, eval mode) on seeded
weights and log-mel input, used to pin oracle/whisper_ref.py.

The reference's encoder restates the same published architecture
(crates/fmd-core/src/model/whisper_encoder.rs); its checkpoint names are the
`transformers` state-dict names under `model.whisper_encoder.`.

Run from the repository root:  python tests/golden/make_whisper_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.whisper_ref import AudioConfig, random_audio_weights  # noqa: E402

CFG = AudioConfig(num_mel_bins=80, d_model=64, encoder_layers=2, encoder_attention_heads=4, encoder_ffn_dim=128,
                  max_source_positions=24, audio_merge_size=4, adaptor_input_dim=256, hidden_size=64)
WEIGHT_SEED = 11
MEL_SEED = 12


def hf_state_dict(w: dict) -> dict:
    sd = {"conv1.weight": w["conv1_w"], "conv1.bias": w["conv1_b"], "conv2.weight": w["conv2_w"],
          "conv2.bias": w["conv2_b"], "embed_positions.weight": w["positions"], "layer_norm.weight": w["ln_w"],
          "layer_norm.bias": w["ln_b"]}
    names = {"q_w": "self_attn.q_proj.weight", "q_b": "self_attn.q_proj.bias", "k_w": "self_attn.k_proj.weight",
             "v_w": "self_attn.v_proj.weight", "v_b": "self_attn.v_proj.bias", "o_w": "self_attn.out_proj.weight",
             "o_b": "self_attn.out_proj.bias", "ln1_w": "self_attn_layer_norm.weight",
             "ln1_b": "self_attn_layer_norm.bias", "fc1_w": "fc1.weight", "fc1_b": "fc1.bias",
             "fc2_w": "fc2.weight", "fc2_b": "fc2.bias", "ln2_w": "final_layer_norm.weight",
             "ln2_b": "final_layer_norm.bias"}
    for i, lw in enumerate(w["layers"]):
        for k, n in names.items():
            sd[f"layers.{i}.{n}"] = lw[k]
    return {k: torch.as_tensor(v) for k, v in sd.items()}


def main() -> None:
    from transformers import WhisperConfig
    from transformers.models.whisper.modeling_whisper import WhisperEncoder

    w = random_audio_weights(CFG, WEIGHT_SEED)
    mel = np.random.default_rng(MEL_SEED).standard_normal((2, CFG.num_mel_bins, 2 * CFG.max_source_positions),
                                                          dtype=np.float32)
    hcfg = WhisperConfig(num_mel_bins=CFG.num_mel_bins, d_model=CFG.d_model, encoder_layers=CFG.encoder_layers,
                         encoder_attention_heads=CFG.encoder_attention_heads, encoder_ffn_dim=CFG.encoder_ffn_dim,
                         max_source_positions=CFG.max_source_positions, decoder_layers=1,
                         decoder_attention_heads=CFG.encoder_attention_heads, decoder_ffn_dim=CFG.encoder_ffn_dim,
                         activation_function="gelu")
    enc = WhisperEncoder(hcfg).eval()
    enc.load_state_dict(hf_state_dict(w), strict=True)
    with torch.no_grad():
        out = enc(torch.as_tensor(mel)).last_hidden_state.numpy()
    np.savez_compressed(Path(__file__).with_name("whisper_tiny.npz"), mel=mel, out=out.astype(np.float32),
                        weight_seed=WEIGHT_SEED)
    print("wrote whisper_tiny.npz", out.shape, float(np.abs(out).max()))


if __name__ == "__main__":
    main()
