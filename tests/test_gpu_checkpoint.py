"""Real-checkpoint loading on the GPU: GGML Q8_0 quantisation on the device
(`fmd_q8_0_quantize_device`) bit for bit against the oracle, and a decoder
loaded from a safetensors checkpoint (reference tensor names) equal to one
loaded from the same values in memory."""

from __future__ import annotations

import ctypes as C
import importlib

import numpy as np
import pytest

from conftest import PKG, tiny_config
from test_checkpoint import write_checkpoint

ckpt = importlib.import_module("fmd_b200.checkpoint")
syn = importlib.import_module("fmd_b200.synthetic")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("src", ["f32", "bf16", "f16"])
def test_device_q8_0_quantiser_is_bit_exact(src):
    import torch

    from oracle import q8_0

    rng = np.random.default_rng(4)
    rows, cols = 257, 1024
    x = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x[0] = 0.0                                    # d == 0: all-zero block
    x[1, :32] = np.arange(32) - 16.0              # exact integers, |q| up to 127
    x[2, :32] = (np.arange(32) + 0.5) / 32 * 3.0  # values landing on .5 steps of x / d
    x[3, 5] = 60000.0                             # one large value dominating its block
    if src == "f32":
        dev, dt, vals = torch.from_numpy(x).cuda(), PKG._lib.DT_F32, x
    elif src == "bf16":
        bits = syn.f32_to_bf16_bits(x)
        dev, dt, vals = torch.from_numpy(bits.view(np.int16)).cuda(), PKG._lib.DT_BF16, syn.bf16_bits_to_f32(bits)
    else:
        h = x.astype(np.float16)
        dev, dt, vals = torch.from_numpy(h).cuda(), PKG._lib.DT_F16, h.astype(np.float32)
    qs = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    d = torch.empty((rows, cols // 32), dtype=torch.int16, device="cuda")
    lib = PKG.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        assert lib.fmd_q8_0_quantize_device(C.c_void_p(dev.data_ptr()), dt, rows, cols, C.c_void_p(qs.data_ptr()),
                                            C.c_void_p(d.data_ptr()), C.c_void_p(stream)) == 0
        torch.cuda.synchronize()
        want_q, want_d = q8_0.quantize(vals)
        assert np.array_equal(qs.cpu().numpy(), want_q)
        assert np.array_equal(d.cpu().numpy().view(np.uint16), want_d.view(np.uint16))
    # shapes the format cannot take, and host pointers, are refused before any launch
    assert lib.fmd_q8_0_quantize_device(C.c_void_p(dev.data_ptr()), dt, rows, 48, C.c_void_p(qs.data_ptr()),
                                        C.c_void_p(d.data_ptr()), C.c_void_p(stream)) == PKG._lib.FMD_EINVAL
    host = np.empty(rows * cols, dtype=np.int8)
    assert lib.fmd_q8_0_quantize_device(C.c_void_p(dev.data_ptr()), dt, rows, cols, C.c_void_p(host.ctypes.data),
                                        C.c_void_p(d.data_ptr()), C.c_void_p(stream)) == PKG._lib.FMD_EINVAL


@pytest.mark.parametrize("prec", ["bf16", "int8"])
def test_decoder_from_checkpoint_equals_in_memory(tmp_path, prec):
    cfg = tiny_config(max_position_embeddings=4096)
    w = syn.make_weights(cfg, seed=6, norm_jitter=0.2)
    write_checkpoint(tmp_path, cfg, w, shards=2)
    got_cfg, loaded = ckpt.load_checkpoint(tmp_path)
    # the same values as f32 arrays in memory (bf16 -> f32 is exact)
    def f32(a):
        a = np.asarray(a)
        return syn.bf16_bits_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)
    mem = {"embed": f32(loaded["embed"]), "norm": f32(loaded["norm"]),
           "layers": [{k: f32(v) for k, v in lw.items()} for lw in loaded["layers"]]}
    rng = np.random.default_rng(3)
    prompt = rng.standard_normal((90, cfg.hidden_size), dtype=np.float32)
    toks = rng.integers(0, cfg.vocab_size, 3)
    outs = []
    for weights in (loaded, mem):
        with PKG.Qwen3Decoder(got_cfg, prec) as dec:
            dec.load_weights(weights)
            dec.reserve(max_slots=1, max_tokens=256, max_rows=128)
            dec.open_slot(0, 100)
            lg, _ = dec.prefill([0], [prompt])
            res = [lg]
            for t in toks:
                lg, _ = dec.decode_step([0], [int(t)])
                res.append(lg)
            outs.append(res)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


def test_audio_encoder_from_checkpoint_equals_in_memory(tmp_path):
    """The audio tower loaded from a checkpoint (bf16 matrices, f32 vectors,
    the reference's tensor names) gives the same frames and embeddings, bit for
    bit, as the same values handed over in memory."""
    import torch

    from oracle.whisper_ref import round_weights
    from test_checkpoint import _small_audio, write_audio_checkpoint

    acfg, w = _small_audio()
    write_audio_checkpoint(tmp_path, acfg, w)
    cfg, wc = ckpt.load_audio_checkpoint(tmp_path)
    wr = round_weights(w, "bf16")
    for k in ("conv1_b", "conv2_b", "ln_w", "ln_b", "ad1_b", "ad2_b", "adn_w", "adn_b"):
        wr[k] = np.asarray(w[k], np.float32)  # vectors stay f32 in the checkpoint
    for lw, src in zip(wr["layers"], w["layers"]):
        for k in ("q_b", "v_b", "o_b", "ln1_w", "ln1_b", "fc1_b", "fc2_b", "ln2_w", "ln2_b"):
            lw[k] = np.asarray(src[k], np.float32)
    mel = np.random.default_rng(92).standard_normal((2, 80, cfg.mel_frames), dtype=np.float32)
    with PKG.AudioEncoder(cfg, wc, "bf16", max_batch=2) as a, PKG.AudioEncoder(cfg, wr, "bf16", max_batch=2) as b:
        fa, fb = a.forward_device(mel), b.forward_device(mel)
        assert torch.equal(fa, fb)
        ea, _ = a.encode_audio_device(mel, [25, 9], [0, 1], 2)
        eb, _ = b.encode_audio_device(mel, [25, 9], [0, 1], 2)
        assert torch.equal(ea, eb)
