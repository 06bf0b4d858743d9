"""ctypes binding of `include/fmd_decoder.h` (libfmd_decoder.so).

The library is built in-tree (`csrc/build.py`) and loaded from the package
directory; there is no CPU fallback -- if the library or a GPU is missing,
calls fail loudly.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libfmd_decoder.so"

# status codes
FMD_OK = 0
FMD_EINVAL = -22
FMD_ENOMEM = -12
FMD_EIO = -5
FMD_EBUSY = -16
FMD_EOVERFLOW = -75
FMD_ENOTSUP = -95
FMD_ETIMEDOUT = -110

# precisions (precision.rs:11-17)
PREC_F32, PREC_F16, PREC_BF16, PREC_INT8, PREC_INT8_BF16 = 0, 1, 2, 3, 4
PRECISIONS = {"f32": PREC_F32, "fp32": PREC_F32, "f16": PREC_F16, "fp16": PREC_F16, "bf16": PREC_BF16,
              "int8": PREC_INT8, "q8_0": PREC_INT8, "int8_bf16": PREC_INT8_BF16}

# host dtypes
DT_F32, DT_F16, DT_BF16, DT_Q8_0 = 0, 1, 2, 3

FINISH_STOP, FINISH_LENGTH, FINISH_ERROR = 0, 1, 2

# every symbol the header declares
EXPORTS = [
    "fmd_create", "fmd_destroy", "fmd_last_error", "fmd_status_string", "fmd_version", "fmd_load_weights",
    "fmd_kv_reserve", "fmd_cache_bytes", "fmd_memory_bytes", "fmd_embed", "fmd_splice_audio", "fmd_slot_open", "fmd_slot_release",
    "fmd_slot_len", "fmd_prefill", "fmd_decode_step", "fmd_engine_load", "fmd_engine_start", "fmd_engine_step",
    "fmd_engine_run", "fmd_engine_fetch",
    "fmd_generate", "fmd_debug_weight", "fmd_debug_kv", "fmd_q8_0_quantize", "fmd_q8_0_quantize_device", "fmd_greedy_pick_noalloc",
    "fmd_debug_wait_timeout", "fmd_debug_paths", "fmd_debug_mma_issue",
    # include/fmd_audio.h
    "fmd_audio_create", "fmd_audio_destroy", "fmd_audio_last_error", "fmd_audio_memory_bytes", "fmd_audio_encode",
    "fmd_audio_encode_audio", "fmd_audio_token_offsets", "fmd_audio_last_timing", "fmd_mel_create", "fmd_mel_destroy", "fmd_mel_last_error",
    "fmd_mel_log_mel", "fmd_mel_filters",
]


class FmdError(RuntimeError):
    """A non-zero status from the library (`crate::error::Error` analogue)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class Config(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32),
        ("num_hidden_layers", C.c_int32), ("num_attention_heads", C.c_int32),
        ("num_key_value_heads", C.c_int32), ("head_dim", C.c_int32), ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_double), ("max_position_embeddings", C.c_int32), ("eos_token_id", C.c_int32),
    ]


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32)]


class LayerWeights(C.Structure):
    _fields_ = [(n, Tensor) for n in (
        "input_layernorm", "post_attention_layernorm", "q_norm", "k_norm", "q_proj", "k_proj", "v_proj",
        "o_proj", "gate_proj", "up_proj", "down_proj")]


class Weights(C.Structure):
    _fields_ = [("embed_tokens", Tensor), ("norm", Tensor), ("lm_head", Tensor),
                ("layers", C.POINTER(LayerWeights))]


class Request(C.Structure):
    _fields_ = [("prompt_len", C.c_int32), ("max_new_tokens", C.c_int32), ("forced_stop", C.c_int32),
                ("reserved", C.c_int32), ("embed_row", C.c_int64)]


class Result(C.Structure):
    _fields_ = [("n_tokens", C.c_int32), ("finish_reason", C.c_int32)]


class Stats(C.Structure):
    _fields_ = [("steps", C.c_int64), ("generated_tokens", C.c_int64), ("prefill_tokens", C.c_int64),
                ("requests_done", C.c_int64), ("generate_seconds", C.c_double), ("device_status", C.c_int32),
                ("reserved", C.c_int32), ("window_steps", C.c_int64), ("window_tokens", C.c_int64),
                ("window_device_ms", C.c_double), ("attn_decode_ms", C.c_double), ("attn_kv_tokens", C.c_int64),
                ("attn_rows", C.c_int64), ("window_mixed_steps", C.c_int64), ("graph_kernels_mixed", C.c_int64),
                ("graph_kernels_decode", C.c_int64), ("lm_head_ms", C.c_double)]


class AudioConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "num_mel_bins", "d_model", "encoder_layers", "encoder_attention_heads", "encoder_ffn_dim",
        "max_source_positions", "audio_merge_size", "adaptor_input_dim", "hidden_size")] + [
        ("adaptor_norm_eps", C.c_float)]


class EncoderLayerWeights(C.Structure):
    _fields_ = [(n, Tensor) for n in (
        "q_proj_w", "q_proj_b", "k_proj_w", "v_proj_w", "v_proj_b", "out_proj_w", "out_proj_b",
        "self_attn_layer_norm_w", "self_attn_layer_norm_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b",
        "final_layer_norm_w", "final_layer_norm_b")]


class AudioWeights(C.Structure):
    _fields_ = [("conv1_w", Tensor), ("conv1_b", Tensor), ("conv2_w", Tensor), ("conv2_b", Tensor),
                ("embed_positions", Tensor), ("layers", C.POINTER(EncoderLayerWeights)),
                ("layer_norm_w", Tensor), ("layer_norm_b", Tensor), ("adaptor_fc1_w", Tensor),
                ("adaptor_fc1_b", Tensor), ("adaptor_fc2_w", Tensor), ("adaptor_fc2_b", Tensor),
                ("adaptor_norm_w", Tensor), ("adaptor_norm_b", Tensor)]


class FeatureConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "feature_size", "sampling_rate", "hop_length", "n_fft", "n_samples", "nb_max_frames")]


_lib = None


def load() -> C.CDLL:
    """Load libfmd_decoder.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FmdError(FMD_EIO, f"{LIB_PATH} is missing: build it with csrc/build.py")
    lib = C.CDLL(str(LIB_PATH))
    P, I32, I64 = C.c_void_p, C.c_int32, C.c_int64
    IP = C.POINTER(C.c_int32)
    sig = {
        "fmd_create": (C.c_int, [C.POINTER(Config), I32, I32, C.POINTER(P)]),
        "fmd_destroy": (C.c_int, [P]),
        "fmd_last_error": (C.c_char_p, [P]),
        "fmd_status_string": (C.c_char_p, [I32]),
        "fmd_version": (C.c_int, []),
        "fmd_load_weights": (C.c_int, [P, C.POINTER(Weights)]),
        "fmd_kv_reserve": (C.c_int, [P, I32, I64, I32]),
        "fmd_cache_bytes": (I64, [C.POINTER(Config), I32, I64, I64]),
        "fmd_memory_bytes": (C.c_int, [P, C.POINTER(I64), C.POINTER(I64), C.POINTER(I64)]),
        "fmd_embed": (C.c_int, [P, IP, I64, P]),
        "fmd_splice_audio": (C.c_int, [P, IP, I64, P, I64, I32, I32, P]),
        "fmd_slot_open": (C.c_int, [P, I32, I32]),
        "fmd_slot_release": (C.c_int, [P, I32]),
        "fmd_slot_len": (C.c_int, [P, I32, IP]),
        "fmd_prefill": (C.c_int, [P, I32, IP, IP, P, I32, C.POINTER(C.c_float), IP]),
        "fmd_decode_step": (C.c_int, [P, I32, IP, IP, C.POINTER(C.c_float), IP]),
        "fmd_engine_load": (C.c_int, [P, C.POINTER(Request), I32, P, I64, I32]),
        "fmd_engine_start": (C.c_int, [P, I32, I32]),
        "fmd_engine_step": (C.c_int, [P, I64, C.POINTER(Stats)]),
        "fmd_engine_run": (C.c_int, [P, I32, I32, I64, C.POINTER(Stats)]),
        "fmd_engine_fetch": (C.c_int, [P, IP, I32, C.POINTER(Result)]),
        "fmd_generate": (C.c_int, [P, C.POINTER(Request), I32, P, I64, I32, I32, I32, IP, I32,
                                   C.POINTER(Result), C.POINTER(Stats)]),
        "fmd_debug_weight": (C.c_int, [P, I32, I32, C.POINTER(C.c_float), I64]),
        "fmd_debug_kv": (C.c_int, [P, I32, I32, I32, I32, P, P]),
        "fmd_q8_0_quantize": (C.c_int, [C.POINTER(C.c_float), I64, I64, P]),
        "fmd_q8_0_quantize_device": (C.c_int, [P, I32, I64, I64, P, P, P]),
        "fmd_greedy_pick_noalloc": (C.c_int, [P, I32, I32, P, P]),
        "fmd_debug_wait_timeout": (C.c_int, [P, I32]),
        "fmd_debug_paths": (C.c_int, [P, C.POINTER(I32)]),
        "fmd_debug_mma_issue": (C.c_int, [P, I32, I32, I32, C.POINTER(C.c_double)]),
        "fmd_audio_create": (C.c_int, [C.POINTER(AudioConfig), C.POINTER(AudioWeights), I32, I32, I32,
                                       C.POINTER(P)]),
        "fmd_audio_destroy": (C.c_int, [P]),
        "fmd_audio_last_error": (C.c_char_p, [P]),
        "fmd_audio_memory_bytes": (C.c_int, [P, C.POINTER(I64), C.POINTER(I64)]),
        "fmd_audio_encode": (C.c_int, [P, P, I32, I32, P]),
        "fmd_audio_encode_audio": (C.c_int, [P, P, I32, I32, IP, IP, I32, I32, P, C.POINTER(I64)]),
        "fmd_audio_token_offsets": (C.c_int, [C.POINTER(AudioConfig), I32, IP, IP, I32, C.POINTER(I64)]),
        "fmd_audio_last_timing": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(I64)]),
        "fmd_mel_create": (C.c_int, [C.POINTER(FeatureConfig), I32, C.POINTER(P)]),
        "fmd_mel_destroy": (C.c_int, [P]),
        "fmd_mel_last_error": (C.c_char_p, [P]),
        "fmd_mel_log_mel": (C.c_int, [P, P, I32, P]),
        "fmd_mel_filters": (C.c_int, [C.POINTER(FeatureConfig), C.POINTER(C.c_float)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, handle=None) -> None:
    if status != FMD_OK:
        lib = load()
        msg = lib.fmd_last_error(handle).decode() if handle else ""
        if not msg:
            msg = lib.fmd_status_string(status).decode()
        raise FmdError(status, msg)
