"""B200-native batched Qwen3 decoder step of fast-moss-diarization.

The hot path of cnmoro/fast-moss-diarization -- the Qwen3 decoder step driven
by `Engine::generate_batch` -- rebuilt as sm_100a kernels behind a C ABI
(`include/fmd_decoder.h`, `libfmd_decoder.so`). This package is the Python
host side: `Qwen3Decoder` (the decoder-forward operator surface of
`qwen3.rs`), `Engine` (continuous batching with on-GPU slot refill),
`AudioEncoder` (the Whisper encoder + VQ adaptor that produce the audio
embeddings) and `MelFrontend` (the log-mel frontend), include/fmd_audio.h; seeded
synthetic workloads, and the request-sharded multi-GPU launcher.
"""

from . import _lib
from ._lib import FmdError
from .audio import AudioConfig, AudioEncoder, AudioFeatures, FeatureConfig, MelFrontend, extract_features
from .config import EOS_TOKEN_ID, TextConfig, parse_precision
from .decoder import Qwen3Decoder
from .engine import BatchStats, Engine, Generated

__all__ = ["AudioConfig", "AudioEncoder", "AudioFeatures", "FeatureConfig", "MelFrontend", "extract_features", "FmdError", "EOS_TOKEN_ID", "TextConfig", "parse_precision", "Qwen3Decoder", "Engine", "BatchStats",
           "Generated", "library_path", "load_library"]


def library_path():
    return _lib.LIB_PATH


def load_library():
    """Load the CUDA library; raises FmdError when it is missing (no fallback)."""
    return _lib.load()
