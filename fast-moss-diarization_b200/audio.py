"""Host side of the audio tower (include/fmd_audio.h): the log-mel frontend,
the Whisper encoder and the VQ adaptor on the GPU.

`MelFrontend` mirrors `MelFrontend::log_mel` (crates/fmd-core/src/audio/mel.rs:84-133)
and `extract_features` the chunk planning of `extract_features`
(crates/fmd-core/src/audio/mod.rs:47-116), with the mel computed on the GPU.

`AudioEncoder` mirrors the reference's `WhisperEncoder::forward`
(crates/fmd-core/src/model/whisper_encoder.rs:142-163) as `forward`, and
`MossModel::encode_audio` (crates/fmd-core/src/model/mod.rs:82-126) as
`encode_audio`: same argument meaning (mel chunks, per-chunk audio token
counts, chunk -> audio mapping, encoder batch) and the same failure for an
audio without chunks. Weights are a dict of host arrays keyed as
`oracle.whisper_ref.random_audio_weights` / `checkpoint.load_audio_checkpoint`
produce them (f32, f16, or bf16 bit patterns as uint16). Outputs live on the
device (torch tensors; torch is only the allocator here) or are copied back as
f32 arrays.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import asdict, dataclass

import numpy as np

from . import _lib
from .config import parse_precision
from .decoder import _host

_LAYER_KEYS = {
    "q_proj_w": "q_w", "q_proj_b": "q_b", "k_proj_w": "k_w", "v_proj_w": "v_w", "v_proj_b": "v_b",
    "out_proj_w": "o_w", "out_proj_b": "o_b", "self_attn_layer_norm_w": "ln1_w",
    "self_attn_layer_norm_b": "ln1_b", "fc1_w": "fc1_w", "fc1_b": "fc1_b", "fc2_w": "fc2_w", "fc2_b": "fc2_b",
    "final_layer_norm_w": "ln2_w", "final_layer_norm_b": "ln2_b",
}
_TOP_KEYS = {
    "conv1_w": "conv1_w", "conv1_b": "conv1_b", "conv2_w": "conv2_w", "conv2_b": "conv2_b",
    "embed_positions": "positions", "layer_norm_w": "ln_w", "layer_norm_b": "ln_b",
    "adaptor_fc1_w": "ad1_w", "adaptor_fc1_b": "ad1_b", "adaptor_fc2_w": "ad2_w", "adaptor_fc2_b": "ad2_b",
    "adaptor_norm_w": "adn_w", "adaptor_norm_b": "adn_b",
}


@dataclass
class AudioConfig:
    """`AudioConfig` (config.rs:61-75) plus the adaptor fields of `ModelConfig`
    (config.rs:78-90); defaults are the Moss checkpoint's Whisper-Medium tower."""
    num_mel_bins: int = 80
    d_model: int = 1024
    encoder_layers: int = 24
    encoder_attention_heads: int = 16
    encoder_ffn_dim: int = 4096
    max_source_positions: int = 1500
    audio_merge_size: int = 4
    adaptor_input_dim: int = 4096
    hidden_size: int = 1024
    adaptor_norm_eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.d_model // self.encoder_attention_heads

    @property
    def mel_frames(self) -> int:
        return 2 * self.max_source_positions

    @property
    def tokens_per_chunk(self) -> int:
        return self.max_source_positions // self.audio_merge_size

    def to_c(self) -> _lib.AudioConfig:
        return _lib.AudioConfig(**asdict(self))

    def oracle_kwargs(self) -> dict:
        return asdict(self)

    @classmethod
    def from_model_config(cls, doc: dict) -> "AudioConfig":
        """From a Moss `config.json` (`ModelConfig`, config.rs:78-90)."""
        a = doc["audio_config"]
        t = doc["text_config"]
        fields = cls.__dataclass_fields__
        kw = {k: a[k] for k in fields if k in a}
        kw.update(audio_merge_size=doc["audio_merge_size"], adaptor_input_dim=doc["adaptor_input_dim"],
                  hidden_size=t["hidden_size"], adaptor_norm_eps=t.get("rms_norm_eps", 1e-6))
        return cls(**kw)


def _mel_host(mel) -> tuple:
    a = np.asarray(mel)
    if a.dtype == np.uint16:
        return np.ascontiguousarray(a), _lib.DT_BF16
    if a.dtype == np.float16:
        return np.ascontiguousarray(a), _lib.DT_F16
    return np.ascontiguousarray(a, dtype=np.float32), _lib.DT_F32


class AudioEncoder:
    def __init__(self, cfg: AudioConfig, weights: dict, precision: str = "bf16", device: int = 0,
                 max_batch: int = 16):
        self.lib = _lib.load()
        self.cfg = cfg
        self.device = device
        self.precision = parse_precision(precision)
        self.act = "bf16" if self.precision in (_lib.PREC_BF16, _lib.PREC_INT8_BF16) else "f16"
        self.max_batch = max_batch
        keep = []

        def t(a):
            arr, dt = _host(a)
            keep.append(arr)
            return _lib.Tensor(arr.ctypes.data, dt)

        layers = (_lib.EncoderLayerWeights * max(1, cfg.encoder_layers))()
        for i, lw in enumerate(weights["layers"][: cfg.encoder_layers]):
            for field, key in _LAYER_KEYS.items():
                setattr(layers[i], field, t(lw[key]))
        w = _lib.AudioWeights()
        for field, key in _TOP_KEYS.items():
            setattr(w, field, t(weights[key]))
        w.layers = layers
        self._h = C.c_void_p()
        st = self.lib.fmd_audio_create(C.byref(cfg.to_c()), C.byref(w), self.precision, device, max_batch,
                                       C.byref(self._h))
        if st != _lib.FMD_OK:
            msg = self.lib.fmd_audio_last_error(self._h).decode() if self._h else ""
            self.close()
            raise _lib.FmdError(st, f"fmd_audio_create: {msg or self.lib.fmd_status_string(st).decode()}")

    # -- lifecycle ---------------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.fmd_audio_destroy(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int) -> None:
        if st != _lib.FMD_OK:
            msg = self.lib.fmd_audio_last_error(self._h).decode()
            raise _lib.FmdError(st, msg or self.lib.fmd_status_string(st).decode())

    def _torch_dtype(self):
        import torch

        return torch.bfloat16 if self.act == "bf16" else torch.float16

    # -- WhisperEncoder::forward ---------------------------------------------------------
    def forward_ptr(self, mel_ptr: int, mel_dtype: int, n_chunks: int, out_ptr: int) -> None:
        """Raw entry: `mel_ptr` host or device (n, n_mels, 2 frames), `out_ptr` device."""
        self._check(self.lib.fmd_audio_encode(self._h, C.c_void_p(mel_ptr), mel_dtype, n_chunks,
                                              C.c_void_p(out_ptr)))

    def forward_device(self, mel):
        """(n, n_mels, 2 x frames) mel (host array) -> device tensor (n, frames, d_model)."""
        import torch

        arr, dt = _mel_host(mel)
        n = arr.shape[0]
        out = torch.empty((n, self.cfg.max_source_positions, self.cfg.d_model), dtype=self._torch_dtype(),
                          device=f"cuda:{self.device}")
        self.forward_ptr(arr.ctypes.data, dt, n, out.data_ptr())
        return out

    def forward(self, mel) -> np.ndarray:
        return self.forward_device(mel).float().cpu().numpy()

    # -- MossModel::encode_audio ------------------------------------------------------
    def _ids(self, chunk_token_lengths, chunk_mapping):
        tl = np.ascontiguousarray(np.asarray(chunk_token_lengths, dtype=np.int32).reshape(-1))
        cm = np.ascontiguousarray(np.asarray(chunk_mapping, dtype=np.int32).reshape(-1))
        if tl.size != cm.size:
            raise ValueError("chunk_token_lengths and chunk_mapping differ in length")
        return tl, cm

    def audio_offsets(self, n_chunks: int, chunk_token_lengths, chunk_mapping, num_audios: int) -> np.ndarray:
        """First output row of every audio (num_audios + 1 entries)."""
        tl, cm = self._ids(chunk_token_lengths, chunk_mapping)
        off = np.zeros(num_audios + 1, dtype=np.int64)
        IP = C.POINTER(C.c_int32)
        self._check(self.lib.fmd_audio_encode_audio(self._h, None, _lib.DT_F32, n_chunks, tl.ctypes.data_as(IP),
                                                    cm.ctypes.data_as(IP), num_audios, 1, None,
                                                    off.ctypes.data_as(C.POINTER(C.c_int64))))
        return off

    def encode_audio_device(self, mel, chunk_token_lengths, chunk_mapping, num_audios: int,
                            encoder_batch: int = 16, out=None):
        """Device tensor (total tokens, hidden) of every audio's embeddings, and
        the per-audio row offsets. `mel` is a host array or a device tensor."""
        import torch

        tl, cm = self._ids(chunk_token_lengths, chunk_mapping)
        if isinstance(mel, torch.Tensor):
            dt = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16}[mel.dtype]
            n, ptr, hold = mel.shape[0], mel.data_ptr(), mel
        else:
            hold, dt = _mel_host(mel)
            n, ptr = hold.shape[0], hold.ctypes.data
        off = self.audio_offsets(n, tl, cm, num_audios)
        if out is None:
            out = torch.empty((int(off[-1]), self.cfg.hidden_size), dtype=self._torch_dtype(),
                              device=f"cuda:{self.device}")
        IP = C.POINTER(C.c_int32)
        self._check(self.lib.fmd_audio_encode_audio(self._h, C.c_void_p(ptr), dt, n, tl.ctypes.data_as(IP),
                                                    cm.ctypes.data_as(IP), num_audios, encoder_batch,
                                                    C.c_void_p(out.data_ptr()),
                                                    off.ctypes.data_as(C.POINTER(C.c_int64))))
        del hold
        return out, off

    def encode_audio(self, mel, chunk_token_lengths, chunk_mapping, num_audios: int,
                     encoder_batch: int = 16) -> list[np.ndarray]:
        """One (tokens, hidden) f32 array per audio, as `MossModel::encode_audio` returns."""
        out, off = self.encode_audio_device(mel, chunk_token_lengths, chunk_mapping, num_audios, encoder_batch)
        host = out.float().cpu().numpy()
        return [host[off[a]:off[a + 1]] for a in range(num_audios)]

    # -- accounting ----------------------------------------------------------------------
    def last_timing(self) -> tuple[float, int]:
        ms, k = C.c_double(), C.c_int64()
        self._check(self.lib.fmd_audio_last_timing(self._h, C.byref(ms), C.byref(k)))
        return ms.value, k.value

    def memory_bytes(self) -> tuple[int, int]:
        w, s = C.c_int64(), C.c_int64()
        self._check(self.lib.fmd_audio_memory_bytes(self._h, C.byref(w), C.byref(s)))
        return w.value, s.value


def token_offsets(cfg: AudioConfig, chunk_token_lengths, chunk_mapping, num_audios: int) -> np.ndarray:
    """First output row of every audio in `encode_audio`'s output
    (`fmd_audio_token_offsets`, host only; num_audios + 1 entries)."""
    lib = _lib.load()
    tl = np.ascontiguousarray(np.asarray(chunk_token_lengths, dtype=np.int32).reshape(-1))
    cm = np.ascontiguousarray(np.asarray(chunk_mapping, dtype=np.int32).reshape(-1))
    if tl.size != cm.size:
        raise ValueError("chunk_token_lengths and chunk_mapping differ in length")
    off = np.zeros(num_audios + 1, dtype=np.int64)
    IP = C.POINTER(C.c_int32)
    st = lib.fmd_audio_token_offsets(C.byref(cfg.to_c()), tl.size, tl.ctypes.data_as(IP), cm.ctypes.data_as(IP),
                                     num_audios, off.ctypes.data_as(C.POINTER(C.c_int64)))
    if st != _lib.FMD_OK:
        raise _lib.FmdError(st, "fmd_audio_token_offsets: bad chunk layout (an audio without chunks, a mapping "
                                "out of range or a negative token count)")
    return off


def encoder_flops(cfg: AudioConfig, n_chunks: int) -> float:
    """Multiply-add FLOPs (x2) of one encoder pass + adaptor over n chunks."""
    D, FF, Tp, F = cfg.d_model, cfg.encoder_ffn_dim, cfg.max_source_positions, cfg.mel_frames
    conv = 2 * F * D * 3 * cfg.num_mel_bins + 2 * Tp * D * 3 * D
    layer = 2 * Tp * (3 * D * D + D * D + 2 * D * FF) + 4 * Tp * Tp * D
    groups = Tp // cfg.audio_merge_size
    adaptor = 2 * groups * cfg.hidden_size * (cfg.adaptor_input_dim + cfg.hidden_size)
    return float(n_chunks) * (conv + cfg.encoder_layers * layer + adaptor)


# ---- log-mel frontend (include/fmd_audio.h: fmd_mel_*) -------------------------------
WHISPER_ENCODER_STRIDE = 2  # config.rs:210


@dataclass
class FeatureConfig:
    """`FeatureConfig` (config.rs:121-166): the Whisper log-mel frontend."""
    feature_size: int = 80
    sampling_rate: int = 16_000
    hop_length: int = 160
    n_fft: int = 400
    n_samples: int = 480_000
    nb_max_frames: int = 3_000

    def to_c(self) -> _lib.FeatureConfig:
        return _lib.FeatureConfig(**asdict(self))


def audio_token_length(num_samples: int, hop_length: int, merge_size: int) -> int:
    """Audio tokens of a chunk of `num_samples` samples (config.rs:212-223)."""
    if num_samples == 0:
        return 0
    return (num_samples - 1) // (hop_length * WHISPER_ENCODER_STRIDE * merge_size) + 1


def plan_chunks(lengths, cfg: FeatureConfig, merge_size: int):
    """Chunk layout of `extract_features` (audio/mod.rs:57-82): 30 s windows per
    waveform (an empty waveform still yields one empty window). Returns
    ([(audio, start, end)], chunk_token_lengths, chunk_mapping, tokens_per_audio)."""
    chunks, tokens, mapping, per_audio = [], [], [], [0] * len(lengths)
    for a, n in enumerate(lengths):
        start, total = 0, max(int(n), 1)
        while start < total:
            end = min(start + cfg.n_samples, int(n))
            t = audio_token_length(end - start, cfg.hop_length, merge_size)
            per_audio[a] += t
            chunks.append((a, start, end))
            tokens.append(t)
            mapping.append(a)
            start += cfg.n_samples
    return chunks, tokens, mapping, per_audio


@dataclass
class AudioFeatures:
    """`AudioFeatures` (audio/mod.rs:17-39) with the mel on the device."""
    mel: object                 # torch tensor (n_chunks, n_mels, frames), f32, on the device
    chunk_token_lengths: list
    chunk_mapping: list
    tokens_per_audio: list

    @property
    def n_chunks(self) -> int:
        return len(self.chunk_token_lengths)


class MelFrontend:
    """`MelFrontend` (mel.rs:29-133) on the GPU."""

    def __init__(self, cfg: FeatureConfig = FeatureConfig(), device: int = 0):
        self.lib = _lib.load()
        self.cfg = cfg
        self.device = device
        self._h = C.c_void_p()
        st = self.lib.fmd_mel_create(C.byref(cfg.to_c()), device, C.byref(self._h))
        if st != _lib.FMD_OK:
            msg = self.lib.fmd_mel_last_error(self._h).decode() if self._h else ""
            self.close()
            raise _lib.FmdError(st, f"fmd_mel_create: {msg or self.lib.fmd_status_string(st).decode()}")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.fmd_mel_destroy(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def n_mels(self) -> int:
        return self.cfg.feature_size

    def num_frames(self, num_samples: int) -> int:  # mel.rs:76-82
        return num_samples // self.cfg.hop_length

    def log_mel_ptr(self, samples_ptr: int, n_chunks: int, out_ptr: int) -> None:
        st = self.lib.fmd_mel_log_mel(self._h, C.c_void_p(samples_ptr), n_chunks, C.c_void_p(out_ptr))
        if st != _lib.FMD_OK:
            raise _lib.FmdError(st, self.lib.fmd_mel_last_error(self._h).decode())

    def log_mel_device(self, windows):
        """(n_chunks, n_samples) zero-padded windows (host array or device
        tensor, f32) -> device tensor (n_chunks, n_mels, frames)."""
        import torch

        if isinstance(windows, torch.Tensor):
            n, ptr, hold = windows.shape[0], windows.data_ptr(), windows
        else:
            hold = np.ascontiguousarray(np.asarray(windows, dtype=np.float32).reshape(-1, self.cfg.n_samples))
            n, ptr = hold.shape[0], hold.ctypes.data
        out = torch.empty((n, self.cfg.feature_size, self.cfg.nb_max_frames), dtype=torch.float32,
                          device=f"cuda:{self.device}")
        self.log_mel_ptr(ptr, n, out.data_ptr())
        del hold
        return out

    def log_mel(self, samples) -> np.ndarray:
        """`MelFrontend::log_mel` of one window of n_samples samples -> (n_mels, frames)."""
        return self.log_mel_device(np.asarray(samples, dtype=np.float32)[None])[0].cpu().numpy()


def extract_features(waveforms, cfg: FeatureConfig, frontend: MelFrontend, merge_size: int) -> AudioFeatures:
    """`extract_features` (audio/mod.rs:47-116): plan the 30 s chunks on the host,
    zero-pad each to the window and run the log-mel frontend on the GPU."""
    chunks, tokens, mapping, per_audio = plan_chunks([len(w) for w in waveforms], cfg, merge_size)
    windows = np.zeros((len(chunks), cfg.n_samples), dtype=np.float32)
    for i, (a, s, e) in enumerate(chunks):
        windows[i, : e - s] = np.asarray(waveforms[a], dtype=np.float32)[s:e]
    mel = frontend.log_mel_device(windows)
    return AudioFeatures(mel, tokens, mapping, per_audio)


def mel_filters(cfg: FeatureConfig = FeatureConfig()) -> np.ndarray:
    """The library's Slaney filterbank (n_mels, n_fft / 2 + 1), host only."""
    lib = _lib.load()
    out = np.empty((cfg.feature_size, cfg.n_fft // 2 + 1), dtype=np.float32)
    st = lib.fmd_mel_filters(C.byref(cfg.to_c()), out.ctypes.data_as(C.POINTER(C.c_float)))
    if st != _lib.FMD_OK:
        raise _lib.FmdError(st, "fmd_mel_filters")
    return out
