"""Qwen3 decoder on the B200: the reference's decoder-forward operator surface.

`Qwen3Decoder` mirrors `crates/fmd-core/src/model/qwen3.rs` -- `load`
(:354-390), `embed` (:405-412), `new_caches` (:415-428), `cache_bytes`
(:431-440), `prefill` (:475-496) + `logits` (:459-463), `decode_step`
(:499-511) -- over the C ABI in `include/fmd_decoder.h`. Differences that
follow from the ragged/paged design: each sequence lives in a *slot* with its
own length (no shared offset, no pad_lengths), and prefill takes a list of
per-sequence embedding blocks instead of one left-padded tensor.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .config import TextConfig, act_dtype_name, parse_precision
from .synthetic import bf16_bits_to_f32

_WHICH = {"qkv": 0, "o": 1, "gate_up": 2, "down": 3, "lm_head": 4}


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _host(a) -> tuple:
    """(contiguous array, FMD_DT_*) of a host tensor: bf16 bit patterns (uint16)
    and f16 are passed as stored (checkpoint views stay memory-mapped),
    anything else as f32."""
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return np.ascontiguousarray(a), _lib.DT_BF16
    if a.dtype == np.float16:
        return np.ascontiguousarray(a), _lib.DT_F16
    return _f32(a), _lib.DT_F32


def _q8_blocks(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """(qs, d) -> GGML 34-byte blocks, shape (rows, cols/32, 34)."""
    rows, cols = qs.shape
    nb = cols // 32
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    out[:, :, :2] = np.ascontiguousarray(d.astype(np.float16)).view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = np.ascontiguousarray(qs).view(np.uint8).reshape(rows, nb, 32)
    return out


class Qwen3Decoder:
    def __init__(self, cfg: TextConfig, precision: str = "bf16", device: int = 0):
        self.lib = _lib.load()
        self.cfg = cfg
        self.precision = parse_precision(precision)
        self.act = act_dtype_name(self.precision)
        self._h = C.c_void_p()
        st = self.lib.fmd_create(C.byref(cfg.to_c()), self.precision, device, C.byref(self._h))
        if st != _lib.FMD_OK:
            raise _lib.FmdError(st, f"fmd_create: {self.lib.fmd_status_string(st).decode()}")
        self._keep: list = []
        self.max_slots = 0

    # -- lifecycle ---------------------------------------------------------------------
    def close(self) -> None:
        if self._h:
            self.lib.fmd_destroy(self._h)
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
        _lib.check(st, self._h)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    # -- weights -------------------------------------------------------------------------
    def load_weights(self, w: dict) -> None:
        """`Qwen3::load` (qwen3.rs:354-390) from a host weight dictionary
        (`synthetic.make_weights`, or `checkpoint.load_checkpoint` for a real
        checkpoint: arrays may be f32, f16 or bf16 bit patterns)."""
        keep: list = []

        def t(arr, dtype=_lib.DT_F32) -> _lib.Tensor:
            if arr is None:
                return _lib.Tensor(None, dtype)
            keep.append(arr)
            return _lib.Tensor(arr.ctypes.data, dtype)

        pre = w.get("q8")
        layers = (_lib.LayerWeights * self.cfg.num_hidden_layers)()
        for i, lw in enumerate(w["layers"]):
            L = layers[i]
            L.input_layernorm = t(*_host(lw["input_norm"]))
            L.post_attention_layernorm = t(*_host(lw["post_norm"]))
            L.q_norm = t(*_host(lw["q_norm"]))
            L.k_norm = t(*_host(lw["k_norm"]))
            for cname, key in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"), ("o_proj", "o"),
                               ("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
                if pre is not None:
                    qs, d = pre["layers"][i][key]
                    setattr(L, cname, t(_q8_blocks(qs, d), _lib.DT_Q8_0))
                else:
                    setattr(L, cname, t(*_host(lw[key])))
        ws = _lib.Weights()
        ws.embed_tokens = t(*_host(w["embed"]))
        ws.norm = t(*_host(w["norm"]))
        head = w.get("lm_head")
        ws.lm_head = t(*_host(head)) if head is not None else _lib.Tensor(None, _lib.DT_F32)
        ws.layers = layers
        keep.append(layers)
        self._check(self.lib.fmd_load_weights(self._h, C.byref(ws)))

    def reserve(self, max_slots: int, max_tokens: int, max_rows: int) -> None:
        """`Qwen3::new_caches` sizing: a paged pool of `max_tokens` positions for
        `max_slots` sequences; up to `max_rows` token rows per forward pass."""
        self._check(self.lib.fmd_kv_reserve(self._h, max_slots, max_tokens, max_rows))
        self.max_slots = max_slots

    def memory_bytes(self) -> dict:
        a, b, c = C.c_int64(), C.c_int64(), C.c_int64()
        self._check(self.lib.fmd_memory_bytes(self._h, C.byref(a), C.byref(b), C.byref(c)))
        return {"weights": a.value, "kv_pool": b.value, "workspace": c.value}

    def cache_bytes(self, batch: int, capacity: int) -> int:
        """`Qwen3::cache_bytes` (qwen3.rs:431-440)."""
        return int(self.lib.fmd_cache_bytes(C.byref(self.cfg.to_c()), self.precision, batch, capacity))

    # -- operators ------------------------------------------------------------------------
    def _act_to_f32(self, bits: np.ndarray) -> np.ndarray:
        if self.act == "bf16":
            return bf16_bits_to_f32(bits)
        return bits.view(np.float16).astype(np.float32)

    def embed(self, ids) -> np.ndarray:
        """`Qwen3::embed` (qwen3.rs:405-412): ids -> (n, hidden) f32 (values of the
        activation-dtype table)."""
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        out = np.empty((ids.size, self.cfg.hidden_size), dtype=np.uint16)
        self._check(self.lib.fmd_embed(self._h, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size,
                                       out.ctypes.data))
        return self._act_to_f32(out)

    def splice_audio(self, token_ids, audio_ptr: int, n_audio: int, audio_dtype: str, audio_token_id: int,
                     out_ptr: int) -> None:
        """`MossModel::splice_audio` (model/mod.rs:134-180) on the GPU: writes the
        prompt rows of `token_ids` (host ids, `audio_token_id` at audio
        positions) to the device buffer at `out_ptr` (len(token_ids) x hidden,
        activation dtype), taking audio positions from the `n_audio` device rows
        at `audio_ptr` ("f32" or the activation dtype), in order. Pointers are
        device addresses (e.g. a torch tensor's `data_ptr()`)."""
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int32).reshape(-1))
        dt = {"f32": _lib.DT_F32, "bf16": _lib.DT_BF16, "f16": _lib.DT_F16}[audio_dtype]
        self._check(self.lib.fmd_splice_audio(self._h, ids.ctypes.data_as(C.POINTER(C.c_int32)), ids.size,
                                              C.c_void_p(audio_ptr), n_audio, dt, audio_token_id,
                                              C.c_void_p(out_ptr)))

    def open_slot(self, slot: int, capacity: int) -> None:
        self._check(self.lib.fmd_slot_open(self._h, slot, capacity))

    def release_slot(self, slot: int) -> None:
        self._check(self.lib.fmd_slot_release(self._h, slot))

    def slot_len(self, slot: int) -> int:
        n = C.c_int32()
        self._check(self.lib.fmd_slot_len(self._h, slot, C.byref(n)))
        return n.value

    def new_caches(self, batch: int, capacity: int) -> list[int]:
        """`Qwen3::new_caches` (qwen3.rs:415-428): opens slots 0..batch-1."""
        for s in range(batch):
            self.open_slot(s, capacity)
        return list(range(batch))

    def prefill(self, slots, embeds, want_logits: bool = True):
        """`Qwen3::prefill` + `Qwen3::logits` (qwen3.rs:475-496, :459-463).

        `embeds` is a list of `(len_i, hidden)` arrays (f32, or uint16 bf16 bits
        when the activation dtype is bf16). Returns `(logits (n, vocab) f32 or
        None, next_ids (n,) int32)` for each sequence's last position."""
        slots = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        blocks = [np.asarray(e).reshape(-1, self.cfg.hidden_size) for e in embeds]
        lens = np.ascontiguousarray(np.array([b.shape[0] for b in blocks], dtype=np.int32))
        if blocks[0].dtype == np.uint16:
            flat = np.ascontiguousarray(np.concatenate(blocks, axis=0))
            dt = _lib.DT_BF16 if self.act == "bf16" else _lib.DT_F16
        else:
            flat = np.ascontiguousarray(np.concatenate(blocks, axis=0), dtype=np.float32)
            dt = _lib.DT_F32
        n = len(slots)
        logits = np.empty((n, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        ids = np.empty(n, dtype=np.int32)
        lp = logits.ctypes.data_as(C.POINTER(C.c_float)) if want_logits else None
        self._check(self.lib.fmd_prefill(self._h, n, slots.ctypes.data_as(C.POINTER(C.c_int32)),
                                         lens.ctypes.data_as(C.POINTER(C.c_int32)), flat.ctypes.data, dt, lp,
                                         ids.ctypes.data_as(C.POINTER(C.c_int32))))
        return logits, ids

    def decode_step(self, slots, ids, want_logits: bool = True):
        """`Qwen3::decode_step` + `argmax_rows` (qwen3.rs:499-511,
        engine.rs:550-559): one token per slot."""
        slots = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        n = len(slots)
        logits = np.empty((n, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        nxt = np.empty(n, dtype=np.int32)
        lp = logits.ctypes.data_as(C.POINTER(C.c_float)) if want_logits else None
        self._check(self.lib.fmd_decode_step(self._h, n, slots.ctypes.data_as(C.POINTER(C.c_int32)),
                                             ids.ctypes.data_as(C.POINTER(C.c_int32)), lp,
                                             nxt.ctypes.data_as(C.POINTER(C.c_int32))))
        return logits, nxt

    # -- inspection -------------------------------------------------------------------------
    def debug_weight(self, layer: int, which: str) -> np.ndarray:
        c = self.cfg
        h, i = c.hidden_size, c.intermediate_size
        shapes = {"qkv": (c.q_dim + 2 * c.kv_dim, h), "o": (h, c.q_dim), "gate_up": (2 * i, h),
                  "down": (h, i), "lm_head": (c.vocab_size, h)}
        out = np.empty(shapes[which], dtype=np.float32)
        self._check(self.lib.fmd_debug_weight(self._h, layer, _WHICH[which],
                                              out.ctypes.data_as(C.POINTER(C.c_float)), out.size))
        return out

    def debug_wait_timeout(self, limit: int) -> None:
        """Run one bounded device wait that runs out (`fmd_debug_wait_timeout`):
        raises FmdError with FMD_ETIMEDOUT, after which the handle stays usable."""
        self._check(self.lib.fmd_debug_wait_timeout(self._h, int(limit)))

    def debug_mma_issue(self, form: int, n: int, iters: int = 4096) -> float:
        """SM cycles per tcgen05.mma (M 128 x N n x K 16) issued by one thread
        of a diverged warp (form 0) or the elected lane of a converged warp
        (form 1, the library's kernels) (`fmd_debug_mma_issue`)."""
        c = C.c_double(0.0)
        self._check(self.lib.fmd_debug_mma_issue(self._h, int(form), int(n), int(iters), C.byref(c)))
        return float(c.value)

    def debug_paths(self) -> dict:
        """Which kernels serve this handle's steps (`fmd_debug_paths`):
        {"layer_tail": decode steps on the persistent layer tail,
        "proj_tc": mixed steps on the persistent projection GEMM,
        "lm_head_tc": the lm_head on the tensor cores,
        "prefill_pp": prefill attention on persistent two-tile CTAs,
        "decode_split": decode-only steps run each half of their rows on its own stream}."""
        f = C.c_int32(0)
        self._check(self.lib.fmd_debug_paths(self._h, C.byref(f)))
        return {"layer_tail": bool(f.value & 1), "proj_tc": bool(f.value & 2), "lm_head_tc": bool(f.value & 4),
                "prefill_pp": bool(f.value & 8), "decode_split": bool(f.value & 16)}

    def debug_kv(self, slot: int, layer: int, pos: int, n: int):
        shape = (n, self.cfg.num_key_value_heads, self.cfg.head_dim)
        k = np.empty(shape, dtype=np.uint16)
        v = np.empty(shape, dtype=np.uint16)
        self._check(self.lib.fmd_debug_kv(self._h, slot, layer, pos, n, k.ctypes.data, v.ctypes.data))
        return self._act_to_f32(k), self._act_to_f32(v)
