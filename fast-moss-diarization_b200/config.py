"""Model shape and precision contract.

`TextConfig` mirrors `crates/fmd-core/src/config.rs:8-58` (explicit head_dim,
eps 1e-6, theta 1e6 defaults); `parse_precision` mirrors
`crates/fmd-core/src/precision.rs:19-29`.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

from . import _lib

EOS_TOKEN_ID = 151_645  # config.rs:110-116, engine.rs:246
DEFAULT_MAX_NEW_TOKENS = 4096  # engine.rs:85-96
ROPE_TABLE_LIMIT = 65_536  # engine.rs:238-243


@dataclass
class TextConfig:
    vocab_size: int = 151_936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 131_072
    eos_token_id: int = EOS_TOKEN_ID

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def kv_repeat(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def n_params(self, with_head: bool = True) -> int:
        """Projection parameters touched per decode step (embedding lookup excluded)."""
        h, i = self.hidden_size, self.intermediate_size
        per_layer = h * (self.q_dim + 2 * self.kv_dim) + self.q_dim * h + 2 * i * h + i * h
        return self.num_hidden_layers * per_layer + (self.vocab_size * h if with_head else 0)

    def kv_bytes_per_token(self, elem: int = 2) -> int:
        """`2 x layers x kv_heads x head_dim x elem` (README.md:130-141 formula)."""
        return 2 * self.num_hidden_layers * self.num_key_value_heads * self.head_dim * elem

    def to_c(self) -> _lib.Config:
        c = _lib.Config()
        for k, v in asdict(self).items():
            setattr(c, k, v)
        return c

    def oracle_kwargs(self) -> dict:
        d = asdict(self)
        d.pop("eos_token_id")
        return d


def parse_precision(name: str) -> int:
    """`Precision::parse` (precision.rs:21-29) plus the int8+bf16 variant."""
    key = name.strip().lower().replace("-", "_")
    aliases = {"float32": "f32", "full": "f32", "float16": "f16", "half": "f16", "bfloat16": "bf16",
               "i8": "int8", "q8": "int8", "q80": "int8"}
    key = aliases.get(key, key)
    if key not in _lib.PRECISIONS:
        raise ValueError(f"unsupported dtype {name!r}; expected one of fp32, fp16, bf16, int8, int8_bf16")
    return _lib.PRECISIONS[key]


def act_dtype_name(precision: int) -> str:
    """`Precision::activation_dtype` (precision.rs:32-41)."""
    return {_lib.PREC_F32: "f32", _lib.PREC_F16: "f16", _lib.PREC_BF16: "bf16", _lib.PREC_INT8: "f16",
            _lib.PREC_INT8_BF16: "bf16"}[precision]
