"""Qwen2 model configuration.

Same interface as the reference's `Qwen2Config` (qweninfer/models/config.py:16-61):
field names follow the Hugging Face checkpoint JSON, and `head_dim`, `n_kv_groups`
and `kv_bytes_per_token` are derived properties.

The CUDA kernels of this package are specialised to the Qwen2-0.5B block shape
(hidden 896, 14 query heads, 2 KV heads, head_dim 64, intermediate 4864); the
number of layers and the vocabulary size are runtime parameters.
`check_supported` states that contract in one place.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from pathlib import Path


@dataclass
class Qwen2Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_position_embeddings: int
    rms_norm_eps: float
    rope_theta: float
    tie_word_embeddings: bool

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def n_kv_groups(self) -> int:
        """Query heads per key/value head (config.py:34-36)."""
        return self.num_attention_heads // self.num_key_value_heads

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        """KV-cache bytes of one token over all layers (config.py:38-45)."""
        per_layer = 2 * self.num_key_value_heads * self.head_dim * dtype_bytes
        return per_layer * self.num_hidden_layers

    @classmethod
    def from_json(cls, path: str | Path) -> "Qwen2Config":
        """Read an HF `config.json` (config.py:47-61)."""
        raw = json.loads(Path(path).read_text())
        return cls(
            vocab_size=raw["vocab_size"],
            hidden_size=raw["hidden_size"],
            intermediate_size=raw["intermediate_size"],
            num_hidden_layers=raw["num_hidden_layers"],
            num_attention_heads=raw["num_attention_heads"],
            num_key_value_heads=raw["num_key_value_heads"],
            max_position_embeddings=raw["max_position_embeddings"],
            rms_norm_eps=raw["rms_norm_eps"],
            rope_theta=raw["rope_theta"],
            tie_word_embeddings=raw.get("tie_word_embeddings", False),
        )

    def to_json(self, path: str | Path) -> None:
        """Write an HF-style `config.json` that `from_json` reads back."""
        raw = asdict(self)
        raw["model_type"] = "qwen2"
        raw["hidden_act"] = "silu"
        Path(path).write_text(json.dumps(raw, indent=1))


# Block shape the CUDA kernels are compiled for (Qwen2-0.5B).
KERNEL_HIDDEN = 896
KERNEL_INTERMEDIATE = 4864
KERNEL_HEADS = 14
KERNEL_KV_HEADS = 2
KERNEL_HEAD_DIM = 64


def qwen2_0p5b(num_hidden_layers: int = 24, vocab_size: int = 151936) -> Qwen2Config:
    """The Qwen2.5-0.5B configuration (layers and vocabulary may be shrunk for tests)."""
    return Qwen2Config(
        vocab_size=vocab_size, hidden_size=896, intermediate_size=4864,
        num_hidden_layers=num_hidden_layers, num_attention_heads=14,
        num_key_value_heads=2, max_position_embeddings=32768,
        rms_norm_eps=1e-6, rope_theta=1000000.0, tie_word_embeddings=True,
    )


def check_supported(cfg: Qwen2Config) -> None:
    """Raise if `cfg` does not fit the compiled kernels."""
    got = (cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads,
           cfg.num_key_value_heads, cfg.head_dim)
    want = (KERNEL_HIDDEN, KERNEL_INTERMEDIATE, KERNEL_HEADS, KERNEL_KV_HEADS,
            KERNEL_HEAD_DIM)
    if got != want:
        raise ValueError(
            "qweninfer_b200 kernels are compiled for hidden/intermediate/heads/kv_heads/"
            f"head_dim = {want}; this config has {got}")
    if cfg.vocab_size % 128 != 0:
        raise ValueError(f"vocab_size must be a multiple of 128, got {cfg.vocab_size}")
    if not cfg.tie_word_embeddings:
        raise ValueError("only tied input/output embeddings are supported (as in Qwen2-0.5B)")
