"""qweninfer/models/qwen2.py: RMSNorm, build_rope_cache, _rotate_half, apply_rope, MLP,
Attention, Block and Qwen2 (from_pretrained, fuse, forward) on the sm_100a kernels."""

from qweninfer_b200.models.config import Qwen2Config
from qweninfer_b200.models.qwen2 import (MLP, Attention, Block, Qwen2, RMSNorm, _rotate_half, apply_rope,
                                         build_rope_cache)

__all__ = ["Qwen2Config", "RMSNorm", "build_rope_cache", "_rotate_half", "apply_rope", "MLP", "Attention",
           "Block", "Qwen2"]
