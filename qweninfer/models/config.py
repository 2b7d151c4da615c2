"""qweninfer/models/config.py: the HF-JSON-named Qwen2Config."""

from qweninfer_b200.models.config import Qwen2Config

__all__ = ["Qwen2Config"]
