"""qweninfer/engine/engine.py: Request, the continuous-batching Engine and autotune_padding."""

from qweninfer_b200.engine.engine import Engine, Request, autotune_padding

__all__ = ["Request", "Engine", "autotune_padding"]
