"""qweninfer/engine/generate.py: single-request greedy generation."""

from qweninfer_b200.engine.generate import generate

__all__ = ["generate"]
