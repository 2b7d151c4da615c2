"""qweninfer/engine/kv_cache.py: the preallocated packed KV cache."""

from qweninfer_b200.engine.kv_cache import KVCache

__all__ = ["KVCache"]
