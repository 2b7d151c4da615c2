"""qweninfer.engine: KVCache (kv_cache.py), Engine / Request / autotune_padding (engine.py)
and generate (generate.py)."""
