"""qweninfer.models: Qwen2Config (config.py) and the Qwen2 model (qwen2.py)."""
