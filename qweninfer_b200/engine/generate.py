"""Single-request greedy generation (QwenInfer's generate, qweninfer/engine/generate.py:18-51).

Prefill once (B = 1, all prompt positions, head on the last one), then one token per
step with one host synchronisation per token (needed to stop on EOS). The decode step
is the same CUDA graph the engine replays at batch size 1.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from qweninfer_b200.engine.kv_cache import KVCache
from qweninfer_b200.engine.runner import DecodeRunner


@torch.inference_mode()
def generate(model, prompt_ids: torch.Tensor, max_new_tokens: int,
             eos_ids: set[int] | None = None, cache: KVCache | None = None,
             on_token: Callable[[int], None] | None = None) -> list[int]:
    """Greedy decoding with a KV cache. prompt_ids: (1, P)."""
    P = prompt_ids.shape[1]
    device = model.device
    if cache is None:
        cache = KVCache(model.cfg, 1, P + max_new_tokens, dtype=model.dtype, device=device)
    runner = DecodeRunner(model, cache, max_batch=1)
    row = cache.row_start
    cache.window = P
    nxt = runner.prefill(row, [int(t) for t in prompt_ids[0].tolist()])
    out: list[int] = []
    for step in range(max_new_tokens):
        tok = nxt
        if eos_ids and tok in eos_ids:
            break
        out.append(tok)
        if on_token is not None:
            on_token(tok)
        pos = P + step
        cache.window = pos + 1
        nxt = int(runner.decode([tok], [pos], row_start=row)[0])
    return out
