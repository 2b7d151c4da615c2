"""Preallocated packed KV cache (QwenInfer's KVCache, qweninfer/engine/kv_cache.py:24-76).

Same layout and interface: K and V are each one allocation of shape
(layers, max_batch rows, kv_heads=2, max_len, head_dim=64), slot j of a row holds the
token at absolute position j, and `row_start` / `window` are set by the caller. One
head of one row is a contiguous run of max_len x 128 bytes, which is what the
attention kernel streams and what `move_row` copies.

On this path the append happens inside the QKV kernel's epilogue (qi_qkv_rope_append),
so `update` exists for API compatibility only; `move_row` runs the qi_move_rows kernel.
"""

from __future__ import annotations

import ctypes as C

import torch

from qweninfer_b200 import _lib
from qweninfer_b200.models.config import Qwen2Config


class KVCache:
    def __init__(self, cfg: Qwen2Config, max_batch: int, max_len: int,
                 dtype: torch.dtype = torch.float16, device: str | torch.device = "cuda") -> None:
        # The kernels read and write a bfloat16 cache (the reference's cache dtype for a
        # bf16 model). A float16 or float32 request (the reference's default is float16)
        # gets the same bfloat16 storage: `dtype` is accepted for API compatibility.
        if dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"KV cache dtype must be bfloat16, float16 or float32; got {dtype}")
        shape = (cfg.num_hidden_layers, max_batch, cfg.num_key_value_heads, max_len, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.max_batch = max_batch
        self.max_len = max_len
        self.window = 0
        self.row_start = 0
        self._native: _lib.QiCache | None = None

    def native(self) -> _lib.QiCache:
        if self._native is None:
            self._native = _lib.QiCache(self.k.data_ptr(), self.v.data_ptr(), self.max_batch, self.max_len)
        return self._native

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor):
        """kv_cache.py:48-63: scatter k/v (B, Hkv, S, hd) at positions (B, S) into rows
        [row_start, row_start + B), return the (B, Hkv, window, hd) history views."""
        B = k.shape[0]
        r = slice(self.row_start, self.row_start + B)
        rows = torch.arange(B, device=k.device).unsqueeze(1)
        self.k[layer, r][rows, :, positions] = k.transpose(1, 2).to(self.k.dtype)
        self.v[layer, r][rows, :, positions] = v.transpose(1, 2).to(self.v.dtype)
        return self.k[layer, r, :, : self.window], self.v[layer, r, :, : self.window]

    def move_row(self, src: int, dst: int, length: int) -> None:
        """kv_cache.py:65-73: copy positions [0, length) of row src to row dst, all layers."""
        self.move_rows([(src, dst, length)])

    def move_rows(self, moves: list[tuple[int, int, int]]) -> None:
        """Apply (src, dst, length) row copies in order, enqueued on the current stream."""
        if not moves:
            return
        _lib.ensure_device(self.k.device)
        flat = (C.c_int * (3 * len(moves)))(*[int(x) for m in moves for x in m])
        _lib.check(_lib.lib().qi_move_rows(self.k.data_ptr(), self.v.data_ptr(), self.k.shape[0],
                                           self.max_batch, self.max_len, flat, len(moves),
                                           _lib.stream_ptr(self.k.device)), "qi_move_rows")

    def memory_bytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()


def _single_layer_view(cache: KVCache, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
    return cache.k[layer], cache.v[layer]
