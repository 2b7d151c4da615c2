"""Preallocated packed KV cache (QwenInfer's KVCache, qweninfer/engine/kv_cache.py:24-76).

Same layout and interface: K and V are each one allocation of shape
(layers, max_batch rows, kv_heads=2, max_len, head_dim=64), slot j of a row holds the
token at absolute position j, and `row_start` / `window` are set by the caller. One
head of one row is a contiguous run of max_len x 128 bytes, which is what the
attention kernel streams and what `move_row` copies.

On this path the append happens inside the QKV kernel's epilogue (qi_qkv_rope_append),
so `update` exists for API compatibility only; `move_row` runs the qi_move_rows kernel.

`PagedKVCache` (no reference counterpart: the reference kept packed rows, README.md:261-266)
stores positions in pages of 128 slots taken from a pool on demand, so the cache holds
the live tokens rather than rows x max_len, and a retired row's hole is filled by moving
page-table entries instead of copying K/V.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
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
            self._native = _lib.QiCache(self.k.data_ptr(), self.v.data_ptr(), self.max_batch, self.max_len,
                                        None, 0, 0, 0)
        return self._native

    # storage management hooks of the paged cache (every slot of a packed row exists)
    def reserve(self, row: int, length: int) -> None:
        """Make positions [0, length) of `row` writable (no-op for packed rows)."""

    def release(self, row: int) -> None:
        """The row's request is gone (no-op for packed rows)."""

    def sync(self) -> None:
        """Publish storage changes to the device before a forward (no-op)."""

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


class PagedKVCache(KVCache):
    """K and V in pages of `page_size` positions (a multiple of 128) from a pool of
    `n_pages` pages per layer: `k`, `v` of shape (layers, n_pages, kv_heads, page_size,
    head_dim) and a page table (max_batch, pages_per_row) int32, -1 for unmapped, on the
    device with a host copy. Pages are taken from the pool as rows grow (`reserve`),
    returned when a row's request ends (`release`), and `move_row` moves page-table
    entries. The default pool (max_batch x pages_per_row pages) never runs out; a smaller
    one raises when it does. Only the forward's tensor-core path reads this layout."""

    def __init__(self, cfg: Qwen2Config, max_batch: int, max_len: int,
                 dtype: torch.dtype = torch.float16, device: str | torch.device = "cuda",
                 page_size: int = 128, n_pages: int | None = None) -> None:
        if dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"KV cache dtype must be bfloat16, float16 or float32; got {dtype}")
        if page_size < 128 or page_size % 128:
            raise ValueError(f"page_size must be a positive multiple of 128; got {page_size}")
        self.page_size = page_size
        self.pages_per_row = -(-max_len // page_size)
        self.n_pages = n_pages if n_pages is not None else max_batch * self.pages_per_row
        if self.n_pages < 1:
            raise ValueError("the pool needs at least one page")
        shape = (cfg.num_hidden_layers, self.n_pages, cfg.num_key_value_heads, page_size, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.max_batch = max_batch
        self.max_len = max_len
        self.window = 0
        self.row_start = 0
        dev = torch.device(device)
        self.table_host = torch.full((max_batch, self.pages_per_row), -1, dtype=torch.int32,
                                     pin_memory=dev.type == "cuda")
        self.table = self.table_host.to(dev)
        self._t = self.table_host.numpy()
        self.mapped = np.zeros(max_batch, dtype=np.int64)   # pages mapped per row (a prefix)
        self.free = list(range(self.n_pages - 1, -1, -1))   # stack of free page ids
        self.dirty = False
        self._native = None

    def native(self) -> _lib.QiCache:
        if self._native is None:
            self._native = _lib.QiCache(self.k.data_ptr(), self.v.data_ptr(), self.max_batch, self.max_len,
                                        self.table.data_ptr(), self.page_size, self.pages_per_row, self.n_pages)
        return self._native

    def reserve(self, row: int, length: int) -> None:
        if not 0 <= row < self.max_batch or not 0 <= length <= self.max_len:
            raise IndexError(f"row {row} / length {length} outside the cache")
        need = -(-length // self.page_size)
        while self.mapped[row] < need:
            if not self.free:
                raise RuntimeError(f"KV page pool of {self.n_pages} pages exhausted")
            self._t[row, self.mapped[row]] = self.free.pop()
            self.mapped[row] += 1
            self.dirty = True

    def release(self, row: int) -> None:
        for j in range(int(self.mapped[row]) - 1, -1, -1):
            self.free.append(int(self._t[row, j]))
            self._t[row, j] = -1
        if self.mapped[row]:
            self.dirty = True
        self.mapped[row] = 0

    def move_row(self, src: int, dst: int, length: int) -> None:
        """Row dst takes over row src's pages (positions [0, length) and any beyond);
        dst's own pages return to the pool and src is left without pages."""
        if src == dst:
            return
        self.release(dst)
        self._t[dst] = self._t[src]
        self.mapped[dst] = self.mapped[src]
        self._t[src] = -1
        self.mapped[src] = 0
        self.dirty = True

    def move_rows(self, moves: list[tuple[int, int, int]]) -> None:
        for src, dst, length in moves:
            self.move_row(src, dst, length)

    def sync(self) -> None:
        if self.dirty:
            self.table.copy_(self.table_host, non_blocking=True)
            self.dirty = False

    def pages_in_use(self) -> int:
        return self.n_pages - len(self.free)

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor):
        raise NotImplementedError("the paged cache is written by the forward's kernels only")


def _single_layer_view(cache: KVCache, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
    return cache.k[layer], cache.v[layer]
