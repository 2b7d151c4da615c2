"""Device side of one engine: prefill and batched decode through `qi_forward`, with the
decode step captured as one CUDA graph per batch size.

Per decode step the host writes the step's token ids, positions and cache rows into a
pinned buffer, copies them to a fixed device buffer (one H2D copy of 12 bytes per row),
replays the graph of that batch size (embedding -> 24 blocks -> head + argmax, ~120
kernels chained with programmatic dependent launch), and reads back one packed argmax
word per row (one D2H copy) — the only host synchronisation of the step, as in the
reference (qweninfer/engine/engine.py:155).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from qweninfer_b200 import _lib
from qweninfer_b200.engine.kv_cache import KVCache, PagedKVCache


class _Staging:
    """[ids | pos | rows | head] int32 for up to n tokens: pinned host + fixed device copy."""

    def __init__(self, n: int, dev: torch.device) -> None:
        self.n = n
        self.h = torch.zeros(3 * n + 1, dtype=torch.int32, pin_memory=True)
        self.d = torch.zeros(3 * n + 1, dtype=torch.int32, device=dev)
        self.np = self.h.numpy()

    def put(self, ids, pos, rows, head: int | None = None) -> None:
        M, n = len(ids), self.n
        self.np[:M] = ids
        self.np[n:n + M] = pos
        self.np[2 * n:2 * n + M] = rows
        if head is not None:
            self.np[3 * n] = head
        self.d.copy_(self.h, non_blocking=True)

    def ptr(self, field: int) -> int:
        return self.d.data_ptr() + 4 * field * self.n


class DecodeRunner:
    """Prefill and decode of one model over one KV cache (see the module docstring)."""

    def __init__(self, model, cache: KVCache, max_batch: int, cuda_graphs: bool = True) -> None:
        self.model = model
        self.cache = cache
        self.dev = model.device
        _lib.ensure_device(self.dev)
        if cache.max_len > model.rope_cos.shape[0]:
            raise ValueError(f"cache max_len {cache.max_len} exceeds the RoPE table "
                             f"({model.rope_cos.shape[0]} positions; raise max_seq_len)")
        self.max_batch = max_batch
        self.cuda_graphs = cuda_graphs
        self.ws = model.workspace(max_batch, cache.max_len)
        self.dec = _Staging(max_batch, self.dev)
        self.pre = _Staging(cache.max_len, self.dev)
        self.h_slots = torch.zeros(max_batch, dtype=torch.int64, pin_memory=True)
        self.d_slots = torch.zeros(max_batch, dtype=torch.int64, device=self.dev)
        self.h_slots_np = self.h_slots.numpy()
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.done = torch.cuda.Event()
        self.steps = 0
        # accounting for benchmarks: kernels launched and bytes moved host<->device
        self.launches = 0
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.kernels_per_forward = lambda M: 1 + 5 * model.cfg.num_hidden_layers + 1
        # a paged cache maps pages before each forward; packed rows need nothing
        self.paged = isinstance(cache, PagedKVCache)

    # ------------------------------------------------------------ helpers

    def _forward(self, st: _Staging, M: int, ws, head_lo: int, n_head: int) -> None:
        if self.paged:
            self.cache.sync()  # new page-table entries, before the kernels read them
        self.launches += self.kernels_per_forward(M)
        _lib.check(_lib.lib().qi_forward(
            C.byref(self.model.native()), C.byref(self.cache.native()), C.byref(ws.struct),
            st.ptr(0), st.ptr(1), st.ptr(2), M, head_lo, 1, n_head, None, 0, 0,
            self.d_slots.data_ptr(), _lib.stream_ptr(self.dev)), "qi_forward")

    def _read(self, k: int) -> np.ndarray:
        self.d2h_bytes += 8 * k
        self.h_slots[:k].copy_(self.d_slots[:k], non_blocking=True)
        self.done.record()
        self.done.synchronize()
        s = self.h_slots_np[:k]
        return (0xFFFFFFFF - (s & 0xFFFFFFFF)).astype(np.int64)

    def _check_ids(self, ids) -> None:
        a = np.asarray(ids)
        if a.min() < 0 or a.max() >= self.model.cfg.vocab_size:
            raise IndexError("token id outside the vocabulary")

    # ---------------------------------------------------------------- API

    @torch.inference_mode()
    def prefill(self, row: int, prompt: list[int]) -> int:
        """B = 1 prefill of `prompt` into cache row `row` at positions 0..P-1; returns the
        greedy next token (engine.py:124-129, generate.py:33-36)."""
        P = len(prompt)
        if P == 0 or P > self.cache.max_len:
            raise ValueError(f"prompt length {P} outside 1..{self.cache.max_len}")
        if not 0 <= row < self.cache.max_batch:
            raise IndexError(f"cache row {row} outside 0..{self.cache.max_batch - 1}")
        self._check_ids(prompt)
        if self.paged:
            self.cache.reserve(row, P)
        self.pre.put(prompt, np.arange(P), np.full(P, row), head=P - 1)
        self.h2d_bytes += self.pre.h.numel() * 4
        ws = self.model.workspace(self.cache.max_len, self.cache.max_len).plan(P, P)
        self._forward(self.pre, P, ws, P - 1, 1)
        return int(self._read(1)[0])

    @torch.inference_mode()
    def prefill_many(self, rows: list[int], prompts: list[list[int]]) -> list[int]:
        """Prefill of several prompts, prompt i into cache row rows[i] at positions
        0..P_i-1, in as few forwards as the staging capacity (cache.max_len tokens)
        allows; returns each prompt's greedy next token. Every token attends to its own
        row only, so this equals one prefill per prompt. In a forward the prompts' last
        tokens are placed after all other tokens: the head tokens are then one contiguous
        range (head_lo = M - n, stride 1)."""
        if len(rows) != len(prompts) or len(set(rows)) != len(rows):
            raise ValueError("one distinct cache row per prompt")
        cap = self.cache.max_len
        for row, p in zip(rows, prompts):
            if not p or len(p) > cap:
                raise ValueError(f"prompt length {len(p)} outside 1..{cap}")
            if not 0 <= row < self.cache.max_batch:
                raise IndexError(f"cache row {row} outside 0..{self.cache.max_batch - 1}")
            self._check_ids(p)
        if self.paged:
            for row, p in zip(rows, prompts):
                self.cache.reserve(row, len(p))
        out: list[int] = []
        i = 0
        while i < len(prompts):
            j, tot = i, 0
            while j < len(prompts) and tot + len(prompts[j]) <= cap:
                tot += len(prompts[j])
                j += 1
            chunk, crow = prompts[i:j], rows[i:j]
            n = len(chunk)
            ids = [t for p in chunk for t in p[:-1]] + [p[-1] for p in chunk]
            pos = [q for p in chunk for q in range(len(p) - 1)] + [len(p) - 1 for p in chunk]
            rws = [r for r, p in zip(crow, chunk) for _ in range(len(p) - 1)] + list(crow)
            M = len(ids)
            self.pre.put(ids, pos, rws)
            self.h2d_bytes += self.pre.h.numel() * 4
            ws = self.model.workspace(cap, cap).plan(M, max(len(p) for p in chunk))
            self._forward(self.pre, M, ws, M - n, n)
            out += [int(t) for t in self._read(n)]
            i = j
        return out

    @torch.inference_mode()
    def decode(self, toks: list[int], pos: list[int], row_start: int = 0) -> np.ndarray:
        """One decode step: token toks[b] at position pos[b] of row row_start + b for every
        b < B; returns the B greedy tokens (engine.py:140-155)."""
        B = len(toks)
        if B == 0 or B > self.max_batch:
            raise ValueError(f"batch {B} outside 1..{self.max_batch}")
        if row_start < 0 or row_start + B > self.cache.max_batch:
            raise IndexError("decode rows outside the cache")
        if max(pos) >= self.cache.max_len or min(pos) < 0:
            raise IndexError(f"position outside 0..{self.cache.max_len - 1}")
        self._check_ids(toks)
        if self.paged:
            for b, q in enumerate(pos):
                self.cache.reserve(row_start + b, int(q) + 1)
            # page-table changes go out before the step, graph replays included (nothing is
            # left to copy when a graph is captured, so no copy is recorded into it)
            self.cache.sync()
        self.dec.put(toks, pos, np.arange(row_start, row_start + B))
        self.h2d_bytes += self.dec.h.numel() * 4
        g = self.graphs.get(B)
        if g is not None:
            g.replay()
        else:
            self.ws.plan(B, 1)  # one token per row: a decode step
            self._forward(self.dec, B, self.ws, 0, B)
            if self.cuda_graphs:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._forward(self.dec, B, self.ws, 0, B)
                self.graphs[B] = g
        self.steps += 1
        return self._read(B)

    @torch.inference_mode()
    def launch_times(self, toks: list[int], pos: list[int], row_start: int = 0) -> list[tuple[str, float]]:
        """The decode step's launches, each timed alone (`qi_forward_launch_times`: an event
        after every launch), as (kind, microseconds); writes the step's K/V like `decode`."""
        B = len(toks)
        if B == 0 or B > self.max_batch or row_start < 0 or row_start + B > self.cache.max_batch:
            raise ValueError("decode batch outside the runner's rows")
        if max(pos) >= self.cache.max_len or min(pos) < 0:
            raise IndexError(f"position outside 0..{self.cache.max_len - 1}")
        self._check_ids(toks)
        if self.paged:
            for b, q in enumerate(pos):
                self.cache.reserve(row_start + b, int(q) + 1)
            self.cache.sync()
        self.dec.put(toks, pos, np.arange(row_start, row_start + B))
        self.ws.plan(B, 1)
        cap = 8 * (2 + 5 * self.model.cfg.num_hidden_layers)
        kinds = (C.c_int * cap)()
        us = (C.c_float * cap)()
        n = C.c_int(0)
        _lib.check(_lib.lib().qi_forward_launch_times(
            C.byref(self.model.native()), C.byref(self.cache.native()), C.byref(self.ws.struct),
            self.dec.ptr(0), self.dec.ptr(1), self.dec.ptr(2), B, 0, 1, B, None, 0, 0,
            self.d_slots.data_ptr(), _lib.stream_ptr(self.dev), kinds, us, cap, C.byref(n)),
            "qi_forward_launch_times")
        return [(_lib.LAUNCH_KINDS[kinds[i]], float(us[i])) for i in range(n.value)]

    def check(self) -> None:
        """Raise if a kernel recorded a timed-out wait (synchronises)."""
        self.ws.check()
        self.model.workspace(self.cache.max_len, self.cache.max_len).check()
