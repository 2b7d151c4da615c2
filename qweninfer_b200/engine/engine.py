"""Continuous-batching engine (QwenInfer's Engine, qweninfer/engine/engine.py:42-233).

The scheduler is the reference's, decision for decision — admission into row
len(active), one batched decode over rows 0..n-1 (plus pad rows at position 0), EOS /
length stopping, retirement highest row first with the last row moved into the hole,
`run` returning requests sorted by rid — so the same request trace yields the same
slots, positions, lengths and row moves. What changes is the device side
(`DecodeRunner`): prefill and decode run as single native forwards, each decode batch
size is one CUDA graph, and per step the host moves 12 bytes per row in and 8 bytes per
row out.

Every scheduler action can be recorded (`record=True`) in the same per-step form as the
test oracle's trace: {"admit": [[rid, row, P, tok]...], "decode": [rows_total,
[[rid, row, tok_in, pos]...]], "move": [[src, dst, len]...], "done": [rid...]}.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

import torch

from qweninfer_b200.engine.kv_cache import KVCache, PagedKVCache
from qweninfer_b200.engine.runner import DecodeRunner


@dataclass
class Request:
    """engine.py:42-58."""
    rid: int
    prompt: list[int]
    max_new_tokens: int
    output: list[int] = field(default_factory=list)
    arrival: float = 0.0
    first_token: float | None = None
    finished: float | None = None
    length: int = 0
    last: int = 0

    @property
    def done(self) -> bool:
        return self.finished is not None


class Engine:
    # Device side; a test may substitute doubles with the same interface.
    cache_cls = KVCache
    runner_cls = DecodeRunner

    def __init__(self, model, max_slots: int, max_len: int, eos_ids: set[int] | None = None,
                 static: bool = False, max_prefills_per_step: int | None = None,
                 pad_to: list[int] | None = None, cuda_graphs: bool = True,
                 record: bool = False, batch_prefill: bool = True, page_size: int = 0,
                 kv_pages: int | None = None) -> None:
        """engine.py:62-98. Extra keywords: `cuda_graphs` (capture each decode batch size),
        `record` (keep a per-step trace of scheduler actions in `self.trace`),
        `batch_prefill` (prefill a step's admissions together; same decisions) and
        `page_size` (> 0: a PagedKVCache of pages of that many positions, `kv_pages` pages
        per layer; row moves then move page-table entries; same decisions)."""
        if pad_to is not None:
            if len(pad_to) <= max_slots or any(pad_to[n] < n for n in range(max_slots + 1)):
                raise ValueError("pad_to needs an entry n -> size >= n for n = 0..max_slots")
        rows = max([max_slots] + (pad_to[: max_slots + 1] if pad_to else []))
        self.model = model
        self.device = model.norm.weight.device
        if page_size:
            self.cache = PagedKVCache(model.cfg, rows, max_len, dtype=model.dtype, device=self.device,
                                      page_size=page_size, n_pages=kv_pages)
        else:
            self.cache = self.cache_cls(model.cfg, rows, max_len, dtype=model.dtype, device=self.device)
        self.max_slots, self.max_len = max_slots, max_len
        self.eos_ids = eos_ids or set()
        self.static = static
        self.max_prefills = max_prefills_per_step
        self.batch_prefill = batch_prefill
        self.pad_to = pad_to
        self.waiting: deque[Request] = deque()
        self.active: list[Request] = []
        self.runner = self.runner_cls(model, self.cache, max_batch=rows, cuda_graphs=cuda_graphs)
        self.trace: list[dict] | None = [] if record else None
        self._rec: dict | None = None

    def submit(self, req: Request) -> None:
        """engine.py:100-105."""
        if len(req.prompt) + req.max_new_tokens > self.max_len:
            raise ValueError(f"request {req.rid} needs {len(req.prompt) + req.max_new_tokens}"
                             f" tokens, capacity is {self.max_len}")
        req.arrival = req.arrival or time.perf_counter()
        self.waiting.append(req)

    def _release(self, row: int) -> None:
        """A row's request is gone: a paged cache takes its pages back (a cache without
        storage management, like the packed one, has nothing to do)."""
        release = getattr(self.cache, "release", None)
        if release is not None:
            release(row)

    def _finish_check(self, req: Request, tok: int) -> bool:
        """engine.py:109-113."""
        if tok in self.eos_ids:
            return True
        req.output.append(tok)
        return len(req.output) >= req.max_new_tokens

    def _admit(self) -> list[Request]:
        """engine.py:115-138: prefill of waiting requests into row len(active), the same
        requests into the same rows as the reference's one-at-a-time loop. Runs of
        requests that keep their slot after prefill (no EOS ids, max_new_tokens > 1) are
        prefilled together (runner.prefill_many); a request that may finish at its first
        token is prefilled alone, because the next request reuses its row."""
        done = []
        if self.static and self.active:
            return done
        admitted = 0
        while (self.waiting and len(self.active) < self.max_slots
               and (self.max_prefills is None or admitted < self.max_prefills)):
            run: list[Request] = []
            if self.batch_prefill and not self.eos_ids:
                while (self.waiting and len(self.active) + len(run) < self.max_slots
                       and (self.max_prefills is None or admitted + len(run) < self.max_prefills)
                       and self.waiting[0].max_new_tokens > 1):
                    run.append(self.waiting.popleft())
            if not run:
                run = [self.waiting.popleft()]
            rows = [len(self.active) + i for i in range(len(run))]
            self.cache.row_start, self.cache.window = rows[-1], len(run[-1].prompt)
            if len(run) > 1:
                toks = self.runner.prefill_many(rows, [r.prompt for r in run])
            else:
                toks = [self.runner.prefill(rows[0], run[0].prompt)]
            now = time.perf_counter()
            for req, row, tok in zip(run, rows, toks):
                req.first_token = now
                admitted += 1
                if self._rec is not None:
                    self._rec["admit"].append([req.rid, row, len(req.prompt), tok])
                if self._finish_check(req, tok):
                    req.finished = req.first_token
                    done.append(req)
                    self._release(row)  # the next admission reuses the row
                    continue
                req.length, req.last = len(req.prompt), tok
                self.active.append(req)
        return done

    def _decode(self) -> list[int]:
        """engine.py:140-164: one batched step over rows 0..n-1 (+ pad rows)."""
        n = len(self.active)
        self.cache.row_start = 0
        self.cache.window = max(r.length for r in self.active) + 1
        toks = [r.last for r in self.active]
        pos = [r.length for r in self.active]
        if self.pad_to is not None:
            extra = self.pad_to[n] - n
            toks += [0] * extra
            pos += [0] * extra
        if self._rec is not None:
            self._rec["decode"] = [len(toks),
                                   [[r.rid, i, r.last, r.length] for i, r in enumerate(self.active)]
                                   + [[-1, n + j, 0, 0] for j in range(len(toks) - n)]]
        nxt = self.runner.decode(toks, pos)[:n].tolist()
        finished_rows = []
        now = time.perf_counter()
        for i, (req, tok) in enumerate(zip(self.active, nxt)):
            req.length += 1
            req.last = tok
            if self._finish_check(req, tok):
                req.finished = now
                finished_rows.append(i)
        return finished_rows

    def _retire(self, rows: list[int]) -> list[Request]:
        """engine.py:166-179: highest row first; the last row moves into the hole."""
        done = []
        for row in sorted(rows, reverse=True):
            req = self.active[row]
            last = len(self.active) - 1
            if row != last:
                mover = self.active[last]
                self.cache.move_row(src=last, dst=row, length=mover.length)
                if self._rec is not None:
                    self._rec["move"].append([last, row, mover.length])
                self.active[row] = mover
            else:
                self._release(row)
            self.active.pop()
            done.append(req)
        return done

    def step(self) -> list[Request]:
        """engine.py:183-188: one scheduler iteration; returns requests finished in it."""
        if self.trace is not None:
            self._rec = {"admit": [], "decode": None, "move": [], "done": []}
        done = self._admit()
        if self.active:
            done += self._retire(self._decode())
        if self.trace is not None:
            self._rec["done"] = [r.rid for r in done]
            self.trace.append(self._rec)
        return done

    def run(self, requests: list[Request]) -> list[Request]:
        """engine.py:190-196."""
        for r in requests:
            self.submit(r)
        finished: list[Request] = []
        while self.waiting or self.active:
            finished += self.step()
        return sorted(finished, key=lambda r: r.rid)


@torch.inference_mode()
def autotune_padding(model, max_slots: int, max_rows: int | None = None,
                     candidates: list[int] | None = None, context: int = 128,
                     iters: int = 8) -> tuple[list[int], dict[int, float]]:
    """engine.py:199-233: time the decode step at candidate batch sizes (context 128,
    2 warm-up + `iters` timed steps, CUDA events) and map every active count n to the
    fastest candidate >= n."""
    if candidates is None:
        candidates = [1, 2, 4, 8, 12, 16, 20, 24, 28, 32, 40, 48, 56, 64]
    max_rows = max_rows or max_slots
    candidates = sorted({c for c in candidates if c <= max_rows} | {max_slots, max_rows})
    cache = KVCache(model.cfg, max_rows, context + 2, dtype=model.dtype, device=model.device)
    cache.window = context + 1
    runner = DecodeRunner(model, cache, max_batch=max_rows)
    ms: dict[int, float] = {}
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for c in candidates:
        toks, pos = [0] * c, [context] * c
        for i in range(iters + 2):
            if i == 2:
                torch.cuda.synchronize()
                start.record()
            runner.decode(toks, pos)
        stop.record()
        stop.synchronize()
        ms[c] = start.elapsed_time(stop) / iters
    del runner, cache
    torch.cuda.empty_cache()
    pad_to = [0] + [min((c for c in candidates if c >= n), key=lambda c: ms[c])
                    for n in range(1, max_slots + 1)]
    return pad_to, ms
