"""Pure-Python restatement of the reference's continuous-batching scheduler.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`). Restates
qweninfer/engine/engine.py:42-196 with the oracle model (or a stub model that only
drives the bookkeeping) and records a trace of every device-visible action, one record per `step()`:

  {"admit":  [[rid, row, prompt_len, first_token], ...],
   "decode": [rows_total, [[rid, row, token_in, position], ...]] or None,
   "move":   [[src, dst, length], ...],
   "done":   [rid, ...]}                    (pad rows appear with rid -1)

Two schedulers that produce the same records for the same requests made the same
slot, position, length and compaction decisions.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np


@dataclass
class OracleRequest:
    """Request, engine.py:42-58 (timestamps replaced by a finished flag)."""
    rid: int
    prompt: list[int]
    max_new_tokens: int
    output: list[int] = field(default_factory=list)
    length: int = 0
    last: int = 0
    finished: bool = False


def stub_token(token_in: int, position: int, vocab: int) -> int:
    """Deterministic stand-in for argmax(logits) when only bookkeeping is checked."""
    return (token_in * 1103515245 + position * 12345 + 7) % vocab


class StubModel:
    """Drives the scheduler without arithmetic: the "next token" of a query is
    `stub_token(last input id, its position)`."""

    def __init__(self, vocab: int = 1000) -> None:
        self.vocab = vocab

    def next_tokens(self, ids: np.ndarray, positions: np.ndarray) -> list[int]:
        return [stub_token(int(i), int(p), self.vocab) for i, p in zip(ids[:, -1], positions[:, -1])]


class OracleEngine:
    """Engine, engine.py:62-196. `model` is an `OracleModel` (real arithmetic, its cache
    is an `OracleCache`) or a `StubModel` (bookkeeping only, no cache)."""

    def __init__(self, model, max_slots: int, max_len: int, eos_ids: set[int] | None = None,
                 static: bool = False, max_prefills_per_step: int | None = None,
                 pad_to: list[int] | None = None) -> None:
        if pad_to is not None:  # engine.py:81-83
            if len(pad_to) <= max_slots or any(pad_to[n] < n for n in range(max_slots + 1)):
                raise ValueError("pad_to needs an entry n -> size >= n for n = 0..max_slots")
        rows = max([max_slots] + (pad_to[: max_slots + 1] if pad_to else []))  # engine.py:87
        self.model = model
        self.rows = rows
        self.cache = None
        if not isinstance(model, StubModel):
            from oracle.qwen2_ref import OracleCache
            self.cache = OracleCache(model.cfg, rows, max_len)
        self.max_slots, self.max_len = max_slots, max_len
        self.eos_ids = eos_ids or set()
        self.static = static
        self.max_prefills = max_prefills_per_step
        self.pad_to = pad_to
        self.waiting: deque[OracleRequest] = deque()
        self.active: list[OracleRequest] = []
        self.trace: list[dict] = []
        self._rec: dict | None = None

    def submit(self, req: OracleRequest) -> None:  # engine.py:100-105
        if len(req.prompt) + req.max_new_tokens > self.max_len:
            raise ValueError(f"request {req.rid} needs {len(req.prompt) + req.max_new_tokens}"
                             f" tokens, capacity is {self.max_len}")
        self.waiting.append(req)

    def _finish_check(self, req: OracleRequest, tok: int) -> bool:  # engine.py:109-113
        if tok in self.eos_ids:
            return True
        req.output.append(tok)
        return len(req.output) >= req.max_new_tokens

    def _forward_tokens(self, ids: np.ndarray, positions: np.ndarray, last_only: bool) -> list[int]:
        if isinstance(self.model, StubModel):
            return self.model.next_tokens(ids, positions)
        logits = self.model.forward(ids, positions=positions, cache=self.cache, last_only=last_only)
        return [int(t) for t in np.argmax(logits[:, -1], axis=-1)]

    def _admit(self) -> list[OracleRequest]:  # engine.py:115-138
        done = []
        if self.static and self.active:
            return done
        admitted = 0
        while (self.waiting and len(self.active) < self.max_slots
               and (self.max_prefills is None or admitted < self.max_prefills)):
            req = self.waiting.popleft()
            row, P = len(self.active), len(req.prompt)
            if self.cache is not None:
                self.cache.row_start, self.cache.window = row, P
            ids = np.array([req.prompt])
            tok = self._forward_tokens(ids, np.arange(P)[None, :], last_only=True)[0]
            self._rec["admit"].append([req.rid, row, P, tok])
            admitted += 1
            if self._finish_check(req, tok):
                req.finished = True
                done.append(req)
                continue
            req.length, req.last = P, tok
            self.active.append(req)
        return done

    def _decode(self) -> list[int]:  # engine.py:140-164
        n = len(self.active)
        if self.cache is not None:
            self.cache.row_start = 0
            self.cache.window = max(r.length for r in self.active) + 1
        toks = [r.last for r in self.active]
        pos = [r.length for r in self.active]
        if self.pad_to is not None:
            extra = self.pad_to[n] - n
            toks += [0] * extra
            pos += [0] * extra
        self._rec["decode"] = [len(toks),
                               [[r.rid, i, r.last, r.length] for i, r in enumerate(self.active)]
                               + [[-1, n + j, 0, 0] for j in range(len(toks) - n)]]
        nxt = self._forward_tokens(np.array(toks)[:, None], np.array(pos)[:, None], False)[:n]
        finished_rows = []
        for i, (req, tok) in enumerate(zip(self.active, nxt)):
            req.length += 1
            req.last = tok
            if self._finish_check(req, tok):
                req.finished = True
                finished_rows.append(i)
        return finished_rows

    def _retire(self, rows: list[int]) -> list[OracleRequest]:  # engine.py:166-179
        done = []
        for row in sorted(rows, reverse=True):
            req = self.active[row]
            last = len(self.active) - 1
            if row != last:
                mover = self.active[last]
                if self.cache is not None:
                    self.cache.move_row(src=last, dst=row, length=mover.length)
                self._rec["move"].append([last, row, mover.length])
                self.active[row] = mover
            self.active.pop()
            done.append(req)
        return done

    def step(self) -> list[OracleRequest]:  # engine.py:183-188
        self._rec = {"admit": [], "decode": None, "move": [], "done": []}
        done = self._admit()
        if self.active:
            done += self._retire(self._decode())
        self._rec["done"] = [r.rid for r in done]
        self.trace.append(self._rec)
        return done

    def run(self, requests: list[OracleRequest]) -> list[OracleRequest]:  # engine.py:190-196
        for r in requests:
            self.submit(r)
        finished: list[OracleRequest] = []
        while self.waiting or self.active:
            finished += self.step()
        return sorted(finished, key=lambda r: r.rid)


def pad_table(max_slots: int, candidates=(1, 2, 4, 8, 12, 16, 20, 24, 28, 32, 40, 48, 56, 64),
              max_rows: int | None = None, ms: dict[int, float] | None = None) -> list[int]:
    """pad_to table construction of autotune_padding, engine.py:221-232, for a given
    step-time table `ms` (default: time grows with size, so the smallest candidate >= n)."""
    max_rows = max_rows or max_slots
    cands = sorted({c for c in candidates if c <= max_rows} | {max_slots, max_rows})
    if ms is None:
        ms = {c: float(c) for c in cands}
    return [0] + [min((c for c in cands if c >= n), key=lambda c: ms[c]) for n in range(1, max_slots + 1)]
