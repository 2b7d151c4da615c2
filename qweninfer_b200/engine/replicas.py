"""Data-parallel serving replicas: one engine per GPU, one process per rank.

The reference serves from a single engine on one GPU (qweninfer/engine/engine.py:47-196).
A 0.5B model fits every GPU many times over, so the multi-GPU form is independent
replicas: each rank holds the weights (0.99 GB), its own KV cache and its own CUDA graphs,
and serves the requests with ``rid % world == rank``. Nothing crosses ranks on the data
path; the host side below only coordinates through the process group's key-value store:

* every finished request's output is published under ``<prefix>/res/<rid>`` as soon as it
  finishes, so work done by a replica that later fails is kept;
* every rank beats a heartbeat counter while it serves;
* after serving its share a rank records ``done`` for the round; a rank that raises
  records ``failed``; a rank whose heartbeat stops for ``timeout_s`` (it exited, hung or
  never joined) is recorded ``failed`` by whoever notices first (compare-and-set: the
  first decision wins, and a rank that finds itself declared failed stops);
* the survivors then split the failed ranks' unfinished requests among themselves
  (``survivors[rid % len(survivors)]``) and serve them in the next round, until a round
  ends with no new failure.

Every survivor computes the same assignment from the store. A request whose result
appears late (a rank finishing it just after being declared failed) may be served twice;
greedy decoding is deterministic, so both results are identical. The store's host (rank
0 of the process group) must stay up: its failure is not recovered.
"""

from __future__ import annotations

import json
import time
from typing import Callable

from qweninfer_b200.engine.engine import Engine, Request


def shard(requests: list[Request], rank: int, world: int) -> list[Request]:
    """The requests replica `rank` of `world` serves: rid % world == rank."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return [r for r in requests if r.rid % world == rank]


class ReplicaFailed(RuntimeError):
    """Raised on a rank that the other replicas declared failed."""


class ReplicaGroup:
    """One rank's side of a replica fleet.

    engine_factory() builds this rank's engine (called once, before the first heartbeat;
    timeout_s must exceed the spread of engine build times). store: a c10d store shared
    by all ranks, e.g. ``torch.distributed.distributed_c10d._get_default_store()`` after
    ``init_process_group`` or a ``torch.distributed.TCPStore``. serve(requests) returns
    every request of the fleet with its output (on every surviving rank).
    """

    def __init__(self, engine_factory: Callable[[], Engine], rank: int, world: int, store,
                 prefix: str = "qi_replicas", heartbeat_s: float = 0.2, timeout_s: float = 10.0,
                 poll_s: float = 0.05) -> None:
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        self.factory, self.rank, self.world, self.store = engine_factory, rank, world, store
        self.prefix, self.heartbeat_s, self.timeout_s, self.poll_s = prefix, heartbeat_s, timeout_s, poll_s
        self.engine: Engine | None = None
        self.round = 0
        self._last_beat = 0.0
        self.log: list[str] = []

    # ------------------------------------------------------------ store keys
    def _k(self, *parts) -> str:
        return "/".join([self.prefix, *map(str, parts)])

    def _has(self, key: str) -> bool:
        return self.store.check([key])

    def _status(self, rnd: int, r: int) -> str | None:
        key = self._k("status", rnd, r)
        return self.store.get(key).decode() if self._has(key) else None

    def _decide(self, rnd: int, r: int, value: str) -> str:
        """Record `value` for (round, rank) unless a decision exists; returns the decision."""
        return self.store.compare_set(self._k("status", rnd, r), "", value).decode()

    def _beat(self, force: bool = False) -> None:
        now = time.monotonic()
        if force or now - self._last_beat >= self.heartbeat_s:
            self.store.add(self._k("hb", self.rank), 1)
            self._last_beat = now
            if self._status(self.round, self.rank) == "failed":
                raise ReplicaFailed(f"rank {self.rank} was declared failed in round {self.round}")

    def _publish(self, req: Request) -> None:
        self.store.set(self._k("res", req.rid), json.dumps(
            {"rid": req.rid, "output": req.output, "arrival": req.arrival, "first_token": req.first_token,
             "finished": req.finished}))

    # ------------------------------------------------------------ serving
    def _serve(self, reqs: list[Request]) -> None:
        todo = [Request(r.rid, list(r.prompt), r.max_new_tokens) for r in reqs
                if not self._has(self._k("res", r.rid))]
        if not todo:
            return
        eng = self.engine
        for r in todo:
            eng.submit(r)
        while eng.waiting or eng.active:
            for r in eng.step():
                self._publish(r)
            self._beat()

    def _await_round(self, rnd: int, live: list[int]) -> list[int]:
        """Wait until every live rank has a decision for round `rnd`; returns the failed."""
        beats = {r: (None, time.monotonic()) for r in live}
        while True:
            undecided = [r for r in live if self._status(rnd, r) is None]
            if not undecided:
                break
            now = time.monotonic()
            for r in undecided:
                key = self._k("hb", r)
                hb = self.store.add(key, 0) if self._has(key) else None
                last, since = beats[r]
                if hb != last:
                    beats[r] = (hb, now)
                elif now - since > self.timeout_s:
                    if self._decide(rnd, r, "failed") == "failed":
                        self.log.append(f"round {rnd}: rank {r} stopped beating, declared failed")
            self._beat()
            time.sleep(self.poll_s)
        return [r for r in live if self._status(rnd, r) == "failed"]

    def serve(self, requests: list[Request], collect: bool = True) -> list[Request] | None:
        """Serve this rank's share and, with the other survivors, the share of any rank
        that fails; returns all requests with outputs, in rid order (None with
        collect=False: the outputs stay in the store, `results` reads them)."""
        live = list(range(self.world))
        assign = {r: shard(requests, r, self.world) for r in live}
        if self.engine is None:  # before the first heartbeat: building it may take a while
            self.engine = self.factory()
        self._beat(force=True)
        while True:
            try:
                self._serve(assign[self.rank])
            except ReplicaFailed:
                raise
            except BaseException:
                self._decide(self.round, self.rank, "failed")
                raise
            if self._decide(self.round, self.rank, "done") != "done":
                raise ReplicaFailed(f"rank {self.rank} was declared failed in round {self.round}")
            failed = self._await_round(self.round, live)
            if not failed:
                break
            live = [r for r in live if r not in failed]
            left = [q for f in failed for q in assign[f] if not self._has(self._k("res", q.rid))]
            assign = {r: [q for q in left if live[q.rid % len(live)] == r] for r in live}
            self.log.append(f"round {self.round}: ranks {failed} failed, {len(left)} requests reassigned")
            self.round += 1
        return self.results(requests) if collect else None

    def results(self, requests: list[Request]) -> list[Request]:
        """Every request of `requests` with the output published for it."""
        out = []
        for r in sorted(requests, key=lambda q: q.rid):
            d = json.loads(self.store.get(self._k("res", r.rid)).decode())
            q = Request(r.rid, list(r.prompt), r.max_new_tokens)
            q.output, q.first_token, q.finished = d["output"], d["first_token"], d["finished"]
            q.arrival = d.get("arrival", q.arrival)
            out.append(q)
        return out
