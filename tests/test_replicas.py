"""Data-parallel replicas (qweninfer_b200/engine/replicas.py) as world-size-2 process
groups on CPU (gloo), with the engine's device side replaced by the stub doubles of
test_engine_host.py. Failures are made on the host: a rank whose engine raises, a rank
that exits without notice, a rank that never joins. In every case the surviving rank
serves the lost requests and the fleet's outputs equal one engine's outputs."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import time

import pytest

from qweninfer_b200 import synthetic
from qweninfer_b200.engine.engine import Request
from qweninfer_b200.engine.replicas import ReplicaGroup, shard

WORLD = 2
REQS = synthetic.serving_requests(24, 4, 24, 8.0, 0.5, 24, seed=11)


def _requests():
    return [Request(r.rid, list(r.prompt), r.max_new_tokens) for r in REQS]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _engine(fail_after: int | None = None, exit_after: int | None = None):
    from test_engine_host import StubEngine, fake_model
    eng = StubEngine(fake_model(), max_slots=4, max_len=64)
    if fail_after is not None or exit_after is not None:
        decode, calls = eng.runner.decode, [0]

        def flaky(toks, pos, row_start=0):
            calls[0] += 1
            if fail_after is not None and calls[0] > fail_after:
                raise RuntimeError("injected replica failure")
            if exit_after is not None and calls[0] > exit_after:
                os._exit(3)
            return decode(toks, pos, row_start)

        eng.runner.decode = flaky
    return eng


def _worker(rank, port, mode, out_q):
    import torch.distributed as dist
    try:
        if mode == "never_joins" and rank == 1:
            return
        if mode == "never_joins":
            store = dist.TCPStore("127.0.0.1", port, WORLD, is_master=True, wait_for_workers=False,
                                  timeout=__import__("datetime").timedelta(seconds=60))
        else:
            dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
            store = dist.distributed_c10d._get_default_store()
        fail = {"raises": dict(fail_after=3), "exits": dict(exit_after=3)}.get(mode, {}) if rank == 1 else {}
        grp = ReplicaGroup(lambda: _engine(**fail), rank, WORLD, store, timeout_s=2.0, poll_s=0.02)
        done = grp.serve(_requests())
        out_q.put((rank, "ok", {r.rid: r.output for r in done}, grp.log))
        if mode == "all_alive":
            dist.barrier()  # both alive: the ordinary collective path still works
    except Exception as e:  # reported to the test; a failed replica is an expected outcome
        out_q.put((rank, "error", repr(e), []))


def _run_fleet(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    deadline = time.time() + 120
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        rank, status, payload, log = q.get()
        res[rank] = (status, payload, log)
    return res, [p.exitcode for p in procs]


def _single_engine_outputs():
    eng = _engine()
    return {r.rid: r.output for r in eng.run(_requests())}


def test_shard_is_a_partition():
    reqs = _requests()
    for world in (1, 2, 3, 8):
        parts = [shard(reqs, r, world) for r in range(world)]
        assert sorted(q.rid for p in parts for q in p) == sorted(q.rid for q in reqs)
        assert all(q.rid % world == r for r, p in enumerate(parts) for q in p)
    with pytest.raises(ValueError):
        shard(reqs, 2, 2)


def test_two_replicas_serve_everything():
    res, codes = _run_fleet("all_alive")
    ref = _single_engine_outputs()
    assert codes == [0, 0]
    for rank in range(WORLD):
        assert res[rank][0] == "ok" and res[rank][1] == ref


@pytest.mark.parametrize("mode", ["raises", "exits", "never_joins"])
def test_failed_replica_work_is_taken_over(mode):
    res, codes = _run_fleet(mode)
    ref = _single_engine_outputs()
    assert res[0][0] == "ok", res
    assert res[0][1] == ref
    if mode == "raises":
        assert res[1][0] == "error" and "injected" in res[1][1]
    if mode == "exits":
        assert codes[1] == 3 and 1 not in res
    assert any("failed" in line for line in res[0][2])
