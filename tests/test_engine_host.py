"""The engine's host bookkeeping, on CPU: with its device side replaced by doubles that
return the oracle's stub tokens, `Engine` must take exactly the reference Engine's
decisions (slot, position, length, padding, row moves, completion order)."""

from __future__ import annotations

import hashlib
import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import golden_json
from oracle.engine_ref import stub_token
from qweninfer_b200 import synthetic
from qweninfer_b200.engine.engine import Engine, Request
from qweninfer_b200.models.config import qwen2_0p5b

VOCAB = 1000


class StubCache:
    def __init__(self, cfg, rows, max_len, dtype=None, device=None):
        self.max_batch, self.max_len = rows, max_len
        self.row_start = self.window = 0

    def move_row(self, src, dst, length):
        assert 0 <= dst < src < self.max_batch and 0 < length <= self.max_len


class StubRunner:
    def __init__(self, model, cache, max_batch, cuda_graphs=True):
        self.cache, self.max_batch = cache, max_batch
        self.batches = []

    def prefill(self, row, prompt):
        assert 0 <= row < self.cache.max_batch
        return stub_token(prompt[-1], len(prompt) - 1, VOCAB)

    def prefill_many(self, rows, prompts):
        assert len(set(rows)) == len(rows)
        self.batches.append(len(rows))
        return [self.prefill(r, p) for r, p in zip(rows, prompts)]

    def decode(self, toks, pos, row_start=0):
        assert len(toks) <= self.max_batch
        return np.array([stub_token(t, p, VOCAB) for t, p in zip(toks, pos)])


class StubEngine(Engine):
    cache_cls = StubCache
    runner_cls = StubRunner


def fake_model():
    return SimpleNamespace(cfg=qwen2_0p5b(), dtype=torch.bfloat16,
                           norm=SimpleNamespace(weight=torch.empty(1)))


def canon_hash(obj) -> str:
    return hashlib.sha256(json.dumps(obj, separators=(",", ":")).encode()).hexdigest()


def run(reqs, **kw):
    eng = StubEngine(fake_model(), record=True, **kw)
    done = eng.run([Request(r.rid, list(r.prompt), r.max_new_tokens) for r in reqs])
    return eng.trace, {str(r.rid): r.output for r in done}, done


@pytest.mark.parametrize("name", ["serve96_slots32", "serve96_slots64_pad", "serve96_slots32_cap4",
                                  "serve96_slots16_static"])
def test_serving_trace_bit_exact(name):
    g = golden_json("sched_traces.json")[name]
    trace, outs, done = run(synthetic.serving96(), **g["kwargs"])
    if "trace" in g:
        assert trace == g["trace"]
    assert canon_hash(trace) == g["sha256"]
    assert canon_hash(outs) == g["outputs_sha256"]
    assert [r.rid for r in done] == sorted(r.rid for r in done)
    assert all(r.first_token is not None and r.finished >= r.first_token for r in done)


@pytest.mark.slow
def test_large_slice_trace_bit_exact():
    g = golden_json("sched_traces.json")["serve3072_rank0of8_slots128"]
    trace, _, _ = run(synthetic.serving3072(0, 8), **g["kwargs"])
    assert canon_hash(trace) == g["sha256"]


def test_small_engine_trace_structure_matches_reference():
    """The real-model reference runs (6 requests): same slots, positions and moves when the
    tokens are ignored (with no EOS, tokens never change a scheduling decision)."""
    gold = golden_json("engine_small.json")
    reqs = [SimpleNamespace(rid=i, prompt=p, max_new_tokens=n)
            for i, (p, n) in enumerate(zip(gold["prompts"], gold["max_new_tokens"]))]

    def strip(trace):
        return [{"admit": [a[:3] for a in t["admit"]],
                 "decode": None if t["decode"] is None else
                 [t["decode"][0], [[x[0], x[1], x[3]] for x in t["decode"][1]]],
                 "move": t["move"], "done": t["done"]} for t in trace]

    for name, r in gold["runs"].items():
        trace, _, _ = run(reqs, **r["kwargs"])
        assert strip(trace) == strip(r["trace"]), name


def test_submit_rejects_oversized_request():
    eng = StubEngine(fake_model(), max_slots=2, max_len=16)
    with pytest.raises(ValueError):
        eng.submit(Request(0, list(range(10)), 7))


def test_pad_to_validation():
    with pytest.raises(ValueError):
        StubEngine(fake_model(), max_slots=4, max_len=16, pad_to=[0, 1, 2])
    with pytest.raises(ValueError):
        StubEngine(fake_model(), max_slots=2, max_len=16, pad_to=[0, 1, 1])


def test_eos_stops_without_appending():
    eng = StubEngine(fake_model(), max_slots=2, max_len=64, eos_ids={stub_token(5, 2, VOCAB)})
    done = eng.run([Request(0, [1, 2, 5], 10)])
    assert done[0].output == []


def _trace_and_batches(reqs, **kw):
    eng = StubEngine(fake_model(), record=True, **kw)
    done = eng.run([Request(r.rid, list(r.prompt), r.max_new_tokens) for r in reqs])
    return eng.trace, {r.rid: r.output for r in done}, eng.runner.batches


@pytest.mark.parametrize("kw", [dict(max_slots=32, max_len=512),
                                dict(max_slots=32, max_len=512, max_prefills_per_step=4),
                                dict(max_slots=8, max_len=512, eos_ids={5, 77})])
def test_batched_prefill_takes_the_same_decisions(kw):
    """Prefilling a step's admissions together admits the same requests into the same
    rows with the same first tokens as the one-at-a-time loop (engine.py:115-138),
    including requests that finish at their first token (max_new_tokens = 1) and
    configurations with EOS ids, which fall back to one prefill per request."""
    reqs = [synthetic.SyntheticRequest(r.rid, r.prompt, 1 if r.rid % 7 == 3 else r.max_new_tokens)
            for r in synthetic.serving96()[:48]]
    t1, o1, b1 = _trace_and_batches(reqs, batch_prefill=True, **kw)
    t0, o0, b0 = _trace_and_batches(reqs, batch_prefill=False, **kw)
    assert t1 == t0 and o1 == o0
    assert b0 == []
    if "eos_ids" in kw:
        assert b1 == []
    else:
        assert max(b1) > 1
