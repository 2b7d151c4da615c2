"""Pin the numpy oracle to the reference: every golden vector in tests/golden was made by
running the reference package itself (tests/golden/make_golden.py)."""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from conftest import golden_json, golden_npz
from oracle import OracleModel, OracleRequest, oracle_generate
from oracle.engine_ref import OracleEngine, StubModel, pad_table
from oracle.qwen2_ref import build_rope_cache

# numpy vs torch fp32 on the same weights: different BLAS, different summation order.
ORACLE_LOGIT_ATOL = 1e-4
ORACLE_HIDDEN_RTOL = 1e-4


def canon_hash(obj) -> str:
    return hashlib.sha256(json.dumps(obj, separators=(",", ":")).encode()).hexdigest()


def test_rope_tables_match_reference():
    g = golden_npz("config0_fp32.npz")
    cos, sin = build_rope_cache(64, 4096, 1e6)
    rows = g["rope_rows"]
    assert np.abs(cos[rows] - g["rope_cos"]).max() < 1e-5
    assert np.abs(sin[rows] - g["rope_sin"]).max() < 1e-5
    # half-split convention: the two halves share their angles
    assert np.array_equal(cos[:, :32], cos[:, 32:])


@pytest.mark.parametrize("variant", ["fp32", "bf16w"])
def test_config0_matches_reference(variant, state_fp32, state_bf16w, full_cfg):
    """CPU reference run: 64-token prompt, prefill + 32 greedy tokens."""
    g = golden_npz(f"config0_{variant}.npz")
    state = state_fp32 if variant == "fp32" else state_bf16w
    model = OracleModel(state, vars(full_cfg))
    steps: list[np.ndarray] = []
    toks = oracle_generate(model, g["prompt"].tolist(), 32, step_logits=steps)
    assert toks == g["tokens"].tolist()
    L = np.stack(steps)
    sub = L[:, g["logit_idx"]]
    assert np.abs(sub - g["logits_sub"]).max() < ORACLE_LOGIT_ATOL
    assert np.array_equal(np.argmax(L, 1), g["top_idx"][:, 0])
    top_v = np.take_along_axis(L, g["top_idx"], 1)
    assert np.abs(top_v - g["top_val"]).max() < ORACLE_LOGIT_ATOL
    # whole-vector statistics (sum, sum of squares, max)
    L64 = L.astype(np.float64)
    st = np.stack([L64.sum(1), (L64 ** 2).sum(1), L64.max(1)], 1)
    assert np.allclose(st, g["stats"][:, :3], rtol=1e-4, atol=0.5)


def test_hidden_states_match_reference(state_bf16w, full_cfg):
    """Per-layer residual stream at two prompt positions (test_parity.py:195-261 analogue)."""
    g = golden_npz("config0_bf16w.npz")
    model = OracleModel(state_bf16w, vars(full_cfg))
    hidden: list[np.ndarray] = []
    model.forward(g["prompt"][None, :], hidden=hidden)
    got = np.stack([h[0, g["hidden_pos"]] for h in hidden[1:]])      # (24, 2, 896)
    ref = g["hidden"]
    scale = np.abs(ref).max(axis=-1, keepdims=True)
    rel = np.abs(got - ref) / scale
    bad = np.argwhere(rel.max(axis=(1, 2)) > ORACLE_HIDDEN_RTOL)
    assert bad.size == 0, f"first diverging layer {bad[0][0]}: rel {rel.max():.2e}"


def _requests(gold):
    return [OracleRequest(i, list(p), n) for i, (p, n) in enumerate(zip(gold["prompts"], gold["max_new_tokens"]))]


def test_engine_small_matches_reference(oracle_bf16w):
    """6 requests through 2-4 slots on the real model (test_cache.py:93-126 analogue):
    outputs and every scheduler action equal the reference Engine's."""
    gold = golden_json("engine_small.json")
    for i, (p, n) in enumerate(zip(gold["prompts"], gold["max_new_tokens"])):
        assert oracle_generate(oracle_bf16w, p, n) == gold["alone"][str(i)]
    for name, run in gold["runs"].items():
        eng = OracleEngine(oracle_bf16w, **run["kwargs"])
        done = eng.run(_requests(gold))
        assert {str(r.rid): r.output for r in done} == run["outputs"], name
        assert eng.trace == run["trace"], name
        # continuous batching does not change any request's output (test_cache.py:93-113)
        assert run["outputs"] == gold["alone"], name


def _stub_trace(reqs, kwargs):
    eng = OracleEngine(StubModel(1000), **kwargs)
    done = eng.run([OracleRequest(r.rid, r.prompt, r.max_new_tokens) for r in reqs])
    return eng.trace, {str(r.rid): r.output for r in done}


def test_scheduler_traces_match_reference():
    """Bookkeeping of the 96-request serving workload (and variants) is bit-exact."""
    from qweninfer_b200 import synthetic
    gold = golden_json("sched_traces.json")
    w96 = synthetic.serving96()
    for name in ["serve96_slots32", "serve96_slots64_pad", "serve96_slots32_cap4", "serve96_slots16_static"]:
        g = gold[name]
        kwargs = dict(g["kwargs"])
        trace, outs = _stub_trace(w96, kwargs)
        if "trace" in g:
            assert trace == g["trace"], name
        assert canon_hash(trace) == g["sha256"], name
        assert canon_hash(outs) == g["outputs_sha256"], name
    assert gold["serve96_slots64_pad"]["kwargs"]["pad_to"] == pad_table(64)


@pytest.mark.slow
def test_scheduler_trace_large_slice_matches_reference():
    """Rank 0 of 8 of the 3072-request workload: 128 slots, max_len 4096."""
    from qweninfer_b200 import synthetic
    g = golden_json("sched_traces.json")["serve3072_rank0of8_slots128"]
    trace, outs = _stub_trace(synthetic.serving3072(0, 8), g["kwargs"])
    assert canon_hash(trace) == g["sha256"]
    assert len([t for t in trace if t["decode"]]) == g["decode_steps"]
