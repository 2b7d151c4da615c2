"""Whole-model parity at the configurations the benchmarks run, against the fp32 oracle on
the same bf16-rounded weights (the reference's fp32 path; tests/golden pins the oracle).

* Batch-1 decode at contexts of 256 and 1024 tokens (the seed-2 prompts of the batch-1
  latency benchmark): prefill, then 128 decode steps fed the oracle's greedy tokens; the
  logits of every 8th step are compared over the whole vocabulary.
* Ragged decode batches of 22 rows (the serving trace's mean batch) and 128 rows (the
  scaled trace's slot count) at mixed positions, one batched step after per-row prefills.

Bar: max-abs logit error <= 3e-2 and cosine >= 0.9999 per step and row; greedy tokens equal
wherever the oracle's top-2 margin exceeds 3e-2 (the tolerance qweninfer's parity tests
use for its own bf16 path, restated in conftest.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import LOGIT_ATOL, LOGIT_MIN_COS, logit_report, top2_margin
from oracle import OracleCache
from qweninfer_b200 import synthetic
from qweninfer_b200.engine.kv_cache import KVCache

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _check(got: np.ndarray, ref: np.ndarray, what) -> None:
    d, cos = logit_report(got, ref)
    assert d <= LOGIT_ATOL and cos >= LOGIT_MIN_COS, (what, d, cos)
    if top2_margin(ref) > LOGIT_ATOL:
        assert int(np.argmax(got)) == int(np.argmax(ref)), what


@pytest.mark.parametrize("context", [256, 1024])
def test_batch1_decode_at_context(gpu_model, oracle_bf16w, full_cfg, context):
    prompt = synthetic.decode_latency_prompts()[context]
    P, steps = len(prompt), 128
    ocache = OracleCache(vars(full_cfg), 1, P + steps + 1)
    ocache.window = P
    ref = oracle_bf16w.forward(np.array([prompt]), positions=np.arange(P), cache=ocache, last_only=True)[0, -1]
    cache = KVCache(gpu_model.cfg, 1, P + steps + 1, dtype=torch.bfloat16, device="cuda")
    cache.window = P
    got = gpu_model(torch.tensor([prompt]), positions=torch.arange(P), cache=cache, last_only=True,
                    logits_dtype=torch.float32)[0, -1].cpu().numpy()
    _check(got, ref, ("prefill", context))
    for i in range(steps):
        tok = int(np.argmax(ref))  # the oracle's greedy token drives both
        pos = P + i
        ocache.window = cache.window = pos + 1
        ref = oracle_bf16w.forward(np.array([[tok]]), positions=np.array([[pos]]), cache=ocache)[0, -1]
        got = gpu_model(torch.tensor([[tok]]), positions=torch.tensor([[pos]]), cache=cache,
                        logits_dtype=torch.float32)[0, -1]
        if i % 8 == 7:
            _check(got.cpu().numpy(), ref, (context, i))


@pytest.mark.parametrize("B", [22, 128])
def test_ragged_decode_batch(gpu_model, oracle_bf16w, full_cfg, B):
    rng = np.random.default_rng(500 + B)
    lens = rng.integers(4, 64, B)
    prompts = [rng.integers(0, full_cfg.vocab_size, n).tolist() for n in lens]
    max_len = 80
    cache = KVCache(gpu_model.cfg, B, max_len, dtype=torch.bfloat16, device="cuda")
    ocache = OracleCache(vars(full_cfg), B, max_len)
    for b, p in enumerate(prompts):
        cache.row_start = ocache.row_start = b
        cache.window = ocache.window = len(p)
        gpu_model(torch.tensor([p]), positions=torch.arange(len(p)), cache=cache, last_only=True)
        oracle_bf16w.forward(np.array([p]), positions=np.arange(len(p)), cache=ocache, last_only=True)
    toks = rng.integers(0, full_cfg.vocab_size, B)
    pos = lens.astype(np.int64)
    cache.row_start = ocache.row_start = 0
    cache.window = ocache.window = int(pos.max()) + 1
    ref = oracle_bf16w.forward(toks[:, None], positions=pos[:, None], cache=ocache)[:, -1]
    got = gpu_model(torch.tensor(toks[:, None]), positions=torch.tensor(pos[:, None]), cache=cache,
                    logits_dtype=torch.float32)[:, -1].cpu().numpy()
    for b in range(B):
        _check(got[b], ref[b], ("row", b))
