"""The single-launch decode step (`qi_decode_step`, csrc/step.cu) on the GPU, through the C
ABI: logits and greedy tokens against the fp32 oracle and against the per-projection
launches of `qi_forward`, on ragged batches of 1..32 rows at mixed positions.

Bars: per step and row, max-abs logit error <= 3e-2 and cosine >= 0.9999 against the fp32
oracle on the same bf16 weights; <= 5e-3 against the oracle with a bf16 cache (the
storage rounding of the GPU cache) and against `qi_forward` (same arithmetic, another
summation order); greedy tokens equal wherever the reference margin exceeds the bar.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import LOGIT_ATOL, LOGIT_MIN_COS, golden_npz, logit_report, top2_margin
from oracle import OracleCache, oracle_generate
from qweninfer_b200 import _lib
from qweninfer_b200.engine.kv_cache import KVCache

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TIGHT_ATOL = 5e-3


class _Step:
    """Direct calls of qi_decode_step / qi_forward with fp32 logits for M tokens."""

    def __init__(self, model, cache, max_tokens: int = 32) -> None:
        self.model, self.cache = model, cache
        self.ws = model.workspace(max_tokens, cache.max_len)
        self.dev = torch.device("cuda")
        self.V = model.cfg.vocab_size

    def _io(self, toks, pos, rows):
        i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=self.dev)  # noqa: E731
        M = len(toks)
        logits = torch.full((M, self.V), float("nan"), device=self.dev)
        slots = torch.zeros(M, dtype=torch.int64, device=self.dev)
        return M, i32(toks), i32(pos), i32(rows), logits, slots

    def step(self, toks, pos, rows, expect_err: int = 0):
        M, t, p, r, logits, slots = self._io(toks, pos, rows)
        self.ws.plan(M)
        self.ws.err.zero_()
        _lib.check(_lib.lib().qi_decode_step(
            C.byref(self.model.native()), C.byref(self.cache.native()), C.byref(self.ws.struct),
            t.data_ptr(), p.data_ptr(), r.data_ptr(), M, logits.data_ptr(), 0, self.V, slots.data_ptr(),
            _lib.stream_ptr(self.dev)), "qi_decode_step")
        torch.cuda.synchronize()
        assert int(self.ws.err.item()) == expect_err
        idx = (0xFFFFFFFF - (slots.cpu().numpy() & 0xFFFFFFFF)).astype(np.int64)
        return logits.cpu().numpy(), idx

    def forward(self, toks, pos, rows):
        M, t, p, r, logits, slots = self._io(toks, pos, rows)
        self.ws.plan(M)
        _lib.check(_lib.lib().qi_forward(
            C.byref(self.model.native()), C.byref(self.cache.native()), C.byref(self.ws.struct),
            t.data_ptr(), p.data_ptr(), r.data_ptr(), M, 0, 1, M, logits.data_ptr(), 0, self.V, slots.data_ptr(),
            _lib.stream_ptr(self.dev)), "qi_forward")
        torch.cuda.synchronize()
        assert int(self.ws.err.item()) == 0
        return logits.cpu().numpy()


def _prefill(model, cache, rows, prompts):
    """Prompts into their cache rows through the model API (per-projection launches)."""
    for row, p in zip(rows, prompts):
        cache.row_start, cache.window = row, len(p)
        model(torch.tensor([p]), positions=torch.arange(len(p)), cache=cache, last_only=True)
    torch.cuda.synchronize()


def test_step_decode_matches_oracle(gpu_model, oracle_bf16w):
    """Config-0 prompt, then 32 single-row steps through qi_decode_step fed the reference's
    tokens: every step's logits vs the fp32 oracle and the bf16-cache oracle (whole vocabulary)."""
    g0 = golden_npz("config0_bf16w.npz")
    prompt, toks = g0["prompt"].tolist(), g0["tokens"].tolist()
    P = len(prompt)
    cache = KVCache(gpu_model.cfg, 1, P + 33, dtype=torch.bfloat16, device="cuda")
    _prefill(gpu_model, cache, [0], [prompt])
    run = _Step(gpu_model, cache)
    got = [run.step([t], [P + i], [0])[0][0] for i, t in enumerate(toks)]
    ref_f32, ref_b16 = [], []
    oracle_generate(oracle_bf16w, prompt, 32, step_logits=ref_f32)
    oracle_generate(oracle_bf16w, prompt, 32, step_logits=ref_b16, kv_bf16=True)
    for s, g in enumerate(got):
        d, cos = logit_report(g, ref_f32[s + 1])
        assert d <= LOGIT_ATOL and cos >= LOGIT_MIN_COS, (s, d, cos)
        assert np.abs(g - ref_b16[s + 1]).max() <= TIGHT_ATOL, s


@pytest.mark.parametrize("M", [1, 5, 8, 9, 16, 22, 32])
def test_step_matches_forward_on_ragged_batches(gpu_model, M):
    """One decode step of M rows at mixed positions: qi_decode_step vs qi_forward on the
    same cache contents (restored between the two), logits and argmax."""
    rng = np.random.default_rng(100 + M)
    lens = rng.integers(3, 90, M)
    prompts = [rng.integers(0, 151936, n).tolist() for n in lens]
    cache = KVCache(gpu_model.cfg, M, 128, dtype=torch.bfloat16, device="cuda")
    _prefill(gpu_model, cache, list(range(M)), prompts)
    k0, v0 = cache.k.clone(), cache.v.clone()
    run = _Step(gpu_model, cache)
    toks = rng.integers(0, 151936, M).tolist()
    pos, rows = [int(n) for n in lens], list(range(M))
    ref = run.forward(toks, pos, rows)
    k1, v1 = cache.k.clone(), cache.v.clone()
    cache.k.copy_(k0)
    cache.v.copy_(v0)
    got, idx = run.step(toks, pos, rows)
    assert np.abs(got - ref).max() <= TIGHT_ATOL
    for b in range(M):
        assert idx[b] == int(np.argmax(got[b]))
        if top2_margin(ref[b]) > 2 * TIGHT_ATOL:
            assert idx[b] == int(np.argmax(ref[b])), b
    # the appended K/V agree to a bf16 rounding step or two
    dk = (cache.k.float() - k1.float()).abs().max().item()
    dv = (cache.v.float() - v1.float()).abs().max().item()
    assert dk <= 2e-2 and dv <= 2e-2, (dk, dv)


def test_step_ragged_batch_matches_oracle(gpu_model, oracle_bf16w, full_cfg):
    """A ragged decode batch of 22 rows (the serving trace's mean batch) vs the oracle."""
    M = 22
    rng = np.random.default_rng(7)
    lens = rng.integers(8, 48, M)
    prompts = [rng.integers(0, 151936, n).tolist() for n in lens]
    max_len = 64
    cache = KVCache(gpu_model.cfg, M, max_len, dtype=torch.bfloat16, device="cuda")
    _prefill(gpu_model, cache, list(range(M)), prompts)
    ocache = OracleCache(vars(full_cfg), M, max_len, kv_bf16=True)
    for b, p in enumerate(prompts):
        ocache.row_start, ocache.window = b, len(p)
        oracle_bf16w.forward(np.array([p]), positions=np.arange(len(p)), cache=ocache, last_only=True)
    toks = rng.integers(0, 151936, M).tolist()
    pos = [int(n) for n in lens]
    ocache.row_start, ocache.window = 0, max(pos) + 1
    ref = oracle_bf16w.forward(np.array(toks)[:, None], positions=np.array(pos)[:, None], cache=ocache)[:, -1]
    got, idx = _Step(gpu_model, cache).step(toks, pos, list(range(M)))
    for b in range(M):
        d, cos = logit_report(got[b], ref[b])
        assert d <= LOGIT_ATOL and cos >= LOGIT_MIN_COS, (b, d, cos)
        if top2_margin(ref[b]) > LOGIT_ATOL:
            assert idx[b] == int(np.argmax(ref[b])), b


def test_step_reports_out_of_cache_position(gpu_model):
    """A row whose position lies outside the cache is reported (QI_ERR_INDEX); nothing is
    written for it and the other rows' results are unchanged."""
    rng = np.random.default_rng(9)
    M, max_len = 4, 64
    prompts = [rng.integers(0, 151936, n).tolist() for n in (5, 9, 7, 11)]
    cache = KVCache(gpu_model.cfg, M, max_len, dtype=torch.bfloat16, device="cuda")
    _prefill(gpu_model, cache, list(range(M)), prompts)
    k0, v0 = cache.k.clone(), cache.v.clone()
    run = _Step(gpu_model, cache)
    toks = [11, 22, 33, 44]
    pos = [5, 9, 7, 11]
    good, _ = run.step(toks, pos, list(range(M)))
    cache.k.copy_(k0)
    cache.v.copy_(v0)
    bad_pos = list(pos)
    bad_pos[2] = max_len
    got, _ = run.step(toks, bad_pos, list(range(M)), expect_err=_lib.QI_ERR_INDEX)
    keep = [0, 1, 3]
    assert np.abs(got[keep] - good[keep]).max() == 0.0
    assert torch.equal(cache.k[:, 2], k0[:, 2]) and torch.equal(cache.v[:, 2], v0[:, 2])
