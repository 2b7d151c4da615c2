"""The single-launch persistent forward (qi_persistent_plan / qi_persistent_launch, one
cooperative kernel walking a stage table) against the per-stage launches of qi_forward.

Both run the same epilogues and attention units. Up to 16 tokens they also use the same
token tile and stream-K partition, so logits, greedy tokens and the appended K/V must be
bitwise identical. Above that the persistent forward keeps all tokens in one tile while
the per-stage forward splits them into tiles of 16-32, which reassociates the k sums:
logits then agree to 1e-2 max-abs and cosine 0.99999 per row, and the cache per layer to fp32 drift plus bf16 rounding. The
oracle parity of the per-stage path is covered by test_model_gpu.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from qweninfer_b200.engine.kv_cache import KVCache
from qweninfer_b200.engine.runner import DecodeRunner

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _decode(model, cache, toks, pos, persistent, monkeypatch):
    monkeypatch.setenv("QI_PERSISTENT", "1" if persistent else "0")
    cache.k.zero_()
    cache.v.zero_()
    cache.row_start, cache.window = 0, int(pos.max()) + 1
    out = model(toks[:, None], positions=pos[:, None], cache=cache, logits_dtype=torch.float32)[:, -1]
    torch.cuda.synchronize()
    return out.clone(), cache.k.clone(), cache.v.clone()


def _close(ref, got):
    # different k-sum order through 24 layers: ~1e-3 typical, a few e-3 at the extreme of
    # 128 x 151936 logits; bounded like the model tests bound the fp32 reference
    assert (ref[0] - got[0]).abs().max().item() <= 1e-2
    cos = torch.nn.functional.cosine_similarity(ref[0].double(), got[0].double(), dim=-1)
    assert cos.min().item() >= 0.99999
    for a, b in ((ref[1], got[1]), (ref[2], got[2])):
        a, b = a.float().flatten(1), b.float().flatten(1)
        err = (a - b).abs().amax(dim=1) / a.abs().amax(dim=1).clamp_min(1e-6)
        # fp32 drift plus one bf16 rounding flip (one ulp is up to 2^-7 of the value)
        assert bool((err <= 3e-3 + 2 ** -7).all()), err.max().item()


@pytest.mark.parametrize("M", [1, 6, 16, 22, 64, 128])
def test_persistent_decode_matches(gpu_model, M, monkeypatch):
    rng = np.random.default_rng(100 + M)
    toks = torch.tensor(rng.integers(0, gpu_model.cfg.vocab_size, M), dtype=torch.long)
    pos = torch.tensor(rng.integers(0, 300, M), dtype=torch.long)
    cache = KVCache(gpu_model.cfg, M, 320, dtype=torch.bfloat16, device="cuda")
    ref = _decode(gpu_model, cache, toks, pos, False, monkeypatch)
    got = _decode(gpu_model, cache, toks, pos, True, monkeypatch)
    if M <= 16:
        assert torch.equal(ref[0], got[0]), (ref[0] - got[0]).abs().max().item()
        assert torch.equal(ref[1], got[1]) and torch.equal(ref[2], got[2])
    else:
        _close(ref, got)


def test_persistent_prefill_chunk_matches(gpu_model, monkeypatch):
    """A 100-token prefill of one row (M <= 128 runs as one persistent launch)."""
    rng = np.random.default_rng(7)
    prompt = torch.tensor(rng.integers(0, gpu_model.cfg.vocab_size, 100), dtype=torch.long)[None]
    outs = []
    for persistent in (False, True):
        monkeypatch.setenv("QI_PERSISTENT", "1" if persistent else "0")
        cache = KVCache(gpu_model.cfg, 1, 128, dtype=torch.bfloat16, device="cuda")
        cache.window = 100
        logits = gpu_model(prompt, positions=torch.arange(100), cache=cache, logits_dtype=torch.float32)[0]
        torch.cuda.synchronize()
        outs.append((logits, cache.k, cache.v))
    _close(outs[0], outs[1])


def test_persistent_runner_graphs_and_trace(gpu_model, monkeypatch):
    """Graph-captured persistent decode steps match the per-stage runner token for token,
    and the stage trace records a start before monotonically ordered stage finishes."""
    monkeypatch.setenv("QI_PERSISTENT", "0")
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, gpu_model.cfg.vocab_size, n).tolist() for n in (5, 17, 33)]
    seqs = {}
    for persistent in (False, True):
        monkeypatch.setenv("QI_PERSISTENT", "1" if persistent else "0")
        cache = KVCache(gpu_model.cfg, 3, 96, dtype=torch.bfloat16, device="cuda")
        r = DecodeRunner(gpu_model, cache, max_batch=3)
        toks = [r.prefill(i, p) for i, p in enumerate(prompts)]
        pos = [len(p) for p in prompts]
        out = [list(toks)]
        for _ in range(6):
            toks = [int(t) for t in r.decode(toks, pos)]
            pos = [x + 1 for x in pos]
            out.append(list(toks))
        r.check()
        seqs[persistent] = out
        if persistent:
            tr = r.ws.persist_trace.cpu().numpy().astype(np.int64)
            n = 1 + 5 * gpu_model.cfg.num_hidden_layers + 1
            assert tr[n] > 0 and tr[n] <= tr[0]
            assert np.all(np.diff(tr[:n]) >= 0)
    assert seqs[False] == seqs[True]
