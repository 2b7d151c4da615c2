"""qi_attention_noalloc: attention for callers that cannot allocate device memory (for
example a C or Go program binding libqi.so that only holds device pointers to its own
tensors, or a service whose device memory is fixed at start-up). Its scratch lives in a
static array inside the library, so the caller passes only inputs and outputs.

Checked through the C ABI against qi_attention (the same kernel with caller-provided
scratch) on two calls in a row with different shapes — the second call sees whatever the
first left in the shared array — and for rejection of sizes beyond the fixed capacity.
Kept in its own file, collected last, and self-contained (fresh process or after the
other tests).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bf16_round
from qweninfer_b200 import _lib

pytestmark = pytest.mark.gpu

ATOL = 1e-5  # the attention kernel's tolerance in tests/test_kernels_gpu.py


def _case(M: int, max_len: int, seed: int):
    rng = np.random.default_rng(seed)
    rows_total = 3
    kc = bf16_round(rng.standard_normal((rows_total, 2, max_len, 64)).astype(np.float32))
    vc = bf16_round(rng.standard_normal((rows_total, 2, max_len, 64)).astype(np.float32))
    q = (2 * rng.standard_normal((M, 896))).astype(np.float32)
    pos = rng.integers(0, max_len, M)
    pos[0] = max_len - 1  # a query that reads every slot of its row
    rows = rng.integers(0, rows_total, M)
    dev = torch.device("cuda")
    t = dict(
        q=torch.from_numpy(q).to(dev),
        k=torch.from_numpy(kc).to(torch.bfloat16).to(dev),
        v=torch.from_numpy(vc).to(torch.bfloat16).to(dev),
        pos=torch.from_numpy(pos.astype(np.int32)).to(dev),
        rows=torch.from_numpy(rows.astype(np.int32)).to(dev),
    )
    return t


def _with_scratch(t, M, max_len):
    from qweninfer_b200.models.qwen2 import _AttnScratch
    ws = _AttnScratch(M, max_len, torch.device("cuda"))
    out = torch.empty(M, 896, device="cuda")
    _lib.check(_lib.lib().qi_attention(
        t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["pos"].data_ptr(), t["rows"].data_ptr(),
        M, max_len, ws.split_keys, ws.max_splits, out.data_ptr(), ws.part.data_ptr(), ws.counters.data_ptr(),
        ws.err.data_ptr(), _lib.stream_ptr()), "qi_attention")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _without_scratch(t, M, max_len, with_err: bool = True, expect_err: int = 0):
    out = torch.full((M, 896), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda") if with_err else None
    _lib.check(_lib.lib().qi_attention_noalloc(
        t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["pos"].data_ptr(), t["rows"].data_ptr(),
        M, max_len, out.data_ptr(), None if err is None else err.data_ptr(), _lib.stream_ptr()),
        "qi_attention_noalloc")
    torch.cuda.synchronize()
    if err is not None:
        assert int(err.item()) == expect_err
    return out.cpu().numpy()


def test_attention_without_allocation_matches_scratch_variant():
    _lib.ensure_device(torch.device("cuda", torch.cuda.current_device()))
    # two calls in a row, different shapes: the second reuses the shared array
    for M, max_len, seed in [(40, 2048, 1), (5, 700, 2)]:
        t = _case(M, max_len, seed)
        ref = _with_scratch(t, M, max_len)
        got = _without_scratch(t, M, max_len)
        assert np.abs(got - ref).max() <= ATOL, (M, max_len)


def test_attention_without_allocation_accepts_null_err():
    """`err` may be NULL (include/qi.h): valid inputs give the same output."""
    _lib.ensure_device(torch.device("cuda", torch.cuda.current_device()))
    M, max_len = 6, 300
    t = _case(M, max_len, 3)
    ref = _with_scratch(t, M, max_len)
    got = _without_scratch(t, M, max_len, with_err=False)
    assert np.abs(got - ref).max() <= ATOL


def test_attention_without_allocation_reports_out_of_cache_position():
    """A position outside the cache is reported as QI_ERR_INDEX in `err`; nothing is read
    or written for that token and every other token's output is unchanged."""
    _lib.ensure_device(torch.device("cuda", torch.cuda.current_device()))
    M, max_len, bad = 5, 400, 2
    t = _case(M, max_len, 4)
    ref = _with_scratch(t, M, max_len)
    t["pos"][bad] = max_len  # one past the last slot of its row
    got = _without_scratch(t, M, max_len, expect_err=_lib.QI_ERR_INDEX)
    keep = [i for i in range(M) if i != bad]
    assert np.abs(got[keep] - ref[keep]).max() <= ATOL
    assert np.isnan(got[bad]).all()  # the bad token's output is left as it was


def test_attention_without_allocation_rejects_oversized_calls():
    _lib.ensure_device(torch.device("cuda", torch.cuda.current_device()))
    L = _lib.lib()
    s = _lib.stream_ptr()
    assert L.qi_attention_noalloc(1, 1, 1, 1, 1, 65, 512, 1, None, s) == _lib.QI_ERR_TOO_LARGE
    assert L.qi_attention_noalloc(1, 1, 1, 1, 1, 4, 2049, 1, None, s) == _lib.QI_ERR_TOO_LARGE
