"""Host-side launch plans of the forward (no GPU needed): attention key splits and the
token tiles of the tensor-core projections. The kernels rely on these invariants: every
key of a row is covered by some split, a decode launch whose splits merge inside one
thread-block cluster has at most 8 of them, split sizes are whole 128-key tiles, and the
token tiles never shrink as the token count grows (a workspace sized for its largest
forward then covers every smaller one)."""

from __future__ import annotations

import pytest

from qweninfer_b200.models.qwen2 import _split_plan, gate_up_tile, token_tile


@pytest.mark.parametrize("max_len", [1, 96, 128, 129, 512, 1000, 1024, 1025, 2048, 4096, 32768])
@pytest.mark.parametrize("M", [1, 22, 64, 65, 128, 129, 512])
def test_split_plan_covers_every_key(M, max_len):
    split, n = _split_plan(M, max_len)
    assert split % 128 == 0 and split >= 128
    assert n >= 1 and split * n >= max_len
    assert split * (n - 1) < max_len  # no split that can never hold a key
    assert n <= 128  # the merge's capacity


@pytest.mark.parametrize("M", [1, 22, 128])
@pytest.mark.parametrize("max_len", [96, 256, 512, 1000, 1024])
def test_short_rows_are_one_split(M, max_len):
    split, n = _split_plan(M, max_len)
    assert n == 1 and split >= max_len


@pytest.mark.parametrize("M,plan", [(1, (512, 8)), (32, (512, 8)), (33, (2048, 2)), (64, (2048, 2)),
                                    (128, (2048, 2))])
def test_long_context_decode_splits(M, plan):
    """Up to batch 32 the splits of a 4096-slot row fill one thread-block cluster (8)."""
    assert _split_plan(M, 4096) == plan


def test_prefill_splits_are_coarse():
    assert _split_plan(512, 512) == (512, 1)
    assert _split_plan(129, 4096) == (4096, 1)
    assert _split_plan(4096, 8192) == (4096, 2)


@pytest.mark.parametrize("rule", [token_tile, gate_up_tile])
def test_token_tiles_non_decreasing_powers_of_two(rule):
    prev = 0
    for M in range(1, 2049):
        t = rule(M)
        assert 8 <= t <= 128 and t & (t - 1) == 0
        assert t >= prev, M
        prev = t


def test_token_tile_rules():
    assert [token_tile(M) for M in (1, 8, 9, 96, 97, 384, 385)] == [8, 8, 16, 16, 32, 32, 64]
    assert [gate_up_tile(M) for M in (1, 8, 9, 32, 33, 384, 385)] == [8, 8, 32, 32, 64, 64, 128]
