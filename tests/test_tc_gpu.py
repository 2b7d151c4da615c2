"""Tensor-core projection path (tcgen05 UMMA, TMEM, stream-K) through the C ABI.

qi_act_tiles must produce the documented activation-tile layout bit for bit;
qi_tc_linear must match an fp64 x @ W^T (optionally RMS-normalised) for every token
count, inner size and stream-K partition, and a token's result must not depend on how
many other tokens share the launch (batch invariance of the engine's decode).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import bf16_round, rmsnorm
from qweninfer_b200 import _lib
from qweninfer_b200.models.qwen2 import tile_weight


def token_tile(M: int) -> int:
    """Every valid token tile is exercised: the power of two >= M, 8..128 (the forward's own
    choice is smaller; the kernels accept any of them)."""
    nt = 8
    while nt < M and nt < 128:
        nt *= 2
    return nt


DEV = "cuda"
_KEEP: list[torch.Tensor] = []


def dev(t: torch.Tensor) -> torch.Tensor:
    t = t.to(DEV)
    _KEEP.append(t)
    return t


@pytest.fixture(autouse=True)
def _keep_alive():
    yield
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    _KEEP.clear()


def act_offset(t, k, part, K, NT):
    nt, tl = t // NT, t % NT
    return ((nt * (K // 64) + (k >> 6)) * (2 * NT * 64) + part * NT * 64 + (tl >> 3) * 512
            + ((k & 63) >> 3) * 64 + (tl & 7) * 8 + (k & 7))


def host_act_tiles(x: np.ndarray, NT: int, norm_w=None) -> np.ndarray:
    """Expected qi_act_tiles output as uint16 bf16 bit patterns."""
    M, K = x.shape
    Mp = -(-M // NT) * NT
    v = np.zeros((Mp, K), np.float32)
    v[:M] = x * (norm_w if norm_w is not None else 1.0)
    hi = bf16_round(v)
    lo = bf16_round(v - hi)
    out = np.zeros(Mp * K * 2, np.uint16)
    t, k = np.meshgrid(np.arange(Mp), np.arange(K), indexing="ij")
    for part, arr in ((0, hi), (1, lo)):
        out[act_offset(t, k, part, K, NT)] = (arr.view(np.uint32) >> 16).astype(np.uint16)
    return out


# ------------------------------------------------ stream-K arithmetic (host mirror)

def test_stream_k_partition_arithmetic():
    """Every unit has one owner; a tile's contributors are owner(first)..owner(last); each
    contributor's partial lands in a distinct (cta, slot) with at most 2 slots per CTA."""
    for KB in (1, 14, 76):
        for tiles in (1, 7, 9, 76, 1187):
            U = KB * tiles
            for G in sorted({1, 2, 3, 7, 63, 126, 148, U}):
                if G > U:
                    continue
                start = [c * U // G for c in range(G + 1)]
                owner = lambda u: ((u + 1) * G - 1) // U  # noqa: E731
                for u in range(0, U, max(1, U // 500)):
                    c = owner(u)
                    assert start[c] <= u < start[c + 1]
                used = set()
                for T in range(tiles):
                    cf, cl = owner(T * KB), owner(T * KB + KB - 1)
                    if cf == cl:
                        continue
                    for cc in range(cf, cl + 1):
                        slot = 0 if start[cc] >= T * KB else 1
                        assert (cc, slot) not in used
                        used.add((cc, slot))


# ------------------------------------------------------------------- GPU tests

@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(1, 896), (5, 896), (22, 896), (130, 896), (7, 4864)])
def test_act_tiles_layout(M, K):
    _lib.ensure_device(torch.device(DEV, 0))
    rng = np.random.default_rng(M + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32) if K == 896 else None
    NT = token_tile(M)
    Mp = -(-M // NT) * NT
    act = dev(torch.full((Mp * K * 2,), 7, dtype=torch.int16))
    ss = dev(torch.full((7 * Mp,), -1.0)) if K == 896 else None
    _lib.check(_lib.lib().qi_act_tiles(dev(torch.from_numpy(x)).data_ptr(),
                                       None if w is None else dev(torch.from_numpy(w)).data_ptr(), M, K, NT,
                                       act.data_ptr(), None if ss is None else ss.data_ptr(), Mp,
                                       _lib.stream_ptr()), "act_tiles")
    got = act.cpu().numpy().view(np.uint16)
    assert np.array_equal(got, host_act_tiles(x, NT, w))
    if ss is not None:
        s = ss.cpu().numpy().reshape(7, Mp)
        assert np.allclose(s[0, :M], (x.astype(np.float64) ** 2).sum(1), rtol=1e-5)
        assert np.all(s[1:, :M] == 0)


def _tc_linear(w_bf: np.ndarray, x: np.ndarray, ctas=0, norm_w=None):
    n_rows, K = w_bf.shape
    M = x.shape[0]
    NT = token_tile(M)
    Mp = -(-M // NT) * NT
    act = dev(torch.zeros(Mp * K * 2, dtype=torch.int16))
    ss = dev(torch.zeros(7 * Mp)) if norm_w is not None else None
    L = _lib.lib()
    s = _lib.stream_ptr()
    _lib.check(L.qi_act_tiles(dev(torch.from_numpy(x)).data_ptr(),
                              None if norm_w is None else dev(torch.from_numpy(norm_w)).data_ptr(), M, K, NT,
                              act.data_ptr(), None if ss is None else ss.data_ptr(), Mp, s), "act_tiles")
    wt = dev(tile_weight(torch.from_numpy(w_bf).to(torch.bfloat16)))
    out = dev(torch.full((M, n_rows), float("nan")))
    scratch = dev(torch.empty(148 * 2 * 128 * NT))
    counters = dev(torch.zeros(4096, dtype=torch.int32))
    err = dev(torch.zeros(1, dtype=torch.int32))
    _lib.check(L.qi_tc_linear(wt.data_ptr(), n_rows, K, act.data_ptr(), M, NT,
                              None if ss is None else ss.data_ptr(), Mp, C.c_float(1e-6), out.data_ptr(), n_rows,
                              scratch.data_ptr(), scratch.numel(), counters.data_ptr(), 4096, ctas, err.data_ptr(),
                              s), "tc_linear")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(counters.abs().sum()) == 0, "stream-K counters must be left at zero"
    return out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8, 9, 22, 64, 100, 128, 200, 300])
@pytest.mark.parametrize("n_rows,K", [(1152, 896), (896, 4864)])
def test_tc_linear_matches_fp64(M, n_rows, K):
    _lib.ensure_device(torch.device(DEV, 0))
    rng = np.random.default_rng(M * 7 + K)
    w = bf16_round(rng.normal(0, 0.02, (n_rows, K)).astype(np.float32))
    x = rng.standard_normal((M, K)).astype(np.float32)
    got = _tc_linear(w, x)
    ref = x.astype(np.float64) @ w.T.astype(np.float64)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 2e-5, err


@pytest.mark.gpu
@pytest.mark.parametrize("ctas", [1, 2, 5, 13, 64, 148])
def test_tc_linear_stream_k_partitions(ctas):
    """Tiles split across 1..14 contributors (fix-up by the last arrival) and CTAs that
    span tile boundaries give the same product."""
    _lib.ensure_device(torch.device(DEV, 0))
    rng = np.random.default_rng(ctas)
    w = bf16_round(rng.normal(0, 0.02, (1152, 896)).astype(np.float32))
    x = rng.standard_normal((22, 896)).astype(np.float32)
    got = _tc_linear(w, x, ctas=ctas)
    ref = x.astype(np.float64) @ w.T.astype(np.float64)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-5


@pytest.mark.gpu
def test_tc_linear_rms_folding():
    """Norm weight folded into the activations, per-token RMS applied in the epilogue."""
    _lib.ensure_device(torch.device(DEV, 0))
    rng = np.random.default_rng(11)
    w = bf16_round(rng.normal(0, 0.02, (1152, 896)).astype(np.float32))
    nw = bf16_round((1 + 0.1 * rng.standard_normal(896)).astype(np.float32))
    x = (3 * rng.standard_normal((13, 896))).astype(np.float32)
    got = _tc_linear(w, x, norm_w=nw)
    ref = rmsnorm(x, nw, 1e-6).astype(np.float64) @ w.T.astype(np.float64)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-5


@pytest.mark.gpu
def test_tc_linear_batch_invariant():
    """A token's output does not depend on the other tokens of the launch (token tile 8,
    32 or 128): the engine's batched decode equals each request decoded alone."""
    _lib.ensure_device(torch.device(DEV, 0))
    rng = np.random.default_rng(12)
    w = bf16_round(rng.normal(0, 0.02, (9728, 896)).astype(np.float32))
    x = rng.standard_normal((100, 896)).astype(np.float32)
    full = _tc_linear(w, x)
    for M in (1, 5, 22):
        part = _tc_linear(w, x[:M])
        assert np.array_equal(part, full[:M]), M


def decode_act_tiles(act: np.ndarray, M: int, K: int, NT: int) -> np.ndarray:
    """hi + lo of activation tiles (uint16 bf16 bit patterns) as fp32 (M, K)."""
    t, k = np.meshgrid(np.arange(M), np.arange(K), indexing="ij")
    hi = (act[act_offset(t, k, 0, K, NT)].astype(np.uint32) << 16).view(np.float32)
    lo = (act[act_offset(t, k, 1, K, NT)].astype(np.uint32) << 16).view(np.float32)
    return hi + lo


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 22, 100])
def test_tc_gate_up_swiglu_matches_fp64(M):
    """qi_tc_gate_up_swiglu (the forward's gate/up launch): RMSNorm folded, interleaved
    gate/up rows, SwiGLU, activation tiles for the down projection."""
    _lib.ensure_device(torch.device(DEV, 0))
    rng = np.random.default_rng(40 + M)
    wg = bf16_round(rng.normal(0, 0.02, (4864, 896)).astype(np.float32))
    wu = bf16_round(rng.normal(0, 0.02, (4864, 896)).astype(np.float32))
    w = np.empty((9728, 896), np.float32)  # the fused layout: gate row 2i, up row 2i+1
    w[0::2], w[1::2] = wg, wu
    nw = bf16_round((1 + 0.1 * rng.standard_normal(896)).astype(np.float32))
    x = (2 * rng.standard_normal((M, 896))).astype(np.float32)
    NT = token_tile(M)
    Mp = -(-M // NT) * NT
    L = _lib.lib()
    s = _lib.stream_ptr()
    act = dev(torch.zeros(Mp * 896 * 2, dtype=torch.int16))
    ss = dev(torch.zeros(7 * Mp))
    _lib.check(L.qi_act_tiles(dev(torch.from_numpy(x)).data_ptr(), dev(torch.from_numpy(nw)).data_ptr(), M, 896, NT,
                              act.data_ptr(), ss.data_ptr(), Mp, s), "act_tiles")
    wt = dev(tile_weight(torch.from_numpy(w).to(torch.bfloat16)))
    out = dev(torch.zeros(Mp * 4864 * 2, dtype=torch.int16))
    scratch = dev(torch.empty(148 * 2 * 128 * NT))
    counters = dev(torch.zeros(4096, dtype=torch.int32))
    err = dev(torch.zeros(1, dtype=torch.int32))
    _lib.check(L.qi_tc_gate_up_swiglu(wt.data_ptr(), act.data_ptr(), M, NT, ss.data_ptr(), Mp, C.c_float(1e-6),
                                      out.data_ptr(), scratch.data_ptr(), scratch.numel(), counters.data_ptr(), 4096,
                                      0, err.data_ptr(), s), "tc_gate_up_swiglu")
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(counters.abs().sum()) == 0
    got = decode_act_tiles(out.cpu().numpy().view(np.uint16), M, 4864, NT)
    xn = rmsnorm(x, nw, 1e-6).astype(np.float64)
    g, u = xn @ wg.T.astype(np.float64), xn @ wu.T.astype(np.float64)
    ref = g / (1 + np.exp(-g)) * u
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-5
