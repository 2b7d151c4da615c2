"""Per-kernel parity on the GPU, through the C ABI, against the numpy oracle on the same
seeded inputs (bf16-valued weights and caches, fp32 arithmetic on both sides).

Tolerances: fp32 component ops 2e-5 absolute (the reference's own component tolerance,
test_parity.py:43); kernels that write the bf16 cache are compared with one bf16 ulp.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import bf16_round, rmsnorm
from oracle.qwen2_ref import apply_rope as oracle_rope
from qweninfer_b200 import _lib
from qweninfer_b200.models.qwen2 import (MLP, RMSNorm, apply_rope, build_rope_cache, rope_pair_order,
                                         tile_weight)
from qweninfer_b200.models.config import qwen2_0p5b

pytestmark = pytest.mark.gpu

TOL_F32 = 2e-5
DEV = "cuda"


def bf16_tensor(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


# Device buffers handed to the C ABI as raw pointers must outlive the asynchronous
# launch: every helper below keeps its tensor referenced until the test has synchronised.
_KEEP: list[torch.Tensor] = []


def dev(t: torch.Tensor) -> torch.Tensor:
    t = t.to(DEV)
    _KEEP.append(t)
    return t


def f32(a) -> torch.Tensor:
    return dev(torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)))


def i32(a) -> torch.Tensor:
    return dev(torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)))


def stream() -> int:
    return _lib.stream_ptr(torch.device(DEV))


@pytest.fixture(scope="module", autouse=True)
def _init():
    _lib.ensure_device(torch.device(DEV, torch.cuda.current_device()))


@pytest.fixture(autouse=True)
def _keep_alive():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def err_word() -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=DEV)


def assert_no_device_error(err: torch.Tensor) -> None:
    torch.cuda.synchronize()
    assert int(err.item()) == 0


# ------------------------------------------------------------------ components

def test_rmsnorm_kernel():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 896)).astype(np.float32)
    w = (rng.standard_normal(896) * 0.1 + 1.0).astype(np.float32)
    mod = RMSNorm(896, 1e-6).to(DEV)
    with torch.no_grad():
        mod.weight.copy_(torch.from_numpy(w))
    got = mod(f32(x)).cpu().numpy()
    assert np.abs(got - rmsnorm(x, w, 1e-6)).max() < TOL_F32


def test_rope_kernel_half_split_convention():
    rng = np.random.default_rng(1)
    B, S = 2, 11
    q = rng.standard_normal((B, 14, S, 64)).astype(np.float32)
    k = rng.standard_normal((B, 2, S, 64)).astype(np.float32)
    pos = rng.integers(0, 4096, (B, S))
    cos, sin = build_rope_cache(64, 4096, 1e6)
    gq, gk = apply_rope(f32(q), f32(k), cos, sin, torch.from_numpy(pos))
    eq, ek = oracle_rope(q, k, cos.numpy(), sin.numpy(), pos)
    assert np.abs(gq.cpu().numpy() - eq).max() < TOL_F32
    assert np.abs(gk.cpu().numpy() - ek).max() < TOL_F32


def test_mlp_kernels():
    cfg = qwen2_0p5b(1, 256)
    torch.manual_seed(0)
    mlp = MLP(cfg)
    with torch.no_grad():
        for p in mlp.parameters():
            p.normal_(0, 0.02)
    wg = bf16_round(mlp.gate_proj.weight.detach().numpy())
    wu = bf16_round(mlp.up_proj.weight.detach().numpy())
    wd = bf16_round(mlp.down_proj.weight.detach().numpy())
    mlp.fuse()
    mlp.to(DEV)
    rng = np.random.default_rng(2)
    for M in (1, 3, 8, 13):
        x = rng.standard_normal((M, 896)).astype(np.float32)
        got = mlp(f32(x)).cpu().numpy()
        g, u = x @ wg.T, x @ wu.T
        ref = ((g / (1 + np.exp(-g))) * u) @ wd.T
        assert np.abs(got - ref).max() < TOL_F32 * max(1.0, np.abs(ref).max()), M


# ------------------------------------------------------- fused projection ops

def _qkv_setup(seed=3):
    rng = np.random.default_rng(seed)
    w = bf16_round(rng.normal(0, 0.02, (1152, 896)).astype(np.float32))
    b = bf16_round(rng.normal(0, 0.02, 1152).astype(np.float32))
    ln = bf16_round((1.0 + rng.normal(0, 0.1, 896)).astype(np.float32))
    order = rope_pair_order(18).numpy()
    w_t = tile_weight(bf16_tensor(w)[order]).to(DEV)
    b_t = f32(b[order])
    return rng, w, b, ln, w_t, b_t


@pytest.mark.parametrize("M", [1, 2, 5, 9, 40])
def test_qkv_rope_append(M):
    rng, w, b, ln, w_t, b_t = _qkv_setup()
    rows_total, max_len = 6, 300
    x = rng.standard_normal((M, 896)).astype(np.float32) * 3
    pos = rng.integers(0, max_len, M)
    rows = rng.integers(0, rows_total, M)
    # distinct (row, pos) slots so the expected cache content is unambiguous
    pos = (np.arange(M) * 7 + pos) % max_len
    rows = np.arange(M) % rows_total
    cos, sin = build_rope_cache(64, 4096, 1e6)
    kc = torch.zeros(rows_total, 2, max_len, 64, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = torch.empty(M, 896, device=DEV)
    err = err_word()
    _lib.check(_lib.lib().qi_qkv_rope_append(
        f32(x).data_ptr(), f32(ln).data_ptr(), C.c_float(1e-6), w_t.data_ptr(), b_t.data_ptr(),
        dev(cos).data_ptr(), dev(sin).data_ptr(), i32(pos).data_ptr(), i32(rows).data_ptr(), M,
        kc.data_ptr(), vc.data_ptr(), max_len, q.data_ptr(), err.data_ptr(), stream()), "qkv")
    assert_no_device_error(err)
    xn = rmsnorm(x, ln, 1e-6)
    qkv = xn @ w.T + b
    qh = qkv[:, :896].reshape(M, 14, 1, 64).transpose(0, 1, 2, 3)
    kh = qkv[:, 896:1024].reshape(M, 2, 1, 64)
    vh = qkv[:, 1024:].reshape(M, 2, 64)
    eq, ek = oracle_rope(qh, kh, cos.numpy(), sin.numpy(), pos[:, None])
    assert np.abs(q.cpu().numpy() - eq.reshape(M, 896)).max() < TOL_F32 * 10
    kc_h = kc.float().cpu().numpy()
    vc_h = vc.float().cpu().numpy()
    for t in range(M):
        gk = kc_h[rows[t], :, pos[t]]
        gv = vc_h[rows[t], :, pos[t]]
        assert np.all(np.abs(gk - ek[t, :, 0]) <= np.abs(ek[t, :, 0]) * 2 ** -8 + 1e-6), t
        assert np.all(np.abs(gv - vh[t]) <= np.abs(vh[t]) * 2 ** -8 + 1e-6), t
    # nothing else was written
    written = np.zeros((rows_total, max_len), bool)
    written[rows, pos] = True
    k_slots = kc_h.transpose(0, 2, 1, 3)   # (rows, max_len, 2, 64)
    v_slots = vc_h.transpose(0, 2, 1, 3)
    assert np.all(k_slots[~written] == 0) and np.all(v_slots[~written] == 0)


@pytest.mark.parametrize("M,max_len,positions", [
    (1, 64, [0]),
    (1, 1024, [1023]),
    (3, 512, [5, 127, 128]),
    (5, 1024, [0, 129, 255, 256, 1000]),
    (70, 700, None),
    # the scaled serving cache (max_len 4096): up to 32 queries 8 splits of 512 keys merged in
    # a cluster, more queries 2 splits of 2048
    (2, 4096, [4095, 2047]),
    (64, 4096, None),
    (128, 4096, None),
    # 16 splits of 512: merged by the last-arriving split through global scratch
    (4, 8192, [8191, 5000, 100, 4096]),
])
def test_attention_ragged(M, max_len, positions):
    """The per-token kernel (decode batches and short prompts) against an fp64 reference.
    Its tensor-core products carry q and p as hi/lo bf16 pairs (~16 mantissa bits), so the
    bar is the reference's own fp32 component tolerance, 2e-5 (measured up to 1.3e-5)."""
    from qweninfer_b200.models.qwen2 import _AttnScratch
    rng = np.random.default_rng(M * 1000 + max_len)
    rows_total = 4
    kc = bf16_round(rng.standard_normal((rows_total, 2, max_len, 64)).astype(np.float32))
    vc = bf16_round(rng.standard_normal((rows_total, 2, max_len, 64)).astype(np.float32))
    q = rng.standard_normal((M, 896)).astype(np.float32) * 2
    pos = np.array(positions) if positions is not None else rng.integers(0, max_len, M)
    rows = rng.integers(0, rows_total, M)
    ws = _AttnScratch(M, max_len, torch.device(DEV))
    out = torch.empty(M, 896, device=DEV)
    kcd, vcd = bf16_tensor(kc).to(DEV), bf16_tensor(vc).to(DEV)
    for rep in range(2):  # second call checks the counters were left at zero
        _lib.check(_lib.lib().qi_attention(
            f32(q).data_ptr(), kcd.data_ptr(), vcd.data_ptr(), i32(pos).data_ptr(), i32(rows).data_ptr(), M,
            max_len, ws.split_keys, ws.max_splits, out.data_ptr(), ws.part.data_ptr(), ws.counters.data_ptr(),
            ws.err.data_ptr(), stream()), "attention")
        assert_no_device_error(ws.err)
        assert int(ws.counters.abs().sum()) == 0
        got = out.cpu().numpy()
        for t in range(M):
            n = pos[t] + 1
            for h in range(14):
                g = h // 7
                s = (kc[rows[t], g, :n] @ q[t, h * 64:(h + 1) * 64].astype(np.float64)) / 8.0
                p = np.exp(s - s.max())
                ref = (p / p.sum()) @ vc[rows[t], g, :n]
                assert np.abs(got[t, h * 64:(h + 1) * 64] - ref).max() < TOL_F32, (t, h)


def _prefill_layout(lens, rows):
    """A batched prefill's query tokens (DecodeRunner.prefill_many): every prompt's tokens but
    the last in order, then all prompts' last tokens."""
    pos = [q for n in lens for q in range(n - 1)] + [n - 1 for n in lens]
    rws = [r for n, r in zip(lens, rows) for _ in range(n - 1)] + list(rows)
    return np.array(pos), np.array(rws)


PREFILL_CASES = ["one_prompt", "batched", "ragged", "long", "bad_position"]


@pytest.mark.parametrize("case", PREFILL_CASES)
def test_attention_prefill_blocks(case):
    """More than 128 queries run the block kernel (16 consecutive tokens of one row as one
    tcgen05 tile, else token by token on CUDA cores) vs an fp64 reference; a query outside
    the cache is reported and its output left untouched."""
    from qweninfer_b200.models.qwen2 import _AttnScratch
    rng = np.random.default_rng(40 + PREFILL_CASES.index(case))
    max_len, rows_total = 512, 4
    if case == "one_prompt":
        pos, rows = np.arange(300), np.full(300, 2)
    elif case == "batched":
        pos, rows = _prefill_layout([150, 37, 200, 1], [3, 0, 1, 2])
    elif case == "ragged":  # every block mixes rows: the token-by-token path
        pos, rows = rng.integers(0, max_len, 200), rng.integers(0, rows_total, 200)
    elif case == "long":
        max_len = 4096
        pos, rows = _prefill_layout([1100, 700], [1, 3])
    else:
        pos, rows = np.arange(160), np.full(160, 1)
        pos[37] = max_len
    M = len(pos)
    kc = bf16_round(rng.standard_normal((rows_total, 2, max_len, 64)).astype(np.float32))
    vc = bf16_round(rng.standard_normal((rows_total, 2, max_len, 64)).astype(np.float32))
    q = rng.standard_normal((M, 896)).astype(np.float32) * 2
    ws = _AttnScratch(M, max_len, torch.device(DEV))
    out = torch.full((M, 896), 7.0, device=DEV)
    kcd, vcd = bf16_tensor(kc).to(DEV), bf16_tensor(vc).to(DEV)
    _lib.check(_lib.lib().qi_attention(
        f32(q).data_ptr(), kcd.data_ptr(), vcd.data_ptr(), i32(pos).data_ptr(), i32(rows).data_ptr(), M,
        max_len, ws.split_keys, ws.max_splits, out.data_ptr(), ws.part.data_ptr(), ws.counters.data_ptr(),
        ws.err.data_ptr(), stream()), "attention")
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    bad = pos >= max_len
    assert int(ws.err.item()) == (_lib.QI_ERR_INDEX if bad.any() else 0)
    assert (got[bad] == 7.0).all()
    qd = q.astype(np.float64).reshape(M, 14, 64)
    for t in np.flatnonzero(~bad):
        n = pos[t] + 1
        for g in range(2):
            s = qd[t, 7 * g:7 * g + 7] @ kc[rows[t], g, :n].T.astype(np.float64) / 8.0   # (7, n)
            pr = np.exp(s - s.max(axis=1, keepdims=True))
            ref = (pr / pr.sum(axis=1, keepdims=True)) @ vc[rows[t], g, :n]
            err = np.abs(got[t].reshape(14, 64)[7 * g:7 * g + 7] - ref).max()
            # tensor-core blocks carry q and p as hi + lo bf16 (~16 significant bits, the
            # precision of the o projection's operand): scores within ~1e-5 relative, and
            # rows over a few dozen keys, where single terms dominate, within 1e-4
            assert err < 1e-4, (t, g, err)


@pytest.mark.parametrize("M", [1, 4, 11])
def test_residual_projections(M):
    rng = np.random.default_rng(5)
    wo = bf16_round(rng.normal(0, 0.02, (896, 896)).astype(np.float32))
    wd = bf16_round(rng.normal(0, 0.02, (896, 4864)).astype(np.float32))
    a = rng.standard_normal((M, 896)).astype(np.float32)
    h = rng.standard_normal((M, 4864)).astype(np.float32)
    x0 = rng.standard_normal((M, 896)).astype(np.float32)
    x = f32(x0)
    err = err_word()
    L = _lib.lib()
    _lib.check(L.qi_o_proj_residual(f32(a).data_ptr(), dev(tile_weight(bf16_tensor(wo))).data_ptr(), M,
                                    x.data_ptr(), err.data_ptr(), stream()), "o")
    ref = x0 + a @ wo.T
    assert np.abs(x.cpu().numpy() - ref).max() < 5e-5
    _lib.check(L.qi_down_residual(f32(h).data_ptr(), dev(tile_weight(bf16_tensor(wd))).data_ptr(), M,
                                  x.data_ptr(), err.data_ptr(), stream()), "down")
    ref = ref + h @ wd.T
    assert np.abs(x.cpu().numpy() - ref).max() < 1e-4
    assert_no_device_error(err)


@pytest.mark.parametrize("M,vocab", [(1, 151936), (3, 151936), (11, 4096)])
def test_lm_head_logits_and_argmax(M, vocab):
    rng = np.random.default_rng(7)
    E = bf16_round(rng.normal(0, 0.02, (vocab, 896)).astype(np.float32))
    nw = bf16_round((1 + rng.normal(0, 0.1, 896)).astype(np.float32))
    x = rng.standard_normal((M, 896)).astype(np.float32) * 5
    Et = tile_weight(bf16_tensor(E)).to(DEV)
    logits = torch.empty(M, vocab, device=DEV)
    slots = torch.zeros(M, dtype=torch.int64, device=DEV)
    err = err_word()
    _lib.check(_lib.lib().qi_lm_head_argmax(f32(x).data_ptr(), 896, f32(nw).data_ptr(), C.c_float(1e-6),
                                            Et.data_ptr(), vocab, M, logits.data_ptr(), 0, vocab,
                                            slots.data_ptr(), err.data_ptr(), stream()), "lm_head")
    assert_no_device_error(err)
    ref = rmsnorm(x, nw, 1e-6) @ E.T
    got = logits.cpu().numpy()
    assert np.abs(got - ref).max() < 5e-5
    idx = (0xFFFFFFFF - (slots.cpu().numpy() & 0xFFFFFFFF))
    assert np.array_equal(idx, np.argmax(got, 1))   # argmax of the very logits written


def test_lm_head_ties_pick_lowest_index():
    vocab, M = 4096, 2
    rng = np.random.default_rng(8)
    E = bf16_round(rng.normal(0, 0.02, (vocab, 896)).astype(np.float32))
    E[3001] = E[17] = E[2500] = 0.5   # identical best rows
    x = np.ones((M, 896), np.float32)
    nw = np.ones(896, np.float32)
    Et = tile_weight(bf16_tensor(E)).to(DEV)
    slots = torch.zeros(M, dtype=torch.int64, device=DEV)
    err = err_word()
    _lib.check(_lib.lib().qi_lm_head_argmax(f32(x).data_ptr(), 896, f32(nw).data_ptr(), C.c_float(1e-6),
                                            Et.data_ptr(), vocab, M, None, 0, 0, slots.data_ptr(),
                                            err.data_ptr(), stream()), "lm_head")
    idx = 0xFFFFFFFF - (slots.cpu().numpy() & 0xFFFFFFFF)
    assert idx.tolist() == [17, 17]


def test_embed_gather():
    rng = np.random.default_rng(9)
    vocab = 1024
    E = bf16_round(rng.standard_normal((vocab, 896)).astype(np.float32))
    ids = np.array([0, 5, 1023, 5, 77])
    x = torch.empty(len(ids), 896, device=DEV)
    slots = torch.full((len(ids),), -1, dtype=torch.int64, device=DEV)
    _lib.check(_lib.lib().qi_embed(dev(tile_weight(bf16_tensor(E))).data_ptr(), vocab, i32(ids).data_ptr(),
                                   len(ids), x.data_ptr(), slots.data_ptr(), None, stream()), "embed")
    assert np.array_equal(x.cpu().numpy(), E[ids])
    assert int(slots.abs().sum()) == 0


def test_move_rows_kernel():
    from qweninfer_b200.engine.kv_cache import KVCache
    cfg = qwen2_0p5b(3, 256)
    cache = KVCache(cfg, 5, 96, dtype=torch.bfloat16, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(0)
    cache.k.copy_(torch.randn(cache.k.shape, generator=g, device=DEV).to(torch.bfloat16))
    cache.v.copy_(torch.randn(cache.v.shape, generator=g, device=DEV).to(torch.bfloat16))
    k0, v0 = cache.k.clone(), cache.v.clone()
    moves = [(4, 1, 50), (3, 0, 96), (2, 3, 1)]
    cache.move_rows(moves)
    for s, d, n in moves:
        k0[:, d, :, :n] = k0[:, s, :, :n]
        v0[:, d, :, :n] = v0[:, s, :, :n]
    torch.cuda.synchronize()
    assert torch.equal(cache.k, k0) and torch.equal(cache.v, v0)
