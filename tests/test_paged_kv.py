"""The paged KV cache (PagedKVCache; no reference counterpart: QwenInfer keeps packed rows).

CPU: the host-side page allocator (reserve / release / move_row, pool exhaustion) and the
engine's use of it over the 96-request serving trace, with a runner that reserves what
it writes as the device runner does: the scheduler decisions stay the reference's and
every page comes back to the pool.
GPU: the forward on a paged cache equals the forward on a packed one bit for bit (the
kernels do the same arithmetic, only the K/V addresses differ), across page boundaries,
for prefill and batched decode; an engine on a paged cache, with a pool smaller than
rows x max_len, produces the packed engine's outputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from qweninfer_b200.engine.engine import Engine, Request
from qweninfer_b200.engine.kv_cache import KVCache, PagedKVCache
from qweninfer_b200.models.config import qwen2_0p5b

from test_engine_host import StubRunner, fake_model, stub_token, VOCAB


def small_cache(**kw) -> PagedKVCache:
    return PagedKVCache(qwen2_0p5b(num_hidden_layers=2), 4, 512, device="cpu", **kw)


def test_reserve_maps_a_prefix_of_pages():
    c = small_cache()
    assert c.pages_per_row == 4 and c.n_pages == 16
    c.reserve(1, 129)
    assert (c.table_host[1, :2] >= 0).all() and (c.table_host[1, 2:] == -1).all()
    c.reserve(1, 100)  # already mapped: nothing taken
    assert c.pages_in_use() == 2
    c.reserve(1, 512)
    assert c.pages_in_use() == 4 and len(set(c.table_host[1].tolist())) == 4


def test_release_and_move_row_keep_the_pool_whole():
    c = small_cache(n_pages=5)
    c.reserve(0, 300)   # 3 pages
    c.reserve(3, 10)    # 1 page
    pages3 = c.table_host[3].tolist()
    c.move_row(src=3, dst=0, length=10)   # row 0's 3 pages back, row 3's page moves
    assert c.table_host[0].tolist() == pages3 and (c.table_host[3] == -1).all()
    assert c.pages_in_use() == 1
    c.release(0)
    assert c.pages_in_use() == 0 and sorted(c.free) == list(range(5))


def test_pool_exhaustion_raises():
    c = small_cache(n_pages=2)
    c.reserve(0, 256)
    with pytest.raises(RuntimeError, match="exhausted"):
        c.reserve(1, 1)


def test_page_size_must_be_whole_tiles():
    with pytest.raises(ValueError):
        small_cache(page_size=64)


class ReservingRunner(StubRunner):
    """The device runner's storage calls without a device: reserve before every write,
    and check that every position a forward touches is mapped."""

    def _mapped(self, row, length):
        c = self.cache
        need = -(-length // c.page_size)
        assert (c.table_host[row, :need] >= 0).all(), (row, length)

    def prefill(self, row, prompt):
        self.cache.reserve(row, len(prompt))
        self._mapped(row, len(prompt))
        return stub_token(prompt[-1], len(prompt) - 1, VOCAB)

    def prefill_many(self, rows, prompts):
        return [self.prefill(r, p) for r, p in zip(rows, prompts)]

    def decode(self, toks, pos, row_start=0):
        for b, q in enumerate(pos):
            self.cache.reserve(row_start + b, q + 1)
            self._mapped(row_start + b, q + 1)
        return np.array([stub_token(t, p, VOCAB) for t, p in zip(toks, pos)])


class PagedStubEngine(Engine):
    runner_cls = ReservingRunner


def test_engine_pages_follow_the_live_rows():
    """The 96-request trace on a paged cache: after every step the pages in use are those
    the active rows need (lengths rounded up to pages), and all come back at the end; the
    finished requests and their outputs are the packed engine's."""
    from qweninfer_b200 import synthetic
    from test_engine_host import StubEngine
    reqs = lambda: [Request(r.rid, r.prompt, r.max_new_tokens) for r in synthetic.serving96()]  # noqa: E731
    eng = PagedStubEngine(fake_model(), max_slots=32, max_len=512, page_size=128)
    assert isinstance(eng.cache, PagedKVCache)
    for r in reqs():
        eng.submit(r)
    done = []
    while eng.waiting or eng.active:
        done += eng.step()
        # the active rows hold positions 0 .. length - 1, exactly the pages they need
        assert eng.cache.pages_in_use() == sum(-(-r.length // 128) for r in eng.active)
    assert eng.cache.pages_in_use() == 0
    ref = StubEngine(fake_model(), max_slots=32, max_len=512).run(reqs())
    assert [(r.rid, r.output) for r in sorted(done, key=lambda r: r.rid)] == [(r.rid, r.output) for r in ref]


# ---------------------------------------------------------------------------- GPU


@pytest.mark.gpu
@pytest.mark.slow
def test_paged_forward_equals_packed(gpu_model):
    """Prompts across page boundaries into rows of a paged cache whose pages are scattered
    (reserved out of order), then a batched decode step: logits equal to the packed
    cache's, bit for bit."""
    from qweninfer_b200.engine.runner import DecodeRunner
    rng = np.random.default_rng(12)
    lens = [127, 128, 129, 300, 5]
    prompts = [rng.integers(0, gpu_model.cfg.vocab_size, n).tolist() for n in lens]
    out = []
    for paged in (False, True):
        if paged:
            cache = PagedKVCache(gpu_model.cfg, 6, 512, dtype=torch.bfloat16, device="cuda")
            for row in (5, 3, 1):  # take pages so that rows' pages are not in order
                cache.reserve(row, 256)
            for row in (5, 3, 1):
                cache.release(row)
        else:
            cache = KVCache(gpu_model.cfg, 6, 512, dtype=torch.bfloat16, device="cuda")
        r = DecodeRunner(gpu_model, cache, max_batch=6)
        firsts = [r.prefill(row, p) for row, p in enumerate(prompts)]
        toks = r.decode(firsts, [len(p) for p in prompts])
        logits = gpu_model(torch.tensor([[int(t)] for t in toks]), positions=torch.tensor([[n + 1] for n in lens]),
                           cache=cache, logits_dtype=torch.float32)[:, -1]
        r.check()
        out.append((firsts, toks.tolist(), logits.cpu().numpy()))
    assert out[0][0] == out[1][0] and out[0][1] == out[1][1]
    assert np.array_equal(out[0][2], out[1][2])


@pytest.mark.gpu
@pytest.mark.slow
def test_paged_engine_matches_packed(gpu_model):
    """An engine on a paged cache whose pool (24 pages of 128 positions) is smaller than
    its 8 rows x 512 slots (32 pages) but holds the live tokens (every request needs at
    most 3 pages) serves requests of mixed lengths with the packed engine's outputs, and
    returns every page."""
    rng = np.random.default_rng(21)
    specs = [(int(rng.integers(20, 300)), int(rng.integers(1, 60))) for _ in range(20)]
    reqs = lambda: [Request(i, rng2.integers(0, gpu_model.cfg.vocab_size, p).tolist(), n)  # noqa: E731
                    for i, (p, n) in enumerate(specs)]
    rng2 = np.random.default_rng(22)
    packed = Engine(gpu_model, max_slots=8, max_len=512).run(reqs())
    rng2 = np.random.default_rng(22)
    eng = Engine(gpu_model, max_slots=8, max_len=512, page_size=128, kv_pages=24)
    paged = eng.run(reqs())
    eng.runner.check()
    assert [r.output for r in paged] == [r.output for r in packed]
    assert eng.cache.pages_in_use() == 0
