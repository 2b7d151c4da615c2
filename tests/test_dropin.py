"""The drop-in boundary on CPU: QwenInfer's own import lines (tests/test_parity.py:6-30,
tests/test_cache.py:16-18, tests/conftest.py:42 of the reference) resolve against the
`qweninfer` package here, with the reference's signatures and defaults (names, order and
default values of every parameter, restated below from qweninfer/models/qwen2.py:243-315,
qweninfer/engine/kv_cache.py:24-28, engine.py:62-66 and 199-202, generate.py:18-23)."""

from __future__ import annotations

import inspect

import torch


def _params(fn):
    return [(p.name, p.default) for p in inspect.signature(fn).parameters.values()]


def test_reference_import_lines_resolve():
    from qweninfer.engine.engine import Engine, Request, autotune_padding  # noqa: F401
    from qweninfer.engine.generate import generate  # noqa: F401
    from qweninfer.engine.kv_cache import KVCache  # noqa: F401
    from qweninfer.models.config import Qwen2Config  # noqa: F401
    import qweninfer.models.qwen2 as student
    for name in ("RMSNorm", "build_rope_cache", "_rotate_half", "apply_rope", "MLP", "Attention", "Block",
                 "Qwen2"):
        assert hasattr(student, name), name


def test_signatures_match_the_reference():
    from qweninfer.engine.engine import Engine, autotune_padding
    from qweninfer.engine.generate import generate
    from qweninfer.engine.kv_cache import KVCache
    from qweninfer.models.qwen2 import Qwen2, RMSNorm, apply_rope, build_rope_cache
    assert _params(Qwen2.from_pretrained)[:6] == [
        ("path", inspect.Parameter.empty), ("dtype", torch.float16), ("device", "cuda"), ("max_seq_len", 4096),
        ("fuse", True), ("residual_fp32", True)]
    assert _params(Qwen2.forward)[:5] == [("self", inspect.Parameter.empty), ("input_ids", inspect.Parameter.empty),
                                          ("positions", None), ("cache", None), ("last_only", False)]
    assert _params(Qwen2.__init__)[1:4] == [("cfg", inspect.Parameter.empty), ("max_seq_len", 4096),
                                            ("residual_fp32", False)]
    assert _params(KVCache.__init__)[1:6] == [("cfg", inspect.Parameter.empty), ("max_batch", inspect.Parameter.empty),
                                              ("max_len", inspect.Parameter.empty), ("dtype", torch.float16),
                                              ("device", "cuda")]
    assert [n for n, _ in _params(KVCache.update)] == ["self", "layer", "k", "v", "positions"]
    assert [n for n, _ in _params(KVCache.move_row)] == ["self", "src", "dst", "length"]
    assert _params(generate)[:6] == [("model", inspect.Parameter.empty), ("prompt_ids", inspect.Parameter.empty),
                                     ("max_new_tokens", inspect.Parameter.empty), ("eos_ids", None), ("cache", None),
                                     ("on_token", None)]
    assert _params(Engine.__init__)[1:8] == [
        ("model", inspect.Parameter.empty), ("max_slots", inspect.Parameter.empty),
        ("max_len", inspect.Parameter.empty), ("eos_ids", None), ("static", False),
        ("max_prefills_per_step", None), ("pad_to", None)]
    assert _params(autotune_padding) == [("model", inspect.Parameter.empty), ("max_slots", inspect.Parameter.empty),
                                         ("max_rows", None), ("candidates", None), ("context", 128), ("iters", 8)]
    assert _params(RMSNorm.__init__)[1:] == [("hidden_dim", inspect.Parameter.empty), ("eps", 1e-6)]
    assert [n for n, _ in _params(build_rope_cache)][:3] == ["head_dim", "max_seq_len", "theta"]
    assert [n for n, _ in _params(apply_rope)] == ["q", "k", "cos", "sin", "positions"]


def test_rotate_half_convention():
    from qweninfer.models.qwen2 import _rotate_half
    x = torch.arange(8.0).reshape(1, 8)
    assert _rotate_half(x).tolist() == [[-4.0, -5.0, -6.0, -7.0, 0.0, 1.0, 2.0, 3.0]]


def test_default_dtypes_are_accepted():
    """The reference defaults to float16; the cache is then held in bfloat16 (the kernels'
    storage format) instead of raising."""
    from qweninfer.engine.kv_cache import KVCache
    from qweninfer_b200.models.config import qwen2_0p5b
    c = KVCache(qwen2_0p5b(num_hidden_layers=1), 1, 4, device="cpu")
    assert c.k.dtype == torch.bfloat16 and c.k.shape == (1, 1, 2, 4, 64)
